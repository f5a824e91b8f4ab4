/*
 * gguf.h — GGUF ingest for the host decode loop (libllmtoy_host.so).
 *
 * lth_gguf_open memory-maps a file and parses it as src/gguf/reader.zig does
 * (versions 1-3, typed metadata, tensor infos, data at the first 32-byte
 * boundary after them).  lth_gguf_info prints what `llmtoy info` prints
 * (src/main.zig:520-618).  lth_model_load builds a device model from it:
 * configFromGguf + loadWeights (src/model/loader.zig:37-145) for dense
 * llama-style files, plus the Qwen3-MoE tensors (router, 3-D expert
 * tensors, per-head Q/K norms); the mapped bytes go up through lt_upload.
 */
#ifndef LLMTOY_HOST_GGUF_H
#define LLMTOY_HOST_GGUF_H

#include "decoder.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lth_gguf lth_gguf;
typedef struct lth_loaded lth_loaded;

lt_status lth_gguf_open(const char *path, lth_gguf **out);
void lth_gguf_close(lth_gguf *g);
/* The info report as text into buf (NUL-terminated, cut at size); returns its full length. */
size_t lth_gguf_info(const lth_gguf *g, char *buf, size_t size);
/* Number of tensors, and tensor i's name / ggml type / byte size. */
uint64_t lth_gguf_tensor_count(const lth_gguf *g);
lt_status lth_gguf_tensor(const lth_gguf *g, uint64_t i, const char **name, uint32_t *ggml_type,
                          uint64_t *nbytes);

/* Upload a decoder from an open file onto ctx's device (kv_cap positions
 * of KV cache).  The file may be closed afterwards. */
lt_status lth_model_load(lt_ctx *ctx, const lth_gguf *g, uint32_t kv_cap, lth_loaded **out);
lth_decoder *lth_loaded_decoder(const lth_loaded *m);
/* The shape the loader read: {n_layers, d_model, n_heads, n_kv_heads, head_dim, vocab, n_experts, n_used}. */
void lth_loaded_shape(const lth_loaded *m, uint32_t out[8]);
void lth_loaded_free(lth_loaded *m);

#ifdef __cplusplus
}
#endif
#endif
