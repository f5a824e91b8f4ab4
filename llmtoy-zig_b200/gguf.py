"""GGUF files for the seeded synthetic models (the benchmark configs are
specified as "emitted from a seed as a synthetic GGUF file").

The container is the one src/gguf/reader.zig parses: magic "GGUF", version 3,
u64 tensor and metadata counts, typed key/value pairs, tensor infos
(name, dims innermost first, ggml type, data offset), tensor data from the
first 32-byte boundary after the infos (types.zig ALIGNMENT), each tensor at
a 32-byte aligned offset.  Tensor names and metadata keys follow the
llama.cpp convention the reference loader reads (src/model/loader.zig:1-20,
configFromGguf at :37-83), plus the MoE names llama.cpp uses for Qwen3-MoE
(ffn_gate_inp, ffn_{gate,up,down}_exps, attn_{q,k}_norm).
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

MAGIC = 0x46554747
ALIGNMENT = 32
# MetaValueType (src/gguf/types.zig:6-20)
U8, I8, U16, I16, U32, I32, F32V, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(v) -> tuple[int, bytes]:
    if isinstance(v, bool):
        return BOOL, struct.pack("<B", int(v))
    if isinstance(v, int):
        return (U32, struct.pack("<I", v)) if 0 <= v < 2 ** 32 else (U64, struct.pack("<Q", v))
    if isinstance(v, float):
        return F32V, struct.pack("<f", v)
    if isinstance(v, str):
        return STRING, _str(v)
    if isinstance(v, (list, tuple)):
        if not v:
            return ARRAY, struct.pack("<IQ", U32, 0)
        t0, _ = _value(v[0])
        return ARRAY, struct.pack("<IQ", t0, len(v)) + b"".join(_value(x)[1] for x in v)
    raise TypeError(type(v))


def write_gguf(path, metadata: dict, tensors: list) -> None:
    """tensors: (name, ggml_type, dims innermost first, raw bytes) in file order."""
    head = struct.pack("<IIQQ", MAGIC, 3, len(tensors), len(metadata))
    for k, v in metadata.items():
        t, b = _value(v)
        head += _str(k) + struct.pack("<I", t) + b
    offsets, off = [], 0
    for _, _, _, data in tensors:
        offsets.append(off)
        off += (len(memoryview(data).cast("B")) + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT
    for (name, t, dims, _), o in zip(tensors, offsets):
        head += _str(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
        head += struct.pack("<IQ", t, o)
    pad = (-len(head)) % ALIGNMENT
    with open(path, "wb") as f:
        f.write(head + b"\0" * pad)
        for (_, _, _, data), o in zip(tensors, offsets):
            b = memoryview(np.ascontiguousarray(data)).cast("B")
            f.write(b)
            f.write(b"\0" * ((-len(b)) % ALIGNMENT))


def model_tensors(m, arch: str) -> tuple[dict, list]:
    """Metadata and tensors of a synth.DecoderModel under llama.cpp names."""
    F32 = 0
    d = m.d_model
    meta = {
        "general.architecture": arch,
        "general.name": f"llmtoy-zig synthetic {arch}",
        f"{arch}.context_length": 4096,
        f"{arch}.embedding_length": d,
        f"{arch}.block_count": m.n_layers,
        f"{arch}.attention.head_count": m.n_heads,
        f"{arch}.attention.head_count_kv": m.n_kv_heads,
        f"{arch}.attention.key_length": m.head_dim,
        f"{arch}.attention.value_length": m.head_dim,
        f"{arch}.feed_forward_length": m.d_ffn if m.d_ffn else m.d_expert,
        f"{arch}.attention.layer_norm_rms_epsilon": float(m.eps),
        f"{arch}.rope.freq_base": float(m.rope_theta),
        f"{arch}.vocab_size": m.vocab,
        "tokenizer.ggml.bos_token_id": 1,
        "tokenizer.ggml.eos_token_id": 2,
    }
    if m.n_experts:
        meta[f"{arch}.expert_count"] = m.n_experts
        meta[f"{arch}.expert_used_count"] = m.k
        meta[f"{arch}.expert_feed_forward_length"] = m.d_expert
    nq, nkv = m.n_heads * m.head_dim, m.n_kv_heads * m.head_dim
    ts = [("token_embd.weight", m.emb_type, [d, m.vocab], m.token_emb)]
    for i, L in enumerate(m.layers):
        p = f"blk.{i}."
        ts += [(p + "attn_norm.weight", F32, [d], L.attn_norm),
               (p + "attn_q.weight", L.attn_type, [d, nq], L.wq),
               (p + "attn_k.weight", L.attn_type, [d, nkv], L.wk),
               (p + "attn_v.weight", L.attn_type, [d, nkv], L.wv),
               (p + "attn_output.weight", L.attn_type, [nq, d], L.wo)]
        if L.qkv_bias is not None:
            b = L.qkv_bias
            ts += [(p + "attn_q.bias", F32, [nq], b[:nq]), (p + "attn_k.bias", F32, [nkv], b[nq:nq + nkv]),
                   (p + "attn_v.bias", F32, [nkv], b[nq + nkv:])]
        if L.q_norm is not None:
            ts += [(p + "attn_q_norm.weight", F32, [m.head_dim], L.q_norm),
                   (p + "attn_k_norm.weight", F32, [m.head_dim], L.k_norm)]
        ts.append((p + "ffn_norm.weight", F32, [d], L.ffn_norm))
        if L.moe is None:
            ts += [(p + "ffn_gate.weight", L.ffn_type, [d, m.d_ffn], L.ffn_gate),
                   (p + "ffn_up.weight", L.ffn_type, [d, m.d_ffn], L.ffn_up),
                   (p + "ffn_down.weight", L.ffn_type, [m.d_ffn, d], L.ffn_down)]
        else:
            E, Fe = m.n_experts, m.d_expert
            ts += [(p + "ffn_gate_inp.weight", F32, [d, E], L.moe.router),
                   (p + "ffn_gate_exps.weight", L.moe.gate_type, [d, Fe, E], L.moe.gate),
                   (p + "ffn_up_exps.weight", L.moe.gate_type, [d, Fe, E], L.moe.up),
                   (p + "ffn_down_exps.weight", L.moe.down_type, [Fe, d, E], L.moe.down)]
    ts += [("output_norm.weight", F32, [d], m.out_norm), ("output.weight", m.lm_type, [d, m.vocab], m.lm_head)]
    return meta, ts


def write_model(path, m, arch: str | None = None) -> Path:
    """Write a synth.DecoderModel as a GGUF file (arch: "qwen2" dense, "qwen3moe" MoE)."""
    arch = arch or ("qwen3moe" if m.n_experts else "qwen2")
    meta, ts = model_tensors(m, arch)
    write_gguf(path, meta, ts)
    return Path(path)
