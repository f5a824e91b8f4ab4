"""Seeded synthetic GGUF tensors with the value distributions of the benchmark configs.

Every generator takes a ``numpy.random.Generator`` (PCG64) and returns raw GGUF
bytes in the reference's block layouts (src/quant/dequant.zig):

* Q4_K (144 B / 256): f16 d ~ U(1e-3, 4e-3), f16 dmin ~ U(0, 2e-3), uniform
  6-bit scales/mins and uniform nibbles (uniform random bytes give both).
* Q6_K (210 B / 256): uniform ql/qh bytes, uniform int8 scales, f16 d ~ U(1e-3, 4e-3).
* Q8_0 (34 B / 32): f16 d = 0.02/127 * U(0.5, 1.5), int8 quants uniform in [-127, 127].
* Q5_0 (22 B / 32), Q5_1 (24 B / 32), IQ4_NL (18 B / 32), Q5_K (176 B / 256),
  Q3_K (110 B / 256): uniform random bytes with finite f16 scales of the same
  weight magnitude (~0.02); these formats appear in no benchmark config.
* router weights f32 N(0, 0.02); hidden states f32 N(0, 1).

``stamp_d`` reproduces the reference's GPU fuzz generator instead: every f16
scale field set to 0x21CD (~0.012) over random bytes (src/gpu/matvec.zig:4568-4586).
"""
from __future__ import annotations

import numpy as np

F32, F16, Q8_0, Q4_K, Q6_K = 0, 1, 8, 12, 14
Q5_0, Q5_1, Q3_K, Q5_K, IQ4_NL = 6, 7, 11, 13, 20
BLOCK = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210), Q5_0: (32, 22),
         Q5_1: (32, 24), IQ4_NL: (32, 18), Q5_K: (256, 176), Q3_K: (256, 110)}

CONFIG_SEED_BASE = 0x11A70000


def config_seed(index: int) -> int:
    return CONFIG_SEED_BASE + index


def _f16_bytes(vals: np.ndarray) -> np.ndarray:
    return vals.astype(np.float16).view(np.uint8).reshape(-1, 2)


def q4k_blocks(rng: np.random.Generator, n: int, stamp_d: bool = False) -> np.ndarray:
    b = rng.integers(0, 256, size=(n, 144), dtype=np.uint8)
    if stamp_d:
        b[:, 0], b[:, 1], b[:, 2], b[:, 3] = 0xCD, 0x21, 0xCD, 0x21
    else:
        b[:, 0:2] = _f16_bytes(rng.uniform(1e-3, 4e-3, n))
        b[:, 2:4] = _f16_bytes(rng.uniform(0.0, 2e-3, n))
    return b


def q6k_blocks(rng: np.random.Generator, n: int, stamp_d: bool = False) -> np.ndarray:
    b = rng.integers(0, 256, size=(n, 210), dtype=np.uint8)
    if stamp_d:
        b[:, 208], b[:, 209] = 0xCD, 0x21
    else:
        b[:, 208:210] = _f16_bytes(rng.uniform(1e-3, 4e-3, n))
    return b


def other_blocks(rng: np.random.Generator, t: int, n: int) -> np.ndarray:
    """Random blocks of the further formats with their f16 scale fields set."""
    b = rng.integers(0, 256, size=(n, BLOCK[t][1]), dtype=np.uint8)
    if t == Q5_0:
        b[:, 0:2] = _f16_bytes(0.02 / 16.0 * rng.uniform(0.5, 1.5, n))
    elif t == Q5_1:
        b[:, 0:2] = _f16_bytes(0.04 / 31.0 * rng.uniform(0.5, 1.5, n))
        b[:, 2:4] = _f16_bytes(-0.02 * rng.uniform(0.5, 1.5, n))
    elif t == IQ4_NL:
        b[:, 0:2] = _f16_bytes(0.02 / 127.0 * rng.uniform(0.5, 1.5, n))
    elif t == Q5_K:
        b[:, 0:2] = _f16_bytes(rng.uniform(5e-4, 2e-3, n))
        b[:, 2:4] = _f16_bytes(rng.uniform(0.0, 1e-3, n))
    elif t == Q3_K:
        b[:, 108:110] = _f16_bytes(rng.uniform(1e-4, 4e-4, n))
    return b


def q8_0_blocks(rng: np.random.Generator, n: int, stamp_d: bool = False) -> np.ndarray:
    b = np.empty((n, 34), dtype=np.uint8)
    if stamp_d:
        b[:, 2:] = rng.integers(0, 256, size=(n, 32), dtype=np.uint8)
        b[:, 0], b[:, 1] = 0xCD, 0x21
    else:
        b[:, 2:] = rng.integers(-127, 128, size=(n, 32), dtype=np.int8).view(np.uint8)
        b[:, 0:2] = _f16_bytes(0.02 / 127.0 * rng.uniform(0.5, 1.5, n))
    return b


def matrix(rng: np.random.Generator, ggml_type: int, rows: int, cols: int, stamp_d: bool = False) -> np.ndarray:
    """rows x cols tensor as GGUF bytes, shape [rows, rowBytes]."""
    elems, nbytes = BLOCK[ggml_type]
    if cols % elems:
        raise ValueError(f"cols {cols} not a multiple of {elems}")
    nb = rows * (cols // elems)
    if ggml_type == Q4_K:
        blk = q4k_blocks(rng, nb, stamp_d)
    elif ggml_type == Q6_K:
        blk = q6k_blocks(rng, nb, stamp_d)
    elif ggml_type == Q8_0:
        blk = q8_0_blocks(rng, nb, stamp_d)
    elif ggml_type in (Q5_0, Q5_1, IQ4_NL, Q5_K, Q3_K):
        blk = other_blocks(rng, ggml_type, nb)
    elif ggml_type == F32:
        blk = rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float32).view(np.uint8)
    elif ggml_type == F16:
        blk = rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float16).view(np.uint8)
    else:
        raise ValueError(ggml_type)
    return np.ascontiguousarray(blk).reshape(rows, (cols // elems) * nbytes)


def router_weights(rng: np.random.Generator, n_experts: int, d_model: int) -> np.ndarray:
    return rng.normal(0.0, 0.02, size=(n_experts, d_model)).astype(np.float32)


def hidden(rng: np.random.Generator, n_tok: int, d_model: int) -> np.ndarray:
    return rng.normal(0.0, 1.0, size=(n_tok, d_model)).astype(np.float32)


class MoeLayer:
    """One MoE FFN layer of the config-1 shape (router + SwiGLU experts)."""

    def __init__(self, rng: np.random.Generator, d_model: int = 2048, n_experts: int = 128, d_expert: int = 768,
                 gate_type: int = Q4_K, down_type: int = Q4_K, fused: bool = False):
        self.d_model, self.n_experts, self.d_expert = d_model, n_experts, d_expert
        self.gate_type, self.down_type, self.fused = gate_type, down_type, fused
        self.router = router_weights(rng, n_experts, d_model)
        if fused:
            self.gate = matrix(rng, gate_type, n_experts * 2 * d_expert, d_model)
            self.up = None
        else:
            self.gate = matrix(rng, gate_type, n_experts * d_expert, d_model)
            self.up = matrix(rng, gate_type, n_experts * d_expert, d_model)
        self.down = matrix(rng, down_type, n_experts * d_model, d_expert)

    @property
    def expert_bytes(self) -> int:
        """Weight bytes one selected expert streams (gate + up + down)."""
        e = self.n_experts
        return (self.gate.nbytes + (self.up.nbytes if self.up is not None else 0) + self.down.nbytes) // e


class DecoderLayer:
    """Attention + FFN weights of one decoder layer (GGUF bytes, f32 norms)."""

    def __init__(self, rng, d: int, n_heads: int, n_kv: int, hd: int, attn_type: int, qk_norm: bool,
                 qkv_bias: bool, norms_random: bool, d_ffn: int, ffn_type: int, moe: "MoeLayer | None"):
        nq, nkv = n_heads * hd, n_kv * hd
        norm = (lambda n: rng.uniform(0.5, 1.5, n).astype(np.float32)) if norms_random else \
            (lambda n: np.ones(n, np.float32))
        self.attn_norm, self.ffn_norm = norm(d), norm(d)
        self.wq = matrix(rng, attn_type, nq, d)
        self.wk = matrix(rng, attn_type, nkv, d)
        self.wv = matrix(rng, attn_type, nkv, d)
        self.wo = matrix(rng, attn_type, d, nq)
        self.attn_type = attn_type
        self.q_norm = norm(hd) if qk_norm else None
        self.k_norm = norm(hd) if qk_norm else None
        self.qkv_bias = rng.normal(0.0, 0.02, nq + 2 * nkv).astype(np.float32) if qkv_bias else None
        self.moe = moe
        if moe is None:
            self.ffn_type = ffn_type
            self.ffn_gate = matrix(rng, ffn_type, d_ffn, d)
            self.ffn_up = matrix(rng, ffn_type, d_ffn, d)
            self.ffn_down = matrix(rng, ffn_type, d, d_ffn)

    @property
    def wqkv(self) -> np.ndarray:
        """Q, K and V rows stacked (one matvec on the device)."""
        return np.concatenate([self.wq, self.wk, self.wv], axis=0)


class DecoderModel:
    """Seeded synthetic decoder: config 0 (dense Qwen2-0.5B shape: Q8_0
    everywhere, consecutive-pair RoPE) or config 2 (Qwen3-30B-A3B shape:
    Q8_0 attention with per-head Q/K RMSNorm and NeoX RoPE, Q4_K MoE FFN with
    renormalised top-k, Q6_K lm_head), at any size."""

    def __init__(self, rng, n_layers: int, d_model: int, n_heads: int, n_kv_heads: int, head_dim: int, vocab: int,
                 d_ffn: int = 0, n_experts: int = 0, k: int = 0, d_expert: int = 0, attn_type: int = Q8_0,
                 emb_type: int = Q8_0, lm_type: int = Q8_0, ffn_type: int = Q8_0, expert_type: int = Q4_K,
                 qk_norm: bool = False, qkv_bias: bool = False, rope_neox: bool = False, norm_topk: bool = False,
                 norms_random: bool = False, eps: float = 1e-6, rope_theta: float = 1e6):
        self.n_layers, self.d_model, self.n_heads, self.n_kv_heads = n_layers, d_model, n_heads, n_kv_heads
        self.head_dim, self.vocab, self.d_ffn = head_dim, vocab, d_ffn
        self.n_experts, self.k, self.d_expert = n_experts, k, d_expert
        self.emb_type, self.lm_type, self.attn_type = emb_type, lm_type, attn_type
        self.ffn_type, self.expert_type = ffn_type, expert_type
        self.rope_neox, self.norm_topk, self.eps, self.rope_theta = rope_neox, norm_topk, eps, rope_theta
        self.token_emb = matrix(rng, emb_type, vocab, d_model)
        self.layers = []
        for _ in range(n_layers):
            moe = MoeLayer(rng, d_model, n_experts, d_expert, expert_type, expert_type) if n_experts else None
            self.layers.append(DecoderLayer(rng, d_model, n_heads, n_kv_heads, head_dim, attn_type, qk_norm,
                                            qkv_bias, norms_random, d_ffn, ffn_type, moe))
        self.out_norm = (rng.uniform(0.5, 1.5, d_model) if norms_random else np.ones(d_model)).astype(np.float32)
        self.lm_head = matrix(rng, lm_type, vocab, d_model)


def config0_model(rng, n_layers: int = 24, vocab: int = 151936, **kw) -> DecoderModel:
    """Config 0: dense Qwen2-0.5B shape, all Q8_0."""
    return DecoderModel(rng, n_layers, 896, 14, 2, 64, vocab, d_ffn=4864, **kw)


def config2_model(rng, n_layers: int = 48, vocab: int = 151936, **kw) -> DecoderModel:
    """Config 2: Qwen3-30B-A3B shape, Q8_0 attention, Q4_K experts, Q6_K lm_head."""
    return DecoderModel(rng, n_layers, 2048, 32, 4, 128, vocab, n_experts=128, k=8, d_expert=768,
                        lm_type=Q6_K, qk_norm=True, rope_neox=True, norm_topk=True, **kw)


class GemmaLayer:
    """One Gemma 4 decoder layer (src/model/gemma4/weights.zig) with a seeded
    per-tensor quantisation mix; tensors whose columns are not a multiple of
    256 are Q8_0 (the K-quants need whole superblocks)."""

    def __init__(self, rng, d, n_heads, n_kv, hd, d_ffn, n_experts, d_expert, is_swa, pick, norms_random, wv=True):
        self.is_swa, self.n_kv_heads, self.head_dim = is_swa, n_kv, hd
        nq, nkv = n_heads * hd, n_kv * hd
        norm = (lambda n: rng.uniform(0.5, 1.5, n).astype(np.float32)) if norms_random else \
            (lambda n: np.ones(n, np.float32))
        self.attn_norm, self.post_attention_norm, self.ffn_norm = norm(d), norm(d), norm(d)
        self.pre_ffw_norm_2, self.post_ffw_norm_1, self.post_ffw_norm_2 = norm(d), norm(d), norm(d)
        self.post_ffw_norm = norm(d)
        self.q_norm, self.k_norm = norm(hd), norm(hd)
        self.layer_output_scale = np.float32(rng.uniform(0.5, 1.0) if norms_random else 1.0)
        self.types = {}

        def mat(name, rows, cols, n=1):
            t = pick(cols)
            self.types[name] = t
            return matrix(rng, t, n * rows, cols)

        self.wq = mat("wq", nq, d)
        self.wk = mat("wk", nkv, d)
        self.wv = mat("wv", nkv, d) if wv else None
        self.wo = mat("wo", d, nq)
        self.w_gate = mat("gate", d_ffn, d)
        t = self.types["gate"]  # gate and up share a type (one dense GeGLU pair)
        self.types["up"] = t
        self.w_up = matrix(rng, t, d_ffn, d)
        self.w_down = mat("down", d, d_ffn)
        self.router_w = router_weights(rng, n_experts, d)
        self.router_scale = norm(d)
        self.gate_up_exps = mat("gate_up_exps", 2 * d_expert, d, n_experts)
        self.down_exps = mat("down_exps", d, d_expert, n_experts)
        self.down_exps_scale = rng.uniform(0.5, 1.5, n_experts).astype(np.float32)


class GemmaModel:
    """Config 3: a Gemma-4-26B-A4B-like decoder (sliding-window : global = 5 : 1,
    128 GeGLU experts top-8 + a dense GeGLU FFN, soft-capped logits) with a
    seeded per-tensor mix of 60% Q4_K, 25% Q6_K, 15% Q8_0, Q8_0 where the
    columns are not a multiple of 256."""

    def __init__(self, rng, n_layers=30, d_model=2816, n_heads=16, n_kv_heads=8, head_dim=256, d_ffn=2112,
                 n_experts=128, k=8, d_expert=704, vocab=262144, sliding_window=1024, swa_period=6,
                 norms_random=False, eps=1e-6, rope_theta_swa=1e4, rope_theta_global=1e6, logit_softcap=30.0,
                 lm_type=Q6_K):
        self.n_layers, self.d_model, self.n_heads, self.d_ffn = n_layers, d_model, n_heads, d_ffn
        self.n_experts, self.k, self.d_expert, self.vocab = n_experts, k, d_expert, vocab
        self.sliding_window, self.eps = sliding_window, eps
        self.rope_theta_swa, self.rope_theta_global, self.logit_softcap = rope_theta_swa, rope_theta_global, logit_softcap

        def pick(cols):
            if cols % 256:
                return Q8_0
            u = rng.uniform()
            return Q4_K if u < 0.60 else Q6_K if u < 0.85 else Q8_0

        self.emb_type = pick(d_model)
        self.token_emb = matrix(rng, self.emb_type, vocab, d_model)
        self.layers = [GemmaLayer(rng, d_model, n_heads, n_kv_heads, head_dim, d_ffn, n_experts, d_expert,
                                  (i + 1) % swa_period != 0, pick, norms_random) for i in range(n_layers)]
        self.out_norm = (rng.uniform(0.5, 1.5, d_model) if norms_random else np.ones(d_model)).astype(np.float32)
        self.lm_type = lm_type
        self.lm_head = matrix(rng, lm_type, vocab, d_model)


def cycle_layers(m, n_layers: int, swa_period: int | None = None):
    """Deepen model m to n_layers by cycling its distinct layers (layer i
    shares the weight arrays of layer i % len(m.layers)).  A full-depth model
    then costs the host memory of a few layers while every layer still reads
    its weights from memory far larger than any cache.  swa_period (Gemma 4):
    layer i is sliding-window unless (i + 1) % swa_period == 0, the pattern of
    the full-depth model, whatever the pattern of the layer it shares."""
    base = list(m.layers)
    out = []
    for i in range(n_layers):
        src = base[i % len(base)]
        if swa_period is None:
            out.append(src)
            continue
        lay = object.__new__(type(src))
        lay.__dict__.update(src.__dict__)
        lay.is_swa = (i + 1) % swa_period != 0
        out.append(lay)
    m.layers = out
    m.n_layers = n_layers
    return m
