"""ctypes binding of the CPU oracle (oracle/liboracle.so) for the tests.

Test infrastructure only: the oracle is the checker the CUDA path is compared
with.  Built by `make -C oracle` (or llmtoy-zig_b200/build.py).
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent.parent
LIB = REPO / "oracle" / "liboracle.so"

F32, F16, Q8_0, Q4_K, Q6_K = 0, 1, 8, 12, 14
Q5_0, Q5_1, Q3_K, Q5_K, IQ4_NL = 6, 7, 11, 13, 20


class SoftmaxStats(ctypes.Structure):
    _fields_ = [("max", ctypes.c_float), ("exp_sum", ctypes.c_float)]


_lib = None


def use_library(path) -> None:
    """Load the oracle from another build of oracle.c (the timed CPU baseline's
    -march=native build); only before the first lib() call."""
    global LIB
    if _lib is not None:
        raise RuntimeError("the oracle library is loaded already")
    LIB = Path(path)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB.exists():
        subprocess.run(["make", "-s", "-C", str(REPO / "oracle")], check=True)
    L = ctypes.CDLL(str(LIB))
    P, SZ, U32, F, I = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32, ctypes.c_float, ctypes.c_int
    sig = {
        "orc_f16_to_f32": (F, [ctypes.c_uint16]),
        "orc_f32_to_f16": (ctypes.c_uint16, [F]),
        "orc_row_bytes": (SZ, [U32, SZ]),
        "orc_dequant_row": (I, [P, P, SZ, U32]),
        "orc_dot_q8_0": (F, [P, P, SZ]),
        "orc_dot_q5_0": (F, [P, P, SZ]),
        "orc_dot_iq4_nl": (F, [P, P, SZ]),
        "orc_quantize_q8_1": (None, [P, P, SZ]),
        "orc_dequant_q8_1": (None, [P, P, SZ]),
        "orc_pack_q8_1_x4": (None, [P, SZ, P]),
        "orc_unpack_q8_1_x4": (None, [P, SZ, P]),
        "orc_dotf32": (F, [P, P, SZ]),
        "orc_matvec": (None, [P, P, P, SZ, SZ]),
        "orc_quant_matvec": (I, [P, P, U32, P, SZ, SZ, P]),
        "orc_rmsnorm": (None, [P, P, P, SZ, F]),
        "orc_softmax": (None, [P, SZ]),
        "orc_silu": (F, [F]),
        "orc_gelu": (F, [F]),
        "orc_pool_create": (P, [I]),
        "orc_pool_destroy": (None, [P]),
        "orc_pool_threads": (I, [P]),
        "orc_quant_matvec_par": (I, [P, P, U32, P, SZ, SZ, P, P]),
        "orc_topk_with_softmax_stats": (SoftmaxStats, [P, SZ, P, SZ]),
        "orc_softmax_topk": (None, [P, SZ, P, SZ]),
        "orc_topk_matvec_f32": (SoftmaxStats, [P, P, SZ, SZ, P, P, SZ]),
        "orc_topk_matvec_f32_par": (SoftmaxStats, [P, P, SZ, SZ, P, P, SZ, P]),
        "orc_router_topk_softmax": (None, [P, P, SZ, P, SZ, SZ, P, P]),
        "orc_moe_topk": (None, [P, SZ, P, SZ]),
        "orc_moe_forward": (I, [P, P, SZ, P, U32, P, U32, P, SZ, SZ, SZ, P]),
        "orc_moe_layer": (I, [P, P, SZ, SZ, P, SZ, SZ, I, P, P, P, U32, P, U32, SZ, I, P, P, P]),
        "orc_greedy": (U32, [P, SZ]),
        "orc_rope": (None, [P, SZ, SZ, F, I]),
        "orc_sdp_attn": (None, [P, P, P, P, SZ, SZ, F]),
        "orc_model_step": (I, [P, P, P, SZ, U32, SZ, P, P]),
        "orc_gemma_step": (I, [P, P, P, SZ, U32, SZ, P, P]),
        "orc_rng_seed": (None, [P, ctypes.c_uint64]),
        "orc_rng_float": (F, [P]),
        "orc_sample": (U32, [P, SZ, F, U32, F, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


class Pool:
    def __init__(self, n: int):
        self.ptr = lib().orc_pool_create(n)

    def close(self):
        if self.ptr:
            lib().orc_pool_destroy(self.ptr)
            self.ptr = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def row_bytes(t: int, cols: int) -> int:
    return lib().orc_row_bytes(t, cols)


def dequant(data: np.ndarray, t: int, rows: int, cols: int) -> np.ndarray:
    data = np.ascontiguousarray(data, dtype=np.uint8).reshape(-1)
    rb = row_bytes(t, cols)
    out = np.empty((rows, cols), dtype=np.float32)
    for r in range(rows):
        rc = lib().orc_dequant_row(data[r * rb:].ctypes.data, out[r].ctypes.data, cols, t)
        assert rc == 0
    return out


def quantize_q8_1(x) -> bytes:
    x = f32(x)
    out = np.zeros(x.size // 32 * 36, np.uint8)
    lib().orc_quantize_q8_1(_p(x), _p(out), x.size)
    return out.tobytes()


def dequant_q8_1(data: bytes, n: int) -> np.ndarray:
    raw = np.frombuffer(data, np.uint8).copy()
    out = np.empty(n, np.float32)
    lib().orc_dequant_q8_1(_p(raw), _p(out), n)
    return out


def quant_matvec(mat: np.ndarray, t: int, vec: np.ndarray, rows: int, cols: int, pool: Pool | None = None):
    mat = np.ascontiguousarray(mat, dtype=np.uint8).reshape(-1)
    vec = f32(vec)
    out = np.empty(rows, dtype=np.float32)
    if pool is None:
        buf = np.empty(cols, dtype=np.float32)
        rc = lib().orc_quant_matvec(_p(out), _p(mat), t, _p(vec), rows, cols, _p(buf))
    else:
        n = lib().orc_pool_threads(pool.ptr)
        buf = np.empty(n * cols, dtype=np.float32)
        rc = lib().orc_quant_matvec_par(_p(out), _p(mat), t, _p(vec), rows, cols, _p(buf), pool.ptr)
    assert rc == 0
    return out


def dotf32(a, b) -> float:
    a, b = f32(a), f32(b)
    return lib().orc_dotf32(_p(a), _p(b), a.size)


def topk_stable(scores, k: int):
    s = f32(scores)
    out = np.empty(k, dtype=np.uint32)
    st = lib().orc_topk_with_softmax_stats(_p(s), s.size, _p(out), k)
    return out, (st.max, st.exp_sum)


def router_topk_softmax(router_w: np.ndarray, x: np.ndarray, k: int, pool: Pool | None = None):
    """routerTopKSoftmax: (ids, probabilities of the selected experts)."""
    w = f32(router_w)
    E, d = w.shape
    x = f32(x)
    scores = np.full(E, -999.0, dtype=np.float32)
    ids = np.empty(k, dtype=np.uint32)
    lib().orc_router_topk_softmax(_p(scores), _p(ids), k, _p(w), E, d, _p(x), pool.ptr if pool else None)
    return ids, scores[ids]


def moe_layer(layer, x: np.ndarray, k: int, norm_topk: bool, act: int = 0, expert_scale=None,
              pool: Pool | None = None):
    """orc_moe_layer over T tokens -> (out[T][d], ids[T][k], w[T][k])."""
    x = f32(x)
    T, d = x.shape
    out = np.empty_like(x)
    ids = np.empty((T, k), dtype=np.uint32)
    w = np.empty((T, k), dtype=np.float32)
    es = None if expert_scale is None else f32(expert_scale)
    rc = lib().orc_moe_layer(
        _p(out), _p(x), T, d, _p(f32(layer.router)), layer.n_experts, k, int(norm_topk), _p(es),
        _p(layer.gate), _p(layer.up), layer.gate_type, _p(layer.down), layer.down_type, layer.d_expert, act,
        pool.ptr if pool else None, _p(ids), _p(w))
    assert rc == 0
    return out, ids, w


def greedy(logits) -> int:
    a = f32(logits)
    return int(lib().orc_greedy(_p(a), a.size))


# ── decoder model (orc_model_step) ───────────────────────────────────────────

class OrcLayer(ctypes.Structure):
    P = ctypes.c_void_p
    _fields_ = [("attn_norm", P), ("ffn_norm", P), ("wq", P), ("wk", P), ("wv", P), ("wo", P),
                ("wq_type", ctypes.c_uint32), ("wk_type", ctypes.c_uint32), ("wv_type", ctypes.c_uint32),
                ("wo_type", ctypes.c_uint32), ("q_bias", P), ("k_bias", P), ("v_bias", P), ("q_norm", P),
                ("k_norm", P), ("w_gate", P), ("w_up", P), ("w_down", P), ("ffn_gate_type", ctypes.c_uint32),
                ("ffn_down_type", ctypes.c_uint32), ("router", P), ("e_gate", P), ("e_up", P), ("e_down", P),
                ("e_gate_type", ctypes.c_uint32), ("e_down_type", ctypes.c_uint32)]


class OrcModel(ctypes.Structure):
    SZ = ctypes.c_size_t
    _fields_ = [("n_layers", SZ), ("d_model", SZ), ("n_heads", SZ), ("n_kv_heads", SZ), ("head_dim", SZ),
                ("d_ffn", SZ), ("vocab", SZ), ("n_experts", SZ), ("k", SZ), ("d_expert", SZ),
                ("norm_topk", ctypes.c_int), ("rope_neox", ctypes.c_int), ("eps", ctypes.c_float),
                ("rope_theta", ctypes.c_float), ("token_emb", ctypes.c_void_p), ("emb_type", ctypes.c_uint32),
                ("out_norm", ctypes.c_void_p), ("lm_head", ctypes.c_void_p), ("lm_type", ctypes.c_uint32),
                ("layers", ctypes.POINTER(OrcLayer)), ("kv_f16", ctypes.c_int)]


class OracleDecoder:
    """orc_model_step over a synth.DecoderModel, with its own KV cache (f32, or
    f16-rounded values with kv_f16)."""

    def __init__(self, m, kv_cap: int, pool: Pool | None = None, kv_f16: bool = False):
        self.m, self.cap, self.pool = m, kv_cap, pool
        self._keep = []

        def p(a):
            if a is None:
                return None
            a = np.ascontiguousarray(a)
            self._keep.append(a)
            return a.ctypes.data

        nq, nkv = m.n_heads * m.head_dim, m.n_kv_heads * m.head_dim
        self._layers = (OrcLayer * m.n_layers)()
        for i, L in enumerate(m.layers):
            b = L.qkv_bias
            o = OrcLayer()
            o.attn_norm, o.ffn_norm = p(L.attn_norm), p(L.ffn_norm)
            o.wq, o.wk, o.wv, o.wo = p(L.wq), p(L.wk), p(L.wv), p(L.wo)
            o.wq_type = o.wk_type = o.wv_type = o.wo_type = L.attn_type
            if b is not None:
                o.q_bias, o.k_bias, o.v_bias = p(b[:nq]), p(b[nq:nq + nkv]), p(b[nq + nkv:])
            o.q_norm, o.k_norm = p(L.q_norm), p(L.k_norm)
            if L.moe is None:
                o.w_gate, o.w_up, o.w_down = p(L.ffn_gate), p(L.ffn_up), p(L.ffn_down)
                o.ffn_gate_type = o.ffn_down_type = L.ffn_type
            else:
                o.router = p(f32(L.moe.router))
                o.e_gate, o.e_up, o.e_down = p(L.moe.gate), p(L.moe.up), p(L.moe.down)
                o.e_gate_type, o.e_down_type = L.moe.gate_type, L.moe.down_type
            self._layers[i] = o
        self.model = OrcModel(m.n_layers, m.d_model, m.n_heads, m.n_kv_heads, m.head_dim, m.d_ffn, m.vocab,
                              m.n_experts, m.k, m.d_expert, int(m.norm_topk), int(m.rope_neox), m.eps, m.rope_theta,
                              p(m.token_emb), m.emb_type, p(m.out_norm), p(m.lm_head), m.lm_type, self._layers,
                              int(kv_f16))
        self.kc = np.zeros(m.n_layers * kv_cap * nkv, np.float32)
        self.vc = np.zeros_like(self.kc)

    def step(self, token: int, pos: int) -> np.ndarray:
        logits = np.empty(self.m.vocab, np.float32)
        rc = lib().orc_model_step(ctypes.byref(self.model), _p(self.kc), _p(self.vc), self.cap, token, pos,
                                  _p(logits), self.pool.ptr if self.pool else None)
        assert rc == 0
        return logits

    def generate(self, prompt, n_gen: int):
        """(generated ids, logits of every step) -- the reference generate loop."""
        toks = list(prompt)
        all_logits = []
        for pos in range(len(prompt) + n_gen - 1):
            lg = self.step(toks[pos], pos)
            all_logits.append(lg)
            if pos + 1 >= len(prompt):
                toks.append(greedy(lg))
        return toks[len(prompt):], all_logits


# ── Gemma 4 decoder (orc_gemma_step) ─────────────────────────────────────────

class OrcGemmaLayer(ctypes.Structure):
    P, U = ctypes.c_void_p, ctypes.c_uint32
    _fields_ = [("is_swa", ctypes.c_int), ("n_kv_heads", ctypes.c_size_t),
                ("attn_norm", P), ("post_attention_norm", P), ("q_norm", P), ("k_norm", P), ("ffn_norm", P),
                ("pre_ffw_norm_2", P), ("post_ffw_norm_1", P), ("post_ffw_norm_2", P), ("post_ffw_norm", P),
                ("layer_output_scale", ctypes.c_float),
                ("wq", P), ("wk", P), ("wv", P), ("wo", P), ("wq_type", U), ("wk_type", U), ("wv_type", U),
                ("wo_type", U), ("w_gate", P), ("w_up", P), ("w_down", P), ("gate_type", U), ("up_type", U),
                ("down_type", U), ("router_w", P), ("router_scale", P), ("down_exps_scale", P),
                ("gate_up_exps", P), ("down_exps", P), ("gu_type", U), ("dn_type", U)]


class OrcGemma(ctypes.Structure):
    SZ = ctypes.c_size_t
    _fields_ = [("n_layers", SZ), ("d_model", SZ), ("n_heads", SZ), ("head_dim_swa", SZ), ("head_dim_global", SZ),
                ("d_ffn", SZ), ("d_expert", SZ), ("n_experts", SZ), ("k", SZ), ("vocab", SZ),
                ("sliding_window", SZ), ("eps", ctypes.c_float), ("rope_theta_swa", ctypes.c_float),
                ("logit_softcap", ctypes.c_float), ("rope_freqs", ctypes.c_void_p), ("token_emb", ctypes.c_void_p),
                ("emb_type", ctypes.c_uint32), ("out_norm", ctypes.c_void_p), ("lm_head", ctypes.c_void_p),
                ("lm_type", ctypes.c_uint32), ("layers", ctypes.POINTER(OrcGemmaLayer))]


class OracleGemma:
    """orc_gemma_step over a synth.GemmaModel with its own f32 KV caches."""

    def __init__(self, m, global_cap: int, pool: Pool | None = None):
        self.m, self.cap, self.pool = m, global_cap, pool
        self._keep = []

        def p(a):
            if a is None:
                return None
            a = np.ascontiguousarray(a)
            self._keep.append(a)
            return a.ctypes.data

        self._layers = (OrcGemmaLayer * m.n_layers)()
        total = 0
        for i, L in enumerate(m.layers):
            o = OrcGemmaLayer()
            o.is_swa, o.n_kv_heads = int(L.is_swa), L.n_kv_heads
            for f in ("attn_norm", "post_attention_norm", "q_norm", "k_norm", "ffn_norm", "pre_ffw_norm_2",
                      "post_ffw_norm_1", "post_ffw_norm_2", "post_ffw_norm", "router_scale", "down_exps_scale"):
                setattr(o, f, p(getattr(L, f)))
            o.layer_output_scale = float(L.layer_output_scale)
            o.wq, o.wk, o.wv, o.wo = p(L.wq), p(L.wk), p(L.wv), p(L.wo)
            t = L.types
            o.wq_type, o.wk_type, o.wv_type, o.wo_type = t["wq"], t["wk"], t.get("wv", 0), t["wo"]
            o.w_gate, o.w_up, o.w_down = p(L.w_gate), p(L.w_up), p(L.w_down)
            o.gate_type, o.up_type, o.down_type = t["gate"], t["up"], t["down"]
            o.router_w = p(f32(L.router_w))
            o.gate_up_exps, o.down_exps = p(L.gate_up_exps), p(L.down_exps)
            o.gu_type, o.dn_type = t["gate_up_exps"], t["down_exps"]
            self._layers[i] = o
            cap = m.sliding_window if L.is_swa else global_cap
            total += cap * L.n_kv_heads * L.head_dim
        hd = m.layers[0].head_dim
        self.model = OrcGemma(m.n_layers, m.d_model, m.n_heads, hd, hd, m.d_ffn, m.d_expert, m.n_experts, m.k,
                              m.vocab, m.sliding_window, m.eps, m.rope_theta_swa, m.logit_softcap, None,
                              p(m.token_emb), m.emb_type, p(m.out_norm), p(m.lm_head), m.lm_type, self._layers)
        self.kc = np.zeros(total, np.float32)
        self.vc = np.zeros(total, np.float32)

    def step(self, token: int, pos: int) -> np.ndarray:
        logits = np.empty(self.m.vocab, np.float32)
        rc = lib().orc_gemma_step(ctypes.byref(self.model), _p(self.kc), _p(self.vc), self.cap, token, pos,
                                  _p(logits), self.pool.ptr if self.pool else None)
        assert rc == 0
        return logits

    def generate(self, prompt, n_gen: int):
        toks = list(prompt)
        all_logits = []
        for pos in range(len(prompt) + n_gen - 1):
            lg = self.step(toks[pos], pos)
            all_logits.append(lg)
            if pos + 1 >= len(prompt):
                toks.append(greedy(lg))
        return toks[len(prompt):], all_logits


class Rng:
    """orc_rng: DefaultPrng (xoshiro256++ seeded by SplitMix64)."""

    def __init__(self, seed: int):
        self.state = (ctypes.c_uint64 * 4)()
        lib().orc_rng_seed(self.state, seed)

    def float(self) -> float:
        return lib().orc_rng_float(self.state)

    def words(self) -> list[int]:
        return list(self.state)

    def copy(self) -> "Rng":
        r = Rng(0)
        r.state[:] = self.state[:]
        return r


def sample(logits, temperature: float, top_k: int, top_p: float, rng: Rng) -> int:
    a = f32(logits).copy()
    return int(lib().orc_sample(_p(a), a.size, temperature, top_k, top_p, rng.state))
