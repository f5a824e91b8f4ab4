"""Python binding of the C++ host decode loop (host/decoder.h,
libllmtoy_host.so): forwardOneModel (src/model/forward.zig:229-316) per token
over the C ABI, one captured CUDA graph per step, greedy sampling on the
device.

    ctx = Context(0)
    dec = Decoder(ctx, ModelSpec(...), layers=[LayerSpec(...), ...], ...)
    tokens = dec.generate(prompt, n_gen)
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

from . import Context, LtError, Tensor, _ptr, load_library, LIB_PATH

HOST_LIB_PATH = LIB_PATH.with_name("libllmtoy_host.so")

P = ctypes.c_void_p
U32 = ctypes.c_uint32


class _Layer(ctypes.Structure):
    _fields_ = [("attn_norm", P), ("ffn_norm", P), ("wqkv", P), ("wq", P), ("wk", P), ("wv", P), ("wo", P),
                ("qkv_bias", P), ("q_norm", P), ("k_norm", P), ("ffn_gate", P), ("ffn_up", P), ("ffn_down", P),
                ("router", P), ("exp_gate", P), ("exp_up", P), ("exp_down", P),
                ("post_attention_norm", P), ("pre_ffw_norm_2", P), ("post_ffw_norm_1", P), ("post_ffw_norm_2", P),
                ("post_ffw_norm", P), ("router_scale", P), ("down_exps_scale", P),
                ("layer_output_scale", ctypes.c_float), ("is_swa", U32), ("n_kv_heads", U32), ("head_dim", U32)]


class _Model(ctypes.Structure):
    _fields_ = [("n_layers", U32), ("d_model", U32), ("n_heads", U32), ("n_kv_heads", U32), ("head_dim", U32),
                ("vocab", U32), ("n_used", U32), ("norm_topk", U32), ("rope_neox", U32), ("act", U32),
                ("eps", ctypes.c_float), ("rope_theta", ctypes.c_float), ("kv_cap", U32),
                ("token_emb", P), ("lm_head", P), ("out_norm", P), ("layers", ctypes.POINTER(_Layer)),
                ("family", U32), ("rope_theta_swa", ctypes.c_float), ("logit_softcap", ctypes.c_float),
                ("sliding_window", U32), ("kv_f16", U32)]

LLAMA, GEMMA4 = 0, 1


_host = None


def load_host_library() -> ctypes.CDLL:
    global _host
    if _host is not None:
        return _host
    load_library()  # the C ABI first (the host library links against it)
    if not HOST_LIB_PATH.exists():
        raise RuntimeError(f"{HOST_LIB_PATH} is missing: build it with `python llmtoy-zig_b200/build.py`")
    L = ctypes.CDLL(str(HOST_LIB_PATH))
    I = ctypes.c_int
    sig = {
        "lth_decoder_create": (I, [P, ctypes.POINTER(_Model), ctypes.POINTER(P)]),
        "lth_decoder_free": (None, [P]),
        "lth_decoder_start": (I, [P, P, U32]),
        "lth_decoder_step": (I, [P]),
        "lth_decoder_capture": (I, [P]),
        "lth_decoder_replay": (I, [P, U32]),
        "lth_decoder_run_layers": (I, [P]),
        "lth_decoder_uses_stack": (I, [P]),
        "lth_decoder_logits": (P, [P]),
        "lth_decoder_tokens": (I, [P, P, U32]),
        "lth_generate": (I, [P, P, U32, U32, P]),
        "lth_decoder_set_sampling": (I, [P, ctypes.c_float, U32, ctypes.c_float, ctypes.c_uint64]),
        "lth_gguf_open": (I, [ctypes.c_char_p, ctypes.POINTER(P)]),
        "lth_gguf_close": (None, [P]),
        "lth_gguf_info": (ctypes.c_size_t, [P, P, ctypes.c_size_t]),
        "lth_gguf_tensor_count": (ctypes.c_uint64, [P]),
        "lth_gguf_tensor": (I, [P, ctypes.c_uint64, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(U32),
                                ctypes.POINTER(ctypes.c_uint64)]),
        "lth_model_load": (I, [P, P, U32, ctypes.POINTER(P)]),
        "lth_loaded_decoder": (P, [P]),
        "lth_loaded_shape": (None, [P, ctypes.POINTER(U32)]),
        "lth_loaded_free": (None, [P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _host = L
    return L


def _h(t: Tensor | None):
    return None if t is None else t.handle


@dataclass
class LayerSpec:
    """One decoder layer: Tensors from Context.upload, norms/biases as device
    tensors (torch CUDA float32)."""
    attn_norm: object
    ffn_norm: object
    wo: Tensor
    wqkv: Tensor | None = None
    wq: Tensor | None = None
    wk: Tensor | None = None
    wv: Tensor | None = None
    qkv_bias: object = None
    q_norm: object = None
    k_norm: object = None
    ffn_gate: Tensor | None = None
    ffn_up: Tensor | None = None
    ffn_down: Tensor | None = None
    router: Tensor | None = None
    exp_gate: Tensor | None = None
    exp_up: Tensor | None = None
    exp_down: Tensor | None = None
    # Gemma 4 only
    post_attention_norm: object = None
    pre_ffw_norm_2: object = None
    post_ffw_norm_1: object = None
    post_ffw_norm_2: object = None
    post_ffw_norm: object = None
    router_scale: object = None
    down_exps_scale: object = None
    layer_output_scale: float = 1.0
    is_swa: bool = False
    n_kv_heads: int = 0
    head_dim: int = 0


@dataclass
class ModelSpec:
    d_model: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    vocab: int
    token_emb: Tensor
    lm_head: Tensor
    out_norm: object
    layers: list = field(default_factory=list)
    n_used: int = 0
    norm_topk: bool = False
    rope_neox: bool = False
    act: int = 0
    eps: float = 1e-6
    rope_theta: float = 1e6
    kv_cap: int = 4096
    family: int = 0
    rope_theta_swa: float = 1e4
    logit_softcap: float = 0.0
    sliding_window: int = 0
    kv_f16: bool = False  # f16 KV caches (the reference's GPU format) instead of f32


class Decoder:
    """A greedy decoder over a device model (lth_decoder)."""

    def __init__(self, ctx: Context, spec: ModelSpec | None, _handle: int | None = None):
        self.lib = load_host_library()
        self.ctx, self.spec = ctx, spec
        if _handle is not None:  # owned by a LoadedModel
            self.ptr, self._owned = _handle, False
            return
        self._owned = True
        self._layers = (_Layer * len(spec.layers))()
        for i, L in enumerate(spec.layers):
            self._layers[i] = _Layer(
                _ptr(L.attn_norm), _ptr(L.ffn_norm), _h(L.wqkv), _h(L.wq), _h(L.wk), _h(L.wv), _h(L.wo),
                _ptr(L.qkv_bias), _ptr(L.q_norm), _ptr(L.k_norm), _h(L.ffn_gate), _h(L.ffn_up), _h(L.ffn_down),
                _h(L.router), _h(L.exp_gate), _h(L.exp_up), _h(L.exp_down), _ptr(L.post_attention_norm),
                _ptr(L.pre_ffw_norm_2), _ptr(L.post_ffw_norm_1), _ptr(L.post_ffw_norm_2), _ptr(L.post_ffw_norm),
                _ptr(L.router_scale), _ptr(L.down_exps_scale), L.layer_output_scale, int(L.is_swa), L.n_kv_heads,
                L.head_dim)
        s = spec
        self._model = _Model(len(s.layers), s.d_model, s.n_heads, s.n_kv_heads, s.head_dim, s.vocab, s.n_used,
                             int(s.norm_topk), int(s.rope_neox), s.act, s.eps, s.rope_theta, s.kv_cap,
                             _h(s.token_emb), _h(s.lm_head), _ptr(s.out_norm), self._layers, s.family,
                             s.rope_theta_swa, s.logit_softcap, s.sliding_window, int(s.kv_f16))
        h = P()
        self._check(self.lib.lth_decoder_create(ctx.ptr, ctypes.byref(self._model), ctypes.byref(h)))
        self.ptr = h.value

    def _check(self, st: int) -> None:
        if st != 0:
            msg = self.ctx.lib.lt_last_error(self.ctx.ptr) or b""
            raise LtError(st, msg.decode())

    def close(self) -> None:
        if getattr(self, "ptr", None):
            if self._owned:
                self.lib.lth_decoder_free(self.ptr)
            self.ptr = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # -- step-level control (parity tests, timing) ----------------------------
    def start(self, prompt) -> None:
        arr = (ctypes.c_uint32 * len(prompt))(*[int(t) for t in prompt])
        self._check(self.lib.lth_decoder_start(self.ptr, arr, len(prompt)))

    def step(self) -> None:
        self._check(self.lib.lth_decoder_step(self.ptr))

    def capture(self) -> None:
        self._check(self.lib.lth_decoder_capture(self.ptr))

    def replay(self, n_steps: int) -> None:
        self._check(self.lib.lth_decoder_replay(self.ptr, n_steps))

    def run_layers(self) -> None:
        """The decoder layers alone at the current position (no embedding, logits or advance)."""
        self._check(self.lib.lth_decoder_run_layers(self.ptr))

    @property
    def uses_stack(self) -> bool:
        return bool(self.lib.lth_decoder_uses_stack(self.ptr))

    def logits_ptr(self) -> int:
        return self.lib.lth_decoder_logits(self.ptr)

    def tokens(self, n: int) -> list[int]:
        arr = (ctypes.c_uint32 * n)()
        self._check(self.lib.lth_decoder_tokens(self.ptr, arr, n))
        return list(arr)

    def set_sampling(self, temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0, seed: int = 42) -> None:
        """sample.zig parameters for the following steps (temperature 0: greedy)."""
        self._check(self.lib.lth_decoder_set_sampling(self.ptr, temperature, top_k, top_p, seed))

    def generate(self, prompt, n_gen: int) -> list[int]:
        """Generation (greedy unless set_sampling chose otherwise): prompt ids -> n_gen new ids."""
        arr = (ctypes.c_uint32 * len(prompt))(*[int(t) for t in prompt])
        out = (ctypes.c_uint32 * n_gen)()
        self._check(self.lib.lth_generate(self.ptr, arr, len(prompt), n_gen, out))
        return list(out)


class _Uploads:
    """ctx.upload once per host array: layers that share weight arrays (a
    model whose depth cycles a few distinct layer sets) share device tensors,
    which are read-only."""

    def __init__(self, ctx: Context):
        self.ctx, self.done = ctx, {}

    def __call__(self, a, t, rows, cols, n_experts=0):
        key = (id(a), t, rows, cols, n_experts)
        if key not in self.done:
            self.done[key] = (a, self.ctx.upload(a, t, rows, cols, n_experts=n_experts))
        return self.done[key][1]


def upload_decoder(ctx: Context, m, kv_cap: int = 4096, stacked_qkv: bool = True, kv_f16: bool = False) -> ModelSpec:
    """Upload a synth.DecoderModel (host GGUF bytes) and return its ModelSpec.
    Norm weights and biases go to torch CUDA tensors, which the spec keeps
    alive; stacked_qkv uploads Q, K and V rows as one tensor (one matvec)."""
    import numpy as np
    import torch

    def dev(a):
        return None if a is None else torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()

    d = m.d_model
    up = _Uploads(ctx)
    layers = []
    for L in m.layers:
        nq, nkv = m.n_heads * m.head_dim, m.n_kv_heads * m.head_dim
        ls = LayerSpec(attn_norm=dev(L.attn_norm), ffn_norm=dev(L.ffn_norm),
                       wo=up(L.wo, L.attn_type, d, nq), qkv_bias=dev(L.qkv_bias),
                       q_norm=dev(L.q_norm), k_norm=dev(L.k_norm))
        if stacked_qkv:
            ls.wqkv = ctx.upload(L.wqkv, L.attn_type, nq + 2 * nkv, d)
        else:
            ls.wq = up(L.wq, L.attn_type, nq, d)
            ls.wk = up(L.wk, L.attn_type, nkv, d)
            ls.wv = up(L.wv, L.attn_type, nkv, d)
        if L.moe is None:
            ls.ffn_gate = up(L.ffn_gate, L.ffn_type, m.d_ffn, d)
            ls.ffn_up = up(L.ffn_up, L.ffn_type, m.d_ffn, d)
            ls.ffn_down = up(L.ffn_down, L.ffn_type, d, m.d_ffn)
        else:
            E, F = m.n_experts, m.d_expert
            ls.router = up(L.moe.router, 0, E, d)
            ls.exp_gate = up(L.moe.gate, L.moe.gate_type, F, d, n_experts=E)
            ls.exp_up = up(L.moe.up, L.moe.gate_type, F, d, n_experts=E)
            ls.exp_down = up(L.moe.down, L.moe.down_type, d, F, n_experts=E)
        layers.append(ls)
    return ModelSpec(d_model=d, n_heads=m.n_heads, n_kv_heads=m.n_kv_heads, head_dim=m.head_dim, vocab=m.vocab,
                     token_emb=ctx.upload(m.token_emb, m.emb_type, m.vocab, d),
                     lm_head=ctx.upload(m.lm_head, m.lm_type, m.vocab, d), out_norm=dev(m.out_norm),
                     layers=layers, n_used=m.k, norm_topk=m.norm_topk, rope_neox=m.rope_neox, eps=m.eps,
                     rope_theta=m.rope_theta, kv_cap=kv_cap, kv_f16=kv_f16)


class GgufFile:
    """A memory-mapped GGUF file (lth_gguf_open): metadata, tensors, info report."""

    def __init__(self, path):
        self.lib = load_host_library()
        h = P()
        st = self.lib.lth_gguf_open(str(path).encode(), ctypes.byref(h))
        if st != 0:
            raise LtError(st, f"cannot parse GGUF file {path}")
        self.ptr = h.value

    def info(self) -> str:
        n = self.lib.lth_gguf_info(self.ptr, None, 0)
        buf = ctypes.create_string_buffer(n + 1)
        self.lib.lth_gguf_info(self.ptr, buf, n + 1)
        return buf.value.decode()

    def tensors(self) -> list[tuple[str, int, int]]:
        out = []
        for i in range(self.lib.lth_gguf_tensor_count(self.ptr)):
            nm, t, nb = ctypes.c_char_p(), U32(), ctypes.c_uint64()
            self.lib.lth_gguf_tensor(self.ptr, i, ctypes.byref(nm), ctypes.byref(t), ctypes.byref(nb))
            out.append((nm.value.decode(), t.value, nb.value))
        return out

    def close(self) -> None:
        if self.ptr:
            self.lib.lth_gguf_close(self.ptr)
            self.ptr = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


class LoadedModel:
    """A decoder uploaded from a GGUF file (lth_model_load)."""

    def __init__(self, ctx: Context, gguf: GgufFile, kv_cap: int = 4096):
        self.lib = load_host_library()
        self.ctx = ctx
        h = P()
        st = self.lib.lth_model_load(ctx.ptr, gguf.ptr, kv_cap, ctypes.byref(h))
        if st != 0:
            msg = ctx.lib.lt_last_error(ctx.ptr) or b""
            raise LtError(st, f"model load failed: {msg.decode()}")
        self.ptr = h.value
        sh = (U32 * 8)()
        self.lib.lth_loaded_shape(self.ptr, sh)
        (self.n_layers, self.d_model, self.n_heads, self.n_kv_heads, self.head_dim, self.vocab, self.n_experts,
         self.n_used) = list(sh)
        self.decoder = Decoder(ctx, None, _handle=self.lib.lth_loaded_decoder(self.ptr))

    def generate(self, prompt, n_gen: int) -> list[int]:
        return self.decoder.generate(prompt, n_gen)

    def close(self) -> None:
        if self.ptr:
            self.decoder.close()
            self.lib.lth_loaded_free(self.ptr)
            self.ptr = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def upload_gemma(ctx: Context, m, kv_cap: int = 4096) -> ModelSpec:
    """Upload a synth.GemmaModel (host GGUF bytes) and return its ModelSpec."""
    import numpy as np
    import torch

    def dev(a):
        return None if a is None else torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()

    d, E, F = m.d_model, m.n_experts, m.d_expert
    up = _Uploads(ctx)
    layers = []
    for L in m.layers:
        nq, nkv = m.n_heads * L.head_dim, L.n_kv_heads * L.head_dim
        t = L.types
        ls = LayerSpec(attn_norm=dev(L.attn_norm), ffn_norm=dev(L.ffn_norm), wo=up(L.wo, t["wo"], d, nq),
                       wq=up(L.wq, t["wq"], nq, d), wk=up(L.wk, t["wk"], nkv, d),
                       wv=None if L.wv is None else up(L.wv, t["wv"], nkv, d),
                       q_norm=dev(L.q_norm), k_norm=dev(L.k_norm),
                       ffn_gate=up(L.w_gate, t["gate"], m.d_ffn, d),
                       ffn_up=up(L.w_up, t["up"], m.d_ffn, d),
                       ffn_down=up(L.w_down, t["down"], d, m.d_ffn),
                       router=up(L.router_w, 0, E, d),
                       exp_gate=up(L.gate_up_exps, t["gate_up_exps"], 2 * F, d, n_experts=E),
                       exp_down=up(L.down_exps, t["down_exps"], d, F, n_experts=E),
                       post_attention_norm=dev(L.post_attention_norm), pre_ffw_norm_2=dev(L.pre_ffw_norm_2),
                       post_ffw_norm_1=dev(L.post_ffw_norm_1), post_ffw_norm_2=dev(L.post_ffw_norm_2),
                       post_ffw_norm=dev(L.post_ffw_norm), router_scale=dev(L.router_scale),
                       down_exps_scale=dev(L.down_exps_scale), layer_output_scale=float(L.layer_output_scale),
                       is_swa=L.is_swa, n_kv_heads=L.n_kv_heads, head_dim=L.head_dim)
        layers.append(ls)
    return ModelSpec(d_model=d, n_heads=m.n_heads, n_kv_heads=m.layers[0].n_kv_heads, head_dim=m.layers[0].head_dim,
                     vocab=m.vocab, token_emb=ctx.upload(m.token_emb, m.emb_type, m.vocab, d),
                     lm_head=ctx.upload(m.lm_head, m.lm_type, m.vocab, d), out_norm=dev(m.out_norm), layers=layers,
                     n_used=m.k, norm_topk=False, rope_neox=True, act=1, eps=m.eps, rope_theta=m.rope_theta_global,
                     kv_cap=kv_cap, family=GEMMA4, rope_theta_swa=m.rope_theta_swa, logit_softcap=m.logit_softcap,
                     sliding_window=m.sliding_window)
