"""B200 (sm_100a) backend for llmtoy-zig's quantized MoE forward path.

Python binding of the C ABI in include/llmtoy_cuda.h (libllmtoy_cuda.so, built
in-tree by build.py).  Device buffers are plain integer addresses, so torch
tensors (``t.data_ptr()``) or any other allocator can feed the ops.  There is
no CPU fallback: without the built library or an sm_100 GPU every entry point
raises.

Import with ``importlib.import_module("llmtoy-zig_b200")`` (the directory name
is not a Python identifier).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libllmtoy_cuda.so")

# GGUF type codes (src/gguf/types.zig:23-52)
F32, F16, Q8_0, Q4_K, Q6_K = 0, 1, 8, 12, 14
Q5_0, Q5_1, Q3_K, Q5_K, IQ4_NL = 6, 7, 11, 13, 20
TYPE_NAMES = {F32: "F32", F16: "F16", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K", Q5_0: "Q5_0", Q5_1: "Q5_1",
              Q3_K: "Q3_K", Q5_K: "Q5_K", IQ4_NL: "IQ4_NL"}
BLOCK = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210), Q5_0: (32, 22),
         Q5_1: (32, 24), Q3_K: (256, 110), Q5_K: (256, 176), IQ4_NL: (32, 18)}
ACT_SILU, ACT_GELU_TANH = 0, 1

STATUS = {0: "LT_OK", 1: "LT_EINVAL", 2: "LT_EUNSUPPORTED_TYPE", 3: "LT_ENOMEM",
          4: "LT_ECUDA", 5: "LT_ETIMEOUT", 6: "LT_ENODEV"}

# Every symbol include/llmtoy_cuda.h declares.
EXPORTS = [
    "lt_api_version", "lt_init", "lt_free", "lt_set_stream", "lt_sync", "lt_last_error",
    "lt_status_string", "lt_reserve", "lt_row_bytes", "lt_upload", "lt_upload_from_device",
    "lt_tensor_download", "lt_tensor_describe", "lt_tensor_free", "lt_dequant", "lt_qmatvec",
    "lt_rmsnorm", "lt_softmax", "lt_moe_route", "lt_moe_ffn", "lt_moe_forward", "lt_moe_block", "lt_argmax",
    "lt_profile_enable", "lt_profile_read", "lt_profile_reset", "lt_capture_begin", "lt_capture_end",
    "lt_graph_launch", "lt_graph_free", "lt_moe_ffn_noalloc", "lt_quant_matvec_host", "lt_moe_forward_host",
    "lt_ep_dispatch", "lt_gather_rows", "lt_moe_combine",
    "lt_device_alloc", "lt_device_free", "lt_copy_to_device", "lt_copy_to_host",
    "lt_embed", "lt_qmatvec_add", "lt_attn_prep", "lt_attn_decode", "lt_attn_block", "lt_attn_block_split", "lt_prefetch_next",
    "lt_ffn_block", "lt_greedy_step", "lt_scale", "lt_add_rmsnorm", "lt_norm_pair", "lt_ffn_tail", "lt_softcap",
    "lt_sample_step", "lt_rng_seed", "lt_quantize_q8_1", "lt_dequant_q8_1", "lt_moe_block_scaled",
    "lt_qmatvec_multi", "lt_noalloc_status", "lt_selftest_wait",
    "lt_stack_create", "lt_stack_run", "lt_stack_free", "lt_ep_unique_id", "lt_ep_init", "lt_ep_free",
    "lt_moe_ffn_ep",
]


class LtError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status


class TensorDesc(ctypes.Structure):
    _fields_ = [("ggml_type", ctypes.c_uint32), ("n_experts", ctypes.c_uint32),
                ("rows", ctypes.c_uint64), ("cols", ctypes.c_uint64),
                ("row_bytes", ctypes.c_uint64), ("row_pitch", ctypes.c_uint64)]


class AttnCfg(ctypes.Structure):
    """lt_attn_cfg: geometry of one attention layer."""
    _fields_ = [("n_heads", ctypes.c_uint32), ("n_kv_heads", ctypes.c_uint32), ("head_dim", ctypes.c_uint32),
                ("rope_neox", ctypes.c_uint32), ("rope_theta", ctypes.c_float), ("eps", ctypes.c_float),
                ("scale", ctypes.c_float), ("kv_cap", ctypes.c_uint32), ("window", ctypes.c_uint32),
                ("v_norm", ctypes.c_uint32), ("kv_f16", ctypes.c_uint32)]


class TailIn(ctypes.Structure):
    """lt_ffn_tail_in: the previous Gemma 4 layer's FFN tail, fused into the next attention block."""
    _fields_ = [("f", ctypes.c_void_p), ("w1", ctypes.c_void_p), ("m", ctypes.c_void_p), ("w2", ctypes.c_void_p),
                ("w", ctypes.c_void_p), ("los", ctypes.c_float), ("eps", ctypes.c_float)]


class SampleParams(ctypes.Structure):
    """lt_sample_params (src/model/sample.zig:4-8)."""
    _fields_ = [("temperature", ctypes.c_float), ("top_k", ctypes.c_uint32), ("top_p", ctypes.c_float)]


def rng_seed(seed: int) -> list[int]:
    """DefaultPrng.init(seed): the four xoshiro256++ state words."""
    out = (ctypes.c_uint64 * 4)()
    load_library().lt_rng_seed(seed, out)
    return list(out)


_lib = None


def load_library() -> ctypes.CDLL:
    """Load libllmtoy_cuda.so, failing loudly if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python llmtoy-zig_b200/build.py`")
    lib = ctypes.CDLL(str(LIB_PATH))
    P, U32, U64, I, F, SZ = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
    sig = {
        "lt_api_version": (I, []),
        "lt_init": (I, [I, ctypes.POINTER(P)]),
        "lt_free": (None, [P]),
        "lt_set_stream": (I, [P, P]),
        "lt_sync": (I, [P]),
        "lt_last_error": (ctypes.c_char_p, [P]),
        "lt_status_string": (ctypes.c_char_p, [I]),
        "lt_reserve": (I, [P, U32, U32, U64, U64]),
        "lt_row_bytes": (U64, [U32, U64]),
        "lt_upload": (I, [P, P, SZ, U32, U64, U64, U32, ctypes.POINTER(P)]),
        "lt_upload_from_device": (I, [P, P, SZ, U32, U64, U64, U32, ctypes.POINTER(P)]),
        "lt_tensor_download": (I, [P, P, P, SZ]),
        "lt_tensor_describe": (I, [P, ctypes.POINTER(TensorDesc)]),
        "lt_tensor_free": (I, [P, P]),
        "lt_dequant": (I, [P, P, U64, U64, P]),
        "lt_quantize_q8_1": (I, [P, P, U64, I, P]),
        "lt_dequant_q8_1": (I, [P, P, U64, I, P]),
        "lt_qmatvec": (I, [P, P, U32, P, P, U32]),
        "lt_rmsnorm": (I, [P, P, P, F, U32, U32, P]),
        "lt_softmax": (I, [P, P, U32, U32]),
        "lt_moe_route": (I, [P, P, P, U32, U32, I, P, P, P]),
        "lt_moe_ffn": (I, [P, P, P, P, I, P, U32, P, P, U32, P]),
        "lt_moe_forward": (I, [P, P, P, P, P, I, I, P, P, U32, U32, P, P, P]),
        "lt_moe_block": (I, [P, P, P, P, P, I, I, P, P, F, P, U32, U32, P, P, P]),
        "lt_moe_block_scaled": (I, [P, P, P, P, P, I, I, P, P, P, F, F, P, U32, U32, I, P, P, P]),
        "lt_qmatvec_multi": (I, [P, U32, P, P, P, F, P]),
        "lt_argmax": (I, [P, P, U32, U32, P]),
        "lt_profile_enable": (I, [P, I]),
        "lt_profile_read": (I, [P, U32, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(U64),
                                ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double),
                                ctypes.POINTER(ctypes.c_double)]),
        "lt_profile_reset": (I, [P]),
        "lt_capture_begin": (I, [P]),
        "lt_capture_end": (I, [P, ctypes.POINTER(P)]),
        "lt_graph_launch": (I, [P, P]),
        "lt_graph_free": (I, [P, P]),
        "lt_moe_ffn_noalloc": (I, [P, P, P, P, U32, U32, U32, U64, U64, I, P, U32, P, P, U32, P]),
        "lt_noalloc_status": (I, [P]),
        "lt_selftest_wait": (I, [P, U32, U32]),
        "lt_stack_create": (I, [P, P, U32, P, U32, U32, I, I, F, ctypes.POINTER(P)]),
        "lt_stack_run": (I, [P, P, P, P]),
        "lt_stack_free": (I, [P, P]),
        "lt_ep_unique_id": (I, [P]),
        "lt_ep_init": (I, [P, U32, U32, P, U32, ctypes.POINTER(P)]),
        "lt_ep_free": (I, [P]),
        "lt_moe_ffn_ep": (I, [P, P, P, P, P, P, I, I, P, P, F, P, U32, U32, P]),
        "lt_ep_dispatch": (I, [P, P, U32, U32, U32, U32, P, P, P, P]),
        "lt_gather_rows": (I, [P, P, U64, P, U32, P]),
        "lt_moe_combine": (I, [P, P, U64, P, P, U32, U32, P, P]),
        "lt_device_alloc": (I, [P, SZ, ctypes.POINTER(P)]),
        "lt_device_free": (I, [P, P]),
        "lt_copy_to_device": (I, [P, P, P, SZ]),
        "lt_copy_to_host": (I, [P, P, P, SZ]),
        "lt_embed": (I, [P, P, P, P, P]),
        "lt_qmatvec_add": (I, [P, P, U32, P, P, P, U32]),
        "lt_attn_prep": (I, [P, ctypes.POINTER(AttnCfg), P, P, P, P, P, P]),
        "lt_attn_decode": (I, [P, ctypes.POINTER(AttnCfg), P, P, P, P, P]),
        "lt_greedy_step": (I, [P, P, U32, P, P, P]),
        "lt_ffn_block": (I, [P, P, P, P, I, P, F, P, U32, I, P]),
        "lt_scale": (I, [P, P, U32, U32, F]),
        "lt_add_rmsnorm": (I, [P, P, P, F, U32, U32, P]),
        "lt_norm_pair": (I, [P, P, P, P, F, F, U32, U32, P, P]),
        "lt_ffn_tail": (I, [P, P, P, P, P, P, F, F, U32, U32, P]),
        "lt_softcap": (I, [P, P, U64, F]),
        "lt_sample_step": (I, [P, P, U32, ctypes.POINTER(SampleParams), P, P, P, P]),
        "lt_rng_seed": (None, [U64, ctypes.POINTER(U64)]),
        "lt_attn_block": (I, [P, ctypes.POINTER(AttnCfg), P, P, F, P, P, P, P, P, P, P, P, P]),
        "lt_attn_block_split": (I, [P, ctypes.POINTER(AttnCfg), P, P, F, P, P, P, P, P, P, P, P, P, P, P,
                                    ctypes.POINTER(TailIn), P]),
        "lt_prefetch_next": (I, [P, P, P]),
        "lt_quant_matvec_host": (I, [P, P, P, U32, P, U64, U64]),
        "lt_moe_forward_host": (I, [P, P, P, P, P, I, I, P, P, U32, U32, P, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def row_bytes(ggml_type: int, cols: int) -> int:
    """rowBytes (src/ops/math.zig:194-208)."""
    elems, nbytes = BLOCK[ggml_type]
    return (cols // elems) * nbytes


def _ptr(x) -> int | None:
    """Device address of a torch tensor, or an int address, or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


class Tensor:
    """A GGUF tensor uploaded to the device (RawMatrix, src/model/model_weights.zig:17)."""

    def __init__(self, ctx: "Context", handle: int):
        self._ctx = ctx
        self.handle = handle
        d = TensorDesc()
        ctx._check(ctx.lib.lt_tensor_describe(handle, ctypes.byref(d)))
        self.ggml_type, self.n_experts = d.ggml_type, d.n_experts
        self.rows, self.cols, self.row_bytes, self.row_pitch = d.rows, d.cols, d.row_bytes, d.row_pitch

    @property
    def total_rows(self) -> int:
        return self.rows * max(1, self.n_experts)

    def download(self) -> bytes:
        buf = ctypes.create_string_buffer(self.total_rows * self.row_bytes)
        self._ctx._check(self._ctx.lib.lt_tensor_download(self._ctx.ptr, self.handle, buf, len(buf)))
        return buf.raw

    def free(self) -> None:
        if self.handle:
            self._ctx.lib.lt_tensor_free(self._ctx.ptr, self.handle)
            self.handle = None


class Graph:
    """A captured sequence of ops (lt_capture_begin .. lt_capture_end)."""

    def __init__(self, ctx: "Context", handle: int):
        self._ctx = ctx
        self.handle = handle

    def launch(self) -> None:
        self._ctx._check(self._ctx.lib.lt_graph_launch(self._ctx.ptr, self.handle))

    def free(self) -> None:
        if self.handle:
            self._ctx.lib.lt_graph_free(self._ctx.ptr, self.handle)
            self.handle = None


class Context:
    """One device context (lt_init); ops run on its stream."""

    def __init__(self, device: int = 0):
        self.lib = load_library()
        p = ctypes.c_void_p()
        st = self.lib.lt_init(device, ctypes.byref(p))
        if st != 0:
            raise LtError(st, f"lt_init(device={device}) failed")
        self.ptr = p.value
        self.device = device

    # -- plumbing ---------------------------------------------------------
    def _check(self, st: int) -> None:
        if st != 0:
            msg = self.lib.lt_last_error(self.ptr) if self.ptr else b""
            raise LtError(st, (msg or b"").decode())

    def close(self) -> None:
        if self.ptr:
            self.lib.lt_free(self.ptr)
            self.ptr = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def set_stream(self, stream) -> None:
        """Run ops on a cudaStream_t (int handle or torch.cuda.Stream); None: the context's own
        stream.  Handle 0, torch's default stream, means the legacy default stream
        (cudaStreamLegacy), so work torch queues there orders with these ops."""
        if stream is None:
            handle = None
        else:
            handle = getattr(stream, "cuda_stream", stream)
            handle = handle or 1  # cudaStreamLegacy
        self._check(self.lib.lt_set_stream(self.ptr, handle))

    def sync(self) -> None:
        self._check(self.lib.lt_sync(self.ptr))

    def reserve(self, max_tokens: int, max_k: int, max_d_model: int, max_d_expert: int) -> None:
        self._check(self.lib.lt_reserve(self.ptr, max_tokens, max_k, max_d_model, max_d_expert))

    # -- weights ----------------------------------------------------------
    def upload(self, data, ggml_type: int, rows: int, cols: int, n_experts: int = 0) -> Tensor:
        """Upload GGUF bytes (bytes / numpy array / host torch tensor)."""
        import numpy as np
        arr = np.ascontiguousarray(np.frombuffer(memoryview(data).cast("B"), dtype=np.uint8)
                                   if not isinstance(data, np.ndarray) else data.view(np.uint8).reshape(-1))
        h = ctypes.c_void_p()
        self._check(self.lib.lt_upload(self.ptr, arr.ctypes.data, arr.nbytes, ggml_type, rows, cols,
                                       n_experts, ctypes.byref(h)))
        return Tensor(self, h.value)

    def upload_device(self, dev_tensor, ggml_type: int, rows: int, cols: int, n_experts: int = 0) -> Tensor:
        """Upload GGUF bytes that already sit in device memory (a uint8 CUDA tensor)."""
        h = ctypes.c_void_p()
        nbytes = dev_tensor.numel() * dev_tensor.element_size()
        self._check(self.lib.lt_upload_from_device(self.ptr, dev_tensor.data_ptr(), nbytes, ggml_type, rows,
                                                   cols, n_experts, ctypes.byref(h)))
        return Tensor(self, h.value)

    # -- device ops (asynchronous) ----------------------------------------
    def dequant(self, t: Tensor, row0: int, nrows: int, out) -> None:
        self._check(self.lib.lt_dequant(self.ptr, t.handle, row0, nrows, _ptr(out)))

    def quantize_q8_1(self, x, n: int, out, x4: bool = False) -> None:
        self._check(self.lib.lt_quantize_q8_1(self.ptr, _ptr(x), n, int(x4), _ptr(out)))

    def dequant_q8_1(self, q, n: int, out, x4: bool = False) -> None:
        self._check(self.lib.lt_dequant_q8_1(self.ptr, _ptr(q), n, int(x4), _ptr(out)))

    def qmatvec(self, w: Tensor, x, y, ntok: int = 1, expert: int = 0) -> None:
        self._check(self.lib.lt_qmatvec(self.ptr, w.handle, expert, _ptr(x), _ptr(y), ntok))

    def rmsnorm(self, x, w, eps: float, n: int, ntok: int, y) -> None:
        self._check(self.lib.lt_rmsnorm(self.ptr, _ptr(x), _ptr(w), eps, n, ntok, _ptr(y)))

    def softmax(self, x, n: int, ntok: int = 1) -> None:
        self._check(self.lib.lt_softmax(self.ptr, _ptr(x), n, ntok))

    def argmax(self, x, n: int, ntok: int, idx) -> None:
        self._check(self.lib.lt_argmax(self.ptr, _ptr(x), n, ntok, _ptr(idx)))

    def moe_route(self, router: Tensor, x, ntok: int, k: int, norm_topk: bool, expert_scale, ids, w) -> None:
        self._check(self.lib.lt_moe_route(self.ptr, router.handle, _ptr(x), ntok, k, int(norm_topk),
                                          _ptr(expert_scale), _ptr(ids), _ptr(w)))

    def moe_ffn(self, gate: Tensor, up: Tensor | None, down: Tensor, act: int, x, ntok: int, ids, w, k: int,
                out) -> None:
        self._check(self.lib.lt_moe_ffn(self.ptr, gate.handle, up.handle if up else None, down.handle, act,
                                        _ptr(x), ntok, _ptr(ids), _ptr(w), k, _ptr(out)))

    def moe_forward(self, router: Tensor, gate: Tensor, up: Tensor | None, down: Tensor, act: int,
                    norm_topk: bool, expert_scale, x, ntok: int, k: int, out, ids=None, w=None) -> None:
        self._check(self.lib.lt_moe_forward(self.ptr, router.handle, gate.handle, up.handle if up else None,
                                            down.handle, act, int(norm_topk), _ptr(expert_scale), _ptr(x), ntok,
                                            k, _ptr(out), _ptr(ids), _ptr(w)))

    def moe_block(self, router: Tensor, gate: Tensor, up: Tensor | None, down: Tensor, act: int, norm_topk: bool,
                  expert_scale, norm_w, eps: float, x, ntok: int, k: int, out, ids=None, w=None) -> None:
        """out = x + moe(rmsnorm(x) * norm_w): the fused MoE FFN block of a layer."""
        self._check(self.lib.lt_moe_block(self.ptr, router.handle, gate.handle, up.handle if up else None,
                                          down.handle, act, int(norm_topk), _ptr(expert_scale), _ptr(norm_w), eps,
                                          _ptr(x), ntok, k, _ptr(out), _ptr(ids), _ptr(w)))

    # -- expert parallelism building blocks (see ep.py) --------------------
    def ep_dispatch(self, ids, ntok: int, k: int, n_experts: int, nranks: int, send_counts, send_token, send_local,
                    pair_pos) -> None:
        self._check(self.lib.lt_ep_dispatch(self.ptr, _ptr(ids), ntok, k, n_experts, nranks, _ptr(send_counts),
                                            _ptr(send_token), _ptr(send_local), _ptr(pair_pos)))

    def gather_rows(self, src, cols: int, idx, n: int, dst) -> None:
        self._check(self.lib.lt_gather_rows(self.ptr, _ptr(src), cols, _ptr(idx), n, _ptr(dst)))

    def moe_combine(self, y, cols: int, pair_pos, w, ntok: int, k: int, resid, out) -> None:
        self._check(self.lib.lt_moe_combine(self.ptr, _ptr(y), cols, _ptr(pair_pos), _ptr(w), ntok, k, _ptr(resid),
                                            _ptr(out)))

    # -- device buffers ----------------------------------------------------
    def device_alloc(self, nbytes: int) -> int:
        """A zero-filled device buffer (free with device_free)."""
        p = ctypes.c_void_p()
        self._check(self.lib.lt_device_alloc(self.ptr, nbytes, ctypes.byref(p)))
        return p.value

    def device_free(self, dev: int) -> None:
        self._check(self.lib.lt_device_free(self.ptr, dev))

    def copy_to_device(self, dev, host_array) -> None:
        import numpy as np
        a = np.ascontiguousarray(host_array)
        self._check(self.lib.lt_copy_to_device(self.ptr, _ptr(dev), a.ctypes.data, a.nbytes))
        self.sync()

    def copy_to_host(self, dev, nbytes: int, dtype="float32"):
        """nbytes at a device address -> numpy array of dtype (synchronises)."""
        import numpy as np
        out = np.empty(nbytes // np.dtype(dtype).itemsize, dtype=dtype)
        self._check(self.lib.lt_copy_to_host(self.ptr, out.ctypes.data, _ptr(dev), out.nbytes))
        self.sync()
        return out

    # -- decode-step ops ---------------------------------------------------
    def embed(self, emb: Tensor, tokens, pos, out) -> None:
        self._check(self.lib.lt_embed(self.ptr, emb.handle, _ptr(tokens), _ptr(pos), _ptr(out)))

    def qmatvec_multi(self, ws: list, x, ys: list, norm_w=None, eps: float = 1e-6) -> None:
        """ys[i] = ws[i] . xn for one token, xn = x or rmsnorm(x) * norm_w, in one launch."""
        n = len(ws)
        hw = (ctypes.c_void_p * n)(*[w.handle for w in ws])
        hy = (ctypes.c_void_p * n)(*[_ptr(y) for y in ys])
        self._check(self.lib.lt_qmatvec_multi(self.ptr, n, hw, _ptr(x), _ptr(norm_w), eps, hy))

    def qmatvec_add(self, w: Tensor, x, add, y, ntok: int = 1, expert: int = 0) -> None:
        self._check(self.lib.lt_qmatvec_add(self.ptr, w.handle, expert, _ptr(x), _ptr(add), _ptr(y), ntok))

    def attn_prep(self, cfg: AttnCfg, qkv, q_norm, k_norm, pos, k_cache, v_cache) -> None:
        self._check(self.lib.lt_attn_prep(self.ptr, ctypes.byref(cfg), _ptr(qkv), _ptr(q_norm), _ptr(k_norm),
                                          _ptr(pos), _ptr(k_cache), _ptr(v_cache)))

    def attn_decode(self, cfg: AttnCfg, q, k_cache, v_cache, pos, out) -> None:
        self._check(self.lib.lt_attn_decode(self.ptr, ctypes.byref(cfg), _ptr(q), _ptr(k_cache), _ptr(v_cache),
                                            _ptr(pos), _ptr(out)))

    def moe_block_scaled(self, router: Tensor, gate: Tensor, up: Tensor | None, down: Tensor, act: int,
                         norm_topk: bool, expert_scale, norm_w, router_scale, router_gs: float, eps: float, x,
                         ntok: int, k: int, out, residual: bool = False, ids=None, w=None) -> None:
        """out = (x if residual) + moe(...): experts on rmsnorm(x) * norm_w, router on
        x * rms_inv * router_gs * router_scale (Gemma 4's MoE half)."""
        self._check(self.lib.lt_moe_block_scaled(self.ptr, router.handle, gate.handle, up.handle if up else None,
                                                 down.handle, act, int(norm_topk), _ptr(expert_scale), _ptr(norm_w),
                                                 _ptr(router_scale), router_gs, eps, _ptr(x), ntok, k,
                                                 int(residual), _ptr(out), _ptr(ids), _ptr(w)))

    def attn_block(self, cfg: AttnCfg, x, norm_w, eps: float, wqkv: Tensor, qkv_bias, q_norm, k_norm, pos,
                   k_cache, v_cache, wo: Tensor, out) -> None:
        """out = x + wo . attention(...) for one token: the attention half of a decoder layer."""
        self._check(self.lib.lt_attn_block(self.ptr, ctypes.byref(cfg), _ptr(x), _ptr(norm_w), eps, wqkv.handle,
                                           _ptr(qkv_bias), _ptr(q_norm), _ptr(k_norm), _ptr(pos), _ptr(k_cache),
                                           _ptr(v_cache), wo.handle, _ptr(out)))

    def attn_block_split(self, cfg: AttnCfg, x, norm_w, eps: float, wq: Tensor, wk: Tensor, wv: Tensor | None,
                         qkv_bias, q_norm, k_norm, pos, k_cache, v_cache, wo: Tensor, post_norm, out,
                         tail: tuple | None = None) -> None:
        """attn_block over separate Q/K/V tensors; wv None: V = K; post_norm: out = x + rmsnorm(wo . att) *
        post_norm; tail (f, w1, m, w2, w, los, eps): the block's input is that FFN tail of x."""
        t = None
        if tail is not None:
            f, w1, m, w2, w, los, teps = tail
            t = ctypes.byref(TailIn(_ptr(f), _ptr(w1), _ptr(m), _ptr(w2), _ptr(w), los, teps))
        self._check(self.lib.lt_attn_block_split(self.ptr, ctypes.byref(cfg), _ptr(x), _ptr(norm_w), eps, wq.handle,
                                                 wk.handle, wv.handle if wv else None, _ptr(qkv_bias), _ptr(q_norm),
                                                 _ptr(k_norm), _ptr(pos), _ptr(k_cache), _ptr(v_cache), wo.handle,
                                                 _ptr(post_norm), t, _ptr(out)))

    def prefetch_next(self, a: Tensor | None, b: Tensor | None = None) -> None:
        self._check(self.lib.lt_prefetch_next(self.ptr, a.handle if a else None, b.handle if b else None))

    def ffn_block(self, gate: Tensor, up: Tensor, down: Tensor, act: int, norm_w, eps: float, x, ntok: int,
                  out, residual: bool = True) -> None:
        """out = (x if residual) + down . (act(gate . xn) * (up . xn)), xn = rmsnorm(x) * norm_w."""
        self._check(self.lib.lt_ffn_block(self.ptr, gate.handle, up.handle, down.handle, act, _ptr(norm_w), eps,
                                          _ptr(x), ntok, int(residual), _ptr(out)))

    # -- Gemma 4 layer glue -------------------------------------------------
    def scale(self, x, n: int, ntok: int, s: float) -> None:
        self._check(self.lib.lt_scale(self.ptr, _ptr(x), n, ntok, s))

    def add_rmsnorm(self, y, w, eps: float, n: int, ntok: int, x) -> None:
        self._check(self.lib.lt_add_rmsnorm(self.ptr, _ptr(y), _ptr(w), eps, n, ntok, _ptr(x)))

    def norm_pair(self, x, w, g, gs: float, eps: float, n: int, ntok: int, a, b) -> None:
        self._check(self.lib.lt_norm_pair(self.ptr, _ptr(x), _ptr(w), _ptr(g), gs, eps, n, ntok, _ptr(a), _ptr(b)))

    def ffn_tail(self, f, m, w2, w, los: float, eps: float, n: int, ntok: int, x, w1=None) -> None:
        """m = rmsnorm(m) * w2; x = (x + rmsnorm(f' + m) * w) * los, f' = rmsnorm(f) * w1 when w1 is given."""
        self._check(self.lib.lt_ffn_tail(self.ptr, _ptr(f), _ptr(w1), _ptr(m), _ptr(w2), _ptr(w), los, eps, n, ntok,
                                         _ptr(x)))

    def softcap(self, x, n: int, cap: float) -> None:
        self._check(self.lib.lt_softcap(self.ptr, _ptr(x), n, cap))

    def sample_step(self, logits, n: int, params: SampleParams, rng_state, tokens, pos, n_prompt) -> None:
        self._check(self.lib.lt_sample_step(self.ptr, _ptr(logits), n, ctypes.byref(params), _ptr(rng_state),
                                            _ptr(tokens), _ptr(pos), _ptr(n_prompt)))

    def greedy_step(self, logits, n: int, tokens, pos, n_prompt) -> None:
        """n_prompt: a device word (the prompt length of the token stream)."""
        self._check(self.lib.lt_greedy_step(self.ptr, _ptr(logits), n, _ptr(tokens), _ptr(pos), _ptr(n_prompt)))

    # -- kernel timing / graph capture -------------------------------------
    def profile(self, on: bool) -> None:
        self._check(self.lib.lt_profile_enable(self.ptr, int(on)))

    def profile_reset(self) -> None:
        self._check(self.lib.lt_profile_reset(self.ptr))

    def profile_read(self) -> dict[str, dict]:
        """{label: {count, total_ms, min_ms, max_ms}} of the timed launches."""
        out = {}
        i = 0
        while True:
            lab, cnt = ctypes.c_char_p(), ctypes.c_uint64()
            tot, mn, mx = ctypes.c_double(), ctypes.c_double(), ctypes.c_double()
            st = self.lib.lt_profile_read(self.ptr, i, ctypes.byref(lab), ctypes.byref(cnt), ctypes.byref(tot),
                                          ctypes.byref(mn), ctypes.byref(mx))
            if st != 0:
                break
            out[lab.value.decode()] = {"count": cnt.value, "total_ms": tot.value, "min_ms": mn.value,
                                       "max_ms": mx.value}
            i += 1
        return out

    def capture_begin(self) -> None:
        self._check(self.lib.lt_capture_begin(self.ptr))

    def capture_end(self) -> "Graph":
        g = ctypes.c_void_p()
        self._check(self.lib.lt_capture_end(self.ptr, ctypes.byref(g)))
        return Graph(self, g.value)

    # -- host-buffer entry points (synchronous) ---------------------------
    def quant_matvec_host(self, mat: Tensor, vec, expert: int = 0):
        """quantMatvec on host vectors (src/ops/math.zig:133): numpy f32 in, numpy f32 out."""
        import numpy as np
        v = np.ascontiguousarray(vec, dtype=np.float32)
        out = np.empty(mat.rows, dtype=np.float32)
        self._check(self.lib.lt_quant_matvec_host(self.ptr, out.ctypes.data, mat.handle, expert, v.ctypes.data,
                                                  mat.rows, mat.cols))
        return out

    def moe_forward_host(self, router: Tensor, gate: Tensor, up: Tensor | None, down: Tensor, act: int,
                         norm_topk: bool, expert_scale, x, k: int, out=None, ids=None, w=None):
        """moeForward on host arrays: x[ntok][d] -> (out, ids, w)."""
        import numpy as np
        xx = np.ascontiguousarray(x, dtype=np.float32)
        ntok = xx.shape[0]
        out = np.empty_like(xx) if out is None else out
        ids = np.empty((ntok, k), dtype=np.uint32) if ids is None else ids
        w = np.empty((ntok, k), dtype=np.float32) if w is None else w
        es = None if expert_scale is None else np.ascontiguousarray(expert_scale, dtype=np.float32)
        self._check(self.lib.lt_moe_forward_host(
            self.ptr, router.handle, gate.handle, up.handle if up else None, down.handle, act, int(norm_topk),
            None if es is None else es.ctypes.data, xx.ctypes.data, ntok, k, out.ctypes.data, ids.ctypes.data,
            w.ctypes.data))
        return out, ids, w
