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


class SoftmaxStats(ctypes.Structure):
    _fields_ = [("max", ctypes.c_float), ("exp_sum", ctypes.c_float)]


_lib = None


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
