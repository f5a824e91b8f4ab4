"""The tensor-core grouped expert GEMM (lt_moe_gemm.cu: tcgen05 MMAs with
TMEM accumulators, Q4_K experts) against the CPU oracle.

Batches of at least LLMTOY_TC_MIN_TOKENS tokens (64 by default) with Q4_K
gate/up/down take this path; the `tc` context here sets the threshold to 2 so
small batches exercise it too.  The weights enter the tensor core exactly
(sc*q in f16, dmin*m split into two f16 planes) and the activations as two
f16 planes (about 22 bits), so results agree with the f32 CPU path to the
same MoE tolerance as the CUDA-core kernels.
"""
from __future__ import annotations

import importlib
import os

import numpy as np
import pytest

from test_gpu_parity import MOE_L2_TOL, W_TOL, _upload_layer, bits, dev, empty, host, max_rel, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tc(pkg):
    import torch
    old = os.environ.get("LLMTOY_TC_MIN_TOKENS")
    os.environ["LLMTOY_TC_MIN_TOKENS"] = "2"
    try:
        c = pkg.Context(0)
    finally:
        if old is None:
            del os.environ["LLMTOY_TC_MIN_TOKENS"]
        else:
            os.environ["LLMTOY_TC_MIN_TOKENS"] = old
    c.set_stream(None)  # own stream: inputs are copied synchronously, results read after a device sync
    yield c
    c.close()


def _synth():
    return importlib.import_module("llmtoy-zig_b200.synth")


def _labels(ctx, fn):
    ctx.profile(True)
    ctx.profile_reset()
    fn()
    lab = ctx.profile_read()
    ctx.profile(False)
    ctx.profile_reset()
    return lab


# d, F, E, k, fused gate_up, act, norm_topk, expert scale, T
CASES = [
    (2048, 768, 128, 8, False, 0, True, False, 5),      # config 1 shape, partial tiles
    (2048, 768, 128, 8, False, 0, True, False, 64),
    (1024, 512, 8, 2, False, 0, True, False, 200),      # ~50 tokens per expert: several 32-position tiles
    (1024, 512, 16, 8, True, 1, False, True, 33),       # fused gate_up, GELU, expert scale
    (2048, 256, 32, 4, False, 0, True, False, 40),      # one superblock of down columns
    # 48+ positions per expert on average: 64-position tiles (N = 128 MMAs)
    (2048, 768, 16, 8, False, 0, True, False, 300),
    (1024, 512, 4, 2, True, 1, False, True, 130),       # fused gate_up, GELU, expert scale
]


def _case_id(c):
    return f"d{c[0]}F{c[1]}E{c[2]}k{c[3]}T{c[8]}{'_fused' if c[4] else ''}"


@pytest.mark.parametrize("case", CASES, ids=_case_id)
def test_gemm_moe_forward_vs_oracle(tc, oracle, pool, case):
    d, F, E, k, fused, act, norm, scale, T = case
    rng = np.random.Generator(np.random.PCG64(7000 + d + F + E + T))
    L = _synth().MoeLayer(rng, d, E, F, 12, 12, fused)
    x = rng.normal(0, 1, size=(T, d)).astype(np.float32)
    escale = rng.uniform(0.5, 2.0, E).astype(np.float32) if scale else None
    rt, g, u, dn = _upload_layer(tc, L)
    out, ids, ww = empty(T * d), empty(T * k, "int32"), empty(T * k)
    es = None if escale is None else dev(escale)
    xd = dev(x)
    lab = _labels(tc, lambda: tc.moe_forward(rt, g, u, dn, act, norm, es, xd, T, k, out, ids, ww))
    assert "moe_gemm_gate_up" in lab and "moe_gemm_down" in lab, lab
    got = host(out).reshape(T, d)
    ref, rids, rw = oracle.moe_layer(L, x, k, norm, act, escale, pool)
    assert np.array_equal(host(ids).view(np.uint32).reshape(T, k), rids)
    np.testing.assert_allclose(host(ww).reshape(T, k), rw, rtol=5 * W_TOL, atol=1e-8)
    assert rel_l2(got, ref) < MOE_L2_TOL
    assert max_rel(got, ref) < 1e-3
    tc.sync()
    for t_ in (rt, g, u, dn):
        if t_ is not None:
            t_.free()


def test_gemm_moe_block_and_determinism(tc, oracle, pool):
    """lt_moe_block (norm + residual, in place) through the GEMM path, twice:
    the same bits both times, and the oracle's x + moe(rmsnorm(x))."""
    synth = _synth()
    rng = np.random.Generator(np.random.PCG64(synth.config_seed(1)))
    L = synth.MoeLayer(rng, 2048, 128, 768)
    T = 48
    x = rng.normal(0, 3, size=(T, 2048)).astype(np.float32)
    nw = rng.uniform(0.5, 1.5, 2048).astype(np.float32)
    rt, g, u, dn = _upload_layer(tc, L)
    runs = []
    for _ in range(2):
        xd = dev(x)
        tc.moe_block(rt, g, u, dn, 0, True, None, dev(nw), 1e-6, xd, T, 8, xd)
        runs.append(host(xd).reshape(T, 2048))
    assert np.array_equal(bits(runs[0]), bits(runs[1]))
    xn = np.empty_like(x)
    for t in range(T):
        oracle.lib().orc_rmsnorm(xn[t].ctypes.data, x[t].ctypes.data, nw.ctypes.data, 2048, 1e-6)
    y, _, _ = oracle.moe_layer(L, xn, 8, True, 0, None, pool)
    assert rel_l2(runs[0] - x, y) < MOE_L2_TOL
    tc.sync()
    for t_ in (rt, g, u, dn):
        t_.free()


@pytest.mark.parametrize("T", [70, 300])
def test_gemm_skewed_routing(tc, oracle, T):
    """Every token on the same few experts: one expert gets all T positions
    (several tiles; 64-position tiles at T = 300), the combine still runs in
    slot order."""
    synth = _synth()
    rng = np.random.Generator(np.random.PCG64(31))
    L = synth.MoeLayer(rng, 1024, 16, 512)
    k = 4
    x = rng.normal(0, 1, size=(T, 1024)).astype(np.float32)
    ids = np.stack([np.r_[[3], rng.choice(np.arange(4, 9), size=k - 1, replace=False)] for _ in range(T)])
    ids = ids.astype(np.uint32)
    w = rng.uniform(0.01, 0.3, size=(T, k)).astype(np.float32)
    rt, g, u, dn = _upload_layer(tc, L)
    out = empty(T * 1024)
    tc.moe_ffn(g, u, dn, 0, dev(x), T, dev(ids.view(np.int32)), dev(w), k, out)
    got = host(out).reshape(T, 1024)
    F, d = 512, 1024
    for t in range(0, T, 7):
        ref = np.zeros(d, np.float32)
        for s in range(k):
            e = int(ids[t, s])
            gg = oracle.quant_matvec(L.gate[e * F:(e + 1) * F], 12, x[t], F, d)
            uu = oracle.quant_matvec(L.up[e * F:(e + 1) * F], 12, x[t], F, d)
            h = np.array([oracle.lib().orc_silu(float(v)) for v in gg], np.float32) * uu
            yv = oracle.quant_matvec(L.down[e * d:(e + 1) * d], 12, h, d, F)
            ref = (ref + w[t, s] * yv).astype(np.float32)
        assert rel_l2(got[t], ref) < MOE_L2_TOL
    tc.sync()
    for t_ in (rt, g, u, dn):
        t_.free()


# Stacked-plane schemes: Q6_K and Q8_0 experts, and Q4_K wider than 2048
# columns (config 3's d_model 2816), each against the oracle.
# d, F, E, k, gate/up type, down type, fused gate_up, act, T
Q4, Q6, Q8 = 12, 14, 8
TYPE_CASES = [
    (2048, 768, 32, 8, Q6, Q6, False, 0, 70),
    (2048, 768, 32, 8, Q8, Q8, False, 0, 70),
    (2048, 768, 16, 8, Q4, Q6, False, 0, 100),    # single-plane Q4_K gate/up, stacked Q6_K down
    (2048, 768, 8, 8, Q6, Q8, True, 1, 300),      # fused gate_up, GELU, 64-position tiles
    (2816, 704, 16, 8, Q4, Q8, False, 1, 80),     # config-3 shape: Q4_K over 11 superblocks, Q8_0 down K = 704
    (2816, 704, 16, 8, Q6, Q8, False, 1, 200),
    (1024, 512, 8, 2, Q8, Q6, False, 0, 130),
]


def _type_id(c):
    n = {Q4: "q4k", Q6: "q6k", Q8: "q8_0"}
    return f"d{c[0]}F{c[1]}E{c[2]}T{c[8]}_{n[c[4]]}_{n[c[5]]}{'_fused' if c[6] else ''}"


@pytest.mark.parametrize("case", TYPE_CASES, ids=_type_id)
def test_gemm_stacked_types_vs_oracle(tc, oracle, pool, case):
    d, F, E, k, gt, dt, fused, act, T = case
    rng = np.random.Generator(np.random.PCG64(9100 + d + F + E + T + gt + 3 * dt))
    L = _synth().MoeLayer(rng, d, E, F, gt, dt, fused)
    x = rng.normal(0, 1, size=(T, d)).astype(np.float32)
    rt, g, u, dn = _upload_layer(tc, L)
    out, ids, ww = empty(T * d), empty(T * k, "int32"), empty(T * k)
    xd = dev(x)
    lab = _labels(tc, lambda: tc.moe_forward(rt, g, u, dn, act, True, None, xd, T, k, out, ids, ww))
    assert "moe_gemm_gate_up" in lab and "moe_gemm_down" in lab, lab
    got = host(out).reshape(T, d)
    ref, rids, _ = oracle.moe_layer(L, x, k, True, act, None, pool)
    assert np.array_equal(host(ids).view(np.uint32).reshape(T, k), rids)
    assert np.all(np.isfinite(got))
    assert rel_l2(got, ref) < MOE_L2_TOL
    assert max_rel(got, ref) < 1e-3
    tc.sync()
    for t_ in (rt, g, u, dn):
        if t_ is not None:
            t_.free()
