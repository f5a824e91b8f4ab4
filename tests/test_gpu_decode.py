"""The single-token persistent MoE kernel (lt_moe_decode.cu) against the
multi-kernel path (router -> gate/up -> down) and against the CPU oracle.

A one-token lt_moe_forward / lt_moe_block runs as one persistent kernel when
its per-CTA share fits in shared memory.  Its router arithmetic is the router
kernel's, so expert ids and weights agree with the multi-kernel path bit for
bit; the expert dot products are summed in a different order (64-column
chunks instead of superblocks), so outputs agree to DECODE_VS_MULTI_L2.  The
oracle checks both.  A context created with LLMTOY_DECODE_KERNEL=0 runs the
multi-kernel path.
"""
from __future__ import annotations

import importlib
import os

import numpy as np
import pytest

from test_gpu_parity import MOE_L2_TOL, _upload_layer, bits, dev, empty, host, rel_l2

pytestmark = pytest.mark.gpu

DECODE_VS_MULTI_L2 = 2e-5  # two quantised-activation evaluations of the same layer


@pytest.fixture(scope="module")
def multi_ctx(pkg):
    import torch
    old = os.environ.get("LLMTOY_DECODE_KERNEL")
    os.environ["LLMTOY_DECODE_KERNEL"] = "0"
    try:
        c = pkg.Context(0)
    finally:
        if old is None:
            del os.environ["LLMTOY_DECODE_KERNEL"]
        else:
            os.environ["LLMTOY_DECODE_KERNEL"] = old
    c.set_stream(torch.cuda.current_stream())
    yield c
    c.close()


def _synth():
    return importlib.import_module("llmtoy-zig_b200.synth")


# gate type, down type, d, F, E, k, fused gate_up, act, norm_topk, expert scale
CASES = [
    (12, 12, 2048, 768, 128, 8, False, 0, True, False),   # config 1 (Qwen3-30B-A3B MoE layer)
    (14, 14, 2048, 768, 16, 8, False, 0, True, False),    # Q6_K experts
    (8, 8, 1024, 512, 8, 2, False, 0, False, False),      # Q8_0 experts
    (8, 8, 800, 320, 16, 4, False, 0, True, False),       # Q8_0 rows with a ragged last item
    (12, 14, 2048, 512, 24, 6, False, 0, True, True),     # mixed types, expert scale
    (12, 12, 1024, 512, 32, 16, False, 0, True, False),   # k = 16
    (12, 12, 2048, 768, 32, 1, False, 0, True, False),    # k = 1
    (12, 8, 1024, 256, 16, 8, True, 1, False, True),      # fused gate_up, GELU, expert scale
    (12, 12, 1024, 256, 256, 8, False, 0, True, False),   # 256 experts: several router warps per CTA
    (12, 12, 4096, 256, 16, 4, False, 0, True, False),    # router rows longer than the prefetched chunk
]


def _case_id(c):
    return f"g{c[0]}d{c[1]}_{c[2]}x{c[3]}_E{c[4]}k{c[5]}{'_fused' if c[6] else ''}"


def _layer(case):
    gt, dt, d, F, E, k, fused, act, norm, scale = case
    rng = np.random.Generator(np.random.PCG64(1000 + d + F + E + k))
    L = _synth().MoeLayer(rng, d, E, F, gt, dt, fused)
    x = rng.normal(0, 1, d).astype(np.float32)
    nw = rng.uniform(0.5, 1.5, d).astype(np.float32)
    escale = rng.uniform(0.5, 2.0, E).astype(np.float32) if scale else None
    return L, x, nw, escale


def _run(ctx, L, case, x, nw, escale, block):
    gt, dt, d, F, E, k, fused, act, norm, scale = case
    rt, g, u, dn = _upload_layer(ctx, L)
    es = None if escale is None else dev(escale)
    ids, ww = empty(k, "int32"), empty(k)
    xd = dev(x)
    if block:
        ctx.moe_block(rt, g, u, dn, act, norm, es, dev(nw), 1e-6, xd, 1, k, xd, ids, ww)
        out = xd
    else:
        out = empty(d)
        ctx.moe_forward(rt, g, u, dn, act, norm, es, xd, 1, k, out, ids, ww)
    res = host(out) - (x if block else 0), host(ids).view(np.uint32), host(ww)
    for t_ in (rt, g, u, dn):
        if t_ is not None:
            t_.free()
    return res


@pytest.mark.parametrize("case", CASES, ids=_case_id)
@pytest.mark.parametrize("block", [False, True], ids=["forward", "block"])
def test_decode_kernel_matches_multi_kernel_path(ctx, multi_ctx, case, block):
    L, x, nw, escale = _layer(case)
    o1, i1, w1 = _run(ctx, L, case, x, nw, escale, block)
    o2, i2, w2 = _run(multi_ctx, L, case, x, nw, escale, block)
    assert np.array_equal(i1, i2)
    assert np.array_equal(bits(w1), bits(w2))
    assert rel_l2(o1, o2) < DECODE_VS_MULTI_L2


@pytest.mark.parametrize("case", CASES[:3] + CASES[7:], ids=_case_id)
def test_decode_kernel_vs_oracle(ctx, oracle, pool, case):
    gt, dt, d, F, E, k, fused, act, norm, scale = case
    L, x, nw, escale = _layer(case)
    got, gids, gw = _run(ctx, L, case, x, nw, escale, block=False)
    ref, rids, rw = oracle.moe_layer(L, x[None], k, norm, act, escale, pool)
    assert np.array_equal(gids, rids[0])
    np.testing.assert_allclose(gw, rw[0], rtol=1e-5, atol=1e-8)
    assert rel_l2(got, ref[0]) < MOE_L2_TOL


def test_decode_kernel_is_the_path_taken(ctx, config1_layer_decode):
    """Config 1 at one token runs as the single persistent launch."""
    L = config1_layer_decode
    rt, g, u, dn = _upload_layer(ctx, L)
    x = dev(np.random.Generator(np.random.PCG64(5)).normal(0, 1, 2048).astype(np.float32))
    out = empty(2048)
    ctx.profile(True)
    ctx.profile_reset()
    ctx.moe_forward(rt, g, u, dn, 0, True, None, x, 1, 8, out)
    labels = ctx.profile_read()
    ctx.profile(False)
    ctx.profile_reset()
    assert set(labels) == {"moe_decode"}, labels
    assert labels["moe_decode"]["count"] == 1
    for t_ in (rt, g, u, dn):
        t_.free()


@pytest.fixture(scope="module")
def config1_layer_decode():
    synth = _synth()
    rng = np.random.Generator(np.random.PCG64(synth.config_seed(1)))
    return synth.MoeLayer(rng, 2048, 128, 768)


def test_decode_stack_graph_replay(ctx, multi_ctx, config1_layer_decode):
    """Six chained blocks applied in place (x <- x + moe(rmsnorm(x))), eagerly
    and as a captured graph replayed twice: the runs agree bit for bit with
    each other and closely with the multi-kernel path."""
    import torch
    L = config1_layer_decode
    rng = np.random.Generator(np.random.PCG64(66))
    x0 = rng.normal(0, 1, 2048).astype(np.float32)
    nws = [rng.uniform(0.5, 1.5, 2048).astype(np.float32) for _ in range(6)]

    def stack(c, xd, tensors, nwd):
        rt, g, u, dn = tensors
        for i in range(6):
            c.moe_block(rt, g, u, dn, 0, True, None, nwd[i], 1e-6, xd, 1, 8, xd)

    results = []
    for c in (ctx, multi_ctx):
        tensors = _upload_layer(c, L)
        nwd = [dev(n) for n in nws]
        xd = dev(x0)
        stack(c, xd, tensors, nwd)
        results.append(bits(host(xd)))
        if c is ctx:  # capture on a side stream (the legacy default stream cannot be captured)
            c.reserve(1, 8, 2048, 768)
            side = torch.cuda.Stream()
            xg = dev(x0)
            torch.cuda.synchronize()
            c.set_stream(side)
            try:
                c.capture_begin()
                stack(c, xg, tensors, nwd)
                graph = c.capture_end()
                for _ in range(2):
                    xg.copy_(torch.from_numpy(x0).cuda())
                    torch.cuda.synchronize()
                    graph.launch()
                    results.append(bits(host(xg)))
                graph.free()
            finally:
                c.set_stream(None)  # back to the context's own stream (the session fixture's choice)
        for t_ in tensors:
            if t_ is not None:
                t_.free()
    assert len(results) == 4
    # [0] eager, [1] [2] graph replays (decode kernel); [3] multi-kernel path
    assert np.array_equal(results[0], results[1]) and np.array_equal(results[0], results[2])
    f = [r.view(np.float32) - x0 for r in results]
    assert rel_l2(f[0], f[3]) < 1e-4
    ctx.sync()  # raises if a device-side wait gave up
