"""CUDA path vs the CPU oracle, through the C ABI, on seeded synthetic inputs.

Bars (north star): dequantised values and router ids bit-exact; floating-point
outputs within the stated tolerance.  Matvecs use the reference's own GPU fuzz
metric, max|delta| / max|ref| < 1e-4 (src/gpu/matvec.zig:4609-4618); MoE
layer outputs use relative L2 <= 1e-4 (ten times tighter than the 1e-3 logits
bar).
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MATVEC_TOL = 1e-4
MOE_L2_TOL = 1e-4
W_TOL = 2e-6


def _torch():
    import torch
    return torch


def dev(a: np.ndarray):
    """A device copy, complete before returning: the context runs on its own
    stream, which does not wait for the copy engine's work on torch's."""
    t = _torch().from_numpy(np.ascontiguousarray(a)).cuda()
    _torch().cuda.synchronize()
    return t


def empty(n, dtype="float32"):
    torch = _torch()
    return torch.empty(n, dtype=getattr(torch, dtype), device="cuda")


def host(t) -> np.ndarray:
    _torch().cuda.synchronize()
    return t.cpu().numpy()


def max_rel(got, ref) -> float:
    return float(np.max(np.abs(got - ref)) / (np.max(np.abs(ref)) + 1e-6))


def rel_l2(got, ref) -> float:
    return float(np.linalg.norm(got - ref) / (np.linalg.norm(ref) + 1e-30))


def bits(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


# ── dequant: bit-exact ──────────────────────────────────────────────────────

def test_dequant_golden_bit_exact(ctx, golden):
    for case in golden["dequant"]:
        raw = bytes.fromhex(case["hex"])
        t = ctx.upload(raw, case["type"], 1, case["cols"])
        out = empty(case["cols"])
        ctx.dequant(t, 0, 1, out)
        assert bits(host(out)).tolist() == case["expect"], case["name"]
        t.free()


@pytest.mark.parametrize("ggml_type,rows,cols", [
    (12, 37, 2048), (12, 64, 768), (14, 33, 2048), (14, 17, 2816), (8, 41, 896), (8, 9, 4864),
    (1, 13, 96), (0, 11, 100)])
def test_dequant_matrix_bit_exact(ctx, pkg, oracle, ggml_type, rows, cols):
    import importlib
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.Generator(np.random.PCG64(1000 + ggml_type * 7 + cols))
    mat = synth.matrix(rng, ggml_type, rows, cols)
    t = ctx.upload(mat, ggml_type, rows, cols)
    out = empty(rows * cols)
    ctx.dequant(t, 0, rows, out)
    got = host(out).reshape(rows, cols)
    ref = oracle.dequant(mat, ggml_type, rows, cols)
    assert np.array_equal(bits(got), bits(ref))
    # a row range in the middle
    out2 = empty(3 * cols)
    ctx.dequant(t, 5, 3, out2)
    assert np.array_equal(bits(host(out2).reshape(3, cols)), bits(ref[5:8]))
    t.free()


@pytest.mark.parametrize("ggml_type,cols", [(12, 768), (14, 2816), (8, 896), (8, 4864), (1, 100), (0, 5)])
def test_upload_download_roundtrip(ctx, ggml_type, cols):
    import importlib
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.Generator(np.random.PCG64(77))
    mat = synth.matrix(rng, ggml_type, 5, cols)
    t = ctx.upload(mat, ggml_type, 5, cols)
    assert t.row_pitch % 16 == 0 and t.row_pitch >= t.row_bytes
    assert t.download() == mat.tobytes()
    t.free()


# ── quantMatvec ──────────────────────────────────────────────────────────────

MATVEC_SHAPES = [(12, 768, 2048), (12, 2048, 768), (12, 100, 2816), (14, 1000, 2048), (14, 300, 2816),
                 (8, 896, 896), (8, 128, 4864), (8, 77, 2048), (0, 64, 100), (1, 64, 96)]


@pytest.mark.parametrize("ggml_type,rows,cols", MATVEC_SHAPES)
@pytest.mark.parametrize("ntok", [1, 3, 6])
def test_qmatvec_vs_oracle(ctx, oracle, ggml_type, rows, cols, ntok):
    import importlib
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.Generator(np.random.PCG64(rows * 31 + cols + ggml_type))
    mat = synth.matrix(rng, ggml_type, rows, cols)
    x = rng.normal(0, 1, size=(ntok, cols)).astype(np.float32)
    t = ctx.upload(mat, ggml_type, rows, cols)
    y = empty(ntok * rows)
    ctx.qmatvec(t, dev(x), y, ntok)
    got = host(y).reshape(ntok, rows)
    for i in range(ntok):
        ref = oracle.quant_matvec(mat, ggml_type, x[i], rows, cols)
        assert max_rel(got[i], ref) < MATVEC_TOL, (ggml_type, rows, cols, i)
    t.free()


@pytest.mark.parametrize("ggml_type,rows,cols", [(8, 32, 256), (12, 32, 256), (14, 32, 256),
                                                 (14, 2048, 2816), (12, 4096, 2816), (8, 2048, 704)])
def test_qmatvec_reference_fuzz(ctx, oracle, ggml_type, rows, cols):
    """The reference's GPU fuzz recipe: random bytes, f16 scales stamped to
    0x21CD, x ~ U(-1,1) (src/gpu/matvec.zig:4560-4618, shapes :5247-5767)."""
    import importlib
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.Generator(np.random.PCG64(4242 + ggml_type))
    mat = synth.matrix(rng, ggml_type, rows, cols, stamp_d=True)
    x = (rng.random(cols, dtype=np.float32) - 0.5) * 2.0
    t = ctx.upload(mat, ggml_type, rows, cols)
    y = empty(rows)
    ctx.qmatvec(t, dev(x), y, 1)
    ref = oracle.quant_matvec(mat, ggml_type, x, rows, cols)
    assert max_rel(host(y), ref) < MATVEC_TOL
    t.free()


@pytest.mark.parametrize("ggml_type,rows,cols", [(14, 40000, 2816), (12, 60000, 2048), (8, 50001, 896),
                                                 (13, 40000, 2048), (8, 40001, 2048), (8, 20000, 4096)])
def test_qmatvec_streaming_lm_head(ctx, oracle, ggml_type, rows, cols):
    """One token over an lm_head-sized matrix runs as the persistent streaming
    kernel (per-warp TMA rings; Q8_0 rows of 2048+ columns through the
    wide-row variant with a transpose reduction): against the oracle, and
    against the multi-token kernel on the same row."""
    import importlib
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.Generator(np.random.PCG64(rows + cols + ggml_type))
    mat = synth.matrix(rng, ggml_type, rows, cols)
    x = rng.normal(0, 1, size=(3, cols)).astype(np.float32)
    t = ctx.upload(mat, ggml_type, rows, cols)
    y1, y3 = empty(rows), empty(3 * rows)
    ctx.profile(True)
    ctx.qmatvec(t, dev(x[0]), y1, 1)
    ctx.sync()
    labels = ctx.profile_read()
    ctx.profile_reset()
    ctx.profile(False)
    assert any(k.startswith("qmv_stream") for k in labels), labels
    ctx.qmatvec(t, dev(x), y3, 3)
    got = host(y1)
    ref = oracle.quant_matvec(mat, ggml_type, x[0], rows, cols)
    assert max_rel(got, ref) < MATVEC_TOL
    assert rel_l2(got, host(y3)[:rows]) < 1e-6
    t.free()


def test_qmatvec_expert_slice(ctx, oracle):
    import importlib
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.Generator(np.random.PCG64(5))
    E, F, d = 4, 256, 512
    mat = synth.matrix(rng, 12, E * F, d)
    t = ctx.upload(mat, 12, F, d, n_experts=E)
    x = rng.normal(0, 1, d).astype(np.float32)
    y = empty(F)
    ctx.qmatvec(t, dev(x), y, 1, expert=2)
    ref = oracle.quant_matvec(mat[2 * F:3 * F], 12, x, F, d)
    assert max_rel(host(y), ref) < MATVEC_TOL
    t.free()


# ── router ───────────────────────────────────────────────────────────────────

def _route(ctx, w: np.ndarray, x: np.ndarray, k: int, norm=False, escale=None):
    E, d = w.shape
    T = x.shape[0]
    rt = ctx.upload(np.ascontiguousarray(w, np.float32), 0, E, d)
    ids = empty(T * k, "int32")
    ww = empty(T * k)
    ctx.moe_route(rt, dev(x), T, k, norm, None if escale is None else dev(np.asarray(escale, np.float32)), ids, ww)
    out = host(ids).view(np.uint32).reshape(T, k), host(ww).reshape(T, k)
    rt.free()
    return out


def test_router_golden_closed_form(ctx, golden):
    c = golden["router"]["gpu_router_closed_form"]
    w = np.array(c["weights"], np.float32).reshape(c["rows"], c["cols"])
    ids, ww = _route(ctx, w, np.array([c["vec"]], np.float32), c["k"], escale=c["expert_scale"])
    assert ids[0].tolist() == c["expect_ids"]
    np.testing.assert_allclose(ww[0], c["expect_w"], atol=c["tol"])


def test_router_golden_ties(ctx, golden):
    c = golden["router"]["topk_ties"]
    w = np.array(c["scores"], np.float32).reshape(-1, 1)  # logits == scores with x = [1]
    ids, _ = _route(ctx, w, np.ones((1, 1), np.float32), c["k"])
    assert ids[0].tolist() == c["expect"]


@pytest.mark.parametrize("case", ["topk_matvec_6x5", "par_37x33", "streamed_5x4"])
def test_router_golden_matvecs(ctx, oracle, golden, case):
    c = golden["router"][case]
    w = np.array(c["weights"], np.float32).reshape(c["rows"], c["cols"])
    x = np.array(c["vec"], np.float32)
    ids, ww = _route(ctx, w, x[None], c["k"])
    with oracle.Pool(c.get("threads", 4)) as p:
        rid, rp = oracle.router_topk_softmax(w, x, c["k"], p)
    assert ids[0].tolist() == rid.tolist()
    np.testing.assert_allclose(ww[0], rp, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("E,d,k", [(128, 2048, 8), (128, 2816, 8), (64, 1000, 4), (37, 33, 8), (256, 512, 16),
                                   (8, 64, 1)])
def test_router_ids_bit_exact(ctx, oracle, pool, E, d, k):
    rng = np.random.Generator(np.random.PCG64(E * 1000 + d))
    w = rng.normal(0, 0.02, size=(E, d)).astype(np.float32)
    x = rng.normal(0, 1, size=(40, d)).astype(np.float32)
    for norm in (False, True):
        ids, ww = _route(ctx, w, x, k, norm=norm)
        for t in range(x.shape[0]):
            rid, rp = oracle.router_topk_softmax(w, x[t], k, pool)
            assert ids[t].tolist() == rid.tolist(), (t, norm)
            if norm:
                rp = rp / np.float32(np.sum(rp, dtype=np.float32))
            np.testing.assert_allclose(ww[t], rp, rtol=W_TOL * 5, atol=1e-8)


def test_router_logits_exact_order(ctx, oracle):
    """The GPU logit is dotf32 bit for bit: with near-tied experts the ids
    still agree (a different summation order would flip some)."""
    rng = np.random.Generator(np.random.PCG64(99))
    d, E = 2048, 128
    base = rng.normal(0, 0.02, size=(1, d)).astype(np.float32)
    w = np.repeat(base, E, axis=0)
    w += rng.normal(0, 1e-7, size=w.shape).astype(np.float32)  # logits differ in the last bits
    x = rng.normal(0, 1, size=(16, d)).astype(np.float32)
    ids, _ = _route(ctx, w, x, 8)
    for t in range(16):
        rid, _ = oracle.router_topk_softmax(w, x[t], 8)
        assert ids[t].tolist() == rid.tolist()


# ── MoE layer ────────────────────────────────────────────────────────────────

def _upload_layer(ctx, L):
    E, F, d = L.n_experts, L.d_expert, L.d_model
    rt = ctx.upload(L.router, 0, E, d)
    g = ctx.upload(L.gate, L.gate_type, (F if L.up is not None else 2 * F), d, n_experts=E)
    u = ctx.upload(L.up, L.gate_type, F, d, n_experts=E) if L.up is not None else None
    dn = ctx.upload(L.down, L.down_type, d, F, n_experts=E)
    return rt, g, u, dn


def _check_moe(ctx, oracle, pool, L, x, k, norm, act=0, escale=None):
    rt, g, u, dn = _upload_layer(ctx, L)
    T = x.shape[0]
    out, ids, ww = empty(T * L.d_model), empty(T * k, "int32"), empty(T * k)
    es = None if escale is None else dev(np.asarray(escale, np.float32))
    ctx.moe_forward(rt, g, u, dn, act, norm, es, dev(x), T, k, out, ids, ww)
    got, gids, gw = host(out).reshape(T, -1), host(ids).view(np.uint32).reshape(T, k), host(ww).reshape(T, k)
    ref, rids, rw = oracle.moe_layer(L, x, k, norm, act, escale, pool)
    assert np.array_equal(gids, rids)
    np.testing.assert_allclose(gw, rw, rtol=5 * W_TOL, atol=1e-8)
    assert rel_l2(got, ref) < MOE_L2_TOL
    assert max_rel(got, ref) < 1e-3
    for t_ in (rt, g, u, dn):
        if t_ is not None:
            t_.free()
    return got


@pytest.fixture(scope="module")
def config1_layer(pkg):
    import importlib
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.Generator(np.random.PCG64(synth.config_seed(1)))
    return synth.MoeLayer(rng, 2048, 128, 768)


@pytest.mark.parametrize("T", [1, 16])
def test_moe_config1_vs_oracle(ctx, oracle, pool, config1_layer, T):
    rng = np.random.Generator(np.random.PCG64(T))
    x = rng.normal(0, 1, size=(T, 2048)).astype(np.float32)
    _check_moe(ctx, oracle, pool, config1_layer, x, 8, norm=True)


def test_moe_config1_t512_vs_oracle(ctx, oracle, pool, config1_layer):
    rng = np.random.Generator(np.random.PCG64(512))
    x = rng.normal(0, 1, size=(512, 2048)).astype(np.float32)
    _check_moe(ctx, oracle, pool, config1_layer, x, 8, norm=True)


@pytest.mark.parametrize("gate_type,down_type,d,F,E,k,fused,act,norm,scale", [
    (12, 8, 2816, 704, 16, 8, True, 1, False, True),     # Gemma4-like: fused gate_up, GELU, down_exps_scale
    (14, 14, 2048, 768, 16, 8, False, 0, True, False),   # Q6_K experts
    (8, 8, 1024, 512, 8, 2, False, 0, False, False),     # Q8_0 experts, moeForward semantics
    (12, 12, 2048, 768, 32, 1, False, 0, True, False),   # k = 1
    (12, 12, 1024, 512, 32, 16, False, 0, True, False),  # k = 16
    (12, 14, 2048, 512, 24, 6, False, 0, True, True),    # mixed types, E not a power of two
])
@pytest.mark.parametrize("T", [1, 5])
def test_moe_variants_vs_oracle(ctx, oracle, pool, gate_type, down_type, d, F, E, k, fused, act, norm, scale, T):
    import importlib
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.Generator(np.random.PCG64(d + F + E + k))
    L = synth.MoeLayer(rng, d, E, F, gate_type, down_type, fused)
    x = rng.normal(0, 1, size=(T, d)).astype(np.float32)
    escale = rng.uniform(0.5, 2.0, E).astype(np.float32) if scale else None
    _check_moe(ctx, oracle, pool, L, x, k, norm, act, escale)


@pytest.mark.parametrize("T", [1, 7])
def test_moe_block_vs_oracle(ctx, oracle, pool, config1_layer, T):
    """lt_moe_block: x + moe(rmsnorm(x) * w), norm and residual fused; run in place."""
    L = config1_layer
    rng = np.random.Generator(np.random.PCG64(70 + T))
    x = rng.normal(0, 3, size=(T, 2048)).astype(np.float32)
    nw = rng.uniform(0.5, 1.5, 2048).astype(np.float32)
    rt, g, u, dn = _upload_layer(ctx, L)
    xd = dev(x)
    ids, ww = empty(T * 8, "int32"), empty(T * 8)
    ctx.moe_block(rt, g, u, dn, 0, True, None, dev(nw), 1e-6, xd, T, 8, xd, ids, ww)
    got = host(xd).reshape(T, 2048)
    xn = np.empty_like(x)
    for t in range(T):
        oracle.lib().orc_rmsnorm(xn[t].ctypes.data, x[t].ctypes.data, nw.ctypes.data, 2048, 1e-6)
    y, rids, rw = oracle.moe_layer(L, xn, 8, True, 0, None, pool)
    assert np.array_equal(host(ids).view(np.uint32).reshape(T, 8), rids)
    assert rel_l2(got - x, y) < MOE_L2_TOL
    np.testing.assert_allclose(got, x + y, rtol=1e-4, atol=1e-3 * float(np.abs(y).max()))
    for t_ in (rt, g, u, dn):
        t_.free()


def test_moe_ffn_skewed_routing(ctx, oracle, config1_layer):
    """Dispatch with every token on the same few experts (and one expert hit by
    all tokens): the grouped plan must still combine in slot order."""
    L = config1_layer
    rng = np.random.Generator(np.random.PCG64(3))
    T, k = 24, 8
    x = rng.normal(0, 1, size=(T, 2048)).astype(np.float32)
    ids = np.stack([np.r_[[5], rng.choice(np.arange(6, 14), size=k - 1, replace=False)] for _ in range(T)])
    ids = ids.astype(np.uint32)
    w = rng.uniform(0.01, 0.3, size=(T, k)).astype(np.float32)
    rt, g, u, dn = _upload_layer(ctx, L)
    out = empty(T * 2048)
    ctx.moe_ffn(g, u, dn, 0, dev(x), T, dev(ids.view(np.int32)), dev(w), k, out)
    got = host(out).reshape(T, 2048)
    F, d = L.d_expert, L.d_model
    rb_g, rb_d = 8 * 144, 3 * 144
    for t in range(T):
        ref = np.zeros(d, np.float32)
        for s in range(k):
            e = int(ids[t, s])
            gg = oracle.quant_matvec(L.gate[e * F:(e + 1) * F], 12, x[t], F, d)
            uu = oracle.quant_matvec(L.up[e * F:(e + 1) * F], 12, x[t], F, d)
            h = np.array([oracle.lib().orc_silu(float(v)) for v in gg], np.float32) * uu
            y = oracle.quant_matvec(L.down[e * d:(e + 1) * d], 12, h, d, F)
            ref = (ref + w[t, s] * y).astype(np.float32)
        assert rel_l2(got[t], ref) < MOE_L2_TOL
    del rb_g, rb_d
    for t_ in (rt, g, u, dn):
        t_.free()


def test_moe_deterministic(ctx, config1_layer):
    rt, g, u, dn = _upload_layer(ctx, config1_layer)
    x = dev(np.random.Generator(np.random.PCG64(8)).normal(0, 1, size=(16, 2048)).astype(np.float32))
    outs = []
    for _ in range(3):
        o = empty(16 * 2048)
        ctx.moe_forward(rt, g, u, dn, 0, True, None, x, 16, 8, o)
        outs.append(bits(host(o)))
    assert all(np.array_equal(outs[0], o) for o in outs[1:])
    for t_ in (rt, g, u, dn):
        t_.free()


# ── host-buffer entry points ─────────────────────────────────────────────────

def test_host_entry_points_match_device_ops(ctx, oracle, config1_layer):
    L = config1_layer
    rt, g, u, dn = _upload_layer(ctx, L)
    rng = np.random.Generator(np.random.PCG64(11))
    x = rng.normal(0, 1, size=(3, 2048)).astype(np.float32)
    out_h, ids_h, w_h = ctx.moe_forward_host(rt, g, u, dn, 0, True, None, x, 8)
    o = empty(3 * 2048)
    ids = empty(24, "int32")
    ww = empty(24)
    ctx.moe_forward(rt, g, u, dn, 0, True, None, dev(x), 3, 8, o, ids, ww)
    assert np.array_equal(bits(out_h), bits(host(o).reshape(3, -1)))
    assert np.array_equal(ids_h, host(ids).view(np.uint32).reshape(3, 8))
    # quantMatvec on host vectors == oracle
    y = ctx.quant_matvec_host(g, x[0], expert=7)
    ref = oracle.quant_matvec(L.gate[7 * 768:8 * 768], 12, x[0], 768, 2048)
    assert max_rel(y, ref) < MATVEC_TOL
    for t_ in (rt, g, u, dn):
        t_.free()


# ── greedy / rmsnorm / softmax ───────────────────────────────────────────────

def test_argmax_golden_and_random(ctx, oracle, golden):
    a = golden["misc"]["argmax"]
    v0 = np.array(a[0]["values"], np.float32)
    idx = empty(1, "int32")
    ctx.argmax(dev(v0), v0.size, 1, idx)
    assert int(host(idx)[0]) == a[0]["expect"]
    v1 = np.full(a[1]["n"], -4.0, np.float32)
    v1[a[1]["peaks"]] = 9.0
    ctx.argmax(dev(v1), v1.size, 1, idx)
    assert int(host(idx)[0]) == a[1]["expect"]
    rng = np.random.Generator(np.random.PCG64(1))
    x = rng.normal(0, 1, size=(5, 151936)).astype(np.float32)
    x[2, [100, 150000]] = 50.0  # tie across far-apart blocks
    x[4, :] = 1.0               # all equal -> index 0
    idx5 = empty(5, "int32")
    ctx.argmax(dev(x), 151936, 5, idx5)
    got = host(idx5).tolist()
    assert got == [oracle.greedy(x[i]) for i in range(5)]
    assert got[2] == 100 and got[4] == 0


def test_rmsnorm_softmax_vs_oracle(ctx, oracle, golden):
    rng = np.random.Generator(np.random.PCG64(2))
    for n in (4, 896, 2048, 2816):
        x = rng.normal(0, 1, size=(3, n)).astype(np.float32)
        w = rng.uniform(0.5, 1.5, n).astype(np.float32)
        y = empty(3 * n)
        ctx.rmsnorm(dev(x), dev(w), 1e-6, n, 3, y)
        got = host(y).reshape(3, n)
        for i in range(3):
            ref = np.empty(n, np.float32)
            oracle.lib().orc_rmsnorm(ref.ctypes.data, x[i].ctypes.data, w.ctypes.data, n, 1e-6)
            np.testing.assert_allclose(got[i], ref, rtol=2e-6, atol=1e-7)
    c = golden["misc"]["rmsnorm"]
    y = empty(4)
    ctx.rmsnorm(dev(np.array(c["x"], np.float32)), dev(np.array(c["w"], np.float32)), c["eps"], 4, 1, y)
    np.testing.assert_allclose(host(y), c["expect"], atol=c["tol"])
    for c in golden["misc"]["softmax"]:
        s = dev(np.array(c["x"], np.float32))
        ctx.softmax(s, 3, 1)
        v = host(s)
        assert abs(float(v.sum()) - 1.0) <= c["tol"] and v[2] > v[1] > v[0]


# ── error behaviour (no CPU fallback, clean status codes) ────────────────────

def test_error_paths(ctx, pkg):
    with pytest.raises(pkg.LtError) as e:
        ctx.upload(bytes(18), 2, 1, 32)  # Q4_0: not a supported type
    assert e.value.status == 2
    with pytest.raises(pkg.LtError) as e:
        ctx.upload(bytes(144), 12, 1, 200)  # cols not a multiple of 256
    assert e.value.status == 1
    with pytest.raises(pkg.LtError) as e:
        ctx.upload(bytes(100), 12, 1, 256)  # wrong byte count
    assert e.value.status == 1
    t = ctx.upload(bytes(144 * 4), 12, 2, 256, n_experts=2)
    y = empty(2)
    with pytest.raises(pkg.LtError) as e:
        ctx.qmatvec(t, empty(256), y, 1, expert=2)
    assert e.value.status == 1
    r = ctx.upload(np.zeros((4, 256), np.float32), 0, 4, 256)
    with pytest.raises(pkg.LtError) as e:
        ctx.moe_route(r, empty(256), 1, 5, False, None, empty(5, "int32"), empty(5))  # k > E
    assert e.value.status == 1
    with pytest.raises(pkg.LtError) as e:
        ctx.moe_route(t, empty(256), 1, 1, False, None, empty(1, "int32"), empty(1))  # router not F32
    assert e.value.status == 2
    t.free()
    r.free()
    ctx.sync()


@pytest.mark.parametrize("norm", [False, True])
def test_router_token_major_matches_expert_major(ctx, oracle, norm):
    """Batches of 32+ tokens take the token-major router kernel; its ids,
    weights and normalised/quantised rows equal the expert-major kernel's
    (31 tokens) bit for bit, and the ids equal the oracle's."""
    import importlib
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.Generator(np.random.PCG64(2024))
    E, d, k = 128, 2048, 8
    w = synth.router_weights(rng, E, d)
    x = synth.hidden(rng, 40, d)
    nw = rng.uniform(0.5, 1.5, d).astype(np.float32)
    rt = ctx.upload(w, 0, E, d)
    outs = []
    for T in (31, 40):
        ids, ww = empty(T * k, "int32"), empty(T * k)
        if norm:
            L = synth.MoeLayer(np.random.default_rng(5), d, E, 256, 12, 12)
            g = ctx.upload(L.gate, 12, 256, d, n_experts=E)
            u = ctx.upload(L.up, 12, 256, d, n_experts=E)
            dn = ctx.upload(L.down, 12, d, 256, n_experts=E)
            out = empty(T * d)
            ctx.moe_block(rt, g, u, dn, 0, True, None, dev(nw), 1e-6, dev(x[:T]), T, k, out, ids, ww)
            for t_ in (g, u, dn):
                t_.free()
        else:
            ctx.moe_route(rt, dev(x[:T]), T, k, True, None, ids, ww)
        outs.append((host(ids).reshape(T, k)[:31], host(ww).reshape(T, k)[:31]))
    np.testing.assert_array_equal(outs[0][0], outs[1][0])
    np.testing.assert_array_equal(bits(outs[0][1]), bits(outs[1][1]))
    if not norm:
        for t in range(31):
            rid, _ = oracle.router_topk_softmax(w, x[t], k)
            assert np.array_equal(outs[1][0][t].astype(np.uint32), rid)
    rt.free()


@pytest.mark.parametrize("t,d,F,act", [(8, 896, 4864, 0), (12, 2048, 768, 0), (14, 2816, 2048, 1), (13, 1024, 512, 0)])
@pytest.mark.parametrize("ntok,residual", [(1, True), (1, False), (5, True)])
def test_ffn_block_vs_oracle(ctx, oracle, t, d, F, act, ntok, residual):
    """lt_ffn_block (forward.zig:307-312): out = (x if residual) + down .
    (act(gate . xn) * (up . xn)), xn = rmsnorm(x) * w -- one token through the
    persistent decode kernel's dense mode (Q8_0/Q4_K/Q6_K), the grouped
    kernels otherwise."""
    import importlib
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.Generator(np.random.PCG64(d + F + t))
    gate, up, down = synth.matrix(rng, t, F, d), synth.matrix(rng, t, F, d), synth.matrix(rng, t, d, F)
    nw = rng.uniform(0.5, 1.5, d).astype(np.float32)
    x = rng.normal(0, 1, (ntok, d)).astype(np.float32)
    tg, tu, td = ctx.upload(gate, t, F, d), ctx.upload(up, t, F, d), ctx.upload(down, t, d, F)
    out = empty(ntok * d)
    ctx.ffn_block(tg, tu, td, act, dev(nw), 1e-6, dev(x), ntok, out, residual=residual)
    got = host(out).reshape(ntok, d)
    lib = oracle.lib()
    for i in range(ntok):
        xn = np.empty(d, np.float32)
        lib.orc_rmsnorm(xn.ctypes.data, x[i].ctypes.data, nw.ctypes.data, d, 1e-6)
        g = oracle.quant_matvec(gate, t, xn, F, d)
        u = oracle.quant_matvec(up, t, xn, F, d)
        f = lib.orc_gelu if act else lib.orc_silu
        h = (np.array([f(float(v)) for v in g], np.float32) * u).astype(np.float32)
        ref = oracle.quant_matvec(down, t, h, d, F) + (x[i] if residual else 0)
        assert rel_l2(got[i], ref) < 1e-4, (i, rel_l2(got[i], ref))
    for w in (tg, tu, td):
        w.free()


@pytest.mark.parametrize("T", [1, 6])
def test_moe_ffn_invalid_id_reported(ctx, pkg, oracle, pool, T):
    """An expert id past the tensor is an error the context reports (LT_EINVAL
    at the next sync), with no read outside the weights: the pair contributes
    nothing and the other pairs are unaffected."""
    import importlib
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.Generator(np.random.PCG64(91 + T))
    L = synth.MoeLayer(rng, 512, 8, 256, 12, 12)
    rt, g, u, dn = _upload_layer(ctx, L)
    x = rng.normal(0, 1, (T, 512)).astype(np.float32)
    ids = rng.integers(0, 8, (T, 2)).astype(np.int32)
    ids[0, 1] = 99
    w = np.full((T, 2), 0.5, np.float32)
    out = empty(T * 512)
    ctx.moe_ffn(g, u, dn, 0, dev(x), T, dev(ids), dev(w), 2, out)
    with pytest.raises(pkg.LtError) as e:
        ctx.sync()
    assert e.value.status == 1
    ctx.sync()  # the error word was cleared
    got = host(out).reshape(T, 512)
    assert np.all(np.isfinite(got))
    if T > 1:  # tokens without the bad id match a clean run
        ok = ids.copy()
        ok[0, 1] = 0
        out2 = empty(T * 512)
        ctx.moe_ffn(g, u, dn, 0, dev(x), T, dev(ok), dev(w), 2, out2)
        np.testing.assert_array_equal(host(out2).reshape(T, 512)[1:], got[1:])
    for t_ in (rt, g, u, dn):
        t_.free()


@pytest.mark.parametrize("T,gt", [(1, 12), (1, 14), (1, 8), (3, 12)])
def test_moe_block_scaled_matches_ops(ctx, pkg, T, gt):
    """lt_moe_block_scaled (Gemma 4's MoE half) against the separate ops it
    replaces -- lt_norm_pair, lt_moe_route on the raw-scaled input, lt_moe_ffn on
    the weighted one: the same ids and weights bit for bit (the router input is
    norm_pair's arithmetic), outputs within f32 rounding of the expert kernels'
    different partial-sum grouping (one persistent launch at T = 1; at T = 3
    the ops themselves, bit for bit).  Q6_K and Q8_0 gate/up tiles of this
    shape exceed shared memory: the persistent kernel takes them in rounds."""
    import importlib
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.Generator(np.random.PCG64(2816 + T + gt))
    d, E, F, k = 2816, 32, 704, 8
    L = synth.MoeLayer(rng, d, E, F, gt, 8, fused=True)
    rt, g, u, dn = _upload_layer(ctx, L)
    x = rng.normal(0, 2, (T, d)).astype(np.float32)
    nw = dev(rng.uniform(0.5, 1.5, d).astype(np.float32))
    rs = dev(rng.uniform(0.5, 1.5, d).astype(np.float32))
    es = dev(rng.uniform(0.5, 2.0, E).astype(np.float32))
    gs = float(np.float32(1.0 / np.sqrt(d)))
    out, ids, w = empty(T * d), empty(T * k, "int32"), empty(T * k)
    ctx.profile(True)
    ctx.moe_block_scaled(rt, g, None, dn, 1, False, es, nw, rs, gs, 1e-6, dev(x), T, k, out, False, ids, w)
    ctx.sync()
    labels = ctx.profile_read()
    ctx.profile_reset()
    ctx.profile(False)
    assert ("moe_decode" in labels) == (T == 1), labels
    a, b = empty(T * d), empty(T * d)
    ctx.norm_pair(dev(x), nw, rs, gs, 1e-6, d, T, a, b)
    ids2, w2, out2 = empty(T * k, "int32"), empty(T * k), empty(T * d)
    ctx.moe_route(rt, b, T, k, False, es, ids2, w2)
    ctx.moe_ffn(g, None, dn, 1, a, T, ids2, w2, k, out2)
    np.testing.assert_array_equal(host(ids), host(ids2))
    np.testing.assert_array_equal(bits(host(w)), bits(host(w2)))
    if T == 1:
        assert rel_l2(host(out), host(out2)) < 1e-5
    else:
        np.testing.assert_array_equal(bits(host(out)), bits(host(out2)))
    for t_ in (rt, g, u, dn):
        if t_ is not None:
            t_.free()


@pytest.mark.parametrize("norm", [False, True])
def test_qmatvec_multi_matches_separate(ctx, pkg, norm):
    """lt_qmatvec_multi: three matrices of different types on one input in one
    launch, optionally normalising it first, bit for bit as lt_rmsnorm followed
    by three lt_qmatvec calls."""
    import importlib
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.Generator(np.random.PCG64(77 + int(norm)))
    d = 2816
    shapes = [(12, 4096), (14, 2048), (8, 2048)]
    mats = [synth.matrix(rng, t, r, d) for t, r in shapes]
    ts = [ctx.upload(m, t, r, d) for m, (t, r) in zip(mats, shapes)]
    x = dev(rng.normal(0, 1, d).astype(np.float32))
    nw = dev(rng.uniform(0.5, 1.5, d).astype(np.float32))
    ys = [empty(r) for _, r in shapes]
    ctx.qmatvec_multi(ts, x, ys, nw if norm else None, 1e-6)
    xn = empty(d)
    if norm:
        ctx.rmsnorm(x, nw, 1e-6, d, 1, xn)
    else:
        xn.copy_(x)
    for t, y in zip(ts, ys):
        ref = empty(t.rows if hasattr(t, "rows") else y.numel())
        ctx.qmatvec(t, xn, ref, 1)
        np.testing.assert_array_equal(bits(host(y)), bits(host(ref)))
    for t in ts:
        t.free()
