"""The further GGUF formats (Q5_0, Q5_1, Q5_K, Q3_K, IQ4_NL; src/quant/dequant.zig:
92-134,196-217,307-506,615-660) and the Q8_1 activation blocks (:508-613) on
the GPU against the oracle.

Bars as for Q4_K/Q6_K/Q8_0: dequantised values and embedding rows bit-exact;
matvecs max|d|/max|ref| < 1e-4; MoE layer outputs rel-L2 < 1e-4 with router ids
exact; Q8_1 blocks byte-exact.
"""
from __future__ import annotations

import importlib

import numpy as np
import pytest

from test_gpu_parity import MATVEC_TOL, bits, dev, empty, host, max_rel, _check_moe

pytestmark = pytest.mark.gpu

Q5_0, Q5_1, Q3_K, Q5_K, IQ4_NL = 6, 7, 11, 13, 20
NEW = [Q5_0, Q5_1, Q3_K, Q5_K, IQ4_NL]


def _synth():
    return importlib.import_module("llmtoy-zig_b200.synth")


def _cols(t, wide=False):
    if t in (Q3_K, Q5_K):
        return 2816 if wide else 2048
    return 2080 if wide else 2048  # 65 blocks: the last 8-block item holds one


@pytest.mark.parametrize("t", NEW)
@pytest.mark.parametrize("wide", [False, True])
def test_dequant_bit_exact(ctx, oracle, t, wide):
    rng = np.random.Generator(np.random.PCG64(300 + t))
    rows, cols = 37, _cols(t, wide)
    mat = _synth().matrix(rng, t, rows, cols)
    w = ctx.upload(mat, t, rows, cols)
    out = empty(rows * cols)
    ctx.dequant(w, 0, rows, out)
    ref = oracle.dequant(mat, t, rows, cols)
    np.testing.assert_array_equal(bits(host(out)), bits(ref.reshape(-1)))
    w.free()


@pytest.mark.parametrize("t", NEW)
@pytest.mark.parametrize("wide", [False, True])
@pytest.mark.parametrize("ntok", [1, 3, 6])
def test_qmatvec_vs_oracle(ctx, oracle, t, wide, ntok):
    rng = np.random.Generator(np.random.PCG64(400 + t + ntok))
    rows, cols = 301, _cols(t, wide)
    mat = _synth().matrix(rng, t, rows, cols)
    x = rng.normal(0, 1, size=(ntok, cols)).astype(np.float32)
    w = ctx.upload(mat, t, rows, cols)
    y = empty(ntok * rows)
    ctx.qmatvec(w, dev(x), y, ntok)
    got = host(y).reshape(ntok, rows)
    for i in range(ntok):
        assert max_rel(got[i], oracle.quant_matvec(mat, t, x[i], rows, cols)) < MATVEC_TOL, (t, i)
    w.free()


@pytest.mark.parametrize("t", NEW)
def test_embed_bit_exact(ctx, oracle, t):
    rng = np.random.Generator(np.random.PCG64(500 + t))
    cols = _cols(t)
    emb = _synth().matrix(rng, t, 50, cols)
    et = ctx.upload(emb, t, 50, cols)
    out = empty(cols)
    toks = dev(np.array([49, 3], np.int32))
    for p, tok in enumerate([49, 3]):
        ctx.embed(et, toks, dev(np.array([p], np.int32)), out)
        np.testing.assert_array_equal(bits(host(out)), bits(oracle.dequant(emb[tok], t, 1, cols)[0]))
    et.free()


@pytest.mark.parametrize("gate_type,down_type,d,F,E,k,fused,act", [
    (Q5_K, Q3_K, 2048, 768, 16, 8, False, 0),
    (IQ4_NL, Q5_0, 2816, 704, 16, 8, True, 1),   # Gemma-like fused gate_up, GELU
    (Q5_1, Q5_1, 1024, 512, 8, 2, False, 0),
    (Q3_K, Q5_K, 2048, 512, 24, 6, False, 0),
])
@pytest.mark.parametrize("T", [1, 5])
def test_moe_vs_oracle(ctx, oracle, pool, gate_type, down_type, d, F, E, k, fused, act, T):
    rng = np.random.Generator(np.random.PCG64(600 + d + F + E + k))
    L = _synth().MoeLayer(rng, d, E, F, gate_type, down_type, fused)
    x = rng.normal(0, 1, size=(T, d)).astype(np.float32)
    _check_moe(ctx, oracle, pool, L, x, k, True, act)


def test_q8_1_golden(ctx, golden):
    for c in golden["q8_1"]:
        x = np.array(c["x"], np.float32)
        out = empty(x.size // 32 * 36, "uint8")
        ctx.quantize_q8_1(dev(x), x.size, out)
        assert host(out).tobytes().hex() == c["hex"], c["name"]


@pytest.mark.parametrize("n", [32, 96, 4096, 4128])
def test_q8_1_vs_oracle(ctx, oracle, n):
    rng = np.random.Generator(np.random.PCG64(n))
    x = (rng.normal(0, 2, n) * rng.choice([1e-3, 1.0, 30.0], n)).astype(np.float32)
    x[:32] = 0.0  # an all-zero block
    ref = oracle.quantize_q8_1(x)
    out = empty(n // 32 * 36, "uint8")
    ctx.quantize_q8_1(dev(x), n, out)
    assert host(out).tobytes() == ref
    # the x4 layout equals packQ8_1_x4 of the basic blocks
    nb = n // 32
    x4 = empty((nb + 3) // 4 * 144, "uint8")
    ctx.quantize_q8_1(dev(x), n, x4, x4=True)
    want = np.zeros((nb + 3) // 4 * 144, np.uint8)
    basic = np.frombuffer(ref, np.uint8).copy()
    oracle.lib().orc_pack_q8_1_x4(basic.ctypes.data, nb, want.ctypes.data)
    assert host(x4).tobytes() == want.tobytes()
    # dequant from either layout
    for q, flag in ((out, False), (x4, True)):
        y = empty(n)
        ctx.dequant_q8_1(q, n, y, x4=flag)
        np.testing.assert_array_equal(bits(host(y)), bits(oracle.dequant_q8_1(ref, n)))


def test_unsupported_type_rejected(ctx, pkg):
    with pytest.raises(pkg.LtError) as e:
        ctx.upload(np.zeros(18 * 2, np.uint8), 2, 1, 64)  # Q4_0: not in rowBytes / dequantRow
    assert e.value.status == 2
