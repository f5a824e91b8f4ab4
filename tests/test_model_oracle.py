"""The oracle's decoder pieces against the reference's own unit tests
(src/ops/rope.zig and src/ops/attn.zig test blocks, src/model/forward.zig
"deterministic" test), plus the host library's exported symbols."""
from __future__ import annotations

import ctypes
import importlib
import subprocess

import numpy as np
import pytest

from conftest import REPO


def rope(orc, v, pos, theta, neox=False):
    a = np.ascontiguousarray(v, dtype=np.float32).copy()
    orc.lib().orc_rope(a.ctypes.data, a.size, pos, theta, int(neox))
    return a


def sdp(orc, q, ks, vs, scale):
    q, ks, vs = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, ks, vs))
    out = np.empty(q.size, np.float32)
    orc.lib().orc_sdp_attn(out.ctypes.data, q.ctypes.data, ks.ctypes.data, vs.ctypes.data, ks.size // q.size,
                           q.size, scale)
    return out


@pytest.mark.parametrize("neox", [False, True])
def test_rope_pos0_identity(oracle, neox):  # rope.zig "pos=0 is identity"
    v = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    np.testing.assert_allclose(rope(oracle, v, 0, 10000.0, neox), v, atol=1e-6)


@pytest.mark.parametrize("neox", [False, True])
def test_rope_preserves_pair_magnitude(oracle, neox):  # rope.zig "preserves vector magnitude"
    v = np.array([3.0, 4.0, 1.0, 0.0], np.float32)
    r = rope(oracle, v, 7, 10000.0, neox)
    pairs = [(0, 1), (2, 3)] if not neox else [(0, 2), (1, 3)]
    for i, j in pairs:
        assert abs((v[i] ** 2 + v[j] ** 2) - (r[i] ** 2 + r[j] ** 2)) < 1e-5


def test_rope_same_pos_same_rotation(oracle):  # rope.zig "same pos gives same rotation"
    v = np.array([1.0, 0.0, 0.0, 1.0], np.float32)
    np.testing.assert_array_equal(rope(oracle, v, 5, 10000.0), rope(oracle, v, 5, 10000.0))


def test_sdp_single_position_returns_value(oracle):  # attn.zig "seq_len=1 -> output equals value"
    out = sdp(oracle, [1, 0, 0, 0], [1, 0, 0, 0], [3, 1, 4, 1], 1.0)
    np.testing.assert_allclose(out, [3, 1, 4, 1], atol=1e-5)


def test_sdp_equal_keys_average(oracle):  # attn.zig "equal keys -> average of values"
    out = sdp(oracle, [1, 0], [1, 0, 1, 0], [0, 0, 2, 4], 1.0)
    np.testing.assert_allclose(out, [1, 2], atol=1e-5)


def test_sdp_extreme_scores(oracle):  # attn.zig "extreme score difference"
    out = sdp(oracle, [10], [-10, 10], [99, 7], 1.0)
    np.testing.assert_allclose(out, [7], atol=1e-3)


def _small(synth, moe: bool, **kw):
    rng = np.random.default_rng(5)
    if moe:
        return synth.DecoderModel(rng, 2, 256, 4, 2, 64, 500, n_experts=8, k=2, d_expert=256, lm_type=14,
                                  qk_norm=True, rope_neox=True, norm_topk=True, norms_random=True, **kw)
    return synth.DecoderModel(rng, 2, 256, 4, 2, 64, 500, d_ffn=512, qkv_bias=True, norms_random=True, **kw)


@pytest.mark.parametrize("moe", [False, True])
def test_model_step_deterministic(oracle, moe):  # forward.zig "deterministic -- same input gives same output"
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    m = _small(synth, moe)
    a = oracle.OracleDecoder(m, 32).generate([3, 1, 4], 4)
    b = oracle.OracleDecoder(m, 32).generate([3, 1, 4], 4)
    assert a[0] == b[0]
    for x, y in zip(a[1], b[1]):
        np.testing.assert_array_equal(x, y)
    assert all(0 <= t < 500 for t in a[0])


def test_model_step_single_layer_matches_manual(oracle):
    """One dense layer at position 0 recomputed from the oracle's primitives:
    with one position, attention returns v, so x1 = x + wo.v + ffn."""
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.default_rng(11)
    m = synth.DecoderModel(rng, 1, 256, 4, 2, 64, 300, d_ffn=256, norms_random=True)
    L = m.layers[0]
    x = oracle.dequant(m.token_emb, m.emb_type, m.vocab, 256)[7]
    lib = oracle.lib()

    def norm(v, w):
        o = np.empty_like(v)
        lib.orc_rmsnorm(o.ctypes.data, np.ascontiguousarray(v).ctypes.data, w.ctypes.data, v.size, 1e-6)
        return o

    xb = norm(x, L.attn_norm)
    v = oracle.quant_matvec(L.wv, L.attn_type, xb, 128, 256)
    att = np.concatenate([v[(h // 2) * 64:(h // 2 + 1) * 64] for h in range(4)])
    x1 = (x + oracle.quant_matvec(L.wo, L.attn_type, att, 256, 256)).astype(np.float32)
    xb = norm(x1, L.ffn_norm)
    g = oracle.quant_matvec(L.ffn_gate, L.ffn_type, xb, 256, 256)
    u = oracle.quant_matvec(L.ffn_up, L.ffn_type, xb, 256, 256)
    h = np.array([lib.orc_silu(float(t)) for t in g], np.float32) * u
    x2 = (x1 + oracle.quant_matvec(L.ffn_down, L.ffn_type, h, 256, 256)).astype(np.float32)
    ref = oracle.quant_matvec(m.lm_head, m.lm_type, norm(x2, m.out_norm), 300, 256)
    got = oracle.OracleDecoder(m, 8).step(7, 0)
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-4)


def test_host_library_exports():
    """libllmtoy_host.so exports every lth_* function decoder.h declares."""
    lib = REPO / "llmtoy-zig_b200" / "libllmtoy_host.so"
    if not lib.exists():
        subprocess.run(["python", str(REPO / "llmtoy-zig_b200" / "build.py")], check=True)
    names = [ln.split("(")[0].split()[-1].lstrip("*") for ln in (REPO / "llmtoy-zig_b200" / "host" / "decoder.h")
             .read_text().splitlines() if ln.startswith(("lt_status lth_", "void lth_", "const float *lth_", "int lth_"))]
    assert len(names) == 12
    L = ctypes.CDLL(str(lib))
    for n in names:
        assert hasattr(L, n), n
