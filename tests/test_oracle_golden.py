"""The CPU oracle against the reference's known-answer tests and the golden fixtures.

Pins the oracle before it is trusted as the checker for the CUDA path.
"""
from __future__ import annotations

import math

import numpy as np
import pytest


def _bits(a: np.ndarray) -> list[int]:
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).reshape(-1).tolist()


def test_dequant_fixtures_bit_exact(oracle, golden):
    for case in golden["dequant"]:
        raw = np.frombuffer(bytes.fromhex(case["hex"]), dtype=np.uint8)
        out = oracle.dequant(raw, case["type"], 1, case["cols"])
        assert _bits(out) == case["expect"], case["name"]


def test_row_bytes_matches_types_table(oracle):
    # src/gguf/types.zig:154-160 and src/ops/math.zig:194-208
    assert oracle.row_bytes(oracle.Q8_0, 896) == 28 * 34
    assert oracle.row_bytes(oracle.Q4_K, 2048) == 8 * 144
    assert oracle.row_bytes(oracle.Q6_K, 2816) == 11 * 210
    assert oracle.row_bytes(oracle.F32, 5) == 20
    # src/gguf/types.zig:150-166 for the further formats
    assert oracle.row_bytes(oracle.Q5_0, 64) == 2 * 22
    assert oracle.row_bytes(oracle.Q5_1, 64) == 2 * 24
    assert oracle.row_bytes(oracle.IQ4_NL, 64) == 2 * 18
    assert oracle.row_bytes(oracle.Q5_K, 512) == 2 * 176
    assert oracle.row_bytes(oracle.Q3_K, 512) == 2 * 110
    assert oracle.row_bytes(99, 256) == 0  # unsupported type
    assert oracle.row_bytes(9, 256) == 0  # Q8_1 is an activation format, not a matrix type (math.zig:194-208)


def test_dot_q8_0_matches_dequant_dot(oracle, golden):
    c = golden["dot_q8_0"]
    raw = np.frombuffer(bytes.fromhex(c["hex"]), dtype=np.uint8)
    vec = np.array(c["vec"], dtype=np.float32)
    got = oracle.lib().orc_dot_q8_0(raw.ctypes.data, vec.ctypes.data, 64)
    assert abs(got - c["expect"]) <= c["tol"]


@pytest.mark.parametrize("key,fn", [("dot_q5_0", "orc_dot_q5_0"), ("dot_iq4_nl", "orc_dot_iq4_nl")])
def test_fused_dots_match_dequant_dot(oracle, golden, key, fn):
    """dequant.zig:716-758: dotQ5_0 / dotIQ4NL == dequant + scalar dot (1e-3)."""
    c = golden[key]
    raw = np.frombuffer(bytes.fromhex(c["hex"]), dtype=np.uint8)
    vec = np.array(c["vec"], dtype=np.float32)
    got = getattr(oracle.lib(), fn)(raw.ctypes.data, vec.ctypes.data, 64)
    assert abs(got - c["expect"]) <= c["tol"]


@pytest.mark.parametrize("t", [6, 20, 7, 13, 11])
def test_quant_matvec_paths(oracle, t):
    """quantMatvec (math.zig:133-171): Q5_0 and IQ4_NL rows go through their
    fused dots, the others through dequantRow + dotf32."""
    synth = pytest.importorskip("importlib").import_module("llmtoy-zig_b200.synth")
    rng = np.random.default_rng(t)
    cols = 512
    mat = synth.matrix(rng, t, 5, cols)
    vec = rng.normal(0, 1, cols).astype(np.float32)
    got = oracle.quant_matvec(mat, t, vec, 5, cols)
    rb = oracle.row_bytes(t, cols)
    for r in range(5):
        row = np.ascontiguousarray(mat.reshape(-1)[r * rb:(r + 1) * rb])
        if t in (6, 20):
            fn = oracle.lib().orc_dot_q5_0 if t == 6 else oracle.lib().orc_dot_iq4_nl
            want = fn(row.ctypes.data, vec.ctypes.data, cols)
        else:
            deq = np.ascontiguousarray(oracle.dequant(row, t, 1, cols)[0])
            want = oracle.lib().orc_dotf32(deq.ctypes.data, vec.ctypes.data, cols)
        assert np.float32(got[r]) == np.float32(want)


def test_q8_1_golden(oracle, golden):
    """quantizeQ8_1 bit-exact against the fixture (halves away from zero, zero
    blocks, random rows)."""
    for c in golden["q8_1"]:
        assert oracle.quantize_q8_1(c["x"]).hex() == c["hex"], c["name"]


def test_q8_1_roundtrip_within_bound(oracle):
    """dequant.zig:768-794: |dequant(quantize(x)) - x| <= amax/127 (+1e-5), the
    inputs drawn from DefaultPrng(0xC0FFEE) as the reference's test does."""
    r = oracle.Rng(0xC0FFEE)
    x = np.array([(r.float() - 0.5) * 4.0 for _ in range(128)], np.float32)
    dec = oracle.dequant_q8_1(oracle.quantize_q8_1(x), 128)
    for b in range(4):
        blk = x[32 * b:32 * b + 32]
        assert np.all(np.abs(dec[32 * b:32 * b + 32] - blk) <= np.abs(blk).max() / 127.0 + 1e-5)


def test_q8_1_sum_term(oracle):
    """dequant.zig:796-815: the stored s equals d * sum(q) within 1e-2."""
    r = oracle.Rng(7)
    x = np.array([(r.float() - 0.5) * 3.0 for _ in range(32)], np.float32)
    b = np.frombuffer(oracle.quantize_q8_1(x), np.uint8)
    d, s = (float(np.frombuffer(b[i:i + 2].tobytes(), np.float16)[0]) for i in (0, 2))
    assert abs(d * int(b[4:].view(np.int8).astype(np.int64).sum()) - s) <= 1e-2


def test_q8_1_x4_roundtrip(oracle):
    """dequant.zig:817-829: pack / unpack of one x4 group is byte-exact; a
    partial last group is zero-padded."""
    rng = np.random.default_rng(11)
    basic = rng.integers(0, 256, 4 * 36, dtype=np.uint8)
    x4 = np.zeros(144, np.uint8)
    oracle.lib().orc_pack_q8_1_x4(basic.ctypes.data, 4, x4.ctypes.data)
    back = np.zeros(144, np.uint8)
    oracle.lib().orc_unpack_q8_1_x4(x4.ctypes.data, 1, back.ctypes.data)
    assert back.tobytes() == basic.tobytes()
    x4 = np.full(288, 7, np.uint8)
    oracle.lib().orc_pack_q8_1_x4(basic.ctypes.data, 3, x4.ctypes.data)
    assert x4[12:16].tolist() == [0] * 4 and x4[16 + 96:144].tolist() == [0] * 32 and x4[144:].tolist() == [7] * 144


def test_quant_matvec_f32_equals_matvec(oracle, golden):
    c = golden["misc"]["quant_matvec_f32"]
    mat = np.array(c["mat"], dtype=np.float32)
    vec = np.array(c["vec"], dtype=np.float32)
    got = oracle.quant_matvec(mat.view(np.uint8), oracle.F32, vec, c["rows"], c["cols"])
    want = np.empty(c["rows"], dtype=np.float32)
    oracle.lib().orc_matvec(want.ctypes.data, mat.ctypes.data, vec.ctypes.data, c["rows"], c["cols"])
    np.testing.assert_allclose(got, want, atol=c["tol"])


def test_rmsnorm_softmax_silu(oracle, golden):
    m = golden["misc"]
    x = np.array(m["rmsnorm"]["x"], dtype=np.float32)
    w = np.array(m["rmsnorm"]["w"], dtype=np.float32)
    out = np.empty_like(x)
    oracle.lib().orc_rmsnorm(out.ctypes.data, x.ctypes.data, w.ctypes.data, 4, m["rmsnorm"]["eps"])
    np.testing.assert_allclose(out, m["rmsnorm"]["expect"], atol=m["rmsnorm"]["tol"])
    for c in m["softmax"]:
        s = np.array(c["x"], dtype=np.float32)
        oracle.lib().orc_softmax(s.ctypes.data, s.size)
        assert abs(float(s.sum()) - 1.0) <= c["tol"]
        assert s[2] > s[1] > s[0]
    assert abs(oracle.lib().orc_silu(0.0)) < 1e-6
    assert 0.0 < oracle.lib().orc_silu(1.0) < 1.0


def test_dotf32_tail_lengths(oracle, golden):
    for n in golden["misc"]["dotf32_lengths"]:
        a = np.array([(i + 1) * 0.5 for i in range(n)], dtype=np.float32)
        b = np.array([(n - i) * 0.3 for i in range(n)], dtype=np.float32)
        exp = np.float32(0)
        for i in range(n):
            exp = np.float32(exp + a[i] * b[i])
        assert abs(oracle.dotf32(a, b) - exp) <= 1e-4


def test_topk_stable_ties(oracle, golden):
    c = golden["router"]["topk_ties"]
    ids, _ = oracle.topk_stable(c["scores"], c["k"])
    assert ids.tolist() == c["expect"]


def test_online_softmax_denominator(oracle, golden):
    c = golden["router"]["online_denominator"]
    s = np.array(c["scores"], dtype=np.float32)
    _, (mx, es) = oracle.topk_stable(s, c["k"])
    assert mx == s.max()
    ref = np.float32(0)
    for v in s:
        ref = np.float32(ref + np.float32(math.exp(float(v - s.max()))))
    assert abs(es - ref) <= 1e-6 * ref


def test_softmax_topk_matches_softmax_then_topk(oracle, golden):
    c = golden["router"]["softmax_topk"]
    ref = np.array(c["scores"], dtype=np.float32)
    got = ref.copy()
    oracle.lib().orc_softmax(ref.ctypes.data, ref.size)
    ref_idx = np.empty(c["k"], dtype=np.uint32)
    oracle.lib().orc_moe_topk(ref.ctypes.data, ref.size, ref_idx.ctypes.data, c["k"])
    got_idx = np.empty(c["k"], dtype=np.uint32)
    oracle.lib().orc_softmax_topk(got.ctypes.data, got.size, got_idx.ctypes.data, c["k"])
    assert got_idx.tolist() == ref_idx.tolist()
    np.testing.assert_allclose(got[got_idx], ref[ref_idx], atol=1e-6)


def test_topk_matvec_matches_materialized(oracle, golden):
    c = golden["router"]["topk_matvec_6x5"]
    w = np.array(c["weights"], dtype=np.float32)
    v = np.array(c["vec"], dtype=np.float32)
    logits = np.empty(c["rows"], dtype=np.float32)
    oracle.lib().orc_matvec(logits.ctypes.data, w.ctypes.data, v.ctypes.data, c["rows"], c["cols"])
    ref = logits.copy()
    ref_idx = np.empty(c["k"], dtype=np.uint32)
    oracle.lib().orc_softmax_topk(ref.ctypes.data, ref.size, ref_idx.ctypes.data, c["k"])
    got_idx = np.empty(c["k"], dtype=np.uint32)
    got_sc = np.empty(c["k"], dtype=np.float32)
    st = oracle.lib().orc_topk_matvec_f32(w.ctypes.data, v.ctypes.data, c["rows"], c["cols"], got_idx.ctypes.data,
                                          got_sc.ctypes.data, c["k"])
    assert got_idx.tolist() == ref_idx.tolist()
    np.testing.assert_allclose(got_sc, logits[ref_idx], atol=1e-6)
    np.testing.assert_allclose(np.exp(got_sc - st.max) / st.exp_sum, ref[ref_idx], atol=1e-6)


def test_topk_matvec_parallel_matches_serial(oracle, golden):
    c = golden["router"]["par_37x33"]
    w = np.array(c["weights"], dtype=np.float32)
    v = np.array(c["vec"], dtype=np.float32)
    k = c["k"]
    ri, rs = np.empty(k, np.uint32), np.empty(k, np.float32)
    gi, gs = np.empty(k, np.uint32), np.empty(k, np.float32)
    L = oracle.lib()
    st_ref = L.orc_topk_matvec_f32(w.ctypes.data, v.ctypes.data, 37, 33, ri.ctypes.data, rs.ctypes.data, k)
    with oracle.Pool(c["threads"]) as p:
        st_got = L.orc_topk_matvec_f32_par(w.ctypes.data, v.ctypes.data, 37, 33, gi.ctypes.data, gs.ctypes.data, k,
                                           p.ptr)
    assert st_ref.max == st_got.max
    assert abs(st_ref.exp_sum - st_got.exp_sum) <= 1e-6 * st_ref.exp_sum
    assert ri.tolist() == gi.tolist()
    np.testing.assert_allclose(rs, gs, atol=1e-6)


def test_router_streamed_matches_materialized(oracle, golden):
    c = golden["router"]["streamed_5x4"]
    w = np.array(c["weights"], dtype=np.float32).reshape(c["rows"], c["cols"])
    v = np.array(c["vec"], dtype=np.float32)
    ref = oracle.quant_matvec(w.view(np.uint8), oracle.F32, v, c["rows"], c["cols"])
    ref_idx = np.empty(c["k"], np.uint32)
    oracle.lib().orc_softmax_topk(ref.ctypes.data, ref.size, ref_idx.ctypes.data, c["k"])
    with oracle.Pool(4) as p:
        ids, probs = oracle.router_topk_softmax(w, v, c["k"], p)
    assert ids.tolist() == ref_idx.tolist()
    np.testing.assert_allclose(probs, ref[ref_idx], atol=1e-6)


def test_gpu_router_closed_form_on_oracle(oracle, golden):
    c = golden["router"]["gpu_router_closed_form"]
    w = np.array(c["weights"], dtype=np.float32).reshape(c["rows"], c["cols"])
    ids, probs = oracle.router_topk_softmax(w, np.array(c["vec"], np.float32), c["k"])
    assert ids.tolist() == c["expect_ids"]
    scaled = np.array(c["expert_scale"], np.float32)[ids] * probs
    np.testing.assert_allclose(scaled, c["expect_w"], atol=c["tol"])


def test_greedy_lowest_index(oracle, golden):
    a = golden["misc"]["argmax"]
    assert oracle.greedy(a[0]["values"]) == a[0]["expect"]
    v = np.full(a[1]["n"], -4.0, np.float32)
    v[a[1]["peaks"]] = 9.0
    assert oracle.greedy(v) == a[1]["expect"]


@pytest.mark.parametrize("t", [12, 14, 8, 6, 7, 11, 13, 20])
def test_golden_regenerates_identically(t, golden):
    """The committed fixture equals what gen_golden.py derives (no drift)."""
    import importlib.util
    from pathlib import Path
    spec = importlib.util.spec_from_file_location("gen_golden", Path(__file__).parent / "golden" / "gen_golden.py")
    g = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(g)
    fresh = {c["name"]: c for c in g.dequant_cases()}
    for c in golden["dequant"]:
        if c["type"] == t:
            assert fresh[c["name"]]["expect"] == c["expect"]
