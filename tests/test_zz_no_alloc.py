"""lt_moe_ffn_noalloc: the MoE FFN for callers that cannot allocate device memory.

Such a caller owns every buffer it passes (weights, activations, ids, output)
and cannot call cudaMalloc; the entry point keeps its intermediates in a fixed
device array inside the library.  This checks it through the C ABI against the
allocating entry point lt_moe_ffn on the same inputs, twice in a row (the
shared array keeps the first call's contents, which must not leak into the
second), once on the one-token path and once on the grouped multi-token path.
The file name sorts last so a run that stops at the first failure has already
run every other test.

A second case checks that a fault the kernels detect on the device (an expert
id past n_experts) is reported by lt_noalloc_status on both paths, and that the
next good call starts from a clear error word.
"""
from __future__ import annotations

import ctypes
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-4  # the MoE tolerance of test_gpu_parity.py


def test_moe_ffn_noalloc_matches_moe_ffn(ctx, pkg):
    import torch

    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.Generator(np.random.PCG64(0x5EED))
    d, E, F, k = 2048, 16, 768, 8
    layer = synth.MoeLayer(rng, d, E, F)
    # the caller's own device buffers holding the GGUF bytes
    gate_d = torch.from_numpy(layer.gate.reshape(-1)).cuda()
    up_d = torch.from_numpy(layer.up.reshape(-1)).cuda()
    down_d = torch.from_numpy(layer.down.reshape(-1)).cuda()
    # the allocating path, for comparison
    g = ctx.upload(layer.gate, pkg.Q4_K, F, d, n_experts=E)
    u = ctx.upload(layer.up, pkg.Q4_K, F, d, n_experts=E)
    dn = ctx.upload(layer.down, pkg.Q4_K, d, F, n_experts=E)
    lib = pkg.load_library()
    stream = torch.cuda.current_stream().cuda_stream

    for ntok in (1, 5):  # two calls in a row: direct path, then the grouped path
        x = torch.from_numpy(rng.normal(0, 1, size=(ntok, d)).astype(np.float32)).cuda()
        ids = torch.from_numpy(np.stack([rng.choice(E, size=k, replace=False) for _ in range(ntok)])
                               .astype(np.int32)).cuda()
        w = torch.from_numpy(rng.uniform(0.01, 0.3, size=(ntok, k)).astype(np.float32)).cuda()
        out_ref = torch.empty(ntok, d, device="cuda")
        ctx.moe_ffn(g, u, dn, pkg.ACT_SILU, x, ntok, ids, w, k, out_ref)
        out = torch.full((ntok, d), float("nan"), device="cuda")
        st = lib.lt_moe_ffn_noalloc(ctypes.c_void_p(stream), gate_d.data_ptr(), up_d.data_ptr(), down_d.data_ptr(),
                                    pkg.Q4_K, pkg.Q4_K, E, d, F, pkg.ACT_SILU, x.data_ptr(), ntok, ids.data_ptr(),
                                    w.data_ptr(), k, out.data_ptr())
        assert st == 0, pkg.STATUS.get(st, st)
        torch.cuda.synchronize()
        ref, got = out_ref.cpu().numpy(), out.cpu().numpy()
        rel = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
        assert rel < REL_L2_TOL, (ntok, rel)

    # a request beyond the fixed capacity is refused, not truncated
    big = 4096
    x = torch.zeros(big, d, device="cuda")
    ids = torch.zeros(big, k, dtype=torch.int32, device="cuda")
    w = torch.zeros(big, k, device="cuda")
    out = torch.empty(big, d, device="cuda")
    st = lib.lt_moe_ffn_noalloc(ctypes.c_void_p(stream), gate_d.data_ptr(), up_d.data_ptr(), down_d.data_ptr(),
                                pkg.Q4_K, pkg.Q4_K, E, d, F, pkg.ACT_SILU, x.data_ptr(), big, ids.data_ptr(),
                                w.data_ptr(), k, out.data_ptr())
    assert st == 1  # LT_EINVAL
    for t in (g, u, dn):
        t.free()


def test_moe_ffn_noalloc_reports_bad_expert_id(ctx, pkg):
    """An id >= n_experts is a caller error the kernels find on the device:
    the call itself returns LT_OK (it is asynchronous), lt_noalloc_status then
    returns LT_EINVAL and clears the word, and the next good call reports
    LT_OK with the other tokens' outputs unchanged."""
    import torch

    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.Generator(np.random.PCG64(0xBAD1D))
    d, E, F, k = 2048, 8, 768, 2
    layer = synth.MoeLayer(rng, d, E, F)
    gate_d = torch.from_numpy(layer.gate.reshape(-1)).cuda()
    up_d = torch.from_numpy(layer.up.reshape(-1)).cuda()
    down_d = torch.from_numpy(layer.down.reshape(-1)).cuda()
    lib = pkg.load_library()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def call(x, ids, w, out):
        ntok = x.shape[0]
        return lib.lt_moe_ffn_noalloc(stream, gate_d.data_ptr(), up_d.data_ptr(), down_d.data_ptr(), pkg.Q4_K,
                                      pkg.Q4_K, E, d, F, pkg.ACT_SILU, x.data_ptr(), ntok, ids.data_ptr(),
                                      w.data_ptr(), k, out.data_ptr())

    assert lib.lt_noalloc_status(stream) == 0
    for ntok in (1, 4):  # the one-token path, then the grouped path
        x = torch.from_numpy(rng.normal(0, 1, size=(ntok, d)).astype(np.float32)).cuda()
        good = np.stack([rng.choice(E, size=k, replace=False) for _ in range(ntok)]).astype(np.int32)
        w = torch.from_numpy(rng.uniform(0.1, 0.5, size=(ntok, k)).astype(np.float32)).cuda()
        ref = torch.empty(ntok, d, device="cuda")
        assert call(x, torch.from_numpy(good).cuda(), w, ref) == 0
        assert lib.lt_noalloc_status(stream) == 0
        bad = good.copy()
        bad[ntok - 1, 1] = E + 3  # one pair of the last token names no expert
        out = torch.empty(ntok, d, device="cuda")
        assert call(x, torch.from_numpy(bad).cuda(), w, out) == 0
        assert lib.lt_noalloc_status(stream) == 1  # LT_EINVAL
        assert lib.lt_noalloc_status(stream) == 0  # read and cleared
        if ntok > 1:  # the grouped path skips the bad pair: the other tokens are untouched
            a, b = out[:ntok - 1].cpu().numpy(), ref[:ntok - 1].cpu().numpy()
            assert float(np.linalg.norm(a - b) / np.linalg.norm(b)) < 1e-6
        again = torch.empty(ntok, d, device="cuda")
        assert call(x, torch.from_numpy(good).cuda(), w, again) == 0
        assert lib.lt_noalloc_status(stream) == 0
        np.testing.assert_array_equal(again.cpu().numpy(), ref.cpu().numpy())
