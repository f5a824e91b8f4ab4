"""lt_moe_ffn_noalloc: the MoE FFN for callers that cannot allocate device memory.

Such a caller owns every buffer it passes (weights, activations, ids, output)
and cannot call cudaMalloc; the entry point keeps its intermediates in a fixed
device array inside the library.  This checks it through the C ABI against the
allocating entry point lt_moe_ffn on the same inputs, twice in a row (the
shared array keeps the first call's contents, which must not leak into the
second), once on the one-token path and once on the grouped multi-token path.
The file name sorts last so a run that stops at the first failure has already
run every other test.
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
