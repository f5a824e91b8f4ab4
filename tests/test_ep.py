"""Expert-parallel MoE over gloo ranks on the CPU: the exchange logic of
ExpertParallelMoE (dispatch order, split sizes, the return trip, the
combine) with the CPU ops of ep_cpu_ops.  Every rank checks its tokens
against orc_moe_layer run over the same tokens on one device; the result
must be identical bit for bit, because sharding only moves rows.
"""
from __future__ import annotations

import importlib
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import REPO

CASES = {
    # name: (world, E, k, T per rank, gate type, down type, fused gate_up, norm_w, expert_scale, skew)
    "q4k_w2": (2, 8, 2, [5, 3], 12, 12, False, False, False, False),
    "q8_block_w2": (2, 8, 3, [4, 6], 8, 8, True, True, True, False),
    "ragged_empty_rank_w2": (2, 8, 2, [0, 4], 12, 14, False, True, False, False),
    "skew_w4": (4, 8, 2, [3, 2, 4, 1], 12, 12, False, False, False, True),
}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def build_case(name: str, rank: int):
    """The layer (full and this rank's slice) and every rank's tokens, from a seed."""
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    world, E, k, Ts, gt, dt, fused, normw, escale, skew = CASES[name]
    d, F = 256, 256
    rng = np.random.default_rng(1234)
    layer = synth.MoeLayer(rng, d_model=d, n_experts=E, d_expert=F, gate_type=gt, down_type=dt, fused=fused)
    xs = [synth.hidden(rng, T, d) for T in Ts]
    if skew:  # every token picks experts 0..k-1, all on rank 0
        layer.router[:k] += 0.05
        xs = [(x + 1.0).astype(np.float32) for x in xs]
    nw = rng.uniform(0.5, 1.5, d).astype(np.float32) if normw else None
    es = rng.uniform(0.5, 1.5, E).astype(np.float32) if escale else None
    return layer, xs, nw, es, k, world


def _rank_main(rank: int, name: str, port: int):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    world = CASES[name][0]
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        import oracle_lib as orc
        from ep_cpu_ops import CpuOps
        ep = importlib.import_module("llmtoy-zig_b200.ep")
        layer, xs, nw, es, k, _ = build_case(name, rank)
        E, F, d = layer.n_experts, layer.d_expert, layer.d_model
        lo, hi = ep.expert_range(E, rank, world)
        gate = layer.gate.reshape(E, -1)[lo:hi].reshape(-1)
        up = None if layer.up is None else layer.up.reshape(E, -1)[lo:hi].reshape(-1)
        down = layer.down.reshape(E, -1)[lo:hi].reshape(-1)
        el = ep.EPLayer(router=layer.router, gate=gate, up=up, down=down, n_experts=E, d_model=d,
                        norm_topk=True, expert_scale=es, norm_w=nw)
        moe = ep.ExpertParallelMoE(CpuOps(F, layer.gate_type, layer.down_type), k)
        assert moe.world == world and moe.rank == rank
        x = xs[rank]
        out = moe.forward(el, torch.from_numpy(x)).numpy()

        # the single-device oracle over this rank's tokens
        T = x.shape[0]
        if nw is not None:
            xn = np.empty_like(x)
            for t in range(T):
                orc.lib().orc_rmsnorm(xn[t].ctypes.data, x[t].ctypes.data, nw.ctypes.data, d, 1e-6)
        else:
            xn = x
        if T:
            ref, ids, _ = orc.moe_layer(layer, xn, k, True, expert_scale=es)
            if nw is not None:
                ref = (x + ref).astype(np.float32)
        else:
            ref, ids = np.empty((0, d), np.float32), np.empty((0, k), np.uint32)
        assert out.shape == ref.shape
        np.testing.assert_array_equal(out.view(np.uint32), ref.view(np.uint32))
        sent = moe.last_stats["sent_pairs"]
        assert sent == [int(((ids // (E // world)) == r).sum()) for r in range(world)]
        # every pair is computed exactly once across the ranks
        got = torch.tensor([moe.last_stats["received_pairs"]])
        dist.all_reduce(got)
        assert int(got) == k * sum(CASES[name][3])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name", list(CASES))
def test_ep_gloo_matches_single_device(name):
    world = CASES[name][0]
    mp.start_processes(_rank_main, args=(name, _free_port()), nprocs=world, join=True, start_method="spawn")


def test_ep_cpu_dispatch_is_stable_rank_order():
    from ep_cpu_ops import CpuOps
    ids = torch.tensor([[5, 1], [0, 7], [2, 3], [6, 4]], dtype=torch.int32)
    counts, tok, loc, pos = CpuOps(256, 12, 12).dispatch(ids, 4, 2, 8, 2)
    assert counts.tolist() == [4, 4]
    assert tok.tolist() == [0, 1, 2, 2, 0, 1, 3, 3]
    assert loc.tolist() == [1, 0, 2, 3, 1, 3, 2, 0]
    flat = ids.reshape(-1)
    for i in range(8):  # pair i lands at pos[i] with its own token and local id
        assert tok[pos[i]] == i // 2 and loc[pos[i]] + 4 * (flat[i] // 4) == flat[i]


def test_expert_range():
    ep = importlib.import_module("llmtoy-zig_b200.ep")
    assert ep.expert_range(128, 3, 8) == (48, 64)
    with pytest.raises(ValueError):
        ep.expert_range(128, 0, 3)
