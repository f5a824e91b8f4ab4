"""Failure detection of the expert-parallel layer over gloo ranks on the CPU:
a rank that leaves between steps, a rank that is late, and a rank that stops
joining the exchanges when no heartbeat is attached.  Each survivor must end
with an error in bounded time, never hang, and must learn of a departed rank
before it issues any exchange of the next step (the heartbeat) or from the
process group's short timeout (no heartbeat).

The reference runs on one process and has no such failure mode; its
counterpart is the CPU fallback on a device error
(src/model/gemma4/forward.zig:456-480).
"""
from __future__ import annotations

import datetime
import importlib
import json
import os
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from test_ep import _free_port, build_case


def _layer(rank: int, world: int):
    from ep_cpu_ops import CpuOps
    ep = importlib.import_module("llmtoy-zig_b200.ep")
    layer, xs, nw, es, k, _ = build_case("q4k_w2", rank)
    E, F, d = layer.n_experts, layer.d_expert, layer.d_model
    lo, hi = ep.expert_range(E, rank, world)
    el = ep.EPLayer(router=layer.router, gate=layer.gate.reshape(E, -1)[lo:hi].reshape(-1),
                    up=layer.up.reshape(E, -1)[lo:hi].reshape(-1), down=layer.down.reshape(E, -1)[lo:hi].reshape(-1),
                    n_experts=E, d_model=d, norm_topk=True)
    return ep, el, torch.from_numpy(xs[rank]), CpuOps(F, layer.gate_type, layer.down_type), k


def _rank_main(rank: int, scenario: str, port: int, out_dir: str):
    world = 2
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=30))
    pg_timeout = datetime.timedelta(seconds=3)
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world, timeout=pg_timeout)
    result = {"rank": rank}
    try:
        ep, el, x, ops, k = _layer(rank, world)
        hb = None if scenario == "no_heartbeat" else ep.Heartbeat(store, rank, world, timeout_s=1.0)
        moe = ep.ExpertParallelMoE(ops, k, heartbeat=hb)
        moe.forward(el, x)  # step 0: every rank takes part
        t0 = time.monotonic()
        try:
            if rank == 1 and scenario == "leave":
                hb.leave()  # leaves between steps, nothing in flight
                result["outcome"] = "left"
                return
            if rank == 1 and scenario == "late":
                time.sleep(2.5)  # beyond the other rank's 1 s heartbeat limit
            if rank == 1 and scenario == "no_heartbeat":
                time.sleep(6.0)  # never joins step 1's exchanges while the other waits in them
                result["outcome"] = "absent"
                return
            moe.forward(el, x)  # step 1
            result["outcome"] = "completed"
        except ep.PeerLost as e:
            result.update(outcome="peer_lost", peer=e.rank, step=e.step, why=e.why)
            hb.leave()
        except RuntimeError as e:  # the process group's timeout ended the exchange
            result.update(outcome="collective_error", message=str(e)[:200])
        result["seconds"] = time.monotonic() - t0
    finally:
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump(result, f)
        # rank 0 hosts the store: it stays up until the other rank is done with it
        if rank == 0:
            deadline = time.monotonic() + 15.0
            while not os.path.exists(os.path.join(out_dir, "rank1.json")) and time.monotonic() < deadline:
                time.sleep(0.01)
        if scenario != "no_heartbeat":  # a group whose peer is gone can only be abandoned
            dist.destroy_process_group()


def _run(scenario: str, tmp_path) -> dict:
    mp.start_processes(_rank_main, args=(scenario, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    return {r: json.loads((tmp_path / f"rank{r}.json").read_text()) for r in (0, 1)}


def test_rank_that_leaves_is_reported_before_the_next_step(tmp_path):
    res = _run("leave", tmp_path)
    assert res[1]["outcome"] == "left"
    r0 = res[0]
    assert r0["outcome"] == "peer_lost" and r0["peer"] == 1 and r0["step"] == 1 and r0["why"] == "it left", r0
    assert r0["seconds"] < 1.0, r0  # the leave mark is seen at once, not at the heartbeat limit


def test_late_rank_is_reported_at_the_heartbeat_limit(tmp_path):
    res = _run("late", tmp_path)
    r0, r1 = res[0], res[1]
    assert r0["outcome"] == "peer_lost" and r0["peer"] == 1 and "no heartbeat" in r0["why"], r0
    assert 0.9 < r0["seconds"] < 2.5, r0
    # the late rank, once it arrives, finds the other gone instead of blocking in an exchange
    assert r1["outcome"] == "peer_lost" and r1["peer"] == 0 and r1["why"] == "it left", r1


def test_without_heartbeat_the_process_group_timeout_ends_the_exchange(tmp_path):
    res = _run("no_heartbeat", tmp_path)
    assert res[1]["outcome"] == "absent"
    r0 = res[0]
    assert r0["outcome"] == "collective_error", r0
    assert r0["seconds"] < 6.0, r0
