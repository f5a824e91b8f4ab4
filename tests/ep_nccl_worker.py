"""One rank of the NCCL expert-parallel check (run by test_gpu_ep.py under
torchrun, one process per GPU).  Each rank holds 128/N experts of a
config-1-shaped layer, runs ExpertParallelMoE over its own tokens and checks
them against the CPU oracle; rank 0 prints EP_OK when every rank passed.
"""
from __future__ import annotations

import datetime
import importlib
import os
import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent.parent
sys.path[:0] = [str(REPO), str(REPO / "tests")]


def main() -> int:
    import torch
    import torch.distributed as dist
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    pkg = importlib.import_module("llmtoy-zig_b200")
    ep = importlib.import_module("llmtoy-zig_b200.ep")
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    import oracle_lib as orc

    rng = np.random.default_rng(4242)
    E, d, F, k = 128, 2048, 768, 8
    L = synth.MoeLayer(rng, d_model=d, n_experts=E, d_expert=F)
    Ts = [96 + 37 * r for r in range(world)]  # ragged token counts; >= 64 pairs per rank reach the GEMM path
    xs = [synth.hidden(rng, T, d) for T in Ts]
    nw = rng.uniform(0.5, 1.5, d).astype(np.float32)
    ok = 1
    with pkg.Context(local) as c:
        lo, hi = ep.expert_range(E, rank, world)
        sl = lambda a: np.ascontiguousarray(a.reshape(E, -1)[lo:hi])
        layer = ep.EPLayer(router=c.upload(L.router, 0, E, d),
                           gate=c.upload(sl(L.gate), L.gate_type, F, d, n_experts=hi - lo),
                           up=c.upload(sl(L.up), L.gate_type, F, d, n_experts=hi - lo),
                           down=c.upload(sl(L.down), L.down_type, d, F, n_experts=hi - lo),
                           n_experts=E, d_model=d, norm_w=torch.from_numpy(nw).cuda())
        moe = ep.ExpertParallelMoE(ep.DeviceOps(c, f"cuda:{local}"), k)
        x = xs[rank]
        out = moe.forward(layer, torch.from_numpy(x).cuda())
        got = out.cpu().numpy() - x
        xn = np.empty_like(x)
        for t in range(x.shape[0]):
            orc.lib().orc_rmsnorm(xn[t].ctypes.data, x[t].ctypes.data, nw.ctypes.data, d, 1e-6)
        with orc.Pool(8) as pool:
            ref, _, _ = orc.moe_layer(L, xn, k, True, pool=pool)
        err = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
        print(f"rank {rank}: T={x.shape[0]} received={moe.last_stats['received_pairs']} rel_l2={err:.3e}",
              flush=True)
        ok = int(err < 1e-4)
        flag = torch.tensor([ok], device=f"cuda:{local}")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ok = int(flag.item())
    dist.destroy_process_group()
    if rank == 0 and ok:
        print("EP_OK", flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
