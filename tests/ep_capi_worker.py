"""One rank of the C-ABI expert-parallel check (lt_ep_init / lt_moe_ffn_ep),
run by test_gpu_ep.py under torchrun, one process per GPU.  Rank 0 makes the
NCCL id and shares it over a gloo group; each rank holds 128/N experts of a
config-1-shaped layer and checks its tokens against the CPU oracle; rank 0
prints EP_CAPI_OK when every rank passed.  With --leave, rank 1 then leaves
between steps and rank 0's next call must come back with LT_ETIMEOUT or
LT_ECUDA within the ep's timeout, leaving its context usable.
"""
from __future__ import annotations

import ctypes
import datetime
import importlib
import os
import sys
import time
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
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    pkg = importlib.import_module("llmtoy-zig_b200")
    ep = importlib.import_module("llmtoy-zig_b200.ep")
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    import oracle_lib as orc
    lib = pkg.load_library()

    rng = np.random.default_rng(4343)
    E, d, F, k = 128, 2048, 768, 8
    L = synth.MoeLayer(rng, d_model=d, n_experts=E, d_expert=F)
    Ts = [80 + 29 * r for r in range(world)]  # ragged; >= 64 pairs per rank reach the GEMM path
    xs = [synth.hidden(rng, T, d) for T in Ts]
    nw = rng.uniform(0.5, 1.5, d).astype(np.float32)
    uid = (ctypes.c_uint8 * 128)()
    if rank == 0:
        assert lib.lt_ep_unique_id(uid) == 0
    obj = [bytes(uid)]
    dist.broadcast_object_list(obj, src=0)
    uid = (ctypes.c_uint8 * 128)(*obj[0])
    ok = 1
    with pkg.Context(local) as c:
        c.set_stream(None)
        lo, hi = ep.expert_range(E, rank, world)
        sl = lambda a: np.ascontiguousarray(a.reshape(E, -1)[lo:hi])  # noqa: E731
        router = c.upload(L.router, 0, E, d)
        gate = c.upload(sl(L.gate), L.gate_type, F, d, n_experts=hi - lo)
        up = c.upload(sl(L.up), L.gate_type, F, d, n_experts=hi - lo)
        down = c.upload(sl(L.down), L.down_type, d, F, n_experts=hi - lo)
        h = ctypes.c_void_p()
        st = lib.lt_ep_init(c.ptr, world, rank, uid, 5000, ctypes.byref(h))
        assert st == 0, pkg.STATUS.get(st, st)
        x = torch.from_numpy(xs[rank]).cuda()
        nwd = torch.from_numpy(nw).cuda()
        out = torch.empty_like(x)
        st = lib.lt_moe_ffn_ep(c.ptr, h, router.handle, gate.handle, up.handle, down.handle, pkg.ACT_SILU, 1, None,
                               nwd.data_ptr(), ctypes.c_float(1e-6), x.data_ptr(), x.shape[0], k, out.data_ptr())
        assert st == 0, pkg.STATUS.get(st, st)
        got = out.cpu().numpy() - xs[rank]
        xn = np.empty_like(xs[rank])
        for t in range(xn.shape[0]):
            orc.lib().orc_rmsnorm(xn[t].ctypes.data, xs[rank][t].ctypes.data, nw.ctypes.data, d, 1e-6)
        with orc.Pool(8) as pool:
            ref, _, _ = orc.moe_layer(L, xn, k, True, pool=pool)
        err = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
        print(f"rank {rank}: T={x.shape[0]} rel_l2={err:.3e}", flush=True)
        ok = int(err < 1e-4)
        flag = torch.tensor([ok])
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ok = int(flag.item())
        if "--leave" in sys.argv and world >= 2 and ok:
            dist.barrier()  # every rank is between steps: nothing is in flight
            if rank == 0:  # the next step: rank 1 never joins it
                t0 = time.monotonic()
                st = lib.lt_moe_ffn_ep(c.ptr, h, router.handle, gate.handle, up.handle, down.handle, pkg.ACT_SILU, 1, None,
                                       nwd.data_ptr(), ctypes.c_float(1e-6), x.data_ptr(), x.shape[0], k,
                                       out.data_ptr())
                dt = time.monotonic() - t0
                print(f"rank 0: step without rank 1 -> {pkg.STATUS.get(st, st)} after {dt:.1f} s", flush=True)
                ok = int(st in (4, 5) and dt < 30.0)  # LT_ECUDA (NCCL saw the peer go) or LT_ETIMEOUT
                st2 = lib.lt_moe_ffn_ep(c.ptr, h, router.handle, gate.handle, up.handle, down.handle, pkg.ACT_SILU, 1, None,
                                        nwd.data_ptr(), ctypes.c_float(1e-6), x.data_ptr(), x.shape[0], k,
                                        out.data_ptr())
                ok = ok and st2 == 5  # the aborted ep refuses further calls
                c.sync()  # the context is still usable
                z = torch.zeros(8, device=f"cuda:{local}")
                z[3] = 1.0
                idx = torch.zeros(1, dtype=torch.int32, device=f"cuda:{local}")
                c.argmax(z, 8, 1, idx)
                c.sync()
                ok = ok and int(idx.item()) == 3
                lib.lt_ep_free(h)
            h = None  # rank 1 leaves its communicator to the process exit
            dist.barrier()
        if h is not None:
            lib.lt_ep_free(h)
        for t in (router, gate, up, down):
            t.free()
    if rank == 0 and ok:
        print("EP_CAPI_OK", flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
