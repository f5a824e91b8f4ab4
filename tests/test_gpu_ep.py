"""Expert-parallel building blocks on the GPU (lt_ep_dispatch,
lt_gather_rows, lt_moe_combine) and the whole expert-parallel layer.

The dispatch, gather and combine kernels move and add rows only, so they must
equal their CPU restatements bit for bit.  The whole layer runs its ranks as
threads of one process on one GPU (each with its own context; the all-to-all
is a host-synchronised copy between them), and, with two or more GPUs, as
NCCL ranks under torchrun (ep_nccl_worker.py).  Each rank's output is
checked against the CPU oracle over the same tokens.
"""
from __future__ import annotations

import ctypes
import importlib
import os
import subprocess
import sys
import threading

import numpy as np
import pytest

from conftest import REPO
from test_gpu_parity import MOE_L2_TOL, W_TOL, bits, dev, empty, host, max_rel, rel_l2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("ntok,k,E,nranks", [(1, 1, 8, 1), (5, 2, 8, 2), (700, 8, 128, 8), (333, 3, 64, 4),
                                             (2048, 8, 128, 2), (129, 6, 96, 3)])
def test_ep_dispatch_matches_cpu(ctx, ntok, k, E, nranks):
    from ep_cpu_ops import CpuOps
    import torch
    rng = np.random.default_rng(ntok * 31 + k)
    ids = np.stack([rng.choice(E, size=k, replace=False) for _ in range(ntok)]).astype(np.int32)
    P = ntok * k
    counts, tok, loc, pos = empty(nranks, "int32"), empty(P, "int32"), empty(P, "int32"), empty(P, "int32")
    ctx.ep_dispatch(dev(ids), ntok, k, E, nranks, counts, tok, loc, pos)
    rc, rt, rl, rp = CpuOps(1, 12, 12).dispatch(torch.from_numpy(ids), ntok, k, E, nranks)
    for got, ref in ((counts, rc), (tok, rt), (loc, rl), (pos, rp)):
        np.testing.assert_array_equal(host(got), ref.numpy())


def test_ep_dispatch_rejects_bad_sharding(ctx, pkg):
    ids = dev(np.zeros(4, np.int32))
    bufs = [empty(4, "int32") for _ in range(4)]
    for E, n in ((10, 3), (16, 9), (16, 0)):
        with pytest.raises(pkg.LtError):
            ctx.ep_dispatch(ids, 2, 2, E, n, *bufs)


def test_gather_rows_and_combine_exact(ctx):
    rng = np.random.default_rng(7)
    T, k, d = 37, 4, 2048
    src = rng.normal(size=(T, d)).astype(np.float32)
    idx = rng.integers(0, T, size=T * k).astype(np.int32)
    rows = empty(T * k * d)
    ctx.gather_rows(dev(src), d, dev(idx), T * k, rows)
    np.testing.assert_array_equal(bits(host(rows).reshape(T * k, d)), bits(src[idx]))

    y = rng.normal(size=(T * k, d)).astype(np.float32)
    pos = rng.permutation(T * k).astype(np.int32)
    w = rng.uniform(0, 1, size=T * k).astype(np.float32)
    resid = rng.normal(size=(T, d)).astype(np.float32)
    for r in (None, resid):
        out = empty(T * d)
        ctx.moe_combine(dev(y), d, dev(pos), dev(w), T, k, None if r is None else dev(r), out)
        ref = np.zeros((T, d), np.float32)
        for s in range(k):
            ref += w.reshape(T, k)[:, s:s + 1] * y[pos.reshape(T, k)[:, s]]
        if r is not None:
            ref = r + ref
        np.testing.assert_array_equal(bits(host(out).reshape(T, d)), bits(ref))


class ThreadExchange:
    """all_to_all_single between threads of one process on one GPU: each
    rank publishes its input, all meet at a barrier, each copies its pieces,
    all meet again before any input may change."""

    def __init__(self, world: int):
        self.world = world
        self.barrier = threading.Barrier(world, timeout=120)
        self.slots = [None] * world

    def for_rank(self, rank: int):
        import torch

        def a2a(out, inp, out_splits=None, in_splits=None):
            torch.cuda.synchronize()
            self.slots[rank] = (inp, in_splits)
            self.barrier.wait()
            off = 0
            for src in range(self.world):
                s_inp, s_splits = self.slots[src]
                if s_splits is None:
                    n = s_inp.shape[0] // self.world
                    start = rank * n
                else:
                    n, start = s_splits[rank], sum(s_splits[:rank])
                if n:
                    out[off:off + n].copy_(s_inp[start:start + n])
                off += n
            torch.cuda.synchronize()
            self.barrier.wait()

        return a2a


def _shard_upload(c, L, lo, hi):
    E, F, d = L.n_experts, L.d_expert, L.d_model
    n = hi - lo
    sl = lambda a: np.ascontiguousarray(a.reshape(E, -1)[lo:hi])
    g = c.upload(sl(L.gate), L.gate_type, (F if L.up is not None else 2 * F), d, n_experts=n)
    u = c.upload(sl(L.up), L.gate_type, F, d, n_experts=n) if L.up is not None else None
    dn = c.upload(sl(L.down), L.down_type, d, F, n_experts=n)
    return g, u, dn


@pytest.mark.parametrize("world,Ts,block", [(2, [24, 70], False), (4, [0, 9, 80, 33], True), (2, [1, 1], True)])
def test_ep_threads_vs_oracle(pkg, oracle, pool, world, Ts, block):
    import torch
    ep = importlib.import_module("llmtoy-zig_b200.ep")
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    rng = np.random.default_rng(99 + world)
    L = synth.MoeLayer(rng, d_model=2048, n_experts=128, d_expert=768)
    xs = [synth.hidden(rng, T, 2048) for T in Ts]
    nw = rng.uniform(0.5, 1.5, 2048).astype(np.float32) if block else None
    k = 8
    xch = ThreadExchange(world)
    results, errors = [None] * world, []

    def run(rank):
        try:
            torch.cuda.set_device(0)
            with pkg.Context(0) as c:
                lo, hi = ep.expert_range(128, rank, world)
                g, u, dn = _shard_upload(c, L, lo, hi)
                rt = c.upload(L.router, 0, 128, 2048)
                layer = ep.EPLayer(router=rt, gate=g, up=u, down=dn, n_experts=128, d_model=2048,
                                   norm_w=None if nw is None else dev(nw))
                moe = ep.ExpertParallelMoE(ep.DeviceOps(c, "cuda:0"), k, exchange=xch.for_rank(rank), rank=rank,
                                           world=world)
                out = moe.forward(layer, dev(xs[rank]).reshape(Ts[rank], 2048))
                torch.cuda.synchronize()
                results[rank] = (host(out).reshape(Ts[rank], 2048), moe.last_stats)
        except BaseException as e:  # noqa: BLE001 - reported by the main thread
            errors.append((rank, e))
            xch.barrier.abort()

    threads = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    assert not errors, errors
    assert sum(r[1]["received_pairs"] for r in results) == k * sum(Ts)
    for rank, T in enumerate(Ts):
        got = results[rank][0]
        if T == 0:
            assert got.shape == (0, 2048)
            continue
        x = xs[rank]
        if nw is not None:
            xn = np.empty_like(x)
            for t in range(T):
                oracle.lib().orc_rmsnorm(xn[t].ctypes.data, x[t].ctypes.data, nw.ctypes.data, 2048, 1e-6)
        else:
            xn = x
        ref, _, _ = oracle.moe_layer(L, xn, k, True, pool=pool)
        if nw is not None:
            ref = x + ref
            got, ref = got - x, ref - x  # compare the MoE part, not the residual
        assert rel_l2(got, ref) < MOE_L2_TOL, (rank, rel_l2(got, ref))


def test_ep_nccl_all_gpus():
    """The NCCL expert-parallel layer over every visible GPU (2, 4 or 8 ranks)."""
    import torch
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    n = max(w for w in (2, 4, 8) if w <= n)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr=127.0.0.1", "--master-port=29531", str(REPO / "tests" / "ep_nccl_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "600"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "EP_OK" in r.stdout


def test_ep_capi_single_rank(ctx, pkg, oracle, pool):
    """lt_ep_init / lt_moe_ffn_ep with one rank (NCCL to itself) on the config-1
    shape: the same result as the single-device block and the oracle, on the
    grouped CUDA-core path (5 tokens) and the tensor-core path (80 tokens)."""
    import torch
    synth = importlib.import_module("llmtoy-zig_b200.synth")
    lib = pkg.load_library()
    rng = np.random.default_rng(4444)
    E, d, F, k = 128, 2048, 768, 8
    L = synth.MoeLayer(rng, d_model=d, n_experts=E, d_expert=F)
    nw = rng.uniform(0.5, 1.5, d).astype(np.float32)
    router, gate = ctx.upload(L.router, 0, E, d), ctx.upload(L.gate, L.gate_type, F, d, n_experts=E)
    up, down = ctx.upload(L.up, L.gate_type, F, d, n_experts=E), ctx.upload(L.down, L.down_type, d, F, n_experts=E)
    uid = (ctypes.c_uint8 * 128)()
    assert lib.lt_ep_unique_id(uid) == 0
    h = ctypes.c_void_p()
    st = lib.lt_ep_init(ctx.ptr, 1, 0, uid, 20000, ctypes.byref(h))
    assert st == 0, pkg.STATUS.get(st, st)
    nwd = torch.from_numpy(nw).cuda()
    try:
        for T in (5, 80):
            x = synth.hidden(rng, T, d)
            xd = torch.from_numpy(x).cuda()
            out = torch.empty_like(xd)
            st = lib.lt_moe_ffn_ep(ctx.ptr, h, router.handle, gate.handle, up.handle, down.handle, pkg.ACT_SILU, 1, None,
                                   nwd.data_ptr(), ctypes.c_float(1e-6), xd.data_ptr(), T, k, out.data_ptr())
            assert st == 0, pkg.STATUS.get(st, st)
            single = torch.empty_like(xd)
            ctx.moe_block(router, gate, up, down, pkg.ACT_SILU, True, None, nwd, 1e-6, xd, T, k, single)
            ctx.sync()
            got, one = out.cpu().numpy() - x, single.cpu().numpy() - x
            xn = np.empty_like(x)
            for t in range(T):
                oracle.lib().orc_rmsnorm(xn[t].ctypes.data, x[t].ctypes.data, nw.ctypes.data, d, 1e-6)
            ref, _, _ = oracle.moe_layer(L, xn, k, True, pool=pool)
            assert rel_l2(got, ref) < MOE_L2_TOL, (T, rel_l2(got, ref))
            assert rel_l2(got, one) < MOE_L2_TOL, (T, rel_l2(got, one))
    finally:
        lib.lt_ep_free(h)
        for t in (router, gate, up, down):
            t.free()


def test_ep_capi_all_gpus():
    """lt_moe_ffn_ep over every visible GPU (2, 4 or 8 ranks) against the oracle;
    then one rank leaves between steps and the other's next call returns an
    error within the ep's timeout, its context still usable (NVLS off)."""
    import torch
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    n = max(w for w in (2, 4, 8) if w <= n)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr=127.0.0.1", "--master-port=29533", str(REPO / "tests" / "ep_capi_worker.py"), "--leave"]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "600"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "EP_CAPI_OK" in r.stdout
