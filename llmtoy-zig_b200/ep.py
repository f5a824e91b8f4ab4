"""Expert-parallel MoE FFN: each rank holds a contiguous slice of the experts,
token rows travel to the rank of their expert and back with all-to-alls over
torch.distributed (NCCL between GPUs; gloo for the host-side tests).

The reference runs its MoE on one device (src/model/gemma4/forward.zig:463-479,
src/ops/moe.zig:18-77) and has no expert parallelism.  Sharding keeps its
arithmetic: each (token, slot) pair is computed by the rank that holds its
expert, with the same kernels as the single-device path, and the weighted
combine runs on the token's own rank in slot order (moe_buf zeroed, then
+= w * down for slot 0, 1, ...).

Rank r of N holds experts [r*E/N, (r+1)*E/N) of a layer; the router weights
and per-expert scales are replicated.  One layer over this rank's T tokens:

  1. route     ids[T][k], w[T][k]                       (lt_moe_route)
  2. dispatch  send_counts[N], send_token[P], send_local[P], pair_pos[P]:
               the P = T*k pairs ordered by destination rank, stable within
               a rank                                    (lt_ep_dispatch)
  3. counts    all-to-all of the N counts; both split lists go to the host
  4. pack      send_rows[i] = x[send_token[i]]           (lt_gather_rows)
  5. exchange  rows and local expert ids, all-to-all-v
  6. experts   y_recv = ffn(recv_rows) with k = 1, w = 1 (lt_moe_ffn)
  7. return    all-to-all-v of y_recv, landing in send order
  8. combine   out[t] = resid[t] + sum_s w[t][s] * y_send[pair_pos[t][s]]
                                                         (lt_moe_combine)

With one rank the layer runs the single-device fused path (lt_moe_forward /
lt_moe_block) and nothing is exchanged.  The kernels come from an ops object
(DeviceOps binds the CUDA library); the exchange code is the same for every
ops object, so the host-side tests drive it over gloo with CPU ops.
"""
from __future__ import annotations

import time
from dataclasses import dataclass


@dataclass
class EPLayer:
    """One MoE layer as seen by one rank.

    router, expert_scale: replicated over all n_experts.  gate, up, down:
    this rank's experts only (n_experts / world of them, local ids from 0).
    up is None for a fused gate_up tensor.  norm_w: the pre-FFN RMSNorm
    weight, or None for a bare FFN (out = moe(x))."""
    router: object
    gate: object
    up: object | None
    down: object
    n_experts: int
    d_model: int
    act: int = 0
    norm_topk: bool = True
    expert_scale: object = None
    norm_w: object = None
    eps: float = 1e-6


def expert_range(n_experts: int, rank: int, world: int) -> tuple[int, int]:
    """The experts [lo, hi) that rank holds."""
    if world <= 0 or n_experts % world != 0:
        raise ValueError(f"{n_experts} experts do not shard over {world} ranks")
    per = n_experts // world
    return rank * per, (rank + 1) * per


class DeviceOps:
    """The layer steps as C-ABI kernels on one GPU (torch CUDA tensors in and
    out).  The context runs on torch's current stream, so the NCCL
    collectives torch.distributed issues order after the kernels before them."""

    def __init__(self, ctx, device):
        import torch
        self.torch = torch
        self.ctx = ctx
        self.device = torch.device(device)
        ctx.set_stream(torch.cuda.current_stream(self.device))

    def empty(self, shape, dtype):
        return self.torch.empty(shape, dtype=dtype, device=self.device)

    # A rank with no tokens still takes part in every exchange; its tensors are
    # empty (null data pointers, which the C ABI rejects), so no kernel runs.
    def normed(self, layer: EPLayer, x, T: int):
        if layer.norm_w is None or T == 0:
            return x
        y = self.empty(x.shape, self.torch.float32)
        self.ctx.rmsnorm(x, layer.norm_w, layer.eps, layer.d_model, T, y)
        return y

    def route(self, layer: EPLayer, x, T: int, k: int):
        ids = self.empty((T, k), self.torch.int32)
        w = self.empty((T, k), self.torch.float32)
        if T == 0:
            return ids, w
        self.ctx.moe_route(layer.router, x, T, k, layer.norm_topk, layer.expert_scale, ids, w)
        return ids, w

    def dispatch(self, ids, T: int, k: int, n_experts: int, world: int):
        t = self.torch
        counts = self.empty((world,), t.int32)
        send_token = self.empty((T * k,), t.int32)
        send_local = self.empty((T * k,), t.int32)
        pair_pos = self.empty((T * k,), t.int32)
        if T == 0:
            counts.zero_()
            return counts, send_token, send_local, pair_pos
        self.ctx.ep_dispatch(ids, T, k, n_experts, world, counts, send_token, send_local, pair_pos)
        return counts, send_token, send_local, pair_pos

    def gather(self, x, idx, n: int):
        out = self.empty((n, x.shape[1]), self.torch.float32)
        if n:
            self.ctx.gather_rows(x, x.shape[1], idx, n, out)
        return out

    def experts(self, layer: EPLayer, rows, n: int, local_ids):
        y = self.empty((n, layer.d_model), self.torch.float32)
        if n:
            ones = self.torch.ones((n,), dtype=self.torch.float32, device=self.device)
            self.ctx.moe_ffn(layer.gate, layer.up, layer.down, layer.act, rows, n, local_ids, ones, 1, y)
        return y

    def combine(self, y, pair_pos, w, T: int, k: int, resid):
        out = self.empty((T, y.shape[1]), self.torch.float32)
        if T == 0:
            return out
        self.ctx.moe_combine(y, y.shape[1], pair_pos, w, T, k, resid, out)
        return out

    def local_forward(self, layer: EPLayer, x, T: int, k: int):
        """The whole layer on this device (one rank)."""
        out = self.empty((T, layer.d_model), self.torch.float32)
        if T == 0:
            return out
        if layer.norm_w is None:
            self.ctx.moe_forward(layer.router, layer.gate, layer.up, layer.down, layer.act, layer.norm_topk,
                                 layer.expert_scale, x, T, k, out)
        else:
            self.ctx.moe_block(layer.router, layer.gate, layer.up, layer.down, layer.act, layer.norm_topk,
                               layer.expert_scale, layer.norm_w, layer.eps, x, T, k, out)
        return out


class PeerLost(RuntimeError):
    """A rank did not reach the current step (it left, or is late beyond the
    heartbeat's limit).  Raised on the host before any kernel or collective of
    the step is issued, so nothing of the step is in flight."""

    def __init__(self, rank: int, step: int, why: str):
        super().__init__(f"rank {rank} did not reach step {step}: {why}")
        self.rank, self.step, self.why = rank, step, why


class Heartbeat:
    """Host-side liveness of the ranks over a torch.distributed Store (the
    TCPStore the process group was created with).

    Before step n every rank posts n, then waits up to timeout_s for every
    other rank to post n as well.  A rank that leaves posts a leave mark
    (leave()), so the others stop at their next step at once; a rank that is
    late beyond timeout_s, or died without a mark, is reported when the limit
    runs out.  Either way PeerLost is raised before the step issues a kernel
    or a collective, so the survivors never block inside NCCL on a rank that
    is gone (NCCL collectives on a dead peer end only at the process group's
    own timeout)."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 5.0, prefix: str = "lt_ep"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix = timeout_s, prefix

    def _key(self, kind: str, r: int) -> str:
        return f"{self.prefix}/{kind}/{r}"

    def leave(self) -> None:
        try:
            self.store.set(self._key("left", self.rank), "1")
        except RuntimeError:  # the store's host is gone already: nobody is left to tell
            pass

    def step(self, n: int) -> None:
        """Post step n and wait for every other rank to reach it.  A store
        that cannot be reached (its host process is gone) counts as a lost
        peer too."""
        try:
            self._step(n)
        except RuntimeError as e:
            if isinstance(e, PeerLost):
                raise
            raise PeerLost(-1, n, f"store unreachable ({e})") from e

    def _step(self, n: int) -> None:
        self.store.set(self._key("step", self.rank), str(n))
        deadline = time.monotonic() + self.timeout_s
        for r in range(self.world):
            if r == self.rank:
                continue
            while True:
                if self.store.check([self._key("left", r)]):
                    raise PeerLost(r, n, "it left")
                k = self._key("step", r)
                if self.store.check([k]) and int(self.store.get(k)) >= n:
                    break
                if time.monotonic() > deadline:
                    raise PeerLost(r, n, f"no heartbeat within {self.timeout_s:.1f} s")
                time.sleep(0.002)


class ExpertParallelMoE:
    """Runs MoE layers expert-parallel over a process group.

    ops: DeviceOps (or any object with the same methods).  group: a
    torch.distributed process group, or None for the default one when
    torch.distributed is initialised, else a single rank.  exchange, rank,
    world: a replacement for the all-to-all (called as exchange(out, inp,
    out_splits, in_splits) like all_to_all_single) with this caller's rank
    and the rank count.  Every rank must call forward() for the same layers
    in the same order (each call issues four exchanges).  heartbeat: an
    optional Heartbeat checked before each layer, so that a rank that left or
    stalls is reported (PeerLost) before any exchange of that layer starts."""

    def __init__(self, ops, k: int, group=None, exchange=None, rank: int | None = None, world: int | None = None,
                 heartbeat: Heartbeat | None = None):
        self.ops, self.k, self.group, self.heartbeat = ops, k, group, heartbeat
        self.n_forward = 0
        if exchange is not None:
            self._a2a, self.rank, self.world = exchange, rank, world
        else:
            import torch.distributed as dist
            self.dist = dist
            if dist.is_available() and dist.is_initialized():
                self.world = dist.get_world_size(group)
                self.rank = dist.get_rank(group)
            else:
                self.world, self.rank = 1, 0
        self.last_stats: dict = {}

    def _a2a(self, out, inp, out_splits=None, in_splits=None):
        self.dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def forward(self, layer: EPLayer, x):
        """x: this rank's tokens [T][d_model] f32.  Returns [T][d_model]:
        x + moe(rmsnorm(x) * norm_w) when layer.norm_w is set, else moe(x)."""
        ops, k, world = self.ops, self.k, self.world
        T = x.shape[0]
        if self.heartbeat is not None and world > 1:
            self.heartbeat.step(self.n_forward)
        self.n_forward += 1
        if world == 1:
            return ops.local_forward(layer, x, T, k)
        torch = ops.torch
        xn = ops.normed(layer, x, T)
        ids, w = ops.route(layer, xn, T, k)
        counts, send_token, send_local, pair_pos = ops.dispatch(ids, T, k, layer.n_experts, world)
        recv_counts = torch.empty_like(counts)
        self._a2a(recv_counts, counts)
        splits = torch.cat([counts, recv_counts]).cpu().tolist()  # the one host sync of the layer
        send_splits, recv_splits = splits[:world], splits[world:]
        R = sum(recv_splits)
        send_rows = ops.gather(xn, send_token, T * k)
        recv_rows = ops.empty((R, layer.d_model), torch.float32)
        recv_local = ops.empty((R,), torch.int32)
        self._a2a(recv_rows, send_rows, recv_splits, send_splits)
        self._a2a(recv_local, send_local, recv_splits, send_splits)
        y_recv = ops.experts(layer, recv_rows, R, recv_local)
        y_send = ops.empty((T * k, layer.d_model), torch.float32)
        self._a2a(y_send, y_recv, send_splits, recv_splits)
        self.last_stats = {"sent_pairs": send_splits, "received_pairs": R}
        return ops.combine(y_send, pair_pos, w, T, k, x if layer.norm_w is not None else None)
