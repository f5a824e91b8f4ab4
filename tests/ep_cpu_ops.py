"""The expert-parallel layer steps on the CPU, for the host-side tests of
ExpertParallelMoE (test infrastructure only).

Each step restates what the matching kernel computes, with the oracle for the
arithmetic: routing and the expert FFN follow orc_moe_layer
(src/model/gemma4/forward.zig:463-479 with the router of :648-668), so the
expert-parallel result over any number of ranks must equal orc_moe_layer
over all tokens bit for bit.  Tensors are CPU torch tensors, so the same
exchange code runs over gloo.
"""
from __future__ import annotations

import numpy as np
import torch

import oracle_lib as orc


class CpuOps:
    torch = torch

    def __init__(self, d_expert: int, gate_type: int, down_type: int):
        self.F, self.gate_type, self.down_type = d_expert, gate_type, down_type

    def empty(self, shape, dtype):
        return torch.empty(shape, dtype=dtype)

    def normed(self, layer, x, T: int):
        if layer.norm_w is None:
            return x
        xs = x.numpy()
        out = np.empty_like(xs)
        nw = orc.f32(layer.norm_w)
        for t in range(T):
            orc.lib().orc_rmsnorm(out[t].ctypes.data, xs[t].ctypes.data, nw.ctypes.data, layer.d_model, layer.eps)
        return torch.from_numpy(out)

    def route(self, layer, x, T: int, k: int):
        ids = np.empty((T, k), dtype=np.int32)
        w = np.empty((T, k), dtype=np.float32)
        for t in range(T):
            sel, p = orc.router_topk_softmax(layer.router, x[t].numpy(), k)
            p = p.astype(np.float32)
            if layer.norm_topk:
                s = np.float32(0.0)
                for v in p:
                    s = np.float32(s + v)
                p = (p / s).astype(np.float32)
            if layer.expert_scale is not None:
                p = (orc.f32(layer.expert_scale)[sel] * p).astype(np.float32)
            ids[t], w[t] = sel.astype(np.int32), p
        return torch.from_numpy(ids), torch.from_numpy(w)

    def dispatch(self, ids, T: int, k: int, n_experts: int, world: int):
        flat = ids.numpy().reshape(-1).astype(np.int64)
        per = n_experts // world
        dest = flat // per
        order = np.argsort(dest, kind="stable")
        pair_pos = np.empty(T * k, dtype=np.int32)
        pair_pos[order] = np.arange(T * k, dtype=np.int32)
        counts = np.bincount(dest, minlength=world).astype(np.int32)
        send_token = (order // k).astype(np.int32)
        send_local = (flat[order] - dest[order] * per).astype(np.int32)
        return tuple(torch.from_numpy(a) for a in (counts, send_token, send_local, pair_pos))

    def gather(self, x, idx, n: int):
        return x[idx.long()].contiguous() if n else torch.empty((0, x.shape[1]), dtype=torch.float32)

    def experts(self, layer, rows, n: int, local_ids):
        d, F = layer.d_model, self.F
        y = np.empty((n, d), dtype=np.float32)
        gu_rb = orc.row_bytes(self.gate_type, d)
        dn_rb = orc.row_bytes(self.down_type, F)
        fused = layer.up is None
        gpe = (2 if fused else 1) * F * gu_rb
        silu = orc.lib().orc_silu
        for i in range(n):
            e = int(local_ids[i])
            x = rows[i].numpy()
            g_data = layer.gate[e * gpe:(e + 1) * gpe]
            u_data = g_data[F * gu_rb:] if fused else layer.up[e * F * gu_rb:(e + 1) * F * gu_rb]
            g = orc.quant_matvec(g_data, self.gate_type, x, F, d)
            u = orc.quant_matvec(u_data, self.gate_type, x, F, d)
            h = np.array([silu(float(v)) for v in g], dtype=np.float32) * u
            y[i] = orc.quant_matvec(layer.down[e * d * dn_rb:(e + 1) * d * dn_rb], self.down_type, h, d, F)
        return torch.from_numpy(y)

    def combine(self, y, pair_pos, w, T: int, k: int, resid):
        yv, pp, wv = y.numpy(), pair_pos.numpy().reshape(T, k), w.numpy().reshape(T, k)
        out = np.zeros((T, yv.shape[1]), dtype=np.float32)
        for s in range(k):
            out += wv[:, s:s + 1] * yv[pp[:, s]]
        if resid is not None:
            out = resid.numpy() + out
        return torch.from_numpy(out.astype(np.float32))

    def local_forward(self, layer, x, T: int, k: int):
        raise NotImplementedError("the host tests run two or more ranks")
