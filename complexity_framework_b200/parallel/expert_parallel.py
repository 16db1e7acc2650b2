"""Expert parallelism for the TR-Hash FFN (the reference has none).

Experts are sharded over an EP group: rank r owns experts
``[r*E/P, (r+1)*E/P)``.  Because TR-Hash routes are a pure function of the
token id, every rank knows where each of its (token, slot) assignments goes
before the layer runs.  Dispatch: assignments are ordered by destination rank
(stable, so the plan is deterministic), counts are exchanged, and the token
rows plus the destination-local expert index travel with one all-to-all.
Each rank runs its experts on the rows it received (expert-contiguous), scales
them by the route weight and returns them with the inverse all-to-all
(combine); the shared SwiGLU stays local.  The all-to-alls are autograd
functions whose backward is the reverse exchange.

Expert parameters carry ``_ep_local = True``: data-parallel gradient averaging
must skip them (each rank owns different experts); their gradients are scaled
by 1/P instead because each rank's loss is a mean over its own tokens.
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F


class _AllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, send_splits: List[int], recv_splits: List[int], group):
        ctx.send, ctx.recv, ctx.group = send_splits, recv_splits, group
        out = x.new_empty((sum(recv_splits),) + tuple(x.shape[1:]))
        dist.all_to_all_single(out, x.contiguous(), recv_splits, send_splits, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        out = g.new_empty((sum(ctx.send),) + tuple(g.shape[1:]))
        dist.all_to_all_single(out, g.contiguous(), ctx.send, ctx.recv, group=ctx.group)
        return out, None, None, None


def all_to_all(x, send_splits, recv_splits, group):
    return _AllToAll.apply(x, list(send_splits), list(recv_splits), group)


class ExpertParallelRouted(nn.Module):
    """Routed-expert part of a TRHashEngine with experts sharded over ``group``."""

    def __init__(self, engine, group=None):
        super().__init__()
        self.group = group
        P = dist.get_world_size(group)
        r = dist.get_rank(group)
        E = engine.config.num_experts
        if E % P:
            raise ValueError("num_experts must be divisible by the expert-parallel size")
        self.P, self.rank, self.E, self.E_local = P, r, E, E // P
        lo = r * self.E_local
        self.lo = lo
        for name in ("expert_gate", "expert_up", "expert_down"):
            full = getattr(engine, name)
            p = nn.Parameter(full.detach()[lo:lo + self.E_local].clone())
            p._ep_local = True
            setattr(self, name, p)

    def forward(self, flat_x: torch.Tensor, routes: torch.Tensor,
                route_weights: torch.Tensor, **unused) -> torch.Tensor:
        k, T = routes.shape
        H = flat_x.shape[1]
        P, El = self.P, self.E_local
        flat_routes = routes.reshape(-1)                      # assignment a = j*T + t
        dest = flat_routes // El
        order = torch.sort(dest, stable=True).indices
        tok = order % T
        slot = order // T
        send_counts = torch.bincount(dest, minlength=P)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        send_splits = send_counts.tolist()
        recv_splits = recv_counts.tolist()
        xs = flat_x.index_select(0, tok)
        meta = torch.stack((flat_routes[order] - dest[order] * El,
                            slot), 1)                          # [n_send, 2] int64
        r_meta = torch.empty((sum(recv_splits), 2), dtype=meta.dtype, device=meta.device)
        dist.all_to_all_single(r_meta, meta, recv_splits, send_splits, group=self.group)
        rx = all_to_all(xs, send_splits, recv_splits, self.group)
        rw = route_weights.to(rx.dtype)[r_meta[:, 1]]
        ry = torch.zeros_like(rx)
        for e in range(El):
            idx = (r_meta[:, 0] == e).nonzero(as_tuple=True)[0]
            if idx.numel() == 0:
                # keep every local expert in the graph so its gradient exists
                ry = ry + 0.0 * (self.expert_gate[e].sum() + self.expert_up[e].sum()
                                 + self.expert_down[e].sum())
                continue
            xe = rx.index_select(0, idx)
            h = F.silu(xe @ self.expert_gate[e]) * (xe @ self.expert_up[e])
            ry = ry.index_add(0, idx, (h @ self.expert_down[e]) * rw[idx, None])
        ys = all_to_all(ry, recv_splits, send_splits, self.group)
        out = torch.zeros_like(flat_x)
        return out.index_add(0, tok, ys.to(out.dtype))


def make_expert_parallel(model, group=None) -> nn.Module:
    """Replace each engine's experts by their expert-parallel shard (in place)."""
    for layer in model.layers:
        eng = getattr(layer.mlp, "engine", None)
        if eng is None:
            continue
        ep = ExpertParallelRouted(eng, group)
        del eng.expert_gate, eng.expert_up, eng.expert_down
        eng.ep = ep
    model.ep_group = group
    return model
