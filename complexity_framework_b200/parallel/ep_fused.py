"""Expert parallelism with dispatch and combine over NVLink peer memory.

Experts are sharded over the group (rank q owns experts [q*E/P, (q+1)*E/P)).
TR-Hash routes are a pure function of the token id, so after one tiny
all-gather of every rank's routes (int8) each rank knows the whole plan:
which (rank, token, slot) assignments each expert owner receives, in an
expert-contiguous order, and where each token's results will sit.  Then:

* dispatch: the expert owner PULLS the routed token rows from the token
  owners' symmetric hidden buffers (16-byte NVLink loads, one warp per row,
  ``csrc/ep_fused.cu``) into its expert-contiguous buffer;
* experts: one fused tcgen05 SwiGLU GEMM pair per local expert on its
  contiguous rows (gate|up GEMM with the SwiGLU epilogue, down GEMM);
* combine: the token owner pulls each slot's output row from the expert
  owners and sums them with the route weights in the same kernel.

Backward runs the same two primitives in the opposite roles (the combine's
backward is a weighted dispatch of the output gradient; the dispatch's
backward is a combine of the row gradients).  Every cross-rank read is
preceded by a bounded device barrier on the symmetric signal pads.  This
replaces NCCL all-to-all + index_select / index_add
(``parallel/expert_parallel.py``), which remains the portable path.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from ..ops._ext import require
from .tp_fused import TPWorkspace

ROUND_EP = 3


@dataclass
class EPPlan:
    row_src: torch.Tensor    # [R, 1] int32: p * T + t for dispatch row r on this rank
    row_w: torch.Tensor      # [R, 1] fp32: route weight of that row's slot
    comb_idx: torch.Tensor   # [T, k] int32: q * cap + r, where token t slot j's output sits
    comb_w: torch.Tensor     # [T, k] fp32: route weights
    seg: List[int]           # dispatch rows per local expert
    R: int
    cap: int


def build_plan(routes: torch.Tensor, route_weights: torch.Tensor, E: int, group, cap: int
               ) -> EPPlan:
    """routes [k, T] (this rank's tokens) -> the dispatch / combine index maps."""
    P = dist.get_world_size(group)
    me = dist.get_rank(group)
    k, T = routes.shape
    El = E // P
    r8 = routes.to(torch.int8).contiguous()
    allr = torch.empty(P, k, T, dtype=torch.int8, device=routes.device)
    dist.all_gather_into_tensor(allr, r8, group=group)
    allr = allr.long()                                            # [P, k, T]
    p_idx = torch.arange(P, device=routes.device).view(P, 1, 1).expand(P, k, T)
    j_idx = torch.arange(k, device=routes.device).view(1, k, 1).expand(P, k, T)
    t_idx = torch.arange(T, device=routes.device).view(1, 1, T).expand(P, k, T)
    owner = allr // El
    # dispatch rows of every owner: ordered by (local expert, source rank, token, slot)
    key = ((allr % El) * P + p_idx) * (T * k) + t_idx * k + j_idx
    flat_owner = owner.reshape(-1)
    flat_key = key.reshape(-1)
    order = torch.argsort(flat_owner * (El * P * T * k) + flat_key, stable=True)
    counts = torch.bincount(flat_owner, minlength=P)
    starts = torch.cumsum(counts, 0) - counts
    pos = torch.empty_like(order)
    pos[order] = torch.arange(order.numel(), device=order.device)
    row_in_owner = (pos - starts[flat_owner]).view(P, k, T)       # dispatch row on its owner
    # this rank as expert owner
    mine = order[starts[me]:starts[me] + counts[me]]
    R = int(counts[me])
    if R > cap:
        raise RuntimeError(f"expert-parallel capacity {cap} < {R} dispatched rows")
    sp, sj, st = mine // (k * T), (mine // T) % k, mine % T
    row_src = (sp * T + st).to(torch.int32).view(-1, 1)
    row_w = route_weights.float()[sj].view(-1, 1).contiguous()
    seg = torch.bincount(allr.reshape(-1)[mine] % El, minlength=El).tolist()
    # this rank as token owner
    comb = (owner[me] * cap + row_in_owner[me]).t().contiguous().to(torch.int32)   # [T, k]
    comb_w = route_weights.float().view(1, k).expand(T, k).contiguous()
    return EPPlan(row_src, row_w, comb, comb_w, seg, R, cap)


def _pull(ws: TPWorkspace, name: str, src: torch.Tensor, idx: torch.Tensor,
          w: Optional[torch.Tensor], rows_out: int, residual: Optional[torch.Tensor] = None,
          stride: Optional[int] = None) -> torch.Tensor:
    """Copy ``src`` into this rank's symmetric buffer ``name`` and gather/combine rows
    of every rank's buffer by ``idx`` (after a bounded barrier)."""
    C = require()
    cap_rows = stride if stride is not None else src.shape[0]
    buf, ptrs = ws.buffer(name, (cap_rows, src.shape[1]), torch.bfloat16)
    buf[:src.shape[0]].copy_(src)
    out = torch.empty(rows_out, src.shape[1], device=src.device, dtype=torch.bfloat16)
    if rows_out:
        C.ep_gather_combine(ptrs, idx, w, cap_rows, residual, out, ws.pads, ws.rank, ROUND_EP,
                            ws.epoch(ROUND_EP))
    else:  # still take part in the barrier
        C.tp_barrier(ws.pads, ws.rank, ROUND_EP, ws.epoch(ROUND_EP), src.device.index)
    return out


class DispatchFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, plan: EPPlan, ws: TPWorkspace, name: str):
        ctx.plan, ctx.ws, ctx.name, ctx.T = plan, ws, name, x.shape[0]
        return _pull(ws, name + ".x", x.contiguous(), plan.row_src, None, plan.R)

    @staticmethod
    def backward(ctx, g):
        p = ctx.plan
        dx = _pull(ctx.ws, ctx.name + ".dd", g.contiguous(), p.comb_idx, None, ctx.T,
                   stride=p.cap)
        return dx, None, None, None


class CombineFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, plan: EPPlan, ws: TPWorkspace, name: str):
        ctx.plan, ctx.ws, ctx.name, ctx.R = plan, ws, name, y.shape[0]
        T = plan.comb_idx.shape[0]
        return _pull(ws, name + ".y", y.contiguous(), plan.comb_idx, plan.comb_w, T, stride=plan.cap)

    @staticmethod
    def backward(ctx, g):
        p = ctx.plan
        dy = _pull(ctx.ws, ctx.name + ".dg", g.contiguous(), p.row_src, p.row_w, ctx.R,
                   stride=g.shape[0])
        return dy, None, None, None


class FusedExpertParallelRouted(nn.Module):
    """Routed experts of one TRHashEngine, sharded over ``group``, with NVLink
    dispatch/combine.  Drop-in for ``ExpertParallelRouted``."""

    def __init__(self, engine, ws: TPWorkspace, name: str, capacity_factor: float = 1.0):
        super().__init__()
        self.ws, self.name = ws, name
        P, r = ws.world, ws.rank
        E = engine.config.num_experts
        if E % P:
            raise ValueError("num_experts must be divisible by the expert-parallel size")
        self.E, self.El = E, E // P
        lo = r * self.El
        for nm in ("expert_gate", "expert_up", "expert_down"):
            p = nn.Parameter(getattr(engine, nm).detach()[lo:lo + self.El].clone())
            p._ep_local = True
            setattr(self, nm, p)
        self.capacity_factor = capacity_factor

    def _expert(self, e: int, xe: torch.Tensor) -> torch.Tensor:
        g, u, d = self.expert_gate[e], self.expert_up[e], self.expert_down[e]   # [H,W],[H,W],[W,H]
        W = g.shape[1]
        if xe.is_cuda and xe.dtype == torch.bfloat16 and W % 128 == 0 and xe.shape[0] > 0:
            from ..ops.fused import pack_shared_gate_up, trhash_mlp

            w_gu = pack_shared_gate_up(g.t(), u.t())
            return trhash_mlp(xe, w_gu, d.t(), None, None, W, 1, 0, 1.0)
        return (F.silu(xe @ g) * (xe @ u)) @ d

    def forward(self, flat_x: torch.Tensor, routes: torch.Tensor,
                route_weights: torch.Tensor) -> torch.Tensor:
        k, T = routes.shape
        cap = int(self.capacity_factor * k * T * self.ws.world)
        plan = build_plan(routes, route_weights, self.E, self.ws.group, cap)
        disp = DispatchFn.apply(flat_x, plan, self.ws, self.name)
        outs, s = [], 0
        for e, n in enumerate(plan.seg):
            outs.append(self._expert(e, disp[s:s + n]))
            s += n
        y = torch.cat(outs, 0) if outs else disp
        # keep experts without rows in the graph so their gradients exist
        y = y + 0.0 * sum(p.sum() for p in (self.expert_gate, self.expert_up, self.expert_down))
        return CombineFn.apply(y.to(torch.bfloat16), plan, self.ws, self.name)


def make_fused_expert_parallel(model, group=None, capacity_factor: float = 1.0):
    """Shard every engine's experts over ``group`` with NVLink dispatch/combine."""
    group = group if group is not None else dist.group.WORLD
    ws = TPWorkspace(group)
    for i, layer in enumerate(model.layers):
        eng = getattr(layer.mlp, "engine", None)
        if eng is None:
            continue
        ep = FusedExpertParallelRouted(eng, ws, f"ep{i}", capacity_factor)
        del eng.expert_gate, eng.expert_up, eng.expert_down
        eng.ep = ep
    model.ep_group = group
    model.ep_ws = ws
    return model
