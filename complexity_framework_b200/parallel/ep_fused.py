"""Expert parallelism with dispatch and combine over NVLink peer memory.

Experts are sharded over the group (rank q owns experts [q*E/P, (q+1)*E/P)).
TR-Hash routes are a pure function of the token id, so one all-gather of
the token ids per forward (int32, shared by every layer) gives each rank the
routes of all tokens of all layers, and one deterministic device plan
(``C.moe_plan`` over all experts, identical on every rank) tells each rank
both which rows it receives as an expert owner and where its own tokens'
slots land on every owner -- no per-layer collective, no host sync.  Then:

* dispatch: the expert owner PULLS the routed token rows from the token
  owners' symmetric hidden buffers (16-byte NVLink loads, one warp per row,
  ``csrc/ep_fused.cu``) into its expert-major buffer (256-row padded segments);
* experts: the grouped tcgen05 GEMMs over all local experts at once (gate|up
  with the SwiGLU + route-weight epilogue, down), as in ``ops/grouped.py``;
* combine: the token owner pulls each slot's output row from the expert
  owners and sums them in the same kernel.

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
    """Static-shape dispatch / combine maps of one layer on this rank (device tensors)."""
    row_src: torch.Tensor    # [R, 1] int32: global token p*T + t of local row r, or -1 (padding)
    row_w: torch.Tensor      # [R] fp32: route weight of that row's slot (0 for padding)
    tiles: torch.Tensor      # [R / 256] int32: local expert of each 256-row tile, or -1
    kstart: torch.Tensor     # [El + 1] int32: local expert segment starts (rows)
    comb_idx: torch.Tensor   # [T, k] int32: q * R + r, where token t's slot j output sits
    R: int
    T: int


def rows_bound(assignments: int, experts: int) -> int:
    """Rows of an expert-major layout whose segments start on 256-row tiles."""
    return (assignments + experts * 255 + 255) // 256 * 256


def build_plan(routes_all: torch.Tensor, route_weights: torch.Tensor, E: int, P: int, me: int,
               T: int) -> EPPlan:
    """routes_all [k, P*T] (every rank's tokens, rank-major) -> this rank's maps.

    One deterministic device plan over all experts (``C.moe_plan``: stable
    expert-major order, 256-row padded segments) is computed identically on
    every rank; owner q's rows are the contiguous range of its experts'
    segments, so every rank also knows where its own tokens' slots landed on
    every owner.  No host synchronisation: all shapes are static bounds.
    """
    C = require()
    k = routes_all.shape[0]
    El = E // P
    dev = routes_all.device
    seg, tiles, row_token, row_weight, token_pos = C.moe_plan(
        routes_all.contiguous(), E, route_weights.float().contiguous())
    Rg = row_token.numel()
    R = rows_bound(k * P * T, El)
    base = seg[me * El].long()
    cnt = seg[(me + 1) * El].long() - base
    i = torch.arange(R, device=dev)
    valid = i < cnt
    g = (base + i).clamp(max=Rg - 1)
    row_src = torch.where(valid, row_token[g], -1).to(torch.int32).view(R, 1)
    row_w = torch.where(valid, row_weight[g], 0.0).float()
    ti = torch.arange(R // 256, device=dev)
    tg = tiles[(base // 256 + ti).clamp(max=tiles.numel() - 1)].long()
    own = (ti * 256 < cnt) & (tg >= me * El) & (tg < (me + 1) * El)
    tiles_loc = torch.where(own, tg - me * El, -1).to(torch.int32)
    kstart = (seg[me * El:(me + 1) * El + 1].long() - base).to(torch.int32)
    a = (torch.arange(k, device=dev).view(k, 1) * (P * T) + me * T
         + torch.arange(T, device=dev).view(1, T))
    gr = token_pos[a].long()
    q = routes_all[:, me * T:(me + 1) * T].long() // El
    comb = (q * R + gr - seg.long()[q * El]).t().contiguous().to(torch.int32)
    return EPPlan(row_src, row_w, tiles_loc, kstart, comb, R, T)


def _pull(ws: TPWorkspace, name: str, src: torch.Tensor, idx: torch.Tensor,
          w: Optional[torch.Tensor], rows_out: int, residual: Optional[torch.Tensor] = None,
          stride: Optional[int] = None) -> torch.Tensor:
    """Copy ``src`` into this rank's symmetric buffer ``name`` and gather/combine rows
    of every rank's buffer by ``idx`` (after a bounded barrier; idx < 0 = zero row)."""
    C = require()
    cap_rows = stride if stride is not None else src.shape[0]
    buf, ptrs = ws.buffer(name, (cap_rows, src.shape[1]), torch.bfloat16)
    buf[:src.shape[0]].copy_(src)
    out = torch.empty(rows_out, src.shape[1], device=src.device, dtype=torch.bfloat16)
    C.ep_gather_combine(ptrs, idx, w, cap_rows, residual, out, ws.pads, ws.rank, ROUND_EP,
                        ws.epoch(ROUND_EP))
    return out


class EPGroupedFn(torch.autograd.Function):
    """Expert-parallel routed experts: NVLink dispatch -> grouped tcgen05 gate|up
    (+SwiGLU, route weight) and down GEMMs over all local experts -> NVLink
    combine.  Backward: dispatch of the output gradient, grouped SwiGLU-backward
    and data-gradient GEMMs, combine of the row gradients, and the K-grouped
    split-K weight gradients of every local expert (zeros for experts without
    rows come out of the same launches)."""

    @staticmethod
    def forward(ctx, x, gate, up, down, plan: EPPlan, ws: TPWorkspace, name: str):
        from ..ops.grouped import EPI_STORE, EPI_SWIGLU_FWD, pack_gate_up

        C = require()
        El, H, W = gate.shape
        R, T = plan.R, plan.T
        xs = _pull(ws, name + ".x", x.contiguous(), plan.row_src, None, R, stride=T)
        w_gu = pack_gate_up(gate, up)
        w_d = down.transpose(1, 2).reshape(El * H, W).contiguous()
        gu = torch.empty(R, 2 * W, device=x.device, dtype=torch.bfloat16)
        act = torch.empty(R, W, device=x.device, dtype=torch.bfloat16)
        C.gemm_grouped(xs, False, w_gu, False, R, 2 * W, H, EPI_SWIGLU_FWD, gu=gu, act=act,
                       row_scale=plan.row_w, expert_width=W, mode=1, tile_group=plan.tiles,
                       groups=El, b_stride=2 * W)
        ys = torch.empty(R, H, device=x.device, dtype=torch.bfloat16)
        C.gemm_grouped(act, False, w_d, False, R, H, W, EPI_STORE, out=ys, mode=1,
                       tile_group=plan.tiles, groups=El, b_stride=H)
        out = _pull(ws, name + ".y", ys, plan.comb_idx, None, T, stride=R)
        ctx.save_for_backward(xs, gu, act, w_gu, w_d)
        ctx.plan, ctx.ws, ctx.name, ctx.dims = plan, ws, name, (El, H, W)
        return out

    @staticmethod
    def backward(ctx, dout):
        from ..ops.grouped import (EPI_F32_ATOMIC, EPI_STORE, EPI_SWIGLU_BWD,
                                   unpack_gate_up)

        C = require()
        xs, gu, act, w_gu, w_d = ctx.saved_tensors
        plan, ws, name = ctx.plan, ctx.ws, ctx.name
        El, H, W = ctx.dims
        R, T = plan.R, plan.T
        dys = _pull(ws, name + ".dy", dout.contiguous(), plan.row_src, None, R, stride=T)
        dgu = torch.empty(R, 2 * W, device=dys.device, dtype=torch.bfloat16)
        C.gemm_grouped(dys, False, w_d, True, R, W, H, EPI_SWIGLU_BWD, out=dgu, gu=gu,
                       row_scale=plan.row_w, expert_width=W, mode=1, tile_group=plan.tiles,
                       groups=El, b_stride=H)
        dxs = torch.empty(R, H, device=dys.device, dtype=torch.bfloat16)
        C.gemm_grouped(dgu, False, w_gu, True, R, H, 2 * W, EPI_STORE, out=dxs, mode=1,
                       tile_group=plan.tiles, groups=El, b_stride=2 * W)
        dx = _pull(ws, name + ".dx", dxs, plan.comb_idx, None, T, stride=R)
        dw_gu = torch.zeros(El * 2 * W, H, device=dys.device, dtype=torch.float32)
        C.gemm_grouped(dgu, True, xs, True, 2 * W, H, R, EPI_F32_ATOMIC, out=dw_gu, mode=2,
                       k_start=plan.kstart, groups=El, c_stride=2 * W)
        dw_d = torch.zeros(El * H, W, device=dys.device, dtype=torch.float32)
        C.gemm_grouped(dys, True, act, True, H, W, R, EPI_F32_ATOMIC, out=dw_d, mode=2,
                       k_start=plan.kstart, groups=El, c_stride=H)
        dg, du = unpack_gate_up(dw_gu, El, H, W)
        dd = dw_d.view(El, H, W).transpose(1, 2)
        return (dx, dg.to(torch.bfloat16), du.to(torch.bfloat16), dd.to(torch.bfloat16),
                None, None, None)


class FusedExpertParallelRouted(nn.Module):
    """Routed experts of one TRHashEngine, sharded over ``group``, with NVLink
    dispatch/combine and grouped expert GEMMs.  Drop-in for
    ``ExpertParallelRouted``."""

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
        self.capacity_factor = capacity_factor  # kept for API compatibility: no row is dropped

    def _routes_all(self, routes: torch.Tensor, token_ids: Optional[torch.Tensor], route_fn):
        """[k, P*T] routes of every rank's tokens: from the token ids gathered once
        per forward (routes are a function of the id), else by gathering routes."""
        ws = self.ws
        if token_ids is not None and route_fn is not None:
            cache = getattr(ws, "ep_ids", None)
            if cache is None or cache[0] is not token_ids:
                ids = token_ids.reshape(-1).to(torch.int32).contiguous()
                allids = torch.empty(ws.world * ids.numel(), dtype=torch.int32, device=ids.device)
                dist.all_gather_into_tensor(allids, ids, group=ws.group)
                ws.ep_ids = cache = (token_ids, allids.long())
            return route_fn(cache[1]).reshape(routes.shape[0], -1)
        r8 = routes.to(torch.int8).contiguous()
        allr = torch.empty(ws.world, *r8.shape, dtype=torch.int8, device=routes.device)
        dist.all_gather_into_tensor(allr, r8, group=ws.group)
        return allr.permute(1, 0, 2).reshape(routes.shape[0], -1).long()

    def forward(self, flat_x: torch.Tensor, routes: torch.Tensor, route_weights: torch.Tensor,
                token_ids: Optional[torch.Tensor] = None, route_fn=None) -> torch.Tensor:
        k, T = routes.shape
        W = self.expert_gate.shape[2]
        if not (flat_x.is_cuda and flat_x.dtype == torch.bfloat16 and W % 128 == 0
                and flat_x.shape[1] % 64 == 0):
            raise RuntimeError("fused expert parallelism runs bf16 CUDA experts with widths "
                               "that are multiples of 128")
        allr = self._routes_all(routes, token_ids, route_fn)
        plan = build_plan(allr, route_weights, self.E, self.ws.world, self.ws.rank, T)
        return EPGroupedFn.apply(flat_x, self.expert_gate, self.expert_up, self.expert_down,
                                 plan, self.ws, self.name)


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

    def _new_forward(module, args):  # token ids are gathered once per forward
        ws.ep_ids = None

    model.register_forward_pre_hook(_new_forward)
    return model
