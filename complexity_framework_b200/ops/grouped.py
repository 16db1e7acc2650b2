"""Grouped (expert-contiguous) execution of the routed experts.

Used when the dense-masked formulation would waste too much work (many wide
experts, e.g. 16 experts of width 256).  On CUDA bf16 everything runs on the
sm_100a kernels with no host synchronisation:

* ``C.moe_plan`` orders the T*k (token, slot) assignments by expert (stable,
  deterministic) into segments padded to the 256-row GEMM tile, and tabulates
  the expert of every row tile;
* ``C.moe_gather`` builds the expert-ordered activations;
* one grouped tcgen05 GEMM computes every expert's gate|up projection with the
  SwiGLU epilogue (the route weight of each row applied there), one grouped
  GEMM the down projection, and ``C.moe_combine`` sums each token's k rows;
* backward: a grouped GEMM with the SwiGLU-backward epilogue, a grouped GEMM
  for the input gradient, and two K-grouped split-K GEMMs for the weight
  gradients (each expert's K range read from device memory).

Elsewhere (CPU, fp32) the same plan runs as an eager per-expert loop.
Reference counterpart: sort_pair_hash_by_expert + K4/K5/K6/K7/K9-K12 of
complexity_cuda/triton_token_routed.py:2205-2351,1031-1229,751-838,279-330.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import require

EPI_STORE, EPI_SWIGLU_FWD, EPI_SWIGLU_BWD, EPI_F32_ATOMIC = 0, 2, 3, 7
SWIGLU_BLOCK = 128


def plan(routes: torch.Tensor, num_experts: int):
    """Expert-contiguous order of assignments (eager path).

    Returns (order [T*k] int64 assignment ids sorted by expert, counts [E]).
    Assignment a = j*T + t is route slot j of token t.
    """
    flat = routes.reshape(-1)
    order = torch.sort(flat, stable=True).indices
    counts = torch.bincount(flat, minlength=num_experts)
    return order, counts


def kernel_eligible(flat_x: torch.Tensor, gate: torch.Tensor) -> bool:
    E, H, W = gate.shape
    return (flat_x.is_cuda and flat_x.dtype == torch.bfloat16 and gate.dtype == torch.bfloat16
            and W % SWIGLU_BLOCK == 0 and H % 64 == 0)


def pack_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[E, H, W] x 2 -> [E*2W, H]: per expert, 128-row blocks of gate^T and up^T
    interleaved (the layout of the SwiGLU GEMM epilogue)."""
    E, H, W = gate.shape
    g = gate.transpose(1, 2).reshape(E, W // SWIGLU_BLOCK, 1, SWIGLU_BLOCK, H)
    u = up.transpose(1, 2).reshape(E, W // SWIGLU_BLOCK, 1, SWIGLU_BLOCK, H)
    return torch.cat([g, u], 2).reshape(E * 2 * W, H).contiguous()


def unpack_gate_up(d: torch.Tensor, E: int, H: int, W: int):
    v = d.view(E, W // SWIGLU_BLOCK, 2, SWIGLU_BLOCK, H)
    dg = v[:, :, 0].reshape(E, W, H).transpose(1, 2)
    du = v[:, :, 1].reshape(E, W, H).transpose(1, 2)
    return dg, du


class GroupedExpertsFn(torch.autograd.Function):
    """sum_j w_j * SwiGLU_{routes[j, t]}(x_t) on the grouped sm_100a kernels."""

    @staticmethod
    def forward(ctx, flat_x, routes, slot_w, gate, up, down):
        C = require()
        E, H, W = gate.shape
        k, T = routes.shape
        x = flat_x.contiguous()
        seg, tiles, row_token, row_weight, token_pos = C.moe_plan(
            routes.contiguous().long(), E, slot_w.float().contiguous())
        R = row_token.numel()
        w_gu = pack_gate_up(gate, up)
        w_d = down.transpose(1, 2).reshape(E * H, W).contiguous()
        xs = C.moe_gather(x, row_token, 1.0)
        gu = torch.empty(R, 2 * W, device=x.device, dtype=torch.bfloat16)
        act = torch.empty(R, W, device=x.device, dtype=torch.bfloat16)
        C.gemm_grouped(xs, False, w_gu, False, R, 2 * W, H, EPI_SWIGLU_FWD, gu=gu, act=act,
                       row_scale=row_weight, expert_width=W, mode=1, tile_group=tiles, groups=E,
                       b_stride=2 * W)
        ys = torch.empty(R, H, device=x.device, dtype=torch.bfloat16)
        C.gemm_grouped(act, False, w_d, False, R, H, W, EPI_STORE, out=ys, mode=1,
                       tile_group=tiles, groups=E, b_stride=H)
        out = C.moe_combine(ys, token_pos, k, 1.0)
        ctx.save_for_backward(xs, gu, act, w_gu, w_d, seg, tiles, row_token, row_weight,
                              token_pos)
        ctx.dims = (E, H, W, k)
        return out

    @staticmethod
    def backward(ctx, dout):
        C = require()
        xs, gu, act, w_gu, w_d, seg, tiles, row_token, row_weight, token_pos = ctx.saved_tensors
        E, H, W, k = ctx.dims
        R = row_token.numel()
        dys = C.moe_gather(dout.contiguous(), row_token, 1.0)
        dgu = torch.empty(R, 2 * W, device=dys.device, dtype=torch.bfloat16)
        # d(act) = dY W_down[e] with the SwiGLU backward (and route weight) in the epilogue
        C.gemm_grouped(dys, False, w_d, True, R, W, H, EPI_SWIGLU_BWD, out=dgu, gu=gu,
                       row_scale=row_weight, expert_width=W, mode=1, tile_group=tiles,
                       groups=E, b_stride=H)
        dxs = torch.empty(R, H, device=dys.device, dtype=torch.bfloat16)
        C.gemm_grouped(dgu, False, w_gu, True, R, H, 2 * W, EPI_STORE, out=dxs, mode=1,
                       tile_group=tiles, groups=E, b_stride=2 * W)
        dx = C.moe_combine(dxs, token_pos, k, 1.0)
        # weight gradients: every expert over its own rows (K ranges from the plan)
        dw_gu = torch.zeros(E * 2 * W, H, device=dys.device, dtype=torch.float32)
        C.gemm_grouped(dgu, True, xs, True, 2 * W, H, R, EPI_F32_ATOMIC, out=dw_gu, mode=2,
                       k_start=seg, groups=E, c_stride=2 * W)
        dw_d = torch.zeros(E * H, W, device=dys.device, dtype=torch.float32)
        C.gemm_grouped(dys, True, act, True, H, W, R, EPI_F32_ATOMIC, out=dw_d, mode=2,
                       k_start=seg, groups=E, c_stride=H)
        dg, du = unpack_gate_up(dw_gu, E, H, W)
        dd = dw_d.view(E, H, W).transpose(1, 2)
        return (dx, None, None, dg.to(torch.bfloat16), du.to(torch.bfloat16),
                dd.to(torch.bfloat16))


def routed_experts(flat_x: torch.Tensor, routes: torch.Tensor, route_weights: torch.Tensor,
                   gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor) -> torch.Tensor:
    """sum_j w_j * SwiGLU_{routes[j, t]}(x_t) for every token t."""
    if kernel_eligible(flat_x, gate):
        return GroupedExpertsFn.apply(flat_x, routes, route_weights, gate, up, down)
    k, T = routes.shape
    E = gate.shape[0]
    order, counts = plan(routes, E)
    tok = order % T
    slot = order // T
    xs = flat_x.index_select(0, tok)
    ws = route_weights.to(flat_x.dtype)[slot]
    outs = []
    start = 0
    for e, n in enumerate(counts.tolist()):
        if n == 0:
            continue
        xe = xs[start:start + n]
        h = F.silu(xe @ gate[e]) * (xe @ up[e])
        outs.append((h @ down[e]) * ws[start:start + n, None])
        start += n
    ys = torch.cat(outs, 0) if outs else flat_x.new_zeros(0, flat_x.shape[1])
    out = torch.zeros_like(flat_x)
    return out.index_add(0, tok, ys.to(out.dtype))
