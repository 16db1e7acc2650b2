"""Grouped (expert-contiguous) execution of the routed experts.

Used when the dense-masked formulation would waste too much work (many wide
experts, e.g. 16 experts of width 256).  The planner orders the T*k
(token, slot) assignments by expert with a stable sort, so the plan is
deterministic; each expert then runs one SwiGLU over its contiguous rows and
the weighted results are scattered back to token order.  Reference
counterpart: sort_pair_hash_by_expert + K4/K5/K9 of
complexity_cuda/triton_token_routed.py:2205-2351,1031-1229,279-330.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def plan(routes: torch.Tensor, num_experts: int):
    """Expert-contiguous order of assignments.

    Returns (order [T*k] int64 assignment ids sorted by expert, counts [E]).
    Assignment a = j*T + t is route slot j of token t.
    """
    flat = routes.reshape(-1)
    order = torch.sort(flat, stable=True).indices
    counts = torch.bincount(flat, minlength=num_experts)
    return order, counts


def routed_experts(flat_x: torch.Tensor, routes: torch.Tensor, route_weights: torch.Tensor,
                   gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor) -> torch.Tensor:
    """sum_j w_j * SwiGLU_{routes[j, t]}(x_t) for every token t."""
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
