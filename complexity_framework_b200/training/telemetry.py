"""Routing telemetry for TR-Hash models.

Counterpart of complexity/training/moe_telemetry.py:30-202.  Routes are a
static function of the token id, so expert load is computed from the route
tables and the batch's token ids (one bincount per layer) instead of from
router outputs; across ranks the counts are all-reduced once.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch
import torch.distributed as dist
import torch.nn as nn


def detect_num_experts(model: nn.Module) -> Optional[int]:
    cfg = getattr(model, "config", None)
    n = getattr(cfg, "num_experts", None)
    return int(n) if n else None


def _engines(model: nn.Module):
    return [m for m in model.modules() if type(m).__name__ == "TRHashEngine"]


@torch.no_grad()
def expert_token_counts(model: nn.Module, input_ids: torch.Tensor) -> torch.Tensor:
    """``[layers, E]`` routed-assignment counts for ``input_ids`` (all top-k slots)."""
    rows = []
    ids = input_ids.reshape(-1)
    for eng in _engines(model):
        table = eng.route_table.to(ids.device)  # [k, vocab]
        routes = table[:, ids.clamp(0, table.shape[1] - 1)]
        rows.append(torch.bincount(routes.reshape(-1), minlength=eng.config.num_experts))
    return torch.stack(rows) if rows else torch.zeros(0, 0, dtype=torch.long)


@torch.no_grad()
def global_expert_shares(model: nn.Module, input_ids: torch.Tensor, group=None) -> torch.Tensor:
    c = expert_token_counts(model, input_ids).double()
    if dist.is_available() and dist.is_initialized() and c.numel():
        dist.all_reduce(c, group=group)
    return c / c.sum(dim=1, keepdim=True).clamp_min(1)


@torch.no_grad()
def global_tr_diagnostics(model: nn.Module, input_ids: torch.Tensor, group=None) -> Dict[str, float]:
    """Load-balance summary: max/min share ratio, coefficient of variation and
    normalised entropy of the expert shares (averaged over layers)."""
    s = global_expert_shares(model, input_ids, group)
    if s.numel() == 0:
        return {}
    E = s.shape[1]
    ent = -(s.clamp_min(1e-12) * s.clamp_min(1e-12).log()).sum(1) / torch.log(torch.tensor(float(E)))
    return {"max_min_ratio": float((s.max(1).values / s.min(1).values.clamp_min(1e-12)).mean()),
            "cv": float((s.std(1) / s.mean(1)).mean()),
            "entropy": float(ent.mean()),
            "max_share": float(s.max())}
