"""Causal-LM losses.

* ``causal_lm_loss``: cross-entropy from logits with optional label smoothing
  and z-loss (complexity/core/losses/causal_lm.py:1-104).
* ``causal_lm_loss_from_hidden`` / ``fused_linear_causal_lm_loss``: CE of
  ``hidden @ W^T`` without materialising all logits.  On CUDA bf16 it is the
  sm_100a fused linear-CE (ops.fused.linear_cross_entropy); elsewhere a chunked
  PyTorch loop with per-chunk recomputation (complexity/core/losses/causal_lm.py:106-191,
  fused_ce.py:95-204).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Tuple

import torch
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint as activation_checkpoint

from .layers import use_fused


@dataclass
class CausalLMLossMetrics:
    ce: float
    z_loss: float
    total: float

    def as_dict(self) -> dict:
        return {"ce": self.ce, "z_loss": self.z_loss, "total": self.total}


def causal_lm_loss(logits: torch.Tensor, labels: torch.Tensor, *, label_smoothing: float = 0.0,
                   z_loss_coef: float = 0.0, ignore_index: int = -100, shift: bool = False,
                   sync_metrics: bool = True) -> Tuple[torch.Tensor, CausalLMLossMetrics]:
    if shift:
        logits = logits[..., :-1, :]
        labels = labels[..., 1:]
    V = logits.shape[-1]
    lf = logits.reshape(-1, V).float()
    lb = labels.reshape(-1)
    ce = F.cross_entropy(lf, lb, ignore_index=ignore_index, label_smoothing=label_smoothing)
    total = ce
    z = torch.zeros((), device=lf.device)
    if z_loss_coef > 0:
        valid = lb != ignore_index
        lse = torch.logsumexp(lf, -1)
        z = z_loss_coef * (lse[valid] ** 2).mean() if bool(valid.any()) else z
        total = ce + z
    if sync_metrics:
        metrics = CausalLMLossMetrics(float(ce.detach()), float(z.detach()), float(total.detach()))
    else:
        metrics = CausalLMLossMetrics(float("nan"), float("nan"), float("nan"))
    return total, metrics


def _chunk_ce(h: torch.Tensor, w: torch.Tensor, y: torch.Tensor, ignore_index: int,
              scale: float) -> torch.Tensor:
    logits = F.linear(h, w).float() * scale
    return F.cross_entropy(logits, y, ignore_index=ignore_index, reduction="sum")


def causal_lm_loss_from_hidden(hidden: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor,
                               *, ignore_index: int = -100, chunk_tokens: int = 8192,
                               logit_scale: float = 1.0, checkpoint_chunks: bool = True
                               ) -> torch.Tensor:
    """Mean CE over labels != ignore_index of ``(hidden @ weight.T) * logit_scale``.

    ``hidden [.., H]`` and ``labels [..]`` are aligned (shift beforehand).
    """
    H = hidden.shape[-1]
    h = hidden.reshape(-1, H)
    y = labels.reshape(-1)
    if (use_fused(h) and weight.dtype == torch.bfloat16 and logit_scale == 1.0
            and weight.shape[0] % 32 == 0 and H % 8 == 0):
        from ..ops.fused import linear_cross_entropy

        return linear_cross_entropy(h, weight, y, ignore_index=ignore_index)
    total = h.new_zeros((), dtype=torch.float32)
    for s in range(0, h.shape[0], chunk_tokens):
        hc, yc = h[s:s + chunk_tokens], y[s:s + chunk_tokens]
        if checkpoint_chunks and torch.is_grad_enabled():
            total = total + activation_checkpoint(_chunk_ce, hc, weight, yc, ignore_index,
                                                  logit_scale, use_reentrant=False)
        else:
            total = total + _chunk_ce(hc, weight, yc, ignore_index, logit_scale)
    return total / (y != ignore_index).sum().clamp_min(1)


def fused_linear_causal_lm_loss(hidden: torch.Tensor, weight: torch.Tensor,
                                labels: torch.Tensor, *, ignore_index: int = -100,
                                shift: bool = True) -> torch.Tensor:
    """Reference-compatible entry: ``hidden[:, :-1]`` predicts ``labels[:, 1:]`` when shift."""
    if shift:
        hidden = hidden[..., :-1, :]
        labels = labels[..., 1:]
    return causal_lm_loss_from_hidden(hidden.contiguous(), weight, labels.contiguous(),
                                      ignore_index=ignore_index)
