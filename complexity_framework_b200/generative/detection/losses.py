"""Detection losses.

Counterparts: complexity/generative/detection/losses.py
(``quality_focal_loss``, ``distribution_focal_loss``) and the CIoU box loss.
Quality focal loss (Li et al., 2020, Generalized Focal Loss) trains the class
score towards the IoU of the predicted box for positives and 0 elsewhere,
weighted by |sigmoid(x) - target|^beta.  Distribution focal loss trains the
box-side distribution over integer bins to put its mass on the two bins
around the continuous target.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def quality_focal_loss(logits: torch.Tensor, target: torch.Tensor,
                       beta: float = 2.0) -> torch.Tensor:
    """``logits``/``target`` [..., C]; target is the soft (IoU) label.  Summed."""
    p = logits.sigmoid()
    bce = F.binary_cross_entropy_with_logits(logits, target, reduction="none")
    return (bce * (p - target).abs().pow(beta)).sum()


def distribution_focal_loss(dist_logits: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """``dist_logits`` [N, bins]; ``target`` [N] continuous in [0, bins - 1].  Per-row."""
    bins = dist_logits.shape[-1]
    t = target.clamp(0, bins - 1 - 1e-3)
    left = t.floor().long()
    right = left + 1
    wl = right.float() - t
    wr = t - left.float()
    logp = F.log_softmax(dist_logits, -1)
    return -(logp.gather(-1, left[:, None]).squeeze(-1) * wl
             + logp.gather(-1, right[:, None]).squeeze(-1) * wr)
