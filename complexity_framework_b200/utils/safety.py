"""Representation-level safety clamps.

Counterpart of complexity/utils/safety.py:43-470: a ``SafetyClamp`` limits
the component of a layer's output along a unit "harm direction" to a
threshold (projecting the excess out), ``MultiDirectionSafetyClamp`` does the
same for several orthonormalised directions, ``ContrastiveSafetyLoss`` trains
a direction from paired activations, and ``install_safety`` / ``remove_safety``
attach clamps to decoder layers as forward hooks with running statistics.
"""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Any, Dict, List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class SafetyConfig:
    threshold: float = 2.0
    layers: Optional[List[int]] = None  # default: last third of the layers
    enabled: bool = True


class SafetyClamp(nn.Module):
    def __init__(self, direction: torch.Tensor, threshold: float = 2.0):
        super().__init__()
        self.register_buffer("direction", F.normalize(direction.float().reshape(-1), dim=0))
        self.threshold = threshold
        self.stats = {"calls": 0, "clamped": 0}

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        d = self.direction.to(h.dtype)
        proj = (h * d).sum(-1, keepdim=True)
        excess = (proj - self.threshold).clamp_min(0)
        self.stats["calls"] += 1
        self.stats["clamped"] += int((excess > 0).sum())
        return h - excess * d


class MultiDirectionSafetyClamp(nn.Module):
    def __init__(self, directions: torch.Tensor, threshold: float = 2.0):
        super().__init__()
        q, _ = torch.linalg.qr(directions.float().t())
        self.register_buffer("basis", q.t().contiguous())  # [k, H] orthonormal rows
        self.threshold = threshold

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        B = self.basis.to(h.dtype)
        proj = h @ B.t()
        excess = (proj - self.threshold).clamp_min(0)
        return h - excess @ B


class ContrastiveSafetyLoss(nn.Module):
    """Learn a direction separating harmful from benign activations (margin loss)."""

    def __init__(self, hidden_size: int, margin: float = 1.0):
        super().__init__()
        self.direction = nn.Parameter(torch.randn(hidden_size) / hidden_size ** 0.5)
        self.margin = margin

    def forward(self, harmful: torch.Tensor, benign: torch.Tensor) -> torch.Tensor:
        d = F.normalize(self.direction, dim=0)
        ph, pb = harmful.float() @ d, benign.float() @ d
        return F.relu(self.margin - (ph.mean() - pb.mean())) + 0.01 * (ph.var() + pb.var())


def _find_layers(model: nn.Module) -> List[nn.Module]:
    layers = getattr(model, "layers", None)
    if layers is None:
        raise ValueError("model has no .layers")
    return list(layers)


def install_safety(model: nn.Module, direction: torch.Tensor,
                   config: Optional[SafetyConfig] = None) -> List[Any]:
    cfg = config or SafetyConfig()
    layers = _find_layers(model)
    idx = cfg.layers if cfg.layers is not None else list(range(2 * len(layers) // 3, len(layers)))
    handles = []
    model._safety_clamps = []
    for i in idx:
        clamp = SafetyClamp(direction.to(next(model.parameters()).device), cfg.threshold)
        model._safety_clamps.append(clamp)

        def hook(mod, inp, out, clamp=clamp):
            if isinstance(out, tuple):
                return (clamp(out[0]),) + tuple(out[1:])
            return clamp(out)

        handles.append(layers[i].register_forward_hook(hook))
    model._safety_handles = handles
    return handles


def remove_safety(model: nn.Module) -> None:
    for h in getattr(model, "_safety_handles", []):
        h.remove()
    model._safety_handles = []


def get_safety_stats(model: nn.Module) -> Dict[str, int]:
    clamps = getattr(model, "_safety_clamps", [])
    return {"layers": len(clamps), "calls": sum(c.stats["calls"] for c in clamps),
            "clamped": sum(c.stats["clamped"] for c in clamps)}


def save_harm_direction(direction: torch.Tensor, path) -> None:
    torch.save({"direction": direction.detach().cpu()}, Path(path))


def load_harm_direction(path, device=None) -> torch.Tensor:
    return torch.load(Path(path), map_location=device or "cpu", weights_only=True)["direction"]


class SafetyCallback:
    """Training callback: logs the clamp statistics every ``log_every`` steps and
    resets them every ``reset_stats_every`` (complexity/utils/safety.py:399-440).
    Works both as a Trainer callback (``on_step_end(trainer, step, loss)``) and
    with the reference's ``on_step_end(metrics)`` call."""

    def __init__(self, model: nn.Module, log_every: int = 100, reset_stats_every: int = 1000):
        self.model, self.log_every, self.reset_stats_every = model, log_every, reset_stats_every
        self.step = 0
        self.history: List[Dict[str, int]] = []

    def on_step_end(self, *args, **kwargs) -> None:
        import logging

        self.step += 1
        if self.step % self.log_every == 0:
            st = get_safety_stats(self.model)
            self.history.append({"step": self.step, **st})
            logging.getLogger(__name__).info("Safety stats at step %d: %s", self.step, st)
        if self.step % self.reset_stats_every == 0:
            for c in getattr(self.model, "_safety_clamps", []):
                for k in c.stats:
                    c.stats[k] = 0
