"""Learning-rate schedules: warmup then cosine / linear / constant / WSD.

Same schedule names and shapes as complexity/training/scheduler.py:12-113;
implemented as one ``LambdaLR`` multiplier function per schedule.
"""
from __future__ import annotations

import math
from typing import Optional

import torch


def lr_multiplier(step: int, *, kind: str, warmup: int, total: int, min_ratio: float,
                  wsd_decay_ratio: float = 0.2) -> float:
    if warmup > 0 and step < warmup:
        return (step + 1) / warmup
    if kind == "constant":
        return 1.0
    span = max(1, total - warmup)
    t = min(1.0, max(0.0, (step - warmup) / span))
    if kind in ("cosine", "auto"):
        return min_ratio + (1 - min_ratio) * 0.5 * (1 + math.cos(math.pi * t))
    if kind == "linear":
        return min_ratio + (1 - min_ratio) * (1 - t)
    if kind == "wsd":
        decay_steps = max(1, int(round(span * wsd_decay_ratio)))
        stable_end = total - decay_steps
        if step < stable_end:
            return 1.0
        d = min(1.0, (step - stable_end) / decay_steps)
        return min_ratio + (1 - min_ratio) * 0.5 * (1 + math.cos(math.pi * d))
    raise ValueError(f"unknown lr scheduler {kind!r}")


def build_scheduler(optimizer: torch.optim.Optimizer, *, kind: str = "auto", warmup_steps: int = 0,
                    total_steps: int = 1, min_lr_ratio: float = 0.1,
                    wsd_decay_ratio: float = 0.2) -> torch.optim.lr_scheduler.LambdaLR:
    def fn(step: int) -> float:
        return lr_multiplier(step, kind=kind, warmup=warmup_steps, total=total_steps,
                             min_ratio=min_lr_ratio, wsd_decay_ratio=wsd_decay_ratio)

    return torch.optim.lr_scheduler.LambdaLR(optimizer, fn)


# reference entry points (complexity/training/scheduler.py:12-80)
def resolve_scheduler_name(config, model=None) -> str:
    """``auto`` resolves to cosine; any other name is returned unchanged."""
    name = getattr(config, "lr_scheduler", "auto")
    return "cosine" if name == "auto" else name


def get_lr_scheduler(optimizer: torch.optim.Optimizer, config=None,
                     num_training_steps: Optional[int] = None, model=None,
                     scheduler_type: Optional[str] = None,
                     num_warmup_steps: Optional[int] = None):
    """Scheduler from a ``TrainingConfig`` (or from the explicit arguments)."""
    if config is None:
        if num_training_steps is None:
            raise ValueError("num_training_steps is required when config is not provided")
        kind = scheduler_type or "cosine"
        return build_scheduler(optimizer, kind=kind, warmup_steps=num_warmup_steps or 0,
                               total_steps=num_training_steps)
    kind = scheduler_type or resolve_scheduler_name(config, model)
    return build_scheduler(optimizer, kind=kind,
                           warmup_steps=(config.warmup_steps if num_warmup_steps is None
                                         else num_warmup_steps),
                           total_steps=num_training_steps or config.max_steps,
                           min_lr_ratio=getattr(config, "min_lr_ratio", 0.1),
                           wsd_decay_ratio=getattr(config, "wsd_decay_ratio", 0.2))
