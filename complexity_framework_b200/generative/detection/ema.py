"""Exponential moving average of model weights (counterpart:
complexity/generative/detection/ema.py).  decay ramps as
``decay * (1 - exp(-updates / tau))`` so early averages track the model."""
from __future__ import annotations

import copy
import math

import torch


class ModelEMA:
    def __init__(self, model: torch.nn.Module, decay: float = 0.9999, tau: float = 2000.0):
        self.ema = copy.deepcopy(model).eval()
        for p in self.ema.parameters():
            p.requires_grad_(False)
        self.decay, self.tau, self.updates = decay, tau, 0

    @torch.no_grad()
    def update(self, model: torch.nn.Module) -> None:
        self.updates += 1
        d = self.decay * (1 - math.exp(-self.updates / self.tau))
        msd = model.state_dict()
        for k, v in self.ema.state_dict().items():
            if v.dtype.is_floating_point:
                v.mul_(d).add_(msd[k].detach().to(v.dtype), alpha=1 - d)
            else:
                v.copy_(msd[k])

    def state_dict(self) -> dict:
        return {"ema": self.ema.state_dict(), "updates": self.updates, "decay": self.decay,
                "tau": self.tau}

    def load_state_dict(self, sd: dict) -> None:
        self.ema.load_state_dict(sd["ema"])
        self.updates, self.decay, self.tau = sd["updates"], sd["decay"], sd["tau"]
