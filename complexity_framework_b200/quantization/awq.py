"""AWQ: activation-aware weight quantisation (Lin et al., 2023).

Counterpart of complexity/quantization/awq.py:23-400.  Per linear layer the
mean input magnitude per channel s_x is measured on calibration data; the
weight columns are scaled by s = s_x^alpha (inputs divided by s, folded into
the layer), with alpha grid-searched to minimise the layer-output error of
the group-wise quantised weight.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Iterable, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .quantizer import dequantize_groupwise, quantize_tensor_groupwise


@dataclass
class AWQConfig:
    bits: int = 4
    group_size: int = 128
    zero_point: bool = True
    grid: int = 20


class AWQLinear(nn.Module):
    """Quantised weight with an input-channel scale ``1/s`` applied to x."""

    def __init__(self, lin: nn.Linear, s: torch.Tensor, cfg: AWQConfig):
        super().__init__()
        W = lin.weight.detach().float() * s[None, :]
        q, sc, z = quantize_tensor_groupwise(W, cfg.bits, cfg.group_size, sym=not cfg.zero_point)
        self.register_buffer("q", q)
        self.register_buffer("qscale", sc)
        self.register_buffer("qzero", z)
        self.register_buffer("inv_s", 1.0 / s)
        self.group_size = cfg.group_size
        self.bias = lin.bias

    def forward(self, x):
        w = dequantize_groupwise(self.q, self.qscale, self.qzero, self.group_size, x.dtype)
        return F.linear(x * self.inv_s.to(x.dtype), w, self.bias)


class AWQQuantizer:
    def __init__(self, config: Optional[AWQConfig] = None):
        self.cfg = config or AWQConfig()

    @torch.no_grad()
    def search_scale(self, lin: nn.Linear, x: torch.Tensor) -> torch.Tensor:
        x = x.reshape(-1, x.shape[-1]).float()
        sx = x.abs().mean(0).clamp_min(1e-6)
        W = lin.weight.detach().float()
        ref = x @ W.t()
        best, best_s = float("inf"), torch.ones_like(sx)
        for i in range(self.cfg.grid + 1):
            a = i / self.cfg.grid
            s = sx.pow(a)
            s = s / (s.max() * s.min()).sqrt()
            q, sc, z = quantize_tensor_groupwise(W * s[None, :], self.cfg.bits,
                                                 self.cfg.group_size, sym=not self.cfg.zero_point)
            Wq = dequantize_groupwise(q, sc, z, self.cfg.group_size) / s[None, :]
            err = float((x @ Wq.t() - ref).pow(2).mean())
            if err < best:
                best, best_s = err, s
        return best_s


@torch.no_grad()
def awq_quantize(model: nn.Module, calibration_data: Optional[Iterable[torch.Tensor]],
                 config: Optional[AWQConfig] = None, exclude=("lm_head",)) -> nn.Module:
    q = AWQQuantizer(config)
    inputs: Dict[str, list] = {}
    hooks = []
    for name, m in model.named_modules():
        if isinstance(m, nn.Linear) and not any(e in name for e in exclude):
            inputs[name] = []
            hooks.append(m.register_forward_hook(
                lambda mod, inp, out, n=name: inputs[n].append(inp[0].detach())))
    for b in calibration_data or []:
        model(b)
    for h in hooks:
        h.remove()
    for name, mod in list(model.named_modules()):
        for cname, child in list(mod.named_children()):
            full = f"{name}.{cname}" if name else cname
            if full in inputs and inputs[full]:
                x = torch.cat([t.reshape(-1, t.shape[-1]) for t in inputs[full]])
                setattr(mod, cname, AWQLinear(child, q.search_scale(child, x), q.cfg))
    return model
