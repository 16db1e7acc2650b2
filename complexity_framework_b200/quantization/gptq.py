"""GPTQ post-training quantisation (Frantar et al., 2022).

Counterpart of complexity/quantization/gptq.py:22-420.  For each linear layer
the Hessian H = 2 X^T X of its calibration inputs is accumulated, damped, and
the weight columns are quantised left to right (optionally in descending
order of diag(H)); each column's quantisation error is propagated to the
remaining columns through the upper Cholesky factor of H^-1, in blocks.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Iterable, Optional

import torch
import torch.nn as nn

from .quantizer import Linear4bit, Linear8bit, quantize_tensor_groupwise


@dataclass
class GPTQConfig:
    bits: int = 4
    group_size: int = 128
    damp_percent: float = 0.01
    desc_act: bool = True
    sym: bool = True
    block_size: int = 128


class GPTQSolver:
    def __init__(self, layer: nn.Linear):
        self.layer = layer
        self.H = torch.zeros(layer.in_features, layer.in_features, device=layer.weight.device)
        self.n = 0

    def add_batch(self, x: torch.Tensor) -> None:
        x = x.reshape(-1, x.shape[-1]).float()
        m = x.shape[0]
        self.H *= self.n / (self.n + m)
        self.n += m
        x = x * (2.0 / self.n) ** 0.5
        self.H += x.t() @ x

    @torch.no_grad()
    def quantize(self, cfg: GPTQConfig):
        """Returns ``(codes [rows, cols] int8, scale [rows, groups], zero [rows, groups])``.

        Group parameters are fixed up front from the original weight in natural
        column order ("static groups"), so the codes pack directly into the
        group-wise int4/int8 layout even with the descending-activation column
        order.
        """
        W = self.layer.weight.detach().float().clone()
        H = self.H.clone()
        rows, cols = W.shape
        g = cfg.group_size if cfg.group_size > 0 else cols
        _, scale, zero = quantize_tensor_groupwise(W, cfg.bits, g, cfg.sym)
        dead = torch.diag(H) == 0
        H[dead, dead] = 1
        W[:, dead] = 0
        perm = (torch.argsort(torch.diag(H), descending=True) if cfg.desc_act
                else torch.arange(cols, device=W.device))
        W, H = W[:, perm], H[perm][:, perm]
        damp = cfg.damp_percent * torch.mean(torch.diag(H))
        H += torch.eye(cols, device=H.device) * damp
        Hinv = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(H)), upper=True)
        qmax = 2 ** (cfg.bits - 1) - 1 if cfg.sym else 2 ** cfg.bits - 1
        lo, hi = (-qmax - 1, qmax) if cfg.sym else (0, qmax)
        codes = torch.zeros(rows, cols, dtype=torch.int8, device=W.device)
        gidx = perm // g
        for i1 in range(0, cols, cfg.block_size):
            i2 = min(i1 + cfg.block_size, cols)
            W1 = W[:, i1:i2].clone()
            Err = torch.zeros_like(W1)
            Hi = Hinv[i1:i2, i1:i2]
            for j in range(i2 - i1):
                c = i1 + j
                s_, z_ = scale[:, gidx[c]], zero[:, gidx[c]]
                w = W1[:, j]
                k = torch.clamp(torch.round(w / s_) + z_, lo, hi)
                codes[:, perm[c]] = k.to(torch.int8)
                e = (w - (k - z_) * s_) / Hi[j, j]
                W1[:, j:] -= e[:, None] * Hi[j, j:][None, :]
                Err[:, j] = e
            W[:, i2:] -= Err @ Hinv[i1:i2, i2:]
        return codes, scale, zero


@torch.no_grad()
def gptq_quantize_model(model: nn.Module, calibration_data: Optional[Iterable[torch.Tensor]],
                        config: Optional[GPTQConfig] = None, exclude=("lm_head",)) -> nn.Module:
    """Quantise every ``nn.Linear`` with GPTQ using inputs recorded on
    ``calibration_data``; weights are replaced by their quantised values and
    the layer by the packed int4 / int8 module."""
    cfg = config or GPTQConfig()
    solvers: Dict[str, GPTQSolver] = {}
    hooks = []
    for name, m in model.named_modules():
        if isinstance(m, nn.Linear) and not any(e in name for e in exclude):
            solvers[name] = GPTQSolver(m)
            hooks.append(m.register_forward_hook(
                lambda mod, inp, out, n=name: solvers[n].add_batch(inp[0].detach())))
    for b in calibration_data or []:
        model(b)
    for h in hooks:
        h.remove()
    results = {n: s.quantize(cfg) for n, s in solvers.items() if s.n}
    for name, mod in list(model.named_modules()):
        for cname, child in list(mod.named_children()):
            full = f"{name}.{cname}" if name else cname
            if full in results:
                codes, scale, zero = results[full]
                setattr(mod, cname, GPTQLinear(child, codes, scale, zero, cfg))
    return model


class GPTQLinear(nn.Module):
    """Group-wise quantised weight from GPTQ codes (4-bit codes are packed two per byte)."""

    def __init__(self, lin: nn.Linear, codes, scale, zero, cfg: GPTQConfig):
        super().__init__()
        self.in_features, self.out_features = lin.in_features, lin.out_features
        self.bits, self.group_size, self.sym = cfg.bits, cfg.group_size, cfg.sym
        if cfg.bits == 4:
            self.register_buffer("packed", Linear4bit.pack(codes, cfg.sym))
        else:
            self.register_buffer("codes", codes)
        self.register_buffer("scale", scale)
        self.register_buffer("zero", zero)
        self.bias = lin.bias

    def dequantize(self, dtype=torch.float32):
        from .quantizer import dequantize_groupwise

        if self.bits == 4:
            lo = (self.packed & 0xF).to(torch.int16)
            hi = (self.packed >> 4).to(torch.int16)
            q = torch.stack((lo, hi), -1).view(self.out_features, -1)[:, :self.in_features]
            q = q - 8 if self.sym else q
        else:
            q = self.codes
        return dequantize_groupwise(q, self.scale, self.zero, self.group_size, dtype)

    def forward(self, x):
        return torch.nn.functional.linear(x, self.dequantize(x.dtype), self.bias)


QuantizedLinear = GPTQLinear
GPTQQuantizer = GPTQSolver
