"""Integer-arithmetic building blocks (INT8 serving research).

Counterpart of complexity/core/integer_ops.py:41-195: per-row symmetric INT8
quantisation of weights and activations, INT8 x INT8 -> INT32 matmul with
per-row/per-channel rescaling (``torch._int_mm`` on CUDA, which runs on the
integer tensor-core path; exact integer arithmetic elsewhere), and 256-entry
lookup-table SiLU / sigmoid / softplus over INT8 inputs.
"""
from __future__ import annotations

from typing import Callable, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


def quantize_int8_rows(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """x [.., K] -> (int8 codes, fp32 scale per row) with x ~= codes * scale."""
    scale = x.float().abs().amax(-1, keepdim=True).clamp_min(1e-12) / 127.0
    q = torch.round(x.float() / scale).clamp(-127, 127).to(torch.int8)
    return q, scale


def int8_matmul(qa: torch.Tensor, sa: torch.Tensor, qw: torch.Tensor, sw: torch.Tensor
                ) -> torch.Tensor:
    """(qa [M, K] int8, sa [M, 1]) x (qw [N, K] int8, sw [N, 1]) -> fp32 [M, N]."""
    if qa.is_cuda and qa.shape[0] > 16 and qa.shape[1] % 8 == 0 and qw.shape[0] % 8 == 0:
        acc = torch._int_mm(qa, qw.t().contiguous())
    else:
        acc = qa.to(torch.int32) @ qw.to(torch.int32).t()
    return acc.float() * sa * sw.view(1, -1)


class Int8Linear(nn.Module):
    """Weights and activations both INT8 (dynamic per-token activation scales)."""

    def __init__(self, lin: nn.Linear):
        super().__init__()
        q, s = quantize_int8_rows(lin.weight.detach())
        self.register_buffer("qw", q)
        self.register_buffer("sw", s)
        self.bias = lin.bias

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shp = x.shape
        qa, sa = quantize_int8_rows(x.reshape(-1, shp[-1]))
        y = int8_matmul(qa, sa, self.qw, self.sw).to(x.dtype)
        if self.bias is not None:
            y = y + self.bias
        return y.view(*shp[:-1], -1)


class LUTActivation(nn.Module):
    """Activation evaluated by table lookup on INT8-quantised inputs in [-clip, clip]."""

    def __init__(self, fn: Callable[[torch.Tensor], torch.Tensor], clip: float = 8.0):
        super().__init__()
        self.clip = clip
        grid = torch.arange(-128, 128, dtype=torch.float32) * (clip / 127.0)
        self.register_buffer("table", fn(grid))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        idx = torch.round(x.float().clamp(-self.clip, self.clip) * (127.0 / self.clip)).long()
        return self.table[idx + 128].to(x.dtype)


def lut_silu(clip: float = 8.0) -> LUTActivation:
    return LUTActivation(F.silu, clip)


def lut_sigmoid(clip: float = 8.0) -> LUTActivation:
    return LUTActivation(torch.sigmoid, clip)


def lut_softplus(clip: float = 8.0) -> LUTActivation:
    return LUTActivation(F.softplus, clip)
