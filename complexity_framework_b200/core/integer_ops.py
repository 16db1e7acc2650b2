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


# ------------------------------------------------------- reference entry points
# complexity/core/integer_ops.py:41-195: per-row scales returned squeezed
# ([N] / [M]), INT8 codes over the full [-128, 127] range, and Q7 fixed-point
# (value * 128 as int32) activations by table lookup over [-8, 8].
Q7 = 128
_LUT_LO, _LUT_HI = -8 * Q7, 8 * Q7


def quantize_weight_int8(weight: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    s = weight.float().abs().amax(-1, keepdim=True).clamp_min(1e-8) / 127.0
    return (weight.float() / s).round().clamp(-128, 127).to(torch.int8), s.squeeze(-1)


def quantize_activation_int8(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    return quantize_weight_int8(x)


def _int8_mm(x2: torch.Tensor, w_int8: torch.Tensor, w_scale: torch.Tensor) -> torch.Tensor:
    qa, sa = quantize_activation_int8(x2)
    return int8_matmul(qa, sa[:, None], w_int8, w_scale[:, None])


def int8_linear(x: torch.Tensor, weight_int8: torch.Tensor, weight_scale: torch.Tensor,
                bias: torch.Tensor = None) -> torch.Tensor:
    """y = x W^T with dynamically quantised activations (fp32 out)."""
    y = _int8_mm(x.reshape(-1, x.shape[-1]), weight_int8, weight_scale)
    if bias is not None:
        y = y + bias
    return y.reshape(*x.shape[:-1], weight_int8.shape[0])


def int8_fused_gate_up(x: torch.Tensor, fused_int8: torch.Tensor, fused_scale: torch.Tensor,
                       inter_size: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """One INT8 GEMM against stacked [gate; up] rows, split into (gate, up)."""
    y = _int8_mm(x.reshape(-1, x.shape[-1]), fused_int8, fused_scale)
    g, u = y.split(inter_size, -1)
    return g.reshape(*x.shape[:-1], inter_size), u.reshape(*x.shape[:-1], inter_size)


def _q7_table(fn) -> torch.Tensor:
    grid = torch.arange(_LUT_LO, _LUT_HI + 1, dtype=torch.float32) / Q7
    return (fn(grid) * Q7).round().to(torch.int32)


_Q7_TABLES = {"silu": _q7_table(F.silu), "sigmoid": _q7_table(torch.sigmoid),
              "softplus": _q7_table(F.softplus)}


def _q7_lookup(name: str, x_q7: torch.Tensor, above) -> torch.Tensor:
    t = _Q7_TABLES[name].to(x_q7.device)
    r = t[(x_q7.clamp(_LUT_LO, _LUT_HI) - _LUT_LO).long()]
    r = torch.where(x_q7 > _LUT_HI, above(x_q7), r)
    return torch.where(x_q7 < _LUT_LO, torch.zeros_like(r), r)


def silu_integer(x_q7: torch.Tensor) -> torch.Tensor:
    """SiLU of a Q7 tensor (identity above +8, zero below -8)."""
    return _q7_lookup("silu", x_q7, lambda x: x)


def sigmoid_integer(x_q7: torch.Tensor) -> torch.Tensor:
    return _q7_lookup("sigmoid", x_q7, lambda x: torch.full_like(x, Q7))


def softplus_integer(x_q7: torch.Tensor) -> torch.Tensor:
    return _q7_lookup("softplus", x_q7, lambda x: x)


def silu_multiply_integer(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up in Q7 x Q7 = Q14 integer arithmetic, returned as float."""
    g = silu_integer((gate.float() * Q7).round().to(torch.int32))
    u = (up.float() * Q7).round().to(torch.int32)
    return (g * u).float() / (Q7 * Q7)
