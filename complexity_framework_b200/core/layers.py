"""Normalisation and rotary position layers.

RMSNorm: ``w * (x * rsqrt(mean(x^2) + eps))`` (complexity/core/normalization/norms.py:26-127);
on CUDA bf16 it runs the fused kernel.  RotaryEmbedding keeps the persistent
``inv_freq`` buffer of the checkpoint format and rotate-half RoPE with
cos/sin of ``cat(freqs, freqs)`` (complexity/core/position/rotary.py:17-72);
the fused kernels read the half-width fp32 tables returned by ``tables``.
"""
from __future__ import annotations

import math
from typing import Tuple

import torch
import torch.nn as nn

from .registry import register_normalization, register_position


def use_fused(x: torch.Tensor) -> bool:
    """Whether an activation is eligible for the sm_100a kernels."""
    return x.is_cuda and x.dtype == torch.bfloat16


@register_normalization("rmsnorm")
@register_normalization("rms")
@register_normalization("llama")
class RMSNorm(nn.Module):
    def __init__(self, hidden_size: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.eps = eps
        self.hidden_size = hidden_size

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if use_fused(x) and self.weight.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0:
            from ..ops.fused import rmsnorm

            return rmsnorm(x, self.weight, self.eps)
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return self.weight * y.to(x.dtype)

    def forward_with_skip(self, x: torch.Tensor):
        """``(norm(x), x)`` where gradients of both outputs are summed in one kernel."""
        if use_fused(x) and self.weight.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0:
            from ..ops.fused import rmsnorm_skip

            return rmsnorm_skip(x, self.weight, self.eps)
        return self(x), x

    def extra_repr(self) -> str:
        return f"{self.hidden_size}, eps={self.eps}"


@register_normalization("layernorm")
class LayerNorm(nn.LayerNorm):
    def __init__(self, hidden_size: int, eps: float = 1e-6):
        super().__init__(hidden_size, eps=eps)


@register_normalization("identity")
class IdentityNorm(nn.Module):
    def __init__(self, hidden_size: int = 0, eps: float = 0.0):
        super().__init__()

    def forward(self, x):
        return x


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), -1)


def apply_rotary_pos_emb(q, k, cos, sin):
    """Rotate-half RoPE on [B, H, S, D] tensors with cos/sin of shape [S, D]
    (or any cos/sin already broadcastable against q and k)."""
    if cos.dim() == 2:
        cos = cos[None, None]
        sin = sin[None, None]
    return q * cos + rotate_half(q) * sin, k * cos + rotate_half(k) * sin


@register_position("rope")
@register_position("standard")
class RotaryEmbedding(nn.Module):
    """Rotate-half RoPE.  ``inv_freq`` is the persistent checkpoint buffer; the
    cos/sin caches are fp32 plain attributes built from an fp32 copy of the
    frequencies, so casting the module to bf16 does not degrade positions."""

    def __init__(self, dim: int, max_seq_len: int = 2048, theta: float = 10000.0,
                 scaling: float = 1.0):
        super().__init__()
        self.dim = dim
        self.max_seq_len = max_seq_len
        self.theta = theta
        self.scaling = scaling
        with torch.device("cpu"):  # host copy, also under a meta default device
            inv = 1.0 / (theta ** (torch.arange(0, dim, 2).float() / dim))
            self._inv32 = inv.clone()
        self.register_buffer("inv_freq", inv)
        self._cos: torch.Tensor = torch.empty(0)
        self._sin: torch.Tensor = torch.empty(0)
        self._mscale = 1.0

    def set_inv_freq(self, inv: torch.Tensor) -> None:
        self._inv32 = inv.detach().float().cpu().clone()
        with torch.no_grad():
            self.inv_freq.copy_(inv.to(self.inv_freq.dtype))
        self._cos = torch.empty(0)

    def _build_cache(self, n: int, device) -> None:
        t = torch.arange(n, dtype=torch.float32) / self.scaling
        freqs = torch.outer(t, self._inv32)
        self._cos = (freqs.cos() * self._mscale).to(device)
        self._sin = (freqs.sin() * self._mscale).to(device)

    def tables(self, n: int, device=None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Half-width fp32 (cos, sin) tables [P, dim/2] covering positions [0, n)."""
        device = self.inv_freq.device if device is None else device
        if self._cos.shape[0] < n or self._cos.device != torch.device(device):
            self.max_seq_len = max(n, self.max_seq_len)
            self._build_cache(self.max_seq_len, device)
        return self._cos, self._sin

    def forward(self, seq_len: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Full-width cos/sin of shape [seq_len, dim]."""
        c, s = self.tables(seq_len)
        c, s = c[:seq_len], s[:seq_len]
        return torch.cat((c, c), -1), torch.cat((s, s), -1)

    def rotate(self, q, k, cos, sin):
        return apply_rotary_pos_emb(q, k, cos, sin)


@register_position("dynamic_ntk")
class DynamicNTKRotaryEmbedding(RotaryEmbedding):
    """NTK-aware base rescaling once the sequence outgrows the trained length."""

    def __init__(self, dim: int, max_seq_len: int = 2048, theta: float = 10000.0,
                 scaling_factor: float = 1.0):
        super().__init__(dim, max_seq_len, theta)
        self.trained_len = max_seq_len
        self.scaling_factor = scaling_factor

    def _build_cache(self, n: int, device) -> None:
        if n > self.trained_len:
            base = self.theta * ((self.scaling_factor * n / self.trained_len)
                                 - (self.scaling_factor - 1)) ** (self.dim / (self.dim - 2))
            self._inv32 = 1.0 / (base ** (torch.arange(0, self.dim, 2).float() / self.dim))
        super()._build_cache(n, device)


@register_position("yarn")
class YaRNRotaryEmbedding(RotaryEmbedding):
    """YaRN (arXiv:2309.00071): per-frequency interpolation ramp plus attention temperature."""

    def __init__(self, dim: int, max_seq_len: int = 2048, theta: float = 10000.0,
                 scale: float = 1.0, original_max_position: int = 2048, beta_fast: float = 32.0,
                 beta_slow: float = 1.0):
        super().__init__(dim, max_seq_len, theta)
        if scale > 1.0:
            idx = torch.arange(0, dim, 2).float()
            wavelen = 2 * math.pi * (theta ** (idx / dim))
            ratio = original_max_position / wavelen
            ramp = ((ratio - beta_slow) / (beta_fast - beta_slow)).clamp(0, 1)
            inv = 1.0 / (theta ** (idx / dim))
            self.set_inv_freq(inv / scale * (1 - ramp) + inv * ramp)
            self._mscale = 0.1 * math.log(scale) + 1.0
