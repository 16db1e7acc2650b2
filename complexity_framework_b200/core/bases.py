"""Abstract bases for user-defined attention and MLP modules, and small core
helpers under the reference's names.

Counterparts: complexity/core/attention/base.py:118-180 (``AttentionBase``),
complexity/core/mlp/base.py:182-215 (``MLPBase``),
complexity/core/mlp/deterministic_init.py:37-68
(``deterministic_gaussian_init_``), complexity/core/mlp/fused_activations.py
(``fused_silu_mul``), complexity/core/normalization/norms.py:114-130
(``build_norm``).  A custom module derives from a base, registers with
``register_attention`` / ``register_mlp`` and is then selected by name in
``ModelConfig`` like the built-in ones (which implement the same call
signatures without deriving from these classes).
"""
from __future__ import annotations

from abc import ABC, abstractmethod
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


class AttentionBase(nn.Module, ABC):
    def __init__(self, config):
        super().__init__()
        self.config = config
        self.hidden_size = config.hidden_size
        self.num_heads = config.num_attention_heads
        self.num_kv_heads = config.num_key_value_heads
        self.head_dim = getattr(config, "head_dim", None) or config.hidden_size // self.num_heads
        self.num_kv_groups = self.num_heads // self.num_kv_heads

    @abstractmethod
    def forward(self, hidden_states: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                past_key_value: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                use_cache: bool = False, **kwargs):
        """-> (output [B, S, H], new (k, v) cache or None)."""


class MLPBase(nn.Module, ABC):
    def __init__(self, config):
        super().__init__()
        self.config = config
        self.hidden_size = config.hidden_size
        self.intermediate_size = config.intermediate_size

    def training_control_capabilities(self) -> frozenset:
        return frozenset()

    def training_telemetry(self) -> dict:
        return {}

    @abstractmethod
    def forward(self, hidden_states: torch.Tensor, token_ids: Optional[torch.Tensor] = None,
                **kwargs) -> torch.Tensor:
        """[B, S, H] -> [B, S, H]."""


def deterministic_gaussian_init_(tensor: torch.Tensor, key: int, std: float = 0.02
                                 ) -> torch.Tensor:
    """In-place N(0, std) fill of a 2-D weight from a CPU generator seeded by
    ``key`` (no global RNG state involved; equal keys give equal weights)."""
    if tensor.dim() != 2:
        raise ValueError(f"deterministic_gaussian_init_ expects a 2D tensor, got shape "
                         f"{tuple(tensor.shape)}")
    g = torch.Generator(device="cpu").manual_seed(int(key) & 0x7FFFFFFF)
    w = torch.empty(tensor.shape, dtype=torch.float32).normal_(0.0, std, generator=g)
    with torch.no_grad():
        tensor.copy_(w.to(tensor.device, tensor.dtype))
    return tensor


def fused_silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up (in the models this is fused into the gate|up GEMM)."""
    return F.silu(gate) * up


def build_norm(norm_type: str, hidden_size: int, **kwargs) -> nn.Module:
    from .registry import NORMALIZATION_REGISTRY

    return NORMALIZATION_REGISTRY.build(norm_type, hidden_size, **kwargs)
