"""Dense SwiGLU MLPs of the registry: ``dense`` and
``dense_deterministic``.

Counterpart of complexity/core/mlp/dense_deterministic.py (+ deterministic_init).
On CUDA bf16 the dense SwiGLU runs the same two fused GEMMs as the TR-Hash
shared path (gate|up GEMM with the SwiGLU epilogue, down GEMM with the
residual add).  ``dense_deterministic`` initialises its weights from a
generator seeded by (seed, layer index), independent of the global RNG, so
two runs build identical models regardless of construction order.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from .layers import use_fused
from .registry import register_mlp


@register_mlp("dense")
class DenseSwiGLU(nn.Module):
    def __init__(self, config):
        super().__init__()
        H = config.hidden_size
        A = int(config.shared_intermediate_size or config.intermediate_size or 4 * H)
        self.gate_proj = nn.Linear(H, A, bias=False)
        self.up_proj = nn.Linear(H, A, bias=False)
        self.down_proj = nn.Linear(A, H, bias=False)
        self.width = A

    def forward(self, hidden_states, token_ids=None, residual=None, **kw):
        x = hidden_states
        if use_fused(x) and x.dtype == torch.bfloat16 and self.width % 256 == 0:
            from ..ops.fused import pack_shared_gate_up, trhash_mlp

            w_gu = pack_shared_gate_up(self.gate_proj.weight, self.up_proj.weight)
            return trhash_mlp(x, w_gu, self.down_proj.weight, None, residual, self.width, 1, 0,
                              1.0)
        out = self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))
        return out if residual is None else residual + out


def deterministic_init(module: nn.Module, seed: int, std: float = 0.02) -> None:
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for p in module.parameters():
            p.copy_(torch.randn(p.shape, generator=g) * std)


@register_mlp("dense_deterministic")
class DeterministicDenseMLP(DenseSwiGLU):
    def __init__(self, config, seed: int = 0x5EED):
        super().__init__(config)
        deterministic_init(self, seed + 1000003 * int(getattr(config, "layer_idx", 0)),
                           float(getattr(config, "initializer_range", 0.02)))
        for m in (self.gate_proj, self.up_proj, self.down_proj):
            m._deterministic_init = True


DenseDeterministicMLP = DeterministicDenseMLP   # reference class name
