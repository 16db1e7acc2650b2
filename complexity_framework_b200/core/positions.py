"""Additional position encodings: partial RoPE, ALiBi, learned absolute.

Counterparts: complexity/core/position/rotary.py:87-237 (partial RoPE),
:300-391 (ALiBi, learned).  ALiBi (Press et al., 2022) adds ``-m_h * (i - j)``
to the attention logits with head slopes m_h = 2^(-8 h / H); the attention
layer asks the position module for that bias.
"""
from __future__ import annotations

import math
from typing import Tuple

import torch
import torch.nn as nn

from .layers import RotaryEmbedding, apply_rotary_pos_emb
from .registry import register_position


@register_position("partial_rope")
@register_position("partial")
class PartialRotaryEmbedding(RotaryEmbedding):
    """RoPE on the first ``fraction`` of each head's dimensions; the rest pass through."""

    def __init__(self, dim: int, max_seq_len: int = 2048, theta: float = 10000.0,
                 fraction: float = 0.5, **kw):
        rot = max(2, int(dim * fraction) // 2 * 2)
        super().__init__(rot, max_seq_len, theta)
        self.full_dim = dim
        self.rot_dim = rot

    def rotate(self, q, k, cos, sin):
        r = self.rot_dim
        qr, kr = apply_rotary_pos_emb(q[..., :r], k[..., :r], cos, sin)
        return torch.cat((qr, q[..., r:]), -1), torch.cat((kr, k[..., r:]), -1)


def alibi_slopes(num_heads: int) -> torch.Tensor:
    def pow2(n):
        start = 2 ** (-8.0 / n)
        return [start ** (i + 1) for i in range(n)]

    if math.log2(num_heads).is_integer():
        return torch.tensor(pow2(num_heads))
    p = 2 ** math.floor(math.log2(num_heads))
    return torch.tensor(pow2(p) + pow2(2 * p)[0::2][: num_heads - p])


@register_position("alibi")
class ALiBiPositionalBias(nn.Module):
    """No rotation; ``bias(q_len, kv_len)`` gives the additive [1, H, q, kv] logits bias."""

    uses_bias = True

    def __init__(self, dim: int, max_seq_len: int = 2048, theta: float = 10000.0,
                 num_heads: int = 1, **kw):
        super().__init__()
        self.register_buffer("slopes", alibi_slopes(num_heads), persistent=False)

    def forward(self, seq_len: int) -> Tuple[torch.Tensor, torch.Tensor]:
        return torch.ones(seq_len, 1), torch.zeros(seq_len, 1)

    def rotate(self, q, k, cos, sin):
        return q, k

    def bias(self, q_len: int, kv_len: int, device, dtype) -> torch.Tensor:
        qpos = torch.arange(kv_len - q_len, kv_len, device=device)[:, None]
        kpos = torch.arange(kv_len, device=device)[None, :]
        dist = (qpos - kpos).clamp_min(0).to(torch.float32)
        return (-self.slopes.to(device)[:, None, None] * dist)[None].to(dtype)


@register_position("learned")
class LearnedPositionalEmbedding(nn.Module):
    """Absolute learned position vectors added to the token embeddings (model level)."""

    def __init__(self, max_seq_len: int, hidden_size: int, **kw):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(max_seq_len, hidden_size))
        nn.init.normal_(self.weight, std=0.02)

    def forward(self, hidden: torch.Tensor, offset: int = 0) -> torch.Tensor:
        S = hidden.shape[1]
        return hidden + self.weight[offset:offset + S].to(hidden.dtype)[None]


# reference class names (complexity/core/position/rotary.py:82-394); the
# rotary ones take the same leading (dim, max_seq_len, theta) arguments
from .layers import DynamicNTKRotaryEmbedding as DynamicNTKRoPE  # noqa: E402
from .layers import RotaryEmbedding as StandardRoPE  # noqa: E402
from .layers import YaRNRotaryEmbedding as YaRNRoPE  # noqa: E402

PartialRoPE = PartialRotaryEmbedding
ALiBiPositionBias = ALiBiPositionalBias
LearnedPositionEmbedding = LearnedPositionalEmbedding
