"""Experimental attention variants of the registry (not part of TR-GQA/TR-MHA).

Counterparts: complexity/core/attention/flash_attention.py:33-676 (flash,
sliding-window, sparse, linear, multiscale), token_routed_mha_v2.py (``tr_mha_v2``)
and causal_conv.py (``causal_conv``).  All share the GQA projections and
QK-norm/RoPE of :class:`GroupedQueryAttention` and differ in the core:

* ``flash``          : causal GQA through the sm_100a attention kernel path
* ``sliding_window`` : local causal window (default 512 when not configured)
* ``sparse``         : block-sparse causal pattern, a local band of blocks plus
                       every ``stride``-th block (strided "summary" blocks)
* ``linear``         : causal kernelised attention, phi(x) = elu(x) + 1,
                       running sums over the sequence (O(S) memory per head)
* ``multiscale``     : head groups with windows w, 4w, 16w ... (last is global)
* ``tr_mha_v2``      : full MHA plus token-routed low-rank Q/V adapters: the
                       token id fixes two candidate experts (route table), a
                       context gate reweights them, up-projections start at zero
* ``causal_conv``    : depthwise causal convolution token mixer with a gate
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .attention import AttentionConfig, GroupedQueryAttention, window_mask
from .registry import register_attention


@register_attention("flash")
class FlashGQA(GroupedQueryAttention):
    """Alias of GQA; the fused path already runs the tcgen05 attention kernels."""


@register_attention("sliding_window")
class SlidingWindowAttention(GroupedQueryAttention):
    def __init__(self, config: AttentionConfig):
        if config.sliding_window is None:
            config.sliding_window = int(config.extra.get("window", 512))
        super().__init__(config)


class _CoreOverride(GroupedQueryAttention):
    """GQA whose reference path uses ``_core`` in place of SDPA (no fused path)."""

    def fused_eligible(self, *a, **k) -> bool:
        return False

    def _core_attention(self, q, k, v, attention_mask, q_len, kv_len):
        if self.num_kv_groups > 1:
            k = k.repeat_interleave(self.num_kv_groups, 1)
            v = v.repeat_interleave(self.num_kv_groups, 1)
        return self._core(q, k, v, q_len, kv_len)


def _masked_softmax_attention(q, k, v, allowed: torch.Tensor, scale: float) -> torch.Tensor:
    s = (q.float() @ k.float().transpose(-1, -2)) * scale
    s = s.masked_fill(~allowed, float("-inf"))
    return (torch.softmax(s, -1) @ v.float()).to(q.dtype)


@register_attention("sparse")
class BlockSparseAttention(_CoreOverride):
    def __init__(self, config: AttentionConfig):
        super().__init__(config)
        self.block = int(config.extra.get("block_size", 64))
        self.local_blocks = int(config.extra.get("local_blocks", 4))
        self.stride = int(config.extra.get("stride", 8))

    def pattern(self, q_len, kv_len, device) -> torch.Tensor:
        qpos = torch.arange(kv_len - q_len, kv_len, device=device)[:, None]
        kpos = torch.arange(kv_len, device=device)[None, :]
        qb, kb = qpos // self.block, kpos // self.block
        local = (qb - kb) < self.local_blocks
        strided = (kb % self.stride) == (self.stride - 1)
        return (kpos <= qpos) & (local | strided)

    def _core(self, q, k, v, q_len, kv_len):
        return _masked_softmax_attention(q, k, v, self.pattern(q_len, kv_len, q.device),
                                         self.attn_scale)


@register_attention("linear")
class LinearAttention(_CoreOverride):
    def _core(self, q, k, v, q_len, kv_len):
        phi_q = F.elu(q.float()) + 1
        phi_k = F.elu(k.float()) + 1
        kv = torch.einsum("bhsd,bhse->bhsde", phi_k, v.float()).cumsum(2)[:, :, -q_len:]
        z = phi_k.cumsum(2)[:, :, -q_len:]
        num = torch.einsum("bhsd,bhsde->bhse", phi_q, kv)
        den = torch.einsum("bhsd,bhsd->bhs", phi_q, z).clamp_min(1e-6)[..., None]
        return (num / den).to(q.dtype)


@register_attention("multiscale")
class MultiScaleAttention(_CoreOverride):
    def __init__(self, config: AttentionConfig):
        super().__init__(config)
        self.base_window = int(config.extra.get("window", 64))
        self.num_scales = int(config.extra.get("num_scales", 3))

    def _core(self, q, k, v, q_len, kv_len):
        H = q.shape[1]
        qpos = torch.arange(kv_len - q_len, kv_len, device=q.device)[:, None]
        kpos = torch.arange(kv_len, device=q.device)[None, :]
        causal = kpos <= qpos
        masks = []
        for h in range(H):
            scale_idx = min(h * self.num_scales // H, self.num_scales - 1)
            if scale_idx == self.num_scales - 1:
                masks.append(causal)
            else:
                w = self.base_window * (4 ** scale_idx)
                masks.append(causal & (kpos > qpos - w))
        allowed = torch.stack(masks)[None]
        return _masked_softmax_attention(q, k, v, allowed, self.attn_scale)


@register_attention("tr_mha_v2")
@register_attention("tr_mha")
class TokenRoutedMHA(GroupedQueryAttention):
    def __init__(self, config: AttentionConfig):
        config.num_key_value_heads = config.num_attention_heads
        super().__init__(config)
        ex = config.extra
        self.E = int(ex.get("tr_mha_num_experts", 4))
        self.r = int(ex.get("tr_mha_adapter_rank", 8))
        self.targets = str(ex.get("tr_mha_targets", "qv"))
        H = config.hidden_size
        from ..tr_hash.routing import mix32

        ids = torch.arange(config.vocab_size, dtype=torch.int64)
        h1 = mix32(ids * 2 + 1 + config.layer_idx * 7919) % self.E
        h2 = (h1 + 1 + mix32(ids * 2 + 2 + config.layer_idx * 7919) % (self.E - 1)) % self.E \
            if self.E > 1 else h1
        self.register_buffer("candidates", torch.stack([h1, h2], 1))
        self.gate = nn.Linear(H, self.E, bias=False)
        nn.init.zeros_(self.gate.weight)
        for t in self.targets:
            out = self.num_heads * self.head_dim
            down = nn.Parameter(torch.randn(self.E, H, self.r) / math.sqrt(H))
            up = nn.Parameter(torch.zeros(self.E, self.r, out))
            self.register_parameter(f"{t}_down", down)
            self.register_parameter(f"{t}_up", up)
        self._token_ids: Optional[torch.Tensor] = None

    def fused_eligible(self, *a, **k) -> bool:
        return False

    def set_token_ids(self, token_ids: torch.Tensor) -> None:
        self._token_ids = token_ids

    def _delta(self, x: torch.Tensor, which: str) -> torch.Tensor:
        ids = self._token_ids
        if ids is None:
            return torch.zeros(x.shape[:-1] + (self.num_heads * self.head_dim,), device=x.device,
                               dtype=x.dtype)
        cand = self.candidates.to(x.device)[ids.clamp(0, self.candidates.shape[0] - 1)]  # [B,S,2]
        logits = self.gate(x).gather(-1, cand)
        w = torch.softmax(logits.float(), -1).to(x.dtype)
        down, up = getattr(self, f"{which}_down"), getattr(self, f"{which}_up")
        out = 0
        for j in range(2):
            e = cand[..., j]
            h = torch.einsum("bsh,bshr->bsr", x, down[e])
            out = out + w[..., j:j + 1] * torch.einsum("bsr,bsro->bso", h, up[e])
        return out

    def _project(self, x: torch.Tensor):
        k, q, v = super()._project(x)
        if "q" in self.targets:
            q = q + self._delta(x, "q")
        if "v" in self.targets:
            v = v + self._delta(x, "v")
        return k, q, v


@register_attention("causal_conv")
class CausalConvMixer(nn.Module):
    """Gated depthwise causal convolution over the sequence (attention-free mixer)."""

    def __init__(self, config: AttentionConfig):
        super().__init__()
        H = config.hidden_size
        self.kernel = int(config.extra.get("causal_conv_kernel_size", 4))
        self.in_proj = nn.Linear(H, 2 * H, bias=False)
        self.conv = nn.Conv1d(H, H, self.kernel, groups=H, padding=self.kernel - 1)
        self.o_proj = nn.Linear(H, H, bias=False)

    def forward(self, hidden_states, attention_mask=None, past_key_value=None, use_cache=False,
                residual=None, **kw):
        S = hidden_states.shape[1]
        u, g = self.in_proj(hidden_states).chunk(2, -1)
        c = self.conv(u.transpose(1, 2))[..., :S].transpose(1, 2)
        out = self.o_proj(c * torch.sigmoid(g))
        return (out if residual is None else residual + out), None
