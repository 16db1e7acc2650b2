"""Grouped-query / multi-head / multi-query attention.

Parameters and math follow complexity/core/attention/gqa.py:24-347: separate
``k_proj``/``q_proj``/``v_proj``/``o_proj`` Linears (executed as one fused
K|Q|V projection, concatenation order k, q, v), per-head RMSNorm of q and k
before RoPE, rotate-half RoPE, causal attention with scale 1/sqrt(d) (or 1/d
under muP), optional sliding window, tuple KV cache.

On CUDA bf16 without a cache the layer runs the sm_100a path: tcgen05 GEMM
for K|Q|V, one kernel for QK-norm + RoPE + head-major scatter, the attention
kernel without K/V head replication, and the o_proj GEMM with the residual
add fused into its epilogue.  Paged-KV decoding goes through
``inference.paged`` and calls ``forward_paged``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any, Dict, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .layers import RMSNorm, RotaryEmbedding, rotate_half, use_fused
from .registry import register_attention


@dataclass
class AttentionConfig:
    hidden_size: int = 768
    num_attention_heads: int = 12
    num_key_value_heads: Optional[int] = None
    max_position_embeddings: int = 2048
    rope_theta: float = 10000.0
    attention_dropout: float = 0.0
    use_qk_norm: bool = True
    sliding_window: Optional[int] = None
    use_sdpa: bool = True
    is_causal: bool = True
    rope_type: str = "standard"
    rope_fraction: float = 1.0
    use_mup_attn_scale: bool = False
    norm_eps: float = 1e-6
    layer_idx: int = 0
    vocab_size: int = 32000
    extra: Dict[str, Any] = field(default_factory=dict)

    def __post_init__(self):
        if self.num_key_value_heads is None:
            self.num_key_value_heads = self.num_attention_heads


def window_mask(q_len: int, kv_len: int, window: Optional[int], device, dtype) -> torch.Tensor:
    """Additive [1, 1, q, kv] causal mask; queries occupy the last q_len key positions.

    With ``window`` a query at position p sees keys in (p - window, p].
    """
    qpos = torch.arange(kv_len - q_len, kv_len, device=device)[:, None]
    kpos = torch.arange(kv_len, device=device)[None, :]
    ok = kpos <= qpos
    if window is not None:
        ok = ok & (kpos > qpos - window)
    mask = torch.zeros(q_len, kv_len, device=device, dtype=dtype)
    return mask.masked_fill(~ok, float("-inf"))[None, None]


def build_rotary(config: AttentionConfig, head_dim: int) -> nn.Module:
    """Position module for ``rope_type`` / ``rope_fraction`` (registry names:
    standard/rope, partial_rope, yarn, dynamic_ntk, alibi, learned/none)."""
    from . import positions  # noqa: F401  (registers partial_rope / alibi / learned)
    from .registry import POSITION_REGISTRY

    kind = (config.rope_type or "standard").lower()
    L, th = config.max_position_embeddings, config.rope_theta
    if kind in ("learned", "none", "nope"):
        return NoRotary(head_dim, L, th)
    if kind == "alibi":
        return POSITION_REGISTRY.build("alibi", head_dim, L, th,
                                       num_heads=config.num_attention_heads)
    if config.rope_fraction < 1.0 and kind in ("standard", "rope", "partial_rope", "partial"):
        return POSITION_REGISTRY.build("partial_rope", head_dim, L, th,
                                       fraction=config.rope_fraction)
    if kind in ("standard", "rope", "default"):
        return RotaryEmbedding(head_dim, max_seq_len=L, theta=th)
    return POSITION_REGISTRY.build(kind, head_dim, L, th)


class NoRotary(RotaryEmbedding):
    """Identity rotation (absolute learned positions live at the model input)."""

    def rotate(self, q, k, cos, sin):
        return q, k


@register_attention("gqa")
@register_attention("grouped_query")
class GroupedQueryAttention(nn.Module):
    def __init__(self, config: AttentionConfig):
        super().__init__()
        self.config = config
        self.hidden_size = config.hidden_size
        self.num_heads = config.num_attention_heads
        self.num_kv_heads = config.num_key_value_heads
        self.head_dim = config.hidden_size // config.num_attention_heads
        self.num_kv_groups = self.num_heads // self.num_kv_heads
        H, D = self.hidden_size, self.head_dim
        self.q_proj = nn.Linear(H, self.num_heads * D, bias=False)
        self.k_proj = nn.Linear(H, self.num_kv_heads * D, bias=False)
        self.v_proj = nn.Linear(H, self.num_kv_heads * D, bias=False)
        self.o_proj = nn.Linear(self.num_heads * D, H, bias=False)
        self.use_qk_norm = config.use_qk_norm
        if self.use_qk_norm:
            self.q_norm = RMSNorm(D, eps=config.norm_eps)
            self.k_norm = RMSNorm(D, eps=config.norm_eps)
        self.rotary_emb = build_rotary(config, D)
        self.attention_dropout = config.attention_dropout
        self.sliding_window = config.sliding_window
        self.is_causal = config.is_causal
        self.attn_scale = (1.0 / D) if config.use_mup_attn_scale else 1.0 / math.sqrt(D)

    # --------------------------------------------------------------- helpers
    def kqv_weight(self) -> torch.Tensor:
        ws = (self.k_proj.weight, self.q_proj.weight, self.v_proj.weight)
        if self.training or torch.is_grad_enabled():
            return torch.cat(ws, 0)
        # inference: reuse one concatenated copy while the weights are unchanged
        # (keyed on storage and version counter; dropped by train())
        key = tuple((w.data_ptr(), w._version) for w in ws)
        got = getattr(self, "_kqv_cache", None)
        if got is None or got[0] != key:
            got = self._kqv_cache = (key, torch.cat(ws, 0))
        return got[1]

    def train(self, mode: bool = True):
        self._kqv_cache = None
        return super().train(mode)

    def _tp_out(self, o2: torch.Tensor, residual, N: int, fused_ok: bool) -> torch.Tensor:
        """Tensor parallel: residual + all-reduce of this rank's o_proj partial."""
        from ..parallel.tp_inference import tp_reduce_add

        w = self.o_proj.weight

        def partial(out):
            if fused_ok:
                from ..ops import fused

                return fused.gemm_nt(o2, w, None, out=out)
            y = F.linear(o2, w)
            return y if out is None else out.copy_(y)

        y = tp_reduce_add(getattr(self, "tp_decode", None), getattr(self, "tp_site", 0),
                          partial, N, residual, self.tp_group)
        return y.view(1, N, -1)

    def _project(self, x: torch.Tensor):
        kd = self.num_kv_heads * self.head_dim
        qd = self.num_heads * self.head_dim
        if not self._plain_projections():  # quantised / adapted projection modules
            return self.k_proj(x), self.q_proj(x), self.v_proj(x)
        kqv = F.linear(x, self.kqv_weight())
        return kqv.split((kd, qd, kd), -1)

    def _plain_projections(self) -> bool:
        return all(isinstance(getattr(m, "weight", None), torch.Tensor)
                   for m in (self.k_proj, self.q_proj, self.v_proj, self.o_proj))

    def fused_eligible(self, x: torch.Tensor, attention_mask, past_key_value, use_cache) -> bool:
        return (use_fused(x) and self._plain_projections()
                and self.q_proj.weight.dtype == torch.bfloat16
                and attention_mask is None and past_key_value is None and not use_cache
                and self.is_causal and self.sliding_window is None
                and (self.attention_dropout == 0.0 or not self.training)
                and self.head_dim in (64, 128) and self.hidden_size % 32 == 0
                and type(self.rotary_emb) is RotaryEmbedding)

    # --------------------------------------------------------------- forward
    def forward(self, hidden_states: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                past_key_value: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                use_cache: bool = False, residual: Optional[torch.Tensor] = None, **kwargs):
        """Returns ``(out, new_kv)``; ``out`` includes ``residual`` when one is given."""
        tp = getattr(self, "tp_group", None)
        if tp is not None:
            # tensor parallel: local heads, partial o_proj, one all-reduce, then residual
            from ..parallel.tensor_parallel import copy_to_tp, reduce_from_tp

            x = copy_to_tp(hidden_states, tp)
            if self.fused_eligible(x, attention_mask, past_key_value, use_cache):
                out, kv = self._forward_fused(x, None), None
            else:
                out, kv = self._forward_reference(x, attention_mask, past_key_value, use_cache)
            out = reduce_from_tp(out, tp)
            return (out if residual is None else residual + out), kv
        if self.fused_eligible(hidden_states, attention_mask, past_key_value, use_cache):
            return self._forward_fused(hidden_states, residual), None
        out, kv = self._forward_reference(hidden_states, attention_mask, past_key_value, use_cache)
        return (out if residual is None else residual + out), kv

    def _forward_fused(self, x: torch.Tensor, residual: Optional[torch.Tensor]) -> torch.Tensor:
        from ..ops import attention as attn_ops
        from ..ops import fused

        B, S, _ = x.shape
        kqv = fused.linear(x, self.kqv_weight())
        cp = getattr(self, "cp_group", None)
        pos = None
        if cp is not None:  # context parallel: global positions of this rank's chunk
            from ..parallel.context_parallel import chunk_positions

            layout = getattr(self, "cp_layout", "contiguous")
            pos = chunk_positions(S, cp, x.device, layout).to(torch.int32).expand(B, S).contiguous()
            cos, sin = self.rotary_emb.tables(int(pos.max()) + 1, x.device)
        else:
            cos, sin = self.rotary_emb.tables(S, x.device)
        if self.use_qk_norm:
            qw, kw, eps = self.q_norm.weight, self.k_norm.weight, self.q_norm.eps
        else:
            qw = kw = kqv.new_ones(self.head_dim)
            eps = 1e-6
        q, k, v = fused.qk_norm_rope(kqv, qw, kw, cos, sin, pos, self.num_heads,
                                     self.num_kv_heads, self.head_dim, eps, self.use_qk_norm)
        if cp is not None:
            from ..parallel.context_parallel import context_parallel_attention

            o = context_parallel_attention(q, k, v, cp, causal=True, scale=self.attn_scale,
                                           method=getattr(self, "cp_method", "auto"),
                                           layout=getattr(self, "cp_layout", "contiguous"))
            o = o.transpose(1, 2).reshape(B, S, -1)
        else:
            o = attn_ops.attention(q, k, v, causal=True, scale=self.attn_scale)  # [B, S, Hq*D]
        return fused.linear(o, self.o_proj.weight, residual)

    def forward_sp(self, x_shard: torch.Tensor, residual: torch.Tensor, B: int, S: int,
                   ws, name: str) -> torch.Tensor:
        """Fused sequence-parallel TP: ``x_shard`` [T/P, H] -> [T/P, H] (+ residual).

        K|Q|V is an all-gather GEMM (this rank's heads for all T tokens),
        attention runs on full sequences, o_proj is a reduce-scatter GEMM.
        """
        from ..ops import attention as attn_ops
        from ..ops import fused
        from ..parallel.tp_fused import ag_linear, rs_linear

        kqv = ag_linear(x_shard, self.kqv_weight(), ws, name + ".kqv").view(B, S, -1)
        cos, sin = self.rotary_emb.tables(S, x_shard.device)
        if self.use_qk_norm:
            qw, kw, eps = self.q_norm.weight, self.k_norm.weight, self.q_norm.eps
        else:
            qw = kw = kqv.new_ones(self.head_dim)
            eps = 1e-6
        q, k, v = fused.qk_norm_rope(kqv, qw, kw, cos, sin, None, self.num_heads,
                                     self.num_kv_heads, self.head_dim, eps, self.use_qk_norm)
        o = attn_ops.attention(q, k, v, causal=True, scale=self.attn_scale)  # [B, S, Hq_p*D]
        return rs_linear(o.reshape(B * S, -1), self.o_proj.weight, residual, ws, name + ".o")

    def _forward_reference(self, x, attention_mask, past_key_value, use_cache):
        B, S, _ = x.shape
        k, q, v = self._project(x)
        q = q.view(B, S, self.num_heads, self.head_dim).transpose(1, 2)
        k = k.view(B, S, self.num_kv_heads, self.head_dim).transpose(1, 2)
        v = v.view(B, S, self.num_kv_heads, self.head_dim).transpose(1, 2)
        if self.use_qk_norm:
            q = self.q_norm(q)
            k = self.k_norm(k)
        cp = getattr(self, "cp_group", None)
        if cp is not None:
            # context parallel: this rank's chunk starts at rank * S in the sequence
            from ..parallel.context_parallel import chunk_positions, context_parallel_attention

            layout = getattr(self, "cp_layout", "contiguous")
            pos = chunk_positions(S, cp, q.device, layout)
            cos, sin = self.rotary_emb(int(pos.max()) + 1)
            q, k = self.rotary_emb.rotate(q, k, cos[pos].to(q.dtype), sin[pos].to(q.dtype))
            o = context_parallel_attention(q, k, v, cp, causal=True, scale=self.attn_scale,
                                           method=getattr(self, "cp_method", "auto"),
                                           layout=layout)
            o = o.transpose(1, 2).reshape(B, S, self.num_heads * self.head_dim)
            return self.o_proj(o), None
        past = 0 if past_key_value is None else past_key_value[0].shape[2]
        kv_len = past + S
        cos, sin = self.rotary_emb(kv_len)
        cos = cos[past:].to(q.device, q.dtype)
        sin = sin[past:].to(q.device, q.dtype)
        q, k = self.rotary_emb.rotate(q, k, cos, sin)
        if past_key_value is not None:
            k = torch.cat((past_key_value[0], k), 2)
            v = torch.cat((past_key_value[1], v), 2)
        new_kv = (k, v) if use_cache else None
        o = self._core_attention(q, k, v, attention_mask, S, kv_len)
        o = o.transpose(1, 2).reshape(B, S, self.num_heads * self.head_dim)
        return self.o_proj(o), new_kv

    def _core_attention(self, q, k, v, attention_mask, q_len, kv_len):
        if self.num_kv_groups > 1:
            k = k.repeat_interleave(self.num_kv_groups, 1)
            v = v.repeat_interleave(self.num_kv_groups, 1)
        if self.sliding_window is not None and q_len > self.sliding_window:
            mask = window_mask(q_len, kv_len, self.sliding_window, q.device, q.dtype)
        elif not self.is_causal:
            mask = attention_mask
        elif q_len != kv_len and q_len > 1:
            # a multi-token chunk appended to a cache stays causal inside the chunk
            mask = window_mask(q_len, kv_len, self.sliding_window, q.device, q.dtype)
            if attention_mask is not None:
                mask = mask + attention_mask
        else:
            mask = attention_mask
        if getattr(self.rotary_emb, "uses_bias", False):
            bias = self.rotary_emb.bias(q_len, kv_len, q.device, q.dtype)
            if mask is None and self.is_causal:
                mask = window_mask(q_len, kv_len, self.sliding_window, q.device, q.dtype)
            mask = bias if mask is None else mask + bias
        p = self.attention_dropout if self.training else 0.0
        causal = self.is_causal and mask is None and q_len == kv_len
        return F.scaled_dot_product_attention(q, k, v, attn_mask=mask, dropout_p=p,
                                              is_causal=causal, scale=self.attn_scale)

    # ----------------------------------------------------------- paged decode
    def forward_paged(self, hidden_states: torch.Tensor, cache, layer_idx: int,
                      residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Attention over a paged KV cache (``inference.paged.PagedBatch``).

        ``hidden_states`` is [1, N, H] with N = total new tokens of the batch;
        ``cache`` supplies per-token positions, the page tables and the pools.
        """
        x = hidden_states
        N = x.shape[1]
        kd = self.num_kv_heads * self.head_dim
        qd = self.num_heads * self.head_dim
        fused_ok = use_fused(x) and self.q_proj.weight.dtype == torch.bfloat16
        if fused_ok:
            from ..ops import fused

            kqv = fused.linear(x, self.kqv_weight())
        else:
            kqv = F.linear(x, self.kqv_weight())
        if (fused_ok and type(self.rotary_emb) is RotaryEmbedding and self.head_dim in (64, 128)
                and cache.pool.dtype == torch.bfloat16
                and (not self.use_qk_norm or self.q_norm.weight.dtype == torch.bfloat16)):
            # one kernel: qk-norm + RoPE of the new tokens, k/v straight into the pool
            from ..ops._ext import require

            cos_h, sin_h = self.rotary_emb.tables(cache.max_position + 1, x.device)
            q = torch.empty(N, self.num_heads, self.head_dim, device=x.device, dtype=x.dtype)
            norm = self.use_qk_norm
            require().paged_qkv_rope(kqv.view(N, -1), self.q_norm.weight if norm else None,
                                     self.k_norm.weight if norm else None, cos_h, sin_h,
                                     cache.positions, cache.slots, q, cache.pool.k[layer_idx],
                                     cache.pool.v[layer_idx],
                                     float(self.q_norm.eps) if norm else 0.0)
            o = cache.attend(layer_idx, q, self.attn_scale)
            if getattr(self, "tp_group", None) is not None:
                return self._tp_out(o.reshape(N, qd), residual, N, True)
            return fused.linear(o.reshape(1, N, qd), self.o_proj.weight, residual)
        k, q, v = kqv.view(N, -1).split((kd, qd, kd), -1)
        q = q.reshape(N, self.num_heads, self.head_dim)
        k = k.reshape(N, self.num_kv_heads, self.head_dim)
        v = v.reshape(N, self.num_kv_heads, self.head_dim)
        if self.use_qk_norm:
            q = self.q_norm(q.contiguous())
            k = self.k_norm(k.contiguous())
        if getattr(self.rotary_emb, "uses_bias", False):
            raise NotImplementedError("paged decoding does not support ALiBi attention bias")
        cos_h, sin_h = self.rotary_emb.tables(cache.max_position + 1, x.device)
        pos = cache.positions
        c = torch.cat((cos_h[pos], cos_h[pos]), -1)[:, None].to(q.dtype)
        s = torch.cat((sin_h[pos], sin_h[pos]), -1)[:, None].to(q.dtype)
        q, k = self.rotary_emb.rotate(q, k, c, s)
        cache.write(layer_idx, k, v)
        o = cache.attend(layer_idx, q, self.attn_scale)  # [N, Hq, D]
        if getattr(self, "tp_group", None) is not None:
            return self._tp_out(o.reshape(N, qd), residual, N, fused_ok)
        o = o.reshape(1, N, qd)
        if fused_ok:
            from ..ops import fused

            return fused.linear(o, self.o_proj.weight, residual)
        out = self.o_proj(o)
        return out if residual is None else residual + out


@register_attention("mha")
@register_attention("multi_head")
class MultiHeadAttention(GroupedQueryAttention):
    def __init__(self, config: AttentionConfig):
        config.num_key_value_heads = config.num_attention_heads
        super().__init__(config)


@register_attention("mqa")
@register_attention("multi_query")
class MultiQueryAttention(GroupedQueryAttention):
    def __init__(self, config: AttentionConfig):
        config.num_key_value_heads = 1
        super().__init__(config)
