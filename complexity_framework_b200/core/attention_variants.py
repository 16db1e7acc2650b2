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


# ------------------------------------------------------------- routed Q/O
def routed_projection(x: torch.Tensor, weight: torch.Tensor, sort_idx: torch.Tensor) -> torch.Tensor:
    """Sort-and-split projection: rows of ``x`` taken in ``sort_idx`` order are cut
    into E equal chunks, chunk e is multiplied by ``weight[e]`` ([E, in, out]) and
    the results are scattered back to the original row order.

    Counterpart: complexity/core/triton_kernels.py:262-300 (``routed_proj``).
    One batched GEMM (``torch.bmm`` -> cuBLAS) over the gathered rows.
    """
    shape = x.shape
    flat = x.reshape(-1, shape[-1])
    n, E = flat.shape[0], weight.shape[0]
    if n % E:
        raise ValueError(f"routed projection needs tokens ({n}) divisible by experts ({E})")
    y = torch.bmm(flat[sort_idx].view(E, n // E, -1), weight.to(flat.dtype)).reshape(n, -1)
    out = torch.empty_like(y)
    out[sort_idx] = y
    return out.view(*shape[:-1], -1)


@register_attention("routed_gqa")
@register_attention("sort_split_gqa")
class RoutedGQA(GroupedQueryAttention):
    """GQA whose Q and O projections have E expert weight sets, K/V shared.

    Counterpart: complexity/core/attention/routed_gqa.py:40-171.  With an
    explicit ``sort_idx`` the projections are the counterpart's sort-and-split:
    tokens in ``sort_idx`` order, cut into E equal chunks, chunk e on expert e.
    Without one (the model path), a token's expert is ``token_id % E``, which
    depends on the token alone, so routing is causal and decoding with a cache
    agrees with recomputation (the rank of a token in a sorted batch would let
    later tokens move earlier ones between experts).  Attention itself is full
    causal GQA over all tokens.  The O experts start at zero, as in the
    counterpart, so the layer starts as an identity residual.
    """

    def __init__(self, config: AttentionConfig):
        super().__init__(config)
        self.num_experts = int(config.extra.get("routed_gqa_num_experts", 4))
        H, qd = self.hidden_size, self.num_heads * self.head_dim
        del self.q_proj, self.o_proj
        self.q_proj_w = nn.Parameter(torch.empty(self.num_experts, H, qd))
        self.o_proj_w = nn.Parameter(torch.zeros(self.num_experts, qd, H))
        nn.init.kaiming_uniform_(self.q_proj_w, a=5 ** 0.5)
        self._token_ids: Optional[torch.Tensor] = None
        self._sort_idx: Optional[torch.Tensor] = None

    def fused_eligible(self, *a, **k) -> bool:
        return False

    def set_token_ids(self, token_ids: torch.Tensor) -> None:
        self._token_ids = token_ids

    def _route(self, x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
        if self._sort_idx is not None:
            return routed_projection(x, weight, self._sort_idx)
        ids = self._ids
        flat = x.reshape(-1, x.shape[-1])
        if ids is None:
            return (flat @ weight[0].to(flat.dtype)).view(*x.shape[:-1], -1)
        expert = ids.reshape(-1).to(x.device) % self.num_experts
        out = flat.new_empty(flat.shape[0], weight.shape[-1])
        for e in range(self.num_experts):
            rows = (expert == e).nonzero().squeeze(1)
            out[rows] = flat[rows] @ weight[e].to(flat.dtype)
        return out.view(*x.shape[:-1], -1)

    def kqv_weight(self) -> torch.Tensor:
        raise NotImplementedError("routed_gqa has per-expert Q weights")

    def _project(self, x: torch.Tensor):
        ids = self._token_ids
        n = x.shape[0] * x.shape[1]
        # a decode step sees only the newest tokens' ids
        self._ids = ids[..., -x.shape[1]:] if ids is not None and ids.numel() >= n else None
        if self._ids is not None and self._ids.numel() != n:
            self._ids = None
        return self.k_proj(x), self._route(x, self.q_proj_w), self.v_proj(x)

    def forward(self, hidden_states, attention_mask=None, past_key_value=None, use_cache=False,
                residual=None, sort_idx: Optional[torch.Tensor] = None, **kwargs):
        self._sort_idx = sort_idx
        try:
            return super().forward(hidden_states, attention_mask, past_key_value, use_cache,
                                   residual)
        finally:
            self._sort_idx = None

    def forward_paged(self, *a, **k):
        raise NotImplementedError("routed_gqa decodes with the contiguous KV cache "
                                  "(InferenceEngine cache_type='contiguous' / model.generate)")

    def o_proj(self, o: torch.Tensor) -> torch.Tensor:  # routed output projection
        return self._route(o, self.o_proj_w)


# ------------------------------------------------------------ lexical channels
def _rms(x: torch.Tensor) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + 1e-6)).to(x.dtype)


class _LexicalBase(GroupedQueryAttention):
    """GQA that reads a per-token lexical object vector [B, S, rank].

    The vector is the ``lexical_scale`` keyword when the caller passes one (a
    model-level tied lexical table), else the layer's own zero-initialised
    ``lexical_objects`` table [vocab, rank] looked up by the block's token ids.
    """

    def __init__(self, config: AttentionConfig):
        super().__init__(config)
        self.lexical_object_rank = int(config.extra.get("lexical_object_rank", 16))
        if self.lexical_object_rank <= 0:
            raise ValueError("lexical_object_rank must be positive")
        self.lexical_objects = nn.Embedding(config.vocab_size, self.lexical_object_rank)
        nn.init.zeros_(self.lexical_objects.weight)
        self._token_ids: Optional[torch.Tensor] = None
        self._lex: Optional[torch.Tensor] = None
        self._lex_weight: Optional[torch.Tensor] = None

    def fused_eligible(self, *a, **k) -> bool:
        return False

    def set_token_ids(self, token_ids: torch.Tensor) -> None:
        self._token_ids = token_ids

    def _lexical(self, B: int, S: int) -> torch.Tensor:
        lex = self._lex
        if lex is None:
            if self._token_ids is None or tuple(self._token_ids.shape) != (B, S):
                raise ValueError(f"{type(self).__name__} needs token_ids matching batch and "
                                 "sequence (or a lexical_scale tensor)")
            lex = self.lexical_objects(self._token_ids)
        if tuple(lex.shape) != (B, S, self.lexical_object_rank):
            raise ValueError(f"lexical_scale must be [B, S, {self.lexical_object_rank}], "
                             f"got {tuple(lex.shape)}")
        return lex

    def forward(self, hidden_states, attention_mask=None, past_key_value=None, use_cache=False,
                residual=None, lexical_scale: Optional[torch.Tensor] = None,
                lexical_weight: Optional[torch.Tensor] = None,
                token_ids: Optional[torch.Tensor] = None, **kwargs):
        if token_ids is not None:
            self._token_ids = token_ids
        self._lex, self._lex_weight = lexical_scale, lexical_weight
        try:
            return super().forward(hidden_states, attention_mask, past_key_value, use_cache,
                                   residual)
        finally:
            self._lex = self._lex_weight = None

    def _key_delta(self, B: int, S: int, dtype) -> Optional[torch.Tensor]:
        return None

    def forward_paged(self, *a, **k):
        raise NotImplementedError(f"{type(self).__name__} has no paged decode path (the "
                                  "lexical keys of cached tokens are not stored)")

    def _forward_reference(self, x, attention_mask, past_key_value, use_cache):
        B, S, _ = x.shape
        self._kd = self._key_delta(B, S, x.dtype)
        return super()._forward_reference(x, attention_mask, past_key_value, use_cache)


@register_attention("lexical_gqa")
@register_attention("lexical_bias_gqa")
class LexicalBiasGQA(_LexicalBase):
    """GQA plus a gated lexical score channel: each head's query gains
    ``tanh(gate_h) * rms(Wq_lex x)`` and each key ``rms(Wk_lex (lex + code(id)))``,
    concatenated to the head dimension, V unchanged.

    Counterpart: complexity/core/attention/lexical_gqa.py:13-164.  The softmax
    scale stays 1/sqrt(head_dim) of the base heads, so with the gate at zero
    (its default init) the scores, and the output, are exactly those of GQA.
    ``code(id)`` is a fixed sinusoid of the token id: cos/sin (odd/even
    dimension index d) of (id + 1) * pi * sqrt(d), d = 1..rank.
    """

    def __init__(self, config: AttentionConfig):
        super().__init__(config)
        ex = config.extra
        self.lexical_rank = int(ex.get("lexical_gqa_rank", 16))
        if self.lexical_rank <= 0:
            raise ValueError("lexical_gqa_rank must be positive")
        self.use_token_code = bool(ex.get("lexical_gqa_use_token_code", True))
        self.lexical_q_proj = nn.Linear(self.hidden_size, self.num_heads * self.lexical_rank,
                                        bias=False)
        self.lexical_k_proj = nn.Linear(self.lexical_object_rank,
                                        self.num_kv_heads * self.lexical_rank, bias=False)
        self.lexical_gate = nn.Parameter(torch.full((self.num_heads,),
                                                    float(ex.get("lexical_gqa_gate_init", 0.0))))

    def token_code(self, token_ids: torch.Tensor) -> torch.Tensor:
        d = torch.arange(1, self.lexical_object_rank + 1, device=token_ids.device,
                         dtype=torch.float64)
        ph = (token_ids.double()[..., None] + 1.0) * math.pi * d.sqrt()
        return torch.where(d.long() % 2 == 0, ph.sin(), ph.cos()).float()

    def _forward_reference(self, x, attention_mask, past_key_value, use_cache):
        B, S, _ = x.shape
        lex = self._lexical(B, S)
        if self.use_token_code:
            lex = lex + self.token_code(self._token_ids).to(lex.dtype)
        lq = _rms(self.lexical_q_proj(x).view(B, S, self.num_heads, -1).transpose(1, 2))
        lk = _rms(self.lexical_k_proj(lex.to(x.dtype)).view(B, S, self.num_kv_heads, -1)
                  .transpose(1, 2))
        self._lq = torch.tanh(self.lexical_gate).view(1, -1, 1, 1).to(lq.dtype) * lq
        self._lk = lk
        return super()._forward_reference(x, attention_mask, past_key_value, use_cache)

    def _core_attention(self, q, k, v, attention_mask, q_len, kv_len):
        lk = self._lk
        if k.shape[2] != lk.shape[2]:
            raise ValueError("lexical_gqa: cached decoding is not supported (the lexical keys "
                             "of past tokens are not cached)")
        q = torch.cat((q, self._lq.to(q.dtype)), -1)
        k = torch.cat((k, lk.to(k.dtype)), -1)
        # pad V to the widened head so SDPA accepts it; the extra columns are dropped
        v = F.pad(v, (0, lk.shape[-1]))
        o = super()._core_attention(q, k, v, attention_mask, q_len, kv_len)
        return o[..., :self.head_dim]


class _KeyResidual(_LexicalBase):
    """Adds a per-KV-head gated lexical vector to the keys after QK-norm/RoPE."""

    def __init__(self, config: AttentionConfig):
        super().__init__(config)
        self.lexical_gate = nn.Parameter(torch.full(
            (self.num_kv_heads,), float(config.extra.get("lexical_key_gate_init", 0.05))))

    def _core_attention(self, q, k, v, attention_mask, q_len, kv_len):
        kd = self._kd
        if k.shape[2] != kd.shape[2]:
            raise ValueError(f"{type(self).__name__}: cached decoding is not supported")
        gate = torch.tanh(self.lexical_gate).view(1, -1, 1, 1).to(k.dtype)
        return super()._core_attention(q, k + gate * kd.to(k.dtype), v, attention_mask,
                                       q_len, kv_len)


@register_attention("lexical_key_gqa")
class LexicalKeyGQA(_KeyResidual):
    """Keys gain ``tanh(gate) * rms(lex)`` zero-padded to the head dimension.

    Counterpart: complexity/core/attention/lexical_key_gqa.py:10-60.
    """

    def __init__(self, config: AttentionConfig):
        super().__init__(config)
        if self.lexical_object_rank > self.head_dim:
            raise ValueError("lexical_object_rank cannot exceed the GQA head dimension")

    def _key_delta(self, B, S, dtype):
        lk = F.pad(_rms(self._lexical(B, S)), (0, self.head_dim - self.lexical_object_rank))
        return lk.unsqueeze(1).expand(-1, self.num_kv_heads, -1, -1)


@register_attention("projected_lexical_key_gqa")
class ProjectedLexicalKeyGQA(_KeyResidual):
    """Keys gain ``tanh(gate) * W lex`` (lex optionally weighted per token).

    Counterpart: complexity/core/attention/lexical_key_gqa.py:63-116.
    """

    def __init__(self, config: AttentionConfig):
        super().__init__(config)
        self.lexical_k_proj = nn.Linear(self.lexical_object_rank,
                                        self.num_kv_heads * self.head_dim, bias=False)

    def _key_delta(self, B, S, dtype):
        lex = self._lexical(B, S)
        if self._lex_weight is not None:
            if tuple(self._lex_weight.shape) != (B, S):
                raise ValueError("lexical_weight must be [B, S]")
            lex = lex * self._lex_weight.unsqueeze(-1).to(lex.dtype)
        return self.lexical_k_proj(lex.to(self.lexical_k_proj.weight.dtype)).view(
            B, S, self.num_kv_heads, self.head_dim).transpose(1, 2)


# --------------------------------------------------------- conv + state
def diagonal_decay_scan(u: torch.Tensor, decay: torch.Tensor, s0: torch.Tensor,
                        chunk: int = 64):
    """s_t = decay * s_{t-1} + u_t over dim 1 of u [B, S, H] (decay [H] in (0, 1)).

    Chunked: inside a chunk of C steps the recurrence is one [C, C] lower-
    triangular decay matrix per channel applied with einsum; chunk boundaries
    carry the state sequentially (S / C steps).  Returns (states [B, S, H],
    last state [B, H]), computed in fp32.
    """
    B, S, H = u.shape
    u = u.float()
    ld = decay.float().log()                                    # [H]
    out = []
    s = s0.float()
    for c0 in range(0, S, chunk):
        uc = u[:, c0:c0 + chunk]
        C = uc.shape[1]
        t = torch.arange(C, device=u.device, dtype=torch.float32)
        diff = (t[:, None] - t[None, :])                        # i - j
        w = torch.exp(diff[..., None] * ld).masked_fill((diff < 0)[..., None], 0.0)  # [C,C,H]
        sc = torch.einsum("ijh,bjh->bih", w, uc) + torch.exp((t[:, None] + 1) * ld) * s[:, None]
        out.append(sc)
        s = sc[:, -1]
    return torch.cat(out, 1), s


@register_attention("causal_state_conv")
@register_attention("lexical_object_state")
class CausalStateConvMixer(CausalConvMixer):
    """Gated causal convolution plus a fixed-size diagonal recurrent state.

    Counterpart: complexity/core/attention/causal_state_conv.py:14-123.  The
    local mix c_t (causal depthwise conv of the input) writes into a per-channel
    state with a learned, input-dependent write gate:
    ``s_t = d * s_{t-1} + (1 - d) * sigmoid(up(silu(down(c_t)))) * c_t`` with
    ``d = clamp(sigmoid(b), 0.95, 0.999)``; the output is the gated
    ``o_proj((c + g * s) * sigmoid(gate))``.  The cache is (conv tail, state),
    so decoding one token costs O(H * kernel).
    """

    def __init__(self, config: AttentionConfig):
        super().__init__(config)
        H = config.hidden_size
        rank = int(config.extra.get("causal_state_rank", 16))
        self.state_decay_down = nn.Linear(H, rank, bias=False)
        self.state_decay_up = nn.Linear(rank, H, bias=False)
        # sigmoid(2.944439) = 0.95: the slowest-forgetting end of the clamp starts low
        self.state_decay_bias = nn.Parameter(torch.full((H,), 2.944439))
        self.state_output_gate = nn.Parameter(torch.tensor(0.1))

    def forward(self, hidden_states, attention_mask=None, past_key_value=None, use_cache=False,
                residual=None, **kw):
        B, S, H = hidden_states.shape
        K = self.kernel
        u, g = self.in_proj(hidden_states).chunk(2, -1)
        tail = (past_key_value[0] if past_key_value is not None
                else u.new_zeros(B, K - 1, H))
        s0 = past_key_value[1] if past_key_value is not None else u.new_zeros(B, H)
        ext = torch.cat((tail.to(u.dtype), u), 1)               # [B, K-1+S, H]
        c = F.conv1d(ext.transpose(1, 2), self.conv.weight, self.conv.bias,
                     groups=H).transpose(1, 2)                  # [B, S, H]
        write = torch.sigmoid(self.state_decay_up(F.silu(self.state_decay_down(c))))
        d = torch.sigmoid(self.state_decay_bias.float()).clamp(0.95, 0.999)
        states, s_last = diagonal_decay_scan((1 - d) * write.float() * c.float(), d, s0)
        mixed = c + self.state_output_gate.to(c.dtype) * states.to(c.dtype)
        out = self.o_proj(mixed * torch.sigmoid(g))
        new = (ext[:, -(K - 1):].detach() if K > 1 else ext[:, :0], s_last) if use_cache else None
        return (out if residual is None else residual + out), new


@register_attention("causal_fast_weight_conv")
class CausalFastWeightConvMixer(CausalConvMixer):
    """Gated causal convolution plus a token-addressed fast-weight memory.

    Counterpart: complexity/core/attention/causal_fast_weight_conv.py:22-200.
    The local mix (causal depthwise conv) feeds ``core.associative.
    AssociativeMemory``: addresses from the token ids (and, with a non-zero
    ``causal_contextual_mix_init``, from the local mix), error-correcting
    writes when ``causal_stable_delta``.  The cache is (conv tail, memory
    state, previous address), so decoding one token costs O(H * kernel + r^2).
    """

    def __init__(self, config: AttentionConfig):
        super().__init__(config)
        from .associative import AssociativeMemory

        ex = config.extra
        self.memory = AssociativeMemory(
            config.hidden_size, int(ex.get("causal_state_rank", 16)),
            delta=bool(ex.get("causal_stable_delta", False)),
            contextual_mix_init=float(ex.get("causal_contextual_mix_init", 0.0)),
            output_gate_init=float(ex.get("causal_context_gate_init", 1.0)),
            chunk_size=int(ex.get("causal_delta_chunk_size", 256)))
        self._token_ids: Optional[torch.Tensor] = None

    def set_token_ids(self, token_ids: torch.Tensor) -> None:
        self._token_ids = token_ids

    def forward(self, hidden_states, attention_mask=None, past_key_value=None, use_cache=False,
                residual=None, token_ids: Optional[torch.Tensor] = None, **kw):
        ids = token_ids if token_ids is not None else self._token_ids
        B, S, H = hidden_states.shape
        if ids is None or tuple(ids.shape[-2:]) != (B, S) and ids.shape[-1] < S:
            raise ValueError("causal_fast_weight_conv needs the token ids of its input")
        ids = ids[..., -S:]
        K = self.kernel
        u, g = self.in_proj(hidden_states).chunk(2, -1)
        tail = past_key_value[0] if past_key_value is not None else u.new_zeros(B, K - 1, H)
        ext = torch.cat((tail.to(u.dtype), u), 1)
        c = F.conv1d(ext.transpose(1, 2), self.conv.weight, self.conv.bias,
                     groups=H).transpose(1, 2)
        mem_state = tuple(past_key_value[1:]) if past_key_value is not None else None
        ctx, mem_state = self.memory(c, ids, mem_state)
        out = self.o_proj(c * torch.sigmoid(g)) + ctx.to(c.dtype)
        new = ((ext[:, -(K - 1):].detach() if K > 1 else ext[:, :0],) + tuple(mem_state)
               if use_cache else None)
        return (out if residual is None else residual + out), new


# reference class names (complexity/core/attention/flash_attention.py,
# token_routed_mha.py, token_routed_mha_v2.py)
FlashAttention = FlashGQA
SparseAttention = BlockSparseAttention
TokenRoutedMultiHeadAttention = TokenRoutedMHA
TokenRoutedMultiHeadAttentionV2 = TokenRoutedMHA
