"""Flash attention on the sm_100a kernels (``csrc/flash_fwd.cu``, ``csrc/flash_bwd.cu``).

``flash_attention(q, k, v)``: q ``[B, Hq, S, D]``, k/v ``[B, Hkv, S, D]`` bf16
views with a contiguous last dimension (head-major tensors, or the transposed
view of token-major ``[B, S, Hq, D]`` memory that the QK-norm/RoPE kernel
writes; the kernels read either layout in place through 4-D TMA maps) ->
``[B, S, Hq*D]`` token-major output.  GQA without K/V replication.

The backward returns dq in the memory layout of q (token-major q gives a
token-major dq, which the QK-norm/RoPE backward consumes without a copy),
dk/dv head-major like k/v.

Reference counterpart: F.scaled_dot_product_attention and its autograd
backward in complexity/core/attention/gqa.py:229-265.
"""
from __future__ import annotations

import torch

from ._ext import require


def _inner_contiguous(t: torch.Tensor) -> torch.Tensor:
    if t.stride(-1) != 1 or any(t.stride(i) % 8 for i in range(3) if t.size(i) > 1):
        return t.contiguous()
    return t


def flash_forward(q, k, v, causal: bool, scale: float):
    C = require()
    B, Hq, S, D = q.shape
    out = torch.empty(B, S, Hq * D, device=q.device, dtype=torch.bfloat16)
    lse = torch.empty(B, Hq, S, device=q.device, dtype=torch.float32)
    C.flash_attn_fwd(_inner_contiguous(q), _inner_contiguous(k), _inner_contiguous(v), out, lse,
                     float(scale), bool(causal))
    return out, lse


def flash_backward(q, k, v, out, lse, dout, causal: bool, scale: float):
    """Gradients of ``flash_forward``; ``out``/``dout`` are ``[B, S, Hq*D]``."""
    C = require()
    B, Hq, S, D = q.shape
    q = _inner_contiguous(q)
    k = _inner_contiguous(k)
    v = _inner_contiguous(v)
    o4 = out.view(B, S, Hq, D).transpose(1, 2)
    do4 = dout.contiguous().view(B, S, Hq, D).transpose(1, 2)
    if q.stride(1) == D and q.stride(2) == Hq * D:  # token-major q -> token-major dq
        dq = torch.empty(B, S, Hq, D, device=q.device, dtype=torch.bfloat16).transpose(1, 2)
    else:
        dq = torch.empty(B, Hq, S, D, device=q.device, dtype=torch.bfloat16)
    dk = torch.empty(k.shape, device=k.device, dtype=torch.bfloat16)
    dv = torch.empty(k.shape, device=k.device, dtype=torch.bfloat16)
    C.flash_attn_bwd(q, k, v, o4, lse, do4, dq, dk, dv, float(scale), bool(causal))
    return dq, dk, dv


class FlashAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, scale):
        out, lse = flash_forward(q, k, v, causal, scale)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.causal, ctx.scale = causal, scale
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = flash_backward(q, k, v, out, lse, dout, ctx.causal, ctx.scale)
        return dq, dk, dv, None, None


def flash_attention(q, k, v, *, causal: bool = True, scale: float):
    if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad):
        return FlashAttnFn.apply(q, k, v, causal, scale)
    return flash_forward(q, k, v, causal, scale)[0]
