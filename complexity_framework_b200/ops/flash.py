"""Flash attention on the sm_100a kernels.

``flash_attention(q, k, v)``: q [B,Hq,S,D], k/v [B,Hkv,S,D] (head-major bf16,
GQA without K/V replication) -> [B, S, Hq*D] token-major output.  The forward
is ``csrc/flash_fwd.cu``; the backward is ``csrc/flash_bwd.cu`` when built.
"""
from __future__ import annotations

import torch

from ._ext import require


def flash_forward(q, k, v, causal: bool, scale: float):
    C = require()
    B, Hq, S, D = q.shape
    out = torch.empty(B, S, Hq * D, device=q.device, dtype=torch.bfloat16)
    lse = torch.empty(B, Hq, S, device=q.device, dtype=torch.float32)
    C.flash_attn_fwd(q.contiguous(), k.contiguous(), v.contiguous(), out, lse, float(scale),
                     bool(causal))
    return out, lse


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
        C = require()
        B, Hq, S, D = q.shape
        dq = torch.empty_like(q)
        dk = torch.empty_like(k)
        dv = torch.empty_like(v)
        C.flash_attn_bwd(q, k, v, out, lse, dout.contiguous(), dq, dk, dv, float(ctx.scale),
                         bool(ctx.causal))
        return dq, dk, dv, None, None


def backward_available() -> bool:
    C = require()
    return hasattr(C, "flash_attn_bwd")


def flash_attention(q, k, v, *, causal: bool = True, scale: float):
    if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad):
        return FlashAttnFn.apply(q, k, v, causal, scale)
    return flash_forward(q, k, v, causal, scale)[0]
