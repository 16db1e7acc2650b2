"""Causal GQA/MHA attention entry point for the fused path.

``attention(q, k, v)`` takes ``q [B, Hq, S, D]`` (head-major, or the transposed
view of token-major memory), ``k/v [B, Hkv, S, D]`` (no K/V head replication)
and returns ``[B, S, Hq*D]`` token-major output ready
for the o_proj GEMM.  It dispatches to the sm_100a flash-attention kernel when
the extension provides it, else to PyTorch SDPA with grouped K/V.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import load


def _kernel_available(needs_grad: bool) -> bool:
    C = load()
    if C is None or not hasattr(C, "flash_attn_fwd"):
        return False
    return hasattr(C, "flash_attn_bwd") or not needs_grad


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, causal: bool = True,
              scale: float) -> torch.Tensor:
    B, Hq, S, D = q.shape
    needs_grad = torch.is_grad_enabled() and (q.requires_grad or k.requires_grad
                                              or v.requires_grad)
    if q.shape[-1] in (64, 128) and _kernel_available(needs_grad):
        from .flash import flash_attention

        return flash_attention(q.contiguous(), k, v, causal=causal, scale=scale)
    o = F.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=scale,
                                       enable_gqa=k.shape[1] != Hq)
    # a token-major q gives a token-major o: this reshape is then a view
    return o.transpose(1, 2).reshape(B, S, Hq * D)
