"""Causal GQA/MHA attention entry point for the fused path.

``attention(q, k, v)`` takes ``q [B, Hq, S, D]`` (head-major, or the transposed
view of token-major memory), ``k/v [B, Hkv, S, D]`` (no K/V head replication)
and returns ``[B, S, Hq*D]`` token-major output ready for the o_proj GEMM.

On CUDA bf16 with head_dim 64 or 128 it runs the sm_100a flash-attention
kernels, forward and backward; a missing extension on such inputs raises
(no silent library fallback).  Other inputs (CPU, fp32, other head dims) use
PyTorch SDPA with grouped K/V.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def kernel_eligible(q: torch.Tensor) -> bool:
    return q.is_cuda and q.dtype == torch.bfloat16 and q.shape[-1] in (64, 128)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, causal: bool = True,
              scale: float) -> torch.Tensor:
    B, Hq, S, D = q.shape
    if kernel_eligible(q):
        from .flash import flash_attention

        return flash_attention(q, k, v, causal=causal, scale=scale)
    o = F.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=scale,
                                       enable_gqa=k.shape[1] != Hq)
    # a token-major q gives a token-major o: this reshape is then a view
    return o.transpose(1, 2).reshape(B, S, Hq * D)
