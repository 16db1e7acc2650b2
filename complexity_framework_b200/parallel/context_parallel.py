"""Context (sequence) parallel attention: a sequence too long for one GPU is
split into contiguous chunks, one per rank of ``group``.

The reference bounds sequence length by one device; this adds the two
standard ways to attend across the chunks:

* ``ulysses_attention``: an all-to-all turns [heads, local chunk] into
  [local heads, full sequence], attention runs per head group on the whole
  sequence, a second all-to-all returns to sequence chunks.  Communication is
  4 * (activation size) / P per layer; needs heads divisible by P (K/V heads
  are repeated up to P when there are fewer).
* ``ring_attention``: K/V chunks travel around the ring of ranks (one
  send/receive per step); each rank merges the partial softmax of every chunk
  into its queries with the running max / sum (online softmax).  Causal
  attention skips chunks entirely in the future of the local queries.  In
  backward the K/V chunk travels with its dK/dV accumulators and arrives back
  at its owner after P hops carrying every rank's contribution.

Inputs are head-major ``q [B, Hq, S_local, D]``, ``k/v [B, Hkv, S_local, D]``
(GQA: Hq a multiple of Hkv); rank r holds sequence positions
[r * S_local, (r + 1) * S_local).  On CUDA bf16 the per-block attention runs on
cuDNN's flash kernels (forward returns the block log-sum-exp; backward takes
the global output and log-sum-exp), elsewhere in fp32.  On NCCL the transfers
go over NVLink; the operators are also exercised on gloo ranks.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn.functional as F


def _rank_world(group) -> Tuple[int, int]:
    return dist.get_rank(group), dist.get_world_size(group)


# ------------------------------------------------------------------ Ulysses
def _a2a(x: torch.Tensor, group, scatter_dim: int, gather_dim: int) -> torch.Tensor:
    """Split ``x`` along ``scatter_dim`` into P parts (part j to rank j) and
    concatenate the parts received from ranks 0..P-1 along ``gather_dim``."""
    P = dist.get_world_size(group)
    parts = [c.contiguous() for c in x.chunk(P, scatter_dim)]
    inp = torch.stack(parts)                          # [P, ...]
    out = torch.empty_like(inp)
    dist.all_to_all_single(out, inp, group=group)
    return torch.cat(list(out.unbind(0)), gather_dim)


class _AllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, scatter_dim, gather_dim):
        ctx.group, ctx.dims = group, (scatter_dim, gather_dim)
        return _a2a(x, group, scatter_dim, gather_dim)

    @staticmethod
    def backward(ctx, g):
        s, gdim = ctx.dims
        return _a2a(g.contiguous(), ctx.group, gdim, s), None, None, None


def seq_to_heads(x: torch.Tensor, group) -> torch.Tensor:
    """[B, H, S_local, D] -> [B, H / P, S, D]."""
    return _AllToAll.apply(x, group, 1, 2)


def heads_to_seq(x: torch.Tensor, group) -> torch.Tensor:
    """[B, H / P, S, D] -> [B, H, S_local, D]."""
    return _AllToAll.apply(x, group, 2, 1)


def ulysses_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, group,
                      causal: bool = True, scale: Optional[float] = None) -> torch.Tensor:
    _, P = _rank_world(group)
    Hq, Hkv = q.shape[1], k.shape[1]
    if Hq % P:
        raise ValueError(f"ulysses_attention needs query heads ({Hq}) divisible by {P} ranks")
    if Hkv % P:  # repeat K/V heads so that every rank gets whole groups
        rep = P // math.gcd(Hkv, P)
        k, v = k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1)
    qh, kh, vh = seq_to_heads(q, group), seq_to_heads(k, group), seq_to_heads(v, group)
    o = F.scaled_dot_product_attention(qh, kh, vh, is_causal=causal, scale=scale,
                                       enable_gqa=kh.shape[1] != qh.shape[1])
    return heads_to_seq(o, group)


# --------------------------------------------------------------------- ring
def _ring_pass(tensors, group):
    """Send to rank + 1, receive from rank - 1 (same shapes); returns received."""
    r, P = _rank_world(group)
    nxt, prv = (r + 1) % P, (r - 1) % P
    g_nxt = dist.get_global_rank(group, nxt) if group is not None else nxt
    g_prv = dist.get_global_rank(group, prv) if group is not None else prv
    # contiguous buffers: inputs may be strided views (e.g. head-major q/k/v)
    recv = [torch.empty(t.shape, dtype=t.dtype, device=t.device) for t in tensors]
    ops = [dist.P2POp(dist.isend, t.contiguous(), g_nxt, group) for t in tensors]
    ops += [dist.P2POp(dist.irecv, t, g_prv, group) for t in recv]
    for req in dist.batch_isend_irecv(ops):
        req.wait()
    return recv


def _expand(k: torch.Tensor, groups: int) -> torch.Tensor:
    return k if groups == 1 else k.repeat_interleave(groups, 1)


def _cudnn_blocks(q: torch.Tensor) -> bool:
    """Block attention on cuDNN's flash kernels (they return the log-sum-exp the
    ring merge needs, and their backward takes the global output / LSE)."""
    import os

    return (q.is_cuda and q.dtype in (torch.bfloat16, torch.float16) and q.shape[-1] in (64, 128)
            and os.environ.get("CFB_RING_FP32", "0") != "1")


def _block_forward(q, k, v, causal: bool, scale: float):
    """Attention of q against one K/V chunk: (out fp32 [B, Hq, Sq, D],
    lse fp32 [B, Hq, Sq, 1]); ``causal`` applies the diagonal-block mask."""
    if _cudnn_blocks(q):
        r = torch.ops.aten._scaled_dot_product_cudnn_attention(
            q.contiguous(), k.contiguous(), v.contiguous(), None, True, 0.0, causal, False,
            scale=scale)
        return r[0].float(), r[1].float().reshape(*q.shape[:3], 1)
    G = q.shape[1] // k.shape[1]
    s = q.float() @ _expand(k, G).float().transpose(-1, -2) * scale
    if causal:
        s = s.masked_fill(~torch.ones(s.shape[-2:], dtype=torch.bool, device=s.device).tril(),
                          -math.inf)
    lse = torch.logsumexp(s, -1, keepdim=True)
    return torch.exp(s - lse) @ _expand(v, G).float(), lse


def _block_backward(do, q, k, v, out, lse, causal: bool, scale: float):
    """(dq, dk, dv) of one block given the GLOBAL output and LSE of q's rows
    (so the block's probabilities are exp(s - lse)); dk/dv have K/V's heads."""
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    if _cudnn_blocks(q):
        # undefined sequence-offset tensors select the dense (non-varlen) path;
        # the dropout seeds are read for their device only (dropout 0)
        seed = torch.empty(0, dtype=torch.int64, device=q.device)
        dq, dk, dv = torch.ops.aten._scaled_dot_product_cudnn_attention_backward(
            do.to(q.dtype).contiguous(), q.contiguous(), k.contiguous(), v.contiguous(),
            out.to(q.dtype).contiguous(), lse.reshape(B, Hq, S, 1).contiguous(), seed, seed,
            None, None, None, S, k.shape[2], 0.0, causal, scale=scale)
        return dq.float(), dk.float(), dv.float()
    qf, dof = q.float(), do.float()
    ke, ve = _expand(k, G).float(), _expand(v, G).float()
    s = qf @ ke.transpose(-1, -2) * scale
    if causal:
        s = s.masked_fill(~torch.ones(s.shape[-2:], dtype=torch.bool, device=s.device).tril(),
                          -math.inf)
    p = torch.exp(s - lse)
    delta = (dof * out.float()).sum(-1, keepdim=True)
    ds = p * (dof @ ve.transpose(-1, -2) - delta)
    dq = ds @ ke * scale
    dk = (ds.transpose(-1, -2) @ qf * scale).view(B, Hkv, G, -1, D).sum(2)
    dv = (p.transpose(-1, -2) @ dof).view(B, Hkv, G, -1, D).sum(2)
    return dq, dk, dv


def _chunk_ids(rank: int, P: int, layout: str):
    """Global chunk ids held by ``rank``: contiguous -> [rank] of P chunks;
    zigzag -> [rank, 2P - 1 - rank] of 2P chunks (equal causal work per rank)."""
    return [rank] if layout == "contiguous" else [rank, 2 * P - 1 - rank]


def _pairs(q_ids, k_ids, L: int, causal: bool):
    """(q slice, k slice, diagonal) for every visible (query chunk, key chunk)."""
    out = []
    for i, cq in enumerate(q_ids):
        for j, ck in enumerate(k_ids):
            if causal and ck > cq:
                continue
            out.append((slice(i * L, (i + 1) * L), slice(j * L, (j + 1) * L), causal and ck == cq))
    return out


class _RingAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, group, causal, scale, layout):
        r, P = _rank_world(group)
        B, Hq, S, D = q.shape
        q_ids = _chunk_ids(r, P, layout)
        L = S // len(q_ids)
        lse = torch.full((B, Hq, S, 1), -math.inf, device=q.device)
        acc = torch.zeros(B, Hq, S, D, device=q.device)
        kc, vc = k, v
        for step in range(P):
            src = (r - step) % P
            for qs, ks, diag in _pairs(q_ids, _chunk_ids(src, P, layout), L, causal):
                o_b, lse_b = _block_forward(q[:, :, qs], kc[:, :, ks], vc[:, :, ks], diag, scale)
                new = torch.logaddexp(lse[:, :, qs], lse_b)
                acc[:, :, qs] = (acc[:, :, qs] * torch.exp(lse[:, :, qs] - new)
                                 + o_b * torch.exp(lse_b - new))
                lse[:, :, qs] = new
            if step < P - 1:
                kc, vc = _ring_pass([kc, vc], group)
        out = acc.to(q.dtype)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.group, ctx.causal, ctx.scale, ctx.layout = group, causal, scale, layout
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse = ctx.saved_tensors
        group, causal, scale, layout = ctx.group, ctx.causal, ctx.scale, ctx.layout
        r, P = _rank_world(group)
        q_ids = _chunk_ids(r, P, layout)
        L = q.shape[2] // len(q_ids)
        dq = torch.zeros(q.shape, device=q.device)
        kc, vc = k, v
        dkc = torch.zeros(k.shape, device=k.device)
        dvc = torch.zeros(v.shape, device=v.device)
        for step in range(P):
            src = (r - step) % P
            for qs, ks, diag in _pairs(q_ids, _chunk_ids(src, P, layout), L, causal):
                dq_b, dk_b, dv_b = _block_backward(dout[:, :, qs], q[:, :, qs], kc[:, :, ks],
                                                   vc[:, :, ks], out[:, :, qs], lse[:, :, qs],
                                                   diag, scale)
                dq[:, :, qs] += dq_b
                dkc[:, :, ks] += dk_b
                dvc[:, :, ks] += dv_b
            # the chunk and its gradient move on together; after P hops every
            # chunk is back at its owner with all ranks' contributions
            kc, vc, dkc, dvc = _ring_pass([kc, vc, dkc, dvc], group)
        return dq.to(q.dtype), dkc.to(k.dtype), dvc.to(v.dtype), None, None, None, None


def ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, group,
                   causal: bool = True, scale: Optional[float] = None,
                   layout: str = "contiguous") -> torch.Tensor:
    """``layout`` "zigzag": this rank's sequence is chunks r and 2P-1-r of 2P
    (see ``split_sequence``), balancing causal work over the ranks."""
    if q.shape[1] % k.shape[1]:
        raise ValueError("query heads must be a multiple of key/value heads")
    if layout not in ("contiguous", "zigzag"):
        raise ValueError("layout must be 'contiguous' or 'zigzag'")
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    return _RingAttention.apply(q, k, v, group, causal, scale, layout)


def context_parallel_attention(q, k, v, group, causal: bool = True,
                               scale: Optional[float] = None, method: str = "auto",
                               layout: str = "contiguous"):
    """``method`` "ulysses" when the heads divide over the ranks (fewer, larger
    messages) and the layout is contiguous, "ring" otherwise; ``auto`` picks."""
    P = dist.get_world_size(group)
    if method == "auto":
        method = "ulysses" if (q.shape[1] % P == 0 and layout == "contiguous") else "ring"
    if method == "ulysses":
        if layout != "contiguous":
            raise ValueError("ulysses attention needs the contiguous layout")
        return ulysses_attention(q, k, v, group, causal, scale)
    return ring_attention(q, k, v, group, causal, scale, layout)


def split_sequence(x: torch.Tensor, group, dim: int = 1, layout: str = "contiguous") -> torch.Tensor:
    """This rank's part of ``x`` along ``dim``: chunk r of P (contiguous), or
    chunks r and 2P-1-r of 2P concatenated (zigzag)."""
    r, P = _rank_world(group)
    n = P if layout == "contiguous" else 2 * P
    if x.shape[dim] % n:
        raise ValueError(f"sequence length {x.shape[dim]} not divisible by {n} chunks")
    chunks = x.chunk(n, dim)
    return torch.cat([chunks[c] for c in _chunk_ids(r, P, layout)], dim)


def chunk_positions(seq_len_local: int, group, device=None,
                    layout: str = "contiguous") -> torch.Tensor:
    """Global positions of this rank's part (for RoPE / position embeddings)."""
    r, P = _rank_world(group)
    ids = _chunk_ids(r, P, layout)
    L = seq_len_local // len(ids)
    return torch.cat([torch.arange(c * L, (c + 1) * L, device=device) for c in ids])


def enable_context_parallel(model: torch.nn.Module, group=None, method: str = "auto",
                            layout: str = "contiguous") -> int:
    """Make every attention layer of ``model`` attend across the sequence chunks
    of ``group`` (RoPE at global positions, ring or Ulysses attention); returns
    the number of layers switched.  Feed each rank its chunk of the inputs and
    of the globally shifted labels (``context_parallel_batch``)."""
    n = 0
    for m in model.modules():
        if hasattr(m, "rotary_emb") and hasattr(m, "o_proj") and hasattr(m, "num_kv_heads"):
            m.cp_group = group if group is not None else dist.group.WORLD
            m.cp_method = method
            m.cp_layout = layout
            n += 1
    return n


def context_parallel_batch(input_ids: torch.Tensor, group=None, ignore_index: int = -100,
                           layout: str = "contiguous"):
    """(this rank's input chunk, its next-token labels): labels are shifted over
    the whole sequence before splitting, so a chunk's last position predicts
    the first token of the next rank's chunk."""
    labels = torch.roll(input_ids, -1, dims=1)
    labels[:, -1] = ignore_index
    return (split_sequence(input_ids, group, 1, layout),
            split_sequence(labels, group, 1, layout))
