"""Paged KV cache.

Memory: one pool per layer of ``num_pages`` pages, each page holding
``page_size`` tokens of K and V for all KV heads:
``k_pool[layer] : [num_pages, page_size, Hkv, D]`` (bf16 on GPU).  A sequence
owns a list of pages; the page table maps logical block i of a sequence to a
physical page.  Pages are allocated once per sequence for all layers (the
reference allocated per layer while its pool held all layers) and attention reads the pages in place instead of gathering them into
a new tensor per token (reference kv_cache.py:295-308).

A forward step processes a ragged batch of new tokens (prefill chunks and
single decode tokens of several sequences concatenated, N tokens total).
``PagedBatch`` carries the per-token positions and write slots and the
per-sequence page tables; ``write`` scatters the new K/V into the pools and
``attend`` runs causal attention of each sequence's new queries over all of
its cached keys.  On CUDA ``attend`` calls the sm_100a paged-attention kernel;
elsewhere a PyTorch gather + SDPA reference.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import torch
import torch.nn.functional as F


class OutOfPages(RuntimeError):
    pass


class PagePool:
    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, num_pages: int,
                 page_size: int = 16, dtype=torch.bfloat16, device="cpu"):
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.num_pages = num_pages
        self.page_size = page_size
        self.dtype = dtype
        self.device = torch.device(device)
        shape = (num_layers, num_pages, page_size, num_kv_heads, head_dim)
        self.k = torch.zeros(shape, dtype=dtype, device=self.device)
        self.v = torch.zeros(shape, dtype=dtype, device=self.device)
        self.free: List[int] = list(range(num_pages - 1, -1, -1))
        self.pages: Dict[int, List[int]] = {}
        self.lengths: Dict[int, int] = {}

    # ------------------------------------------------------------ bookkeeping
    def allocate_sequence(self, seq_id: int) -> None:
        if seq_id in self.pages:
            raise ValueError(f"sequence {seq_id} already allocated")
        self.pages[seq_id] = []
        self.lengths[seq_id] = 0

    def free_sequence(self, seq_id: int) -> None:
        for p in self.pages.pop(seq_id, []):
            self.free.append(p)
        self.lengths.pop(seq_id, None)

    def reset(self) -> None:
        for sid in list(self.pages):
            self.free_sequence(sid)

    def reserve(self, seq_id: int, new_tokens: int) -> None:
        """Make room for ``new_tokens`` more tokens of ``seq_id`` (raises OutOfPages)."""
        need = self.lengths[seq_id] + new_tokens
        pages = self.pages[seq_id]
        while len(pages) * self.page_size < need:
            if not self.free:
                raise OutOfPages("KV page pool exhausted")
            pages.append(self.free.pop())

    def can_reserve(self, seq_id: Optional[int], length_after: int, current: int = 0) -> bool:
        have = len(self.pages.get(seq_id, [])) if seq_id is not None else 0
        need = -(-length_after // self.page_size) - have
        return need <= len(self.free)

    def fork_sequence(self, src: int, dst: int) -> None:
        """New sequence ``dst`` with a copy of ``src``'s cached tokens (beam search).

        Full pages are copied whole; the copy is one gather/scatter per pool.
        """
        if dst in self.pages:
            self.free_sequence(dst)
        self.allocate_sequence(dst)
        n = self.lengths[src]
        self.reserve(dst, n)
        k = -(-n // self.page_size)
        if k:
            s_idx = torch.tensor(self.pages[src][:k], device=self.device)
            d_idx = torch.tensor(self.pages[dst][:k], device=self.device)
            self.k[:, d_idx] = self.k[:, s_idx]
            self.v[:, d_idx] = self.v[:, s_idx]
        self.lengths[dst] = n

    def truncate_sequence(self, seq_id: int, length: int) -> None:
        """Drop cached tokens past ``length`` (speculative-decoding rollback);
        pages beyond the new length go back to the free list."""
        length = max(0, min(length, self.lengths[seq_id]))
        self.lengths[seq_id] = length
        keep = -(-length // self.page_size)
        pages = self.pages[seq_id]
        while len(pages) > keep:
            self.free.append(pages.pop())

    def memory_usage(self) -> Dict[str, float]:
        used = self.num_pages - len(self.free)
        per_page = 2 * self.num_layers * self.page_size * self.num_kv_heads * self.head_dim * \
            self.k.element_size()
        return {"pages_used": used, "pages_total": self.num_pages,
                "gb_used": used * per_page / 1e9, "gb_total": self.num_pages * per_page / 1e9}

    def get_seq_len(self, seq_id: int) -> int:
        return self.lengths[seq_id]


@dataclass
class SeqChunk:
    seq_id: int
    start: int      # position of the first new token
    length: int     # number of new tokens


class PagedBatch:
    """Per-step view of the pool for a ragged batch of new tokens."""

    def __init__(self, pool: PagePool, chunks: Sequence[SeqChunk]):
        self.pool = pool
        self.chunks = list(chunks)
        dev = pool.device
        pos, slots, seq_of_tok = [], [], []
        for i, c in enumerate(self.chunks):
            pool.reserve(c.seq_id, c.start + c.length - pool.lengths[c.seq_id])
            pages = pool.pages[c.seq_id]
            for t in range(c.start, c.start + c.length):
                pos.append(t)
                slots.append(pages[t // pool.page_size] * pool.page_size + t % pool.page_size)
                seq_of_tok.append(i)
        self.num_tokens = len(pos)
        self.positions = torch.tensor(pos, dtype=torch.long, device=dev)
        self.slots = torch.tensor(slots, dtype=torch.long, device=dev)
        self.max_position = max(pos) if pos else 0
        cu = [0]
        for c in self.chunks:
            cu.append(cu[-1] + c.length)
        self.cu_q = torch.tensor(cu, dtype=torch.int32, device=dev)
        self.kv_lens = torch.tensor([c.start + c.length for c in self.chunks], dtype=torch.int32,
                                    device=dev)
        max_pages = max(len(pool.pages[c.seq_id]) for c in self.chunks) if self.chunks else 1
        table = torch.zeros(len(self.chunks), max(1, max_pages), dtype=torch.int32)
        for i, c in enumerate(self.chunks):
            pg = pool.pages[c.seq_id]
            table[i, :len(pg)] = torch.tensor(pg, dtype=torch.int32)
        self.page_table = table.to(dev)
        self._cu_host = cu
        # chunks that start a sequence run dense causal flash attention over the
        # chunk itself; the others (decode tokens, continued prefill) read pages
        self.fresh = [i for i, c in enumerate(self.chunks) if c.start == 0 and c.length > 1]
        paged = [i for i in range(len(self.chunks)) if i not in set(self.fresh)]
        self.paged = paged
        tok_idx, pcu = [], [0]
        for i in paged:
            tok_idx.extend(range(cu[i], cu[i + 1]))
            pcu.append(pcu[-1] + self.chunks[i].length)
        self.paged_tokens = torch.tensor(tok_idx, dtype=torch.long, device=dev)
        self.paged_cu = torch.tensor(pcu, dtype=torch.int32, device=dev)
        sel = torch.tensor(paged, dtype=torch.long)
        self.paged_table = table[sel].contiguous().to(dev) if paged else None
        self.paged_kv_lens = (torch.tensor([self.chunks[i].start + self.chunks[i].length
                                            for i in paged], dtype=torch.int32, device=dev))

    def commit(self) -> None:
        """Advance the recorded sequence lengths after the forward step."""
        for c in self.chunks:
            self.pool.lengths[c.seq_id] = max(self.pool.lengths[c.seq_id], c.start + c.length)

    # ---------------------------------------------------------------- compute
    def write(self, layer: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """k, v: [N, Hkv, D] for the N new tokens."""
        P = self.pool
        kf = P.k[layer].view(-1, P.num_kv_heads, P.head_dim)
        vf = P.v[layer].view(-1, P.num_kv_heads, P.head_dim)
        kf.index_copy_(0, self.slots, k.to(P.dtype))
        vf.index_copy_(0, self.slots, v.to(P.dtype))

    def attend(self, layer: int, q: torch.Tensor, scale: float) -> torch.Tensor:
        """Causal attention of q [N, Hq, D] over each sequence's cached keys -> [N, Hq, D]."""
        from ..ops._ext import load

        C = load()
        P = self.pool
        D = q.shape[-1]
        if not (q.is_cuda and C is not None and hasattr(C, "paged_attention")
                and q.dtype == torch.bfloat16 and P.dtype == torch.bfloat16 and D in (64, 128)):
            return self._attend_reference(layer, q, scale)
        from ..ops.flash import flash_forward

        out = torch.empty_like(q)
        Hq, Hkv = q.shape[1], P.num_kv_heads
        for i in self.fresh:
            a, e = self._cu_host[i], self._cu_host[i + 1]
            # the chunk's own K/V were just written; take them from the pool slots
            slots = self.slots[a:e]
            kf = P.k[layer].view(-1, Hkv, D).index_select(0, slots)
            vf = P.v[layer].view(-1, Hkv, D).index_select(0, slots)
            o, _ = flash_forward(q[a:e].transpose(0, 1)[None].contiguous(),
                                 kf.transpose(0, 1)[None].contiguous(),
                                 vf.transpose(0, 1)[None].contiguous(), True, scale)
            out[a:e] = o.view(e - a, Hq, D)
        if self.paged and not self.fresh:  # every token reads pages: no gather/scatter
            C.paged_attention(q.contiguous(), P.k[layer], P.v[layer], self.paged_table,
                              self.paged_cu, self.paged_kv_lens, out, float(scale),
                              int(self.max_q_len()))
        elif self.paged:
            qs = q.index_select(0, self.paged_tokens).contiguous()
            os_ = torch.empty_like(qs)
            C.paged_attention(qs, P.k[layer], P.v[layer], self.paged_table, self.paged_cu,
                              self.paged_kv_lens, os_, float(scale), int(self.max_q_len()))
            out.index_copy_(0, self.paged_tokens, os_)
        return out

    def max_q_len(self) -> int:
        return max((c.length for c in self.chunks), default=1)

    def _attend_reference(self, layer: int, q: torch.Tensor, scale: float) -> torch.Tensor:
        P = self.pool
        out = torch.empty_like(q)
        Hq, Hkv = q.shape[1], P.num_kv_heads
        for i, c in enumerate(self.chunks):
            kv_len = c.start + c.length
            pages = P.pages[c.seq_id][: -(-kv_len // P.page_size)]
            idx = torch.tensor(pages, device=q.device)
            k = P.k[layer][idx].reshape(-1, Hkv, P.head_dim)[:kv_len]
            v = P.v[layer][idx].reshape(-1, Hkv, P.head_dim)[:kv_len]
            qs = q[self._cu_host[i]:self._cu_host[i + 1]]
            qh = qs.transpose(0, 1)[None].float()
            kh = k.transpose(0, 1)[None].float()
            vh = v.transpose(0, 1)[None].float()
            if Hq != Hkv:
                kh = kh.repeat_interleave(Hq // Hkv, 1)
                vh = vh.repeat_interleave(Hq // Hkv, 1)
            qpos = torch.arange(c.start, kv_len, device=q.device)[:, None]
            kpos = torch.arange(kv_len, device=q.device)[None, :]
            mask = torch.zeros(c.length, kv_len, device=q.device)
            mask = mask.masked_fill(kpos > qpos, float("-inf"))
            o = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=mask, scale=scale)
            out[self._cu_host[i]:self._cu_host[i + 1]] = o[0].transpose(0, 1).to(q.dtype)
        return out


class StaticDecodeBatch(PagedBatch):
    """A decode-only batch of ``size`` sequences (one new token each) whose
    device tensors never move, so a forward over it can be captured in a CUDA
    graph once and replayed every step.

    All per-step inputs (token ids, positions, cache slots, kv lengths, page
    table rows) live in ONE int32 device buffer, refilled from a pinned host
    buffer by a single copy.  A row keeps its sequence while that sequence runs,
    so the host only appends a page id when a sequence crosses a page boundary.
    Rows past the live requests are padding: they attend over one scratch page
    reserved at construction and write their K/V there.
    """

    SCRATCH_SEQ = -1

    def __init__(self, pool: PagePool, size: int, max_pages: int, max_position: int):
        self.pool = pool
        self.size, self.max_pages = size, max_pages
        dev = pool.device
        if self.SCRATCH_SEQ not in pool.pages:
            pool.allocate_sequence(self.SCRATCH_SEQ)
            pool.reserve(self.SCRATCH_SEQ, 1)
        self.scratch_page = pool.pages[self.SCRATCH_SEQ][0]
        B = size
        # layout: ids | positions | slots | kv_lens | page table [size, max_pages]
        n = B * (4 + max_pages)
        self.host = torch.zeros(n, dtype=torch.int32).pin_memory()
        self._h = self.host.numpy()
        self.dev = torch.zeros(n, dtype=torch.int32, device=dev)
        self.ids32 = self.dev[0:B]
        self._pos32 = self.dev[B:2 * B]
        self._slots32 = self.dev[2 * B:3 * B]
        self.paged_kv_lens = self.dev[3 * B:4 * B]
        self.paged_table = self.dev[4 * B:].view(B, max_pages)
        self.page_table, self.kv_lens = self.paged_table, self.paged_kv_lens
        self.max_position = max_position
        self.num_tokens = B
        self.chunks = [SeqChunk(-1, 0, 1) for _ in range(B)]
        self.fresh, self.paged = [], list(range(B))
        self._cu_host = list(range(B + 1))
        self.paged_tokens = torch.arange(B, dtype=torch.long, device=dev)
        self.paged_cu = torch.arange(B + 1, dtype=torch.int32, device=dev)
        self.cu_q = self.paged_cu
        # long index tensors the model reads (filled from the int32 buffer by
        # ``expand``, a device op that a captured graph replays)
        self.positions = torch.zeros(B, dtype=torch.long, device=dev)
        self.slots = torch.zeros(B, dtype=torch.long, device=dev)
        self.ids = torch.zeros(B, dtype=torch.long, device=dev)
        self._row_seq = [None] * B   # sequence of each row
        self._row_pages = [0] * B    # pages of that sequence already in the table row
        self._live = []
        for i in range(B):
            self._set_padding(i)

    def _set_padding(self, i: int) -> None:
        B, mp, h = self.size, self.max_pages, self._h
        P = self.pool
        h[4 * B + i * mp:4 * B + (i + 1) * mp] = 0
        h[4 * B + i * mp] = self.scratch_page
        h[i] = 0
        h[B + i] = 0
        h[2 * B + i] = self.scratch_page * P.page_size
        h[3 * B + i] = 1
        self._row_seq[i] = None
        self._row_pages[i] = 0

    def expand(self) -> None:
        self.positions.copy_(self._pos32)
        self.slots.copy_(self._slots32)
        self.ids.copy_(self.ids32)

    def fill(self, entries) -> None:
        """``entries[i] = (seq_id, token, position)`` for row i (at most ``size``
        live rows, the rest padding): reserves the page each new token lands on
        and stages every input with one host-to-device copy."""
        P = self.pool
        B, mp, h = self.size, self.max_pages, self._h
        if len(entries) > B:
            raise ValueError(f"{len(entries)} requests for a decode batch of {B}")
        if self.SCRATCH_SEQ not in P.pages:  # the pool was reset: take a new scratch page
            P.allocate_sequence(self.SCRATCH_SEQ)
            P.reserve(self.SCRATCH_SEQ, 1)
            self.scratch_page = P.pages[self.SCRATCH_SEQ][0]
            for i in range(B):
                self._set_padding(i)
        for i in range(B):
            if i >= len(entries):
                if self._row_seq[i] is not None:
                    self._set_padding(i)
                continue
            sid, tok, t = entries[i]
            if self._row_seq[i] != sid:
                h[4 * B + i * mp:4 * B + (i + 1) * mp] = 0
                self._row_seq[i], self._row_pages[i] = sid, 0
            P.reserve(sid, t + 1 - P.lengths[sid])
            pages = P.pages[sid]
            if len(pages) > mp:
                raise ValueError(f"sequence {sid} needs {len(pages)} pages; the graph holds {mp}")
            for j in range(self._row_pages[i], len(pages)):
                h[4 * B + i * mp + j] = pages[j]
            self._row_pages[i] = len(pages)
            h[i], h[B + i], h[3 * B + i] = tok, t, t + 1
            h[2 * B + i] = pages[t // P.page_size] * P.page_size + t % P.page_size
        self.dev.copy_(self.host, non_blocking=True)
        self._live = [(e[0], e[2]) for e in entries]

    def commit(self) -> None:
        for sid, t in self._live:
            self.pool.lengths[sid] = max(self.pool.lengths[sid], t + 1)

    def max_q_len(self) -> int:
        return 1


class KVCache:
    """Contiguous per-layer KV cache ``[L, B, Hkv, Smax, D]`` (API of the reference KVCache)."""

    def __init__(self, num_layers: int, batch_size: int, num_heads: int, head_dim: int,
                 max_seq_len: int, dtype=torch.float32, device="cpu"):
        shape = (num_layers, batch_size, num_heads, max_seq_len, head_dim)
        self.k = torch.zeros(shape, dtype=dtype, device=device)
        self.v = torch.zeros(shape, dtype=dtype, device=device)
        self.max_seq_len = max_seq_len
        self._len = 0

    def update(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor):
        n = k.shape[2]
        if self._len + n > self.max_seq_len:
            raise ValueError("KV cache full")
        self.k[layer_idx, :, :, self._len:self._len + n] = k
        self.v[layer_idx, :, :, self._len:self._len + n] = v
        return self.get(layer_idx, self._len + n)

    def get(self, layer_idx: int, length: Optional[int] = None):
        n = self._len if length is None else length
        return self.k[layer_idx, :, :, :n], self.v[layer_idx, :, :, :n]

    def advance(self, num_tokens: int = 1) -> None:
        self._len += num_tokens

    def reset(self) -> None:
        self._len = 0

    @property
    def seq_len(self) -> int:
        return self._len

    def memory_usage(self) -> float:
        return 2 * self.k.numel() * self.k.element_size() / 1e9
