"""KV caches under the reference's ``complexity.inference.kv_cache`` API.

Counterpart of complexity/inference/kv_cache.py:19-470 (``CacheConfig``,
``KVCache``, ``PagedKVCache``, ``SlidingWindowCache``, ``create_cache``).
``PagedKVCache`` is the engine's ``PagePool`` (the same page storage the
paged attention kernels read) with the reference's constructor and
``update(seq_id, layer_idx, key, value)``: the new keys / values are
scattered into their pages and the sequence's whole cache comes back as one
gather over its page list (no per-page Python loop).  As in the reference,
``update`` writes at the current length and ``advance`` moves it.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch

from .decoding import SlidingWindowCache as _SlidingWindow
from .paged import KVCache as _Contiguous
from .paged import OutOfPages, PagePool


@dataclass
class CacheConfig:
    num_layers: int
    num_heads: int
    head_dim: int
    max_seq_len: int
    dtype: torch.dtype = torch.float16
    device: str = "cpu"


class KVCache(_Contiguous):
    """Contiguous cache [L, B, H, Smax, D] with the reference's argument order."""

    def __init__(self, num_layers: int, num_heads: int, head_dim: int,
                 max_seq_len: Optional[int] = None, max_length: Optional[int] = None,
                 batch_size: int = 1, dtype=torch.float32, device="cpu"):
        n = max_seq_len if max_seq_len is not None else max_length
        if n is None:
            raise ValueError("max_seq_len or max_length is required")
        super().__init__(num_layers, batch_size, num_heads, head_dim, n, dtype, device)
        self.num_layers, self.num_heads, self.head_dim = num_layers, num_heads, head_dim
        self.batch_size, self.dtype, self.device = batch_size, dtype, device


class SlidingWindowCache(_SlidingWindow):
    def __init__(self, num_layers: int, num_heads: int, head_dim: int, window_size: int = 4096,
                 batch_size: int = 1, dtype=torch.float32, device="cpu", **_):
        super().__init__(num_layers, batch_size, num_heads, head_dim, window_size, dtype, device)


class PagedKVCache(PagePool):
    def __init__(self, num_layers: int, num_heads: int, head_dim: int, page_size: int = 16,
                 num_pages: int = 1024, max_pages: Optional[int] = None,
                 dtype=torch.float32, device="cpu"):
        super().__init__(num_layers, num_heads, head_dim,
                         num_pages if max_pages is None else max_pages, page_size, dtype, device)
        self.num_heads = num_heads

    @property
    def free_pages(self):
        return self.free

    @property
    def page_tables(self) -> Dict[int, list]:
        return self.pages

    def update(self, seq_id: int, layer_idx: int, key: torch.Tensor,
               value: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """``key`` / ``value`` [1, H, n, D] at positions len .. len+n-1;
        returns the sequence's [1, H, len+n, D] keys and values."""
        pos, n = self.lengths[seq_id], key.shape[2]
        pages = self.pages[seq_id]
        while len(pages) * self.page_size < pos + n:
            if not self.free:
                raise OutOfPages("Out of pages")
            pages.append(self.free.pop())
        dev = self.k.device
        t = torch.arange(pos, pos + n, device=dev)
        page_t = torch.tensor(pages, device=dev)
        pg, off = page_t[t // self.page_size], t % self.page_size
        self.k[layer_idx, pg, off] = key[0].transpose(0, 1).to(self.k.dtype)
        self.v[layer_idx, pg, off] = value[0].transpose(0, 1).to(self.v.dtype)
        allt = torch.arange(pos + n, device=dev)
        pa, oa = page_t[allt // self.page_size], allt % self.page_size
        return (self.k[layer_idx, pa, oa].transpose(0, 1)[None],
                self.v[layer_idx, pa, oa].transpose(0, 1)[None])

    def advance(self, seq_id: int, num_tokens: int = 1) -> None:
        self.lengths[seq_id] += num_tokens

    def get_seq_len(self, seq_id: int) -> int:
        return self.lengths.get(seq_id, 0)

    def memory_usage(self) -> Dict[str, float]:
        used = self.num_pages - len(self.free)
        page_bytes = 2 * self.num_layers * self.page_size * self.num_kv_heads * self.head_dim * \
            self.k.element_size()
        mb = 1024 ** 2
        return {"total_mb": self.num_pages * page_bytes / mb, "used_mb": used * page_bytes / mb,
                "free_pages": len(self.free), "used_pages": used}


def create_cache(config: CacheConfig, cache_type: str = "standard", **kwargs):
    base = dict(num_layers=config.num_layers, num_heads=config.num_heads,
                head_dim=config.head_dim, dtype=config.dtype, device=config.device)
    if cache_type == "standard":
        return KVCache(max_seq_len=config.max_seq_len, **base, **kwargs)
    if cache_type == "paged":
        return PagedKVCache(**base, **kwargs)
    if cache_type == "sliding_window":
        return SlidingWindowCache(**base, **kwargs)
    raise ValueError(f"Unknown cache type: {cache_type}")
