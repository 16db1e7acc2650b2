"""Static CUDA-graph shape buckets (reference: complexity/tr_hash/buckets.py:10-46)."""
from __future__ import annotations

from typing import Iterable, Tuple

from .config import GraphBucket, _sorted_unique_buckets


class GraphBucketPlanner:
    """Select the smallest captured (batch, sequence) bucket that holds an input."""

    def __init__(self, buckets: Iterable[GraphBucket]):
        self.buckets: Tuple[GraphBucket, ...] = _sorted_unique_buckets(buckets)
        if not self.buckets:
            raise ValueError("at least one graph bucket is required")

    def select(self, batch_size: int, sequence_length: int) -> GraphBucket:
        if batch_size <= 0 or sequence_length <= 0:
            raise ValueError("batch_size and sequence_length must be positive")
        for bucket in self.buckets:  # sorted by token capacity
            if bucket.batch_size >= batch_size and bucket.sequence_length >= sequence_length:
                return bucket
        raise ValueError(
            f"no CUDA graph bucket fits batch={batch_size}, sequence={sequence_length}; "
            f"largest is {self.buckets[-1]}")
