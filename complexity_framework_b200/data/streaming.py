"""Streaming text datasets and corpus mixtures.

Counterparts: complexity/data/streaming.py:20-400 (``StreamingDataset``,
``ShardedDataset``, ``InterleavedDataset``, ``CachedDataset``) and the
weighted-mixture / replay logic of complexity/training/corpus_mixture.py
(applied here to local token shards; there is no network access).
"""
from __future__ import annotations

import json
import random
from pathlib import Path
from typing import Dict, Iterable, Iterator, List, Optional, Sequence

import numpy as np
import torch
from torch.utils.data import Dataset, IterableDataset

from .token_shards import open_shard_reader, split_bounds


def iter_texts(paths: Sequence[str], text_key: str = "text") -> Iterator[str]:
    """Lines of .txt files or the ``text_key`` field of .jsonl files."""
    for p in paths:
        p = Path(p)
        with p.open("r", encoding="utf-8") as f:
            if p.suffix in (".jsonl", ".json"):
                for line in f:
                    line = line.strip()
                    if line:
                        yield json.loads(line).get(text_key, "")
            else:
                for line in f:
                    if line.strip():
                        yield line.rstrip("\n")


class StreamingDataset(IterableDataset):
    """Tokenise text files on the fly and emit fixed-length windows."""

    def __init__(self, paths: Sequence[str], tokenizer, seq_len: int, *, text_key: str = "text",
                 rank: int = 0, world_size: int = 1, add_eos: bool = True):
        self.paths, self.tok, self.seq_len = list(paths), tokenizer, seq_len
        self.text_key, self.rank, self.world_size, self.add_eos = text_key, rank, world_size, add_eos

    def __iter__(self):
        buf: List[int] = []
        for i, text in enumerate(iter_texts(self.paths, self.text_key)):
            if i % self.world_size != self.rank:
                continue
            buf.extend(self.tok.encode(text))
            if self.add_eos and self.tok.eos_token_id is not None:
                buf.append(self.tok.eos_token_id)
            while len(buf) >= self.seq_len + 1:
                w = torch.tensor(buf[:self.seq_len + 1])
                buf = buf[self.seq_len:]
                yield {"input_ids": w[:-1], "labels": w[1:]}


class ShardedDataset(IterableDataset):
    """Files are split across (rank, worker) streams; each stream reads its own files."""

    def __init__(self, paths: Sequence[str], make_iter, *, rank: int = 0, world_size: int = 1):
        self.paths, self.make_iter, self.rank, self.world_size = list(paths), make_iter, rank, world_size

    def __iter__(self):
        w = torch.utils.data.get_worker_info()
        wid, nw = (0, 1) if w is None else (w.id, w.num_workers)
        sid, ns = self.rank * nw + wid, self.world_size * nw
        for i, p in enumerate(self.paths):
            if i % ns == sid:
                yield from self.make_iter(p)


class InterleavedDataset(IterableDataset):
    """Draw from several iterables with fixed weights (stops when one is exhausted
    unless ``cycle``)."""

    def __init__(self, datasets: Sequence[Iterable], weights: Optional[Sequence[float]] = None,
                 seed: int = 0, cycle: bool = True):
        self.datasets = list(datasets)
        w = np.asarray(weights if weights is not None else [1.0] * len(self.datasets), float)
        self.weights = w / w.sum()
        self.seed, self.cycle = seed, cycle

    def __iter__(self):
        rng = np.random.default_rng(self.seed)
        its = [iter(d) for d in self.datasets]
        while True:
            k = int(rng.choice(len(its), p=self.weights))
            try:
                yield next(its[k])
            except StopIteration:
                if not self.cycle:
                    return
                its[k] = iter(self.datasets[k])
                yield next(its[k])


class CachedDataset(Dataset):
    """Materialise the first ``limit`` items of an iterable (eval sets)."""

    def __init__(self, source: Iterable, limit: int):
        self.items = []
        for i, x in enumerate(source):
            if i >= limit:
                break
            self.items.append(x)

    def __len__(self):
        return len(self.items)

    def __getitem__(self, i):
        return self.items[i]


class TokenShardMixture:
    """Weighted mixture of token shards with a deterministic per-batch plan.

    Batch b of rank r draws ``round(w_k * B)`` windows from shard k (largest
    remainders fill the rest), positions from a generator seeded by
    ``(seed, r, b)`` so resuming at batch b replays exactly.  ``replay`` lists
    (shard index, fraction) pairs that are mixed into every batch on top of
    the base weights (e.g. to revisit an earlier corpus).
    """

    def __init__(self, paths: Sequence[str], weights: Sequence[float], batch_size: int,
                 seq_len: int, *, rank: int = 0, seed: int = 0, split: str = "train",
                 eval_ratio: float = 0.001, replay: Sequence = ()):
        self.readers = []
        self.bounds = []
        for p in paths:
            r, meta = open_shard_reader(p)
            self.readers.append(r)
            self.bounds.append(split_bounds(int(meta["num_tokens"]), seq_len, split, eval_ratio))
        w = np.asarray(weights, float)
        for k, frac in replay:
            w[int(k)] += float(frac) * w.sum()
        self.weights = w / w.sum()
        self.B, self.S, self.rank, self.seed = batch_size, seq_len, rank, seed

    def counts(self) -> np.ndarray:
        raw = self.weights * self.B
        c = np.floor(raw).astype(int)
        for i in np.argsort(-(raw - c))[: self.B - c.sum()]:
            c[i] += 1
        return c

    def batch(self, b: int) -> torch.Tensor:
        g = np.random.default_rng([self.seed, self.rank, b])
        out = torch.empty(self.B, self.S + 1, dtype=torch.long)
        row = 0
        for k, n in enumerate(self.counts()):
            if n == 0:
                continue
            lo, hi = self.bounds[k]
            pos = torch.from_numpy(g.integers(lo, hi - self.S - 1 + 1, size=n).astype(np.int64))
            self.readers[k].gather(pos, out[row:row + n], 2)
            row += n
        return out[torch.from_numpy(g.permutation(self.B))]
