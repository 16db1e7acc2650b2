"""Batch loaders.

``TokenBatchLoader`` is the training input path: a background thread asks the
native shard reader for ``[B, S+1]`` windows written straight into a ring of
pinned host buffers (GIL released during the copy), so the next batch is
ready before the GPU step ends and the host-to-device copy is a single
asynchronous DMA.  ``CUDAPrefetcher`` additionally issues that copy on a side
stream one step ahead.

``DistributedDataLoader`` / ``InfiniteDataLoader`` / ``create_dataloader``
keep the API of complexity/data/dataloader.py:19-230 for map-style and
iterable datasets (rank-sharded sampling, infinite cycling with epochs).
"""
from __future__ import annotations

import queue
import threading
from dataclasses import dataclass
from typing import Any, Iterator, Optional

import numpy as np
import torch
from torch.utils.data import DataLoader, Dataset, DistributedSampler, IterableDataset

from .token_shards import open_shard_reader, split_bounds


@dataclass
class DataConfig:
    batch_size: int = 8
    seq_len: int = 1024
    num_workers: int = 2
    pin_memory: bool = True
    shuffle: bool = True
    drop_last: bool = True
    seed: int = 42
    prefetch_factor: int = 2


class TokenBatchLoader:
    """Infinite (random) or single-pass (sequential) batches from a token shard.

    Yields ``(input_ids, labels)`` views of one pinned ``[B, S+1]`` int64
    buffer; it stays valid until the next ``next()`` call, so copy it to the
    device (or clone it) before asking for the next batch.
    """

    def __init__(self, path, batch_size: int, seq_len: int, *, rank: int = 0, world_size: int = 1,
                 seed: int = 42, split: str = "train", eval_ratio: float = 0.001,
                 order: str = "random", start_batch: int = 0, depth: int = 4, threads: int = 4,
                 pin_memory: Optional[bool] = None, device=None):
        self.reader, self.meta = open_shard_reader(path)
        self.B, self.S = int(batch_size), int(seq_len)
        self.rank, self.world = int(rank), int(world_size)
        self.seed, self.order = int(seed), order
        self.start, self.end = split_bounds(int(self.meta["num_tokens"]), self.S, split,
                                            eval_ratio)
        self.batch_index = int(start_batch)
        self.threads = threads
        pin = torch.cuda.is_available() if pin_memory is None else pin_memory
        self.bufs = [torch.empty(self.B, self.S + 1, dtype=torch.long, pin_memory=pin)
                     for _ in range(depth)]
        if depth < 3:
            raise ValueError("depth must be >= 3")
        # one buffer held by the consumer, one being filled, the rest queued
        self._q: "queue.Queue" = queue.Queue(maxsize=depth - 2)
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self._slot = 0
        # with a device, batches are returned on it; the asynchronous copy out
        # of a pinned slot is fenced by an event before the slot is refilled
        self.device = torch.device(device) if device is not None else None
        self._events = [None] * depth

    def _positions(self, b: int) -> Optional[np.ndarray]:
        if self.order == "sequential":
            first = (b * self.world + self.rank) * self.B
            pos = self.start + (first + np.arange(self.B)) * self.S
            if pos[-1] + self.S + 1 > self.end:
                return None
            return pos
        g = np.random.default_rng([self.seed, self.rank, b])
        return g.integers(self.start, self.end - self.S - 1 + 1, size=self.B)

    def _produce(self) -> None:
        b = self.batch_index
        slot = 0
        while not self._stop.is_set():
            pos = self._positions(b)
            if pos is None:
                self._q.put(None)
                return
            buf = self.bufs[slot]
            ev = self._events[slot]
            if ev is not None:
                ev.synchronize()
            self.reader.gather(torch.from_numpy(np.ascontiguousarray(pos, dtype=np.int64)), buf,
                               self.threads)
            while not self._stop.is_set():
                try:
                    self._q.put((b, slot), timeout=0.1)
                    break
                except queue.Full:
                    continue
            slot = (slot + 1) % len(self.bufs)
            b += 1

    def __iter__(self):
        if self._thread is None:
            self._thread = threading.Thread(target=self._produce, daemon=True)
            self._thread.start()
        return self

    def __next__(self):
        item = self._q.get()
        if item is None:
            raise StopIteration
        b, slot = item
        self.batch_index = b + 1
        buf = self.bufs[slot]
        if self.device is not None and self.device.type == "cuda":
            dev = buf.to(self.device, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record()
            self._events[slot] = ev
            return dev[:, :-1], dev[:, 1:]
        return buf[:, :-1], buf[:, 1:]

    def state_dict(self) -> dict:
        return {"batch_index": self.batch_index}

    def close(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)


class CUDAPrefetcher:
    """Copies the next batch to the GPU on a side stream while the current one is used."""

    def __init__(self, loader, device=None):
        self.it = iter(loader)
        self.device = torch.device(device or "cuda")
        self.stream = torch.cuda.Stream(self.device)
        self._next = None
        self._preload()

    def _preload(self):
        try:
            batch = next(self.it)
        except StopIteration:
            self._next = None
            return
        with torch.cuda.stream(self.stream):
            self._next = tuple(t.to(self.device, non_blocking=True) for t in batch)

    def __iter__(self):
        return self

    def __next__(self):
        if self._next is None:
            raise StopIteration
        torch.cuda.current_stream(self.device).wait_stream(self.stream)
        out = self._next
        for t in out:
            t.record_stream(torch.cuda.current_stream(self.device))
        self._preload()
        return out


class DistributedDataLoader:
    """Rank-sharded DataLoader: a ``DistributedSampler`` for map-style datasets,
    rank/world attributes set on iterable datasets that expose them."""

    def __init__(self, dataset, batch_size: int, *, rank: int = 0, world_size: int = 1,
                 shuffle: bool = True, seed: int = 42, num_workers: int = 0,
                 pin_memory: bool = False, drop_last: bool = True, collate_fn=None):
        self.dataset = dataset
        self.sampler = None
        if isinstance(dataset, IterableDataset):
            for k, v in (("rank", rank), ("world_size", world_size)):
                if hasattr(dataset, k):
                    setattr(dataset, k, v)
            self.loader = DataLoader(dataset, batch_size=batch_size, num_workers=num_workers,
                                     pin_memory=pin_memory, drop_last=drop_last,
                                     collate_fn=collate_fn)
        else:
            self.sampler = DistributedSampler(dataset, num_replicas=world_size, rank=rank,
                                              shuffle=shuffle, seed=seed, drop_last=drop_last)
            self.loader = DataLoader(dataset, batch_size=batch_size, sampler=self.sampler,
                                     num_workers=num_workers, pin_memory=pin_memory,
                                     drop_last=drop_last, collate_fn=collate_fn)

    def set_epoch(self, epoch: int) -> None:
        if self.sampler is not None:
            self.sampler.set_epoch(epoch)

    def __iter__(self):
        return iter(self.loader)

    def __len__(self):
        return len(self.loader)


class InfiniteDataLoader:
    """Cycles a loader forever, bumping the sampler epoch at each pass."""

    def __init__(self, loader):
        self.loader = loader
        self.epoch = 0
        self._it = None

    def __iter__(self):
        return self

    def __next__(self):
        while True:
            if self._it is None:
                if hasattr(self.loader, "set_epoch"):
                    self.loader.set_epoch(self.epoch)
                self._it = iter(self.loader)
            try:
                return next(self._it)
            except StopIteration:
                self._it = None
                self.epoch += 1


def create_dataloader(dataset, config: Optional[DataConfig] = None, *, rank: int = 0,
                      world_size: int = 1, infinite: bool = False, collate_fn=None):
    cfg = config or DataConfig()
    dl = DistributedDataLoader(dataset, cfg.batch_size, rank=rank, world_size=world_size,
                               shuffle=cfg.shuffle, seed=cfg.seed, num_workers=cfg.num_workers,
                               pin_memory=cfg.pin_memory and torch.cuda.is_available(),
                               drop_last=cfg.drop_last, collate_fn=collate_fn)
    return InfiniteDataLoader(dl) if infinite else dl


class SyntheticTokenDataset(IterableDataset):
    """Zipf-distributed random token windows (benchmarks and tests; no files)."""

    def __init__(self, vocab_size: int, seq_len: int, *, zipf_a: float = 1.1, seed: int = 0):
        self.vocab_size, self.seq_len, self.a, self.seed = vocab_size, seq_len, zipf_a, seed

    def __iter__(self):
        g = np.random.default_rng(self.seed)
        while True:
            ids = (g.zipf(self.a, size=self.seq_len + 1) - 1) % self.vocab_size
            t = torch.from_numpy(ids.astype(np.int64))
            yield {"input_ids": t[:-1], "labels": t[1:]}


class BackgroundTokenizer:
    """Tokenize text on a worker thread while the GPU computes; hand out
    ``[max_length + 1]`` training windows from the token stream.

    Counterpart: complexity/gpu/data_loading.py:87-120.  ``submit`` only
    enqueues (the caller never waits for the tokenizer); the worker encodes,
    appends an optional ``eos_id`` separator, and grows the token buffer.
    Consecutive windows share one token (the last target of a window is the
    first input of the next), so no token is dropped between windows.
    ``get_batch`` returns None until a full window is buffered (``block=True``
    waits for one, or until ``close``).
    """

    def __init__(self, tokenizer, max_length: int = 2048, buffer_size: int = 100,
                 eos_id: Optional[int] = None):
        self.tokenizer, self.max_length, self.eos_id = tokenizer, int(max_length), eos_id
        self._texts: "queue.Queue[Optional[str]]" = queue.Queue(maxsize=max(1, buffer_size))
        self._tokens: list = []
        self._cv = threading.Condition()
        self._closed = False
        self._error: Optional[BaseException] = None
        self._worker = threading.Thread(target=self._run, daemon=True)
        self._worker.start()

    def _run(self) -> None:
        while True:
            text = self._texts.get()
            if text is None:
                break
            try:
                ids = list(self.tokenizer.encode(text))
            except BaseException as e:  # surfaced to the consumer
                with self._cv:
                    self._error = e
                    self._cv.notify_all()
                break
            if self.eos_id is not None:
                ids.append(int(self.eos_id))
            with self._cv:
                self._tokens.extend(ids)
                self._cv.notify_all()
        with self._cv:
            self._closed = True
            self._cv.notify_all()

    def submit(self, text: str) -> None:
        if self._closed:
            raise RuntimeError("BackgroundTokenizer is closed")
        self._texts.put(text)

    def buffered_tokens(self) -> int:
        with self._cv:
            return len(self._tokens)

    def get_batch(self, block: bool = False, timeout: Optional[float] = None
                  ) -> Optional[torch.Tensor]:
        need = self.max_length + 1
        with self._cv:
            if block:
                self._cv.wait_for(lambda: len(self._tokens) >= need or self._closed
                                  or self._error is not None, timeout)
            if self._error is not None:
                raise RuntimeError("tokenizer failed in the background") from self._error
            if len(self._tokens) < need:
                return None
            window = self._tokens[:need]
            del self._tokens[:self.max_length]
        return torch.tensor(window, dtype=torch.long)

    def close(self) -> None:
        """Finish the submitted texts and stop the worker."""
        if not self._closed:
            self._texts.put(None)
            self._worker.join()

    def __iter__(self) -> Iterator[torch.Tensor]:
        while True:
            b = self.get_batch(block=True)
            if b is None:
                return
            yield b
