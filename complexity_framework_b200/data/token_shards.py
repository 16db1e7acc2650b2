"""Flat token shards: ``tokens.bin`` (uint16/uint32 ids) + ``tokens.idx.json``.

The on-disk format (file names, ``format`` tag ``complexity-token-shard-v1``
and metadata keys) is the one of complexity/data/token_shards.py:26-124 so
shards written by either framework load in the other.  Reads go through the
native memory-mapped reader (``_io.ShardReader``): batches of windows are
gathered by C++ threads into pinned host tensors, with the GIL released.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path
from typing import Any, Dict, Iterable, Iterator, Optional, Tuple, Union

import numpy as np
import torch
from torch.utils.data import IterableDataset

TOKEN_BIN = "tokens.bin"
TOKEN_INDEX = "tokens.idx.json"
FORMAT = "complexity-token-shard-v1"


def _io():
    from .. import _io  # noqa: WPS433 (native module built next to the package)

    return _io


def dtype_for_vocab(vocab_size: Optional[int]) -> np.dtype:
    return np.dtype(np.uint16) if vocab_size is not None and vocab_size <= 65536 else np.dtype(np.uint32)


def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with path.open("rb") as f:
        for chunk in iter(lambda: f.read(8 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def _arrays(tokens, dtype) -> Iterator[np.ndarray]:
    if isinstance(tokens, (np.ndarray, torch.Tensor)):
        yield np.asarray(tokens, dtype=dtype).reshape(-1)
        return
    buf = []
    for t in tokens:
        if isinstance(t, (int, np.integer)):
            buf.append(int(t))
            if len(buf) >= 1 << 20:
                yield np.asarray(buf, dtype=dtype)
                buf = []
        else:
            if buf:
                yield np.asarray(buf, dtype=dtype)
                buf = []
            yield np.asarray(list(t) if not isinstance(t, np.ndarray) else t, dtype=dtype)
    if buf:
        yield np.asarray(buf, dtype=dtype)


def write_token_shard(output_dir: Union[str, Path], tokens, *, vocab_size: Optional[int] = None,
                      tokenizer: Optional[str] = None, dtype=None,
                      extra_metadata: Optional[Dict[str, Any]] = None) -> Path:
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    np_dtype = np.dtype(dtype) if dtype is not None else dtype_for_vocab(vocab_size)
    bin_path = out / TOKEN_BIN
    n, mx = 0, -1
    with bin_path.open("wb") as f:
        for arr in _arrays(tokens, np_dtype):
            if arr.size:
                mx = max(mx, int(arr.max()))
                arr.tofile(f)
                n += int(arr.size)
    if n == 0:
        raise ValueError("cannot write an empty token shard")
    meta = {"format": FORMAT, "bin": TOKEN_BIN, "dtype": np_dtype.str, "num_tokens": n,
            "max_token_id": mx, "vocab_size": vocab_size, "tokenizer": tokenizer,
            "sha256": _sha256(bin_path)}
    meta.update(extra_metadata or {})
    idx = out / TOKEN_INDEX
    idx.write_text(json.dumps(meta, indent=2, sort_keys=True) + "\n", encoding="utf-8")
    return idx


def read_token_shard_metadata(path: Union[str, Path]) -> Dict[str, Any]:
    idx = Path(path).expanduser() / TOKEN_INDEX
    if not idx.exists():
        raise FileNotFoundError(f"token shard index not found: {idx}")
    meta = json.loads(idx.read_text(encoding="utf-8"))
    if meta.get("format") != FORMAT:
        raise ValueError(f"unsupported token shard format {meta.get('format')!r}")
    return meta


def load_token_shard(path: Union[str, Path], *, mmap_mode: str = "r") -> Tuple[np.memmap, Dict]:
    """numpy memmap view + metadata (for inspection; training reads use ShardReader)."""
    meta = read_token_shard_metadata(path)
    binp = Path(path).expanduser() / meta.get("bin", TOKEN_BIN)
    arr = np.memmap(binp, dtype=np.dtype(meta["dtype"]), mode=mmap_mode,
                    shape=(int(meta["num_tokens"]),))
    return arr, meta


def open_shard_reader(path: Union[str, Path]):
    meta = read_token_shard_metadata(path)
    binp = Path(path).expanduser() / meta.get("bin", TOKEN_BIN)
    return _io().ShardReader(str(binp), np.dtype(meta["dtype"]).itemsize, int(meta["num_tokens"])), meta


def token_shard_frequencies(path: Union[str, Path], vocab_size: int, *, start: int = 0,
                            end: Optional[int] = None, threads: int = 8) -> torch.Tensor:
    """Token counts ``[vocab_size]`` over ``[start, end)`` (ids >= vocab are dropped)."""
    reader, meta = open_shard_reader(path)
    e = int(meta["num_tokens"]) if end is None else int(end)
    return reader.frequencies(int(vocab_size), int(start), e, int(threads))[:vocab_size]


def split_bounds(num_tokens: int, seq_len: int, split: str, eval_ratio: float) -> Tuple[int, int]:
    """Token range of a split: the eval split is the shard's tail."""
    if split == "all" or (split == "train" and eval_ratio <= 0):
        return 0, num_tokens
    if eval_ratio <= 0:
        raise ValueError("eval_ratio must be positive for an eval split")
    ev = max(seq_len + 1, int(num_tokens * eval_ratio))
    ev = min(ev, max(seq_len + 1, num_tokens // 10))
    if split == "train":
        return 0, num_tokens - ev
    if split in ("eval", "val", "validation"):
        return num_tokens - ev, num_tokens
    raise ValueError("split must be one of: all, train, eval, val, validation")


class TokenShardDataset(IterableDataset):
    """Fixed-length LM windows from a token shard.

    ``order="sequential"`` walks non-overlapping windows, interleaved over
    ``world_size`` ranks x DataLoader workers, starting at ``start_sequence``
    (exact resume); ``order="random"`` samples window starts from a seeded
    generator per (rank, worker) stream.  Yields dicts with ``input_ids`` and
    ``labels`` (the window shifted by one).
    """

    def __init__(self, path, seq_len: int, *, rank: int = 0, world_size: int = 1, seed: int = 42,
                 split: str = "train", eval_ratio: float = 0.001, order: str = "random",
                 start_sequence: int = 0):
        if order not in ("random", "sequential"):
            raise ValueError("order must be one of: random, sequential")
        if start_sequence < 0:
            raise ValueError("start_sequence must be non-negative")
        self.path, self.seq_len = str(path), int(seq_len)
        self.rank, self.world_size, self.seed = int(rank), int(world_size), int(seed)
        self.split, self.eval_ratio, self.order = split, float(eval_ratio), order
        self.start_sequence = int(start_sequence)
        self.metadata = read_token_shard_metadata(path)
        self.num_tokens = int(self.metadata["num_tokens"])
        if self.num_tokens < self.seq_len + 2:
            raise ValueError(f"need at least {self.seq_len + 2} tokens, got {self.num_tokens}")
        self.start, self.end = split_bounds(self.num_tokens, self.seq_len, split, self.eval_ratio)
        if self.end - self.start < self.seq_len + 1:
            raise ValueError(f"split {split!r} too small for seq_len={self.seq_len}")

    def _stream(self) -> Tuple[int, int]:
        w = torch.utils.data.get_worker_info()
        wid, nw = (0, 1) if w is None else (w.id, w.num_workers)
        return self.rank * nw + wid, max(1, self.world_size * nw)

    def positions(self, count: int, stream: int = 0, streams: int = 1, cursor: int = 0):
        """Window starts for ``count`` samples of one stream (used by the batch loader)."""
        if self.order == "sequential":
            idx = self.start_sequence + stream + streams * (cursor + np.arange(count))
            pos = self.start + idx * self.seq_len
            return pos[pos + self.seq_len < self.end]
        g = np.random.default_rng(self.seed + 1_000_003 * stream + cursor)
        high = self.end - self.seq_len - 1
        return g.integers(self.start, high + 1, size=count)

    def __iter__(self):
        reader, _ = open_shard_reader(self.path)
        stream, streams = self._stream()
        cursor = 0
        while True:
            pos = self.positions(64, stream, streams, cursor)
            cursor += 64
            if len(pos) == 0:
                return
            out = torch.empty(len(pos), self.seq_len + 1, dtype=torch.long)
            reader.gather(torch.as_tensor(pos, dtype=torch.long), out, 1)
            for row in out:
                yield {"input_ids": row[:-1], "labels": row[1:]}


def iter_texts_from_files(paths, *, input_format: str = "jsonl", text_field: str = "text",
                          limit: int = 0) -> Iterator[str]:
    """Texts of JSONL rows (``text_field``) or whole plain-text files, in order,
    stopping after ``limit`` records when it is positive."""
    seen = 0
    for p in paths:
        p = Path(p)
        if input_format == "jsonl":
            with p.open(encoding="utf-8") as f:
                for line in f:
                    if not line.strip():
                        continue
                    t = json.loads(line).get(text_field, "")
                    if t:
                        yield str(t)
                        seen += 1
                        if limit > 0 and seen >= limit:
                            return
        elif input_format == "text":
            t = p.read_text(encoding="utf-8")
            if t:
                yield t
                seen += 1
                if limit > 0 and seen >= limit:
                    return
        else:
            raise ValueError(f"unsupported input_format {input_format!r} (jsonl or text)")


def build_token_shard_from_texts(texts, tokenizer, output_dir, *, vocab_size: Optional[int] = None,
                                 tokenizer_name: Optional[str] = None, add_eos: bool = True,
                                 dtype=None, extra_metadata: Optional[Dict[str, Any]] = None
                                 ) -> Path:
    """Tokenise text records (EOS after each when the tokenizer has one) into a
    streaming token shard; returns the index file."""
    eos = getattr(tokenizer, "eos_token_id", None)

    def encode(t: str):
        try:
            return tokenizer.encode(t, add_special_tokens=False)
        except TypeError:
            return tokenizer.encode(t)

    def chunks():
        for t in texts:
            ids = list(encode(t))
            if add_eos and eos is not None:
                ids.append(int(eos))
            if ids:
                yield ids

    vs = vocab_size or getattr(tokenizer, "vocab_size", None)
    return write_token_shard(output_dir, chunks(), vocab_size=vs, tokenizer=tokenizer_name,
                             dtype=dtype, extra_metadata=extra_metadata)
