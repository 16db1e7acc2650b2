"""Pretraining corpus mixtures: weighted text streams and pretokenized
row-addressed token mixtures with replay plans and resume-skip.

Formats and rules shared with complexity/training/corpus_mixture.py (so a
mixture built for either framework trains identically in the other):

* manifest ``mixture_manifest.json`` with ``format: tr-hash-token-mixture-v1``,
  ``dtype: uint16``, ``seq_len`` and ``sources: [{name, weight, rows,
  manifest}]``; each source manifest lists ``shards: [{file, rows, tokens,
  bytes?, sha256?}]``; a shard of R rows holds ``R * seq_len + 1`` uint16
  tokens and row i is tokens ``[i*seq_len, (i+1)*seq_len + 1)`` (inputs and
  shifted labels share the boundary token);
* sources are interleaved by weighted fair queuing: the next sample comes
  from the source with the smallest ``emitted / weight``, ties broken by the
  source order (the reference's rule, corpus_mixture.py:480-485);
* rank ``r`` of ``P`` (times data-loader workers) takes the rows ``i`` with
  ``i % shard_count == shard_index`` of each source, counted across its shards;
* a replay plan (``format: tr-hash-token-replay-v1``) is a list of phases,
  each repeated ``passes`` times over selected shard prefixes; its declared
  ``unique_tokens`` / ``trained_tokens`` are checked;
* ``resume_skip_rows`` drops that many of this rank's leading samples so a
  resumed run continues on the next unseen row.

Hub download/caching is not built (no network); everything else — manifest
validation (coverage, shard sizes, duplicate names), replay plans, rank and
worker sharding, resume-skip — is.  ``write_token_mixture`` builds the format
from token arrays.
"""
from __future__ import annotations

import hashlib
import json
import math
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Dict, Iterable, Iterator, Mapping, Optional, Sequence, Tuple, Union

import numpy as np
import torch
from torch.utils.data import IterableDataset, get_worker_info

MIXTURE_FORMAT = "tr-hash-token-mixture-v1"
REPLAY_PLAN_FORMAT = "tr-hash-token-replay-v1"
TOKEN_DTYPE = np.dtype("<u2")


@dataclass(frozen=True)
class TextCorpusSource:
    """One source of a pretraining mixture."""

    name: str
    weight: float
    dataset_id: Optional[str] = None
    config_name: Optional[str] = None
    data_files: Union[str, Sequence[str], None] = None
    text_field: str = "text"
    split: str = "train"

    def validate(self) -> None:
        if not self.name.strip():
            raise ValueError("corpus source name cannot be empty")
        if not 0.0 < self.weight <= 1.0:
            raise ValueError(f"{self.name} weight must be in (0, 1]")
        if (self.dataset_id is None) == (self.data_files is None):
            raise ValueError(f"{self.name} must define exactly one of dataset_id or data_files")
        if not self.text_field.strip():
            raise ValueError(f"{self.name} text_field cannot be empty")


def validate_corpus_mixture(sources: Sequence[TextCorpusSource]) -> None:
    if not sources:
        raise ValueError("corpus mixture cannot be empty")
    for s in sources:
        s.validate()
    names = [s.name for s in sources]
    if len(set(names)) != len(names):
        raise ValueError("corpus source names must be unique")
    total = math.fsum(s.weight for s in sources)
    if abs(total - 1.0) > 1e-9:
        raise ValueError(f"corpus weights must sum to 1.0, got {total:.12f}")


def allocate_weighted_counts(total: int, sources: Sequence[TextCorpusSource]) -> Dict[str, int]:
    """Integer split of ``total`` by the weights: floors, then the largest
    remainders (ties by name) take the leftover units."""
    validate_corpus_mixture(sources)
    if total < 1:
        raise ValueError("weighted allocation total must be positive")
    exact = {s.name: total * s.weight for s in sources}
    counts = {k: int(math.floor(v)) for k, v in exact.items()}
    left = total - sum(counts.values())
    for name in sorted(exact, key=lambda k: (counts[k] - exact[k], k))[:left]:
        counts[name] += 1
    return counts


def next_source(sources: Sequence[TextCorpusSource], counts: Mapping[str, int]) -> TextCorpusSource:
    """Weighted fair queuing: the source furthest below its share (first on ties)."""
    best, key = None, None
    for s in sources:
        k = counts[s.name] / s.weight
        if key is None or k < key:
            best, key = s, k
    return best


def _shard_slot() -> Tuple[int, int]:
    w = get_worker_info()
    return (w.num_workers, w.id) if w is not None else (1, 0)


def _sample(chunk: np.ndarray) -> Dict[str, torch.Tensor]:
    c = torch.from_numpy(chunk.astype(np.int64))
    return {"input_ids": c[:-1].clone(), "labels": c[1:].clone()}


class WeightedStreamingTextDataset(IterableDataset):
    """Text sources tokenized and packed per source (documents never cross
    sources), then interleaved at exact sample-level weights."""

    def __init__(self, *, tokenizer: Any, seq_len: int, sources: Sequence[TextCorpusSource],
                 rank: int = 0, world_size: int = 1,
                 streams: Optional[Mapping[str, Iterable[Mapping[str, Any]]]] = None):
        validate_corpus_mixture(sources)
        if seq_len < 1:
            raise ValueError("seq_len must be positive")
        if rank < 0 or world_size < 1 or rank >= world_size:
            raise ValueError("invalid distributed rank/world_size")
        self.tokenizer, self.seq_len = tokenizer, int(seq_len)
        self.sources = tuple(sources)
        self.rank, self.world_size = int(rank), int(world_size)
        self._streams = streams

    def _stream(self, src: TextCorpusSource) -> Iterator[Mapping[str, Any]]:
        if self._streams is not None:
            if src.name not in self._streams:
                raise ValueError(f"missing provided stream for {src.name}")
            rows: Iterable[Mapping[str, Any]] = self._streams[src.name]
        else:
            if src.data_files is None:
                raise ValueError(f"{src.name}: remote datasets need network access; give "
                                 "data_files (local JSONL) or a provided stream")
            files = [src.data_files] if isinstance(src.data_files, str) else list(src.data_files)

            def read():
                for f in files:
                    with open(f, encoding="utf-8") as fh:
                        for line in fh:
                            if line.strip():
                                yield json.loads(line)
            rows = read()
        workers, wid = _shard_slot()
        count, index = self.world_size * workers, self.rank * workers + wid
        for i, row in enumerate(rows):
            if i % count == index:
                yield row

    def _packed(self, src: TextCorpusSource) -> Iterator[Dict[str, torch.Tensor]]:
        buf = []
        eos = getattr(self.tokenizer, "eos_token_id", None)
        for row in self._stream(src):
            text = row.get(src.text_field, "")
            if not isinstance(text, str) or not text:
                continue
            try:
                ids = self.tokenizer.encode(text, add_special_tokens=False)
            except TypeError:
                ids = self.tokenizer.encode(text)
            buf.extend(int(t) for t in ids)
            if eos is not None:
                buf.append(int(eos))
            while len(buf) >= self.seq_len + 1:
                yield _sample(np.asarray(buf[:self.seq_len + 1]))
                del buf[:self.seq_len]

    def __iter__(self):
        its = {s.name: self._packed(s) for s in self.sources}
        counts = {s.name: 0 for s in self.sources}
        while True:
            s = next_source(self.sources, counts)
            try:
                item = next(its[s.name])
            except StopIteration as exc:
                raise RuntimeError(f"corpus source {s.name!r} exhausted before the token "
                                   "budget") from exc
            counts[s.name] += 1
            yield item


class PretokenizedCorpusMixtureDataset(IterableDataset):
    """Rows of local uint16 token shards, mixed by weight, sharded over ranks
    and data-loader workers, with optional replay plan and resume-skip."""

    def __init__(self, root: Union[str, Path], *, rank: int = 0, world_size: int = 1,
                 replay_plan: Union[str, Path, Mapping[str, Any], None] = None,
                 resume_skip_rows: int = 0, verify_sha256: bool = False):
        root_s = str(root)
        if root_s.startswith("hf://"):
            raise ValueError("hub-hosted mixtures need network access; download the mixture "
                             "and pass its local directory")
        self.root = Path(root)
        path = self.root / "mixture_manifest.json"
        if not path.is_file():
            raise FileNotFoundError(f"pretokenized mixture manifest not found: {path}")
        self.manifest = json.loads(path.read_text(encoding="utf-8"))
        if self.manifest.get("format") != MIXTURE_FORMAT:
            raise ValueError("unsupported pretokenized mixture format")
        if self.manifest.get("dtype") != "uint16":
            raise ValueError("pretokenized mixture must use uint16 tokens")
        self.seq_len = int(self.manifest["seq_len"])
        if rank < 0 or world_size < 1 or rank >= world_size:
            raise ValueError("invalid distributed rank/world_size")
        if resume_skip_rows < 0:
            raise ValueError("resume_skip_rows must be non-negative")
        self.rank, self.world_size = int(rank), int(world_size)
        self.resume_skip_rows = int(resume_skip_rows)
        self.sources = tuple(TextCorpusSource(name=e["name"], weight=float(e["weight"]),
                                              data_files=str(self.root / e["manifest"]))
                             for e in self.manifest["sources"])
        validate_corpus_mixture(self.sources)
        self.rows_by_source = {e["name"]: int(e["rows"]) for e in self.manifest["sources"]}
        self.shards: Dict[str, Dict[str, Mapping[str, Any]]] = {}
        self.shard_order: Dict[str, Tuple[str, ...]] = {}
        self.shard_dir: Dict[str, Path] = {}
        for s in self.sources:
            mpath = Path(s.data_files)
            sm = json.loads(mpath.read_text(encoding="utf-8"))
            if sm.get("format") != MIXTURE_FORMAT or sm.get("dtype") != "uint16":
                raise ValueError(f"unsupported source manifest for {s.name}")
            if int(sm["seq_len"]) != self.seq_len:
                raise ValueError(f"sequence length mismatch for {s.name}")
            shards = sm.get("shards") or []
            if not shards:
                raise ValueError(f"source {s.name} does not contain any token shards")
            files = [str(x["file"]) for x in shards]
            if len(set(files)) != len(files):
                raise ValueError(f"source {s.name} contains duplicate shard filenames")
            if any(Path(f).name != f for f in files):
                raise ValueError(f"source {s.name} shard filenames must not contain directories")
            rows = sum(int(x["rows"]) for x in shards)
            want = self.rows_by_source[s.name]
            if rows != want or int(sm["rows"]) != want:
                raise ValueError(f"source {s.name} shard coverage mismatch: shards={rows}, "
                                 f"source={sm['rows']}, mixture={want}")
            for x in shards:
                r, t = int(x["rows"]), int(x["tokens"])
                if r < 1 or t != r * self.seq_len + 1:
                    raise ValueError(f"invalid shard layout for {s.name}/{x['file']}")
                fp = mpath.parent / str(x["file"])
                nbytes = int(x.get("bytes", t * TOKEN_DTYPE.itemsize))
                if not fp.is_file():
                    raise FileNotFoundError(f"token shard missing: {fp}")
                if fp.stat().st_size != nbytes:
                    raise ValueError(f"corrupt token shard {fp}: {fp.stat().st_size} != {nbytes}")
                if verify_sha256 and x.get("sha256"):
                    if hashlib.sha256(fp.read_bytes()).hexdigest() != x["sha256"]:
                        raise ValueError(f"sha256 mismatch for {fp}")
            self.shards[s.name] = {str(x["file"]): x for x in shards}
            self.shard_order[s.name] = tuple(files)
            self.shard_dir[s.name] = mpath.parent
        self.phases = self._load_plan(replay_plan)
        if self.phases is None:
            self.unique_tokens = sum(self.rows_by_source.values()) * self.seq_len
            self.trained_tokens = self.unique_tokens
        else:
            self.unique_tokens, self.trained_tokens = self._plan_tokens(self.phases)

    # ---------------------------------------------------------------- replay
    def _plan_tokens(self, phases) -> Tuple[int, int]:
        unique: Dict[Tuple[str, str], int] = {}
        trained = 0
        for ph in phases:
            n = 0
            for src, sels in ph["sources"].items():
                for sel in sels:
                    k = (src, sel["file"])
                    unique[k] = max(unique.get(k, 0), sel["rows"])
                    n += sel["rows"]
            trained += n * ph["passes"]
        return sum(unique.values()) * self.seq_len, trained * self.seq_len

    def _load_plan(self, plan):
        if plan is None:
            return None
        if not isinstance(plan, Mapping):
            p = Path(plan)
            if not p.is_file():
                p = self.root / p
            if not p.is_file():
                raise FileNotFoundError(f"token replay plan not found: {plan}")
            plan = json.loads(p.read_text(encoding="utf-8"))
        if plan.get("format") != REPLAY_PLAN_FORMAT:
            raise ValueError("unsupported token replay plan format")
        if int(plan.get("seq_len", -1)) != self.seq_len:
            raise ValueError("token replay plan sequence length mismatch")
        phases = plan.get("phases")
        if not isinstance(phases, list) or not phases:
            raise ValueError("token replay plan must contain at least one phase")
        out = []
        for i, ph in enumerate(phases):
            name = str(ph.get("name", f"phase_{i + 1}"))
            passes = int(ph.get("passes", 1))
            if passes < 1:
                raise ValueError(f"token replay phase {name} passes must be positive")
            srcs = ph.get("sources")
            if not isinstance(srcs, Mapping) or not srcs:
                raise ValueError(f"token replay phase {name} has no sources")
            norm = {}
            for src, sels in srcs.items():
                if src not in self.shards:
                    raise ValueError(f"token replay phase {name} references unknown source {src}")
                if not isinstance(sels, list) or not sels:
                    raise ValueError(f"token replay phase {name}/{src} has no shards")
                seen, items = set(), []
                for sel in sels:
                    f = str(sel["file"])
                    if f in seen:
                        raise ValueError(f"token replay phase {name}/{src} repeats shard {f}")
                    seen.add(f)
                    if f not in self.shards[src]:
                        raise ValueError(f"token replay phase {name}/{src} references unknown "
                                         f"shard {f}")
                    full = int(self.shards[src][f]["rows"])
                    rows = int(sel.get("rows", full))
                    if not 1 <= rows <= full:
                        raise ValueError(f"token replay phase {name}/{src}/{f} rows={rows} "
                                         f"outside 1..{full}")
                    items.append({"file": f, "rows": rows})
                norm[src] = tuple(items)
            out.append({"name": name, "passes": passes, "sources": norm})
        out = tuple(out)
        unique, trained = self._plan_tokens(out)
        for key, got in (("unique_tokens", unique), ("trained_tokens", trained)):
            if key in plan and int(plan[key]) != got:
                raise ValueError(f"token replay plan {key} mismatch: declared={plan[key]}, "
                                 f"actual={got}")
        return out

    # ------------------------------------------------------------- iteration
    def _rows(self, src: str, index: int, count: int,
              selections: Optional[Sequence[Mapping[str, Any]]] = None):
        if selections is None:
            selections = [{"file": f, "rows": int(self.shards[src][f]["rows"])}
                          for f in self.shard_order[src]]
        S = self.seq_len
        global_row = 0
        for sel in selections:
            shard = self.shards[src][sel["file"]]
            full = int(shard["rows"])
            tokens = np.memmap(self.shard_dir[src] / sel["file"], mode="r", dtype=TOKEN_DTYPE)
            if tokens.size != full * S + 1:
                raise ValueError(f"corrupt token shard {sel['file']}")
            rows = int(sel["rows"])
            first = (index - global_row) % count
            for r in range(first, rows, count):
                yield _sample(np.asarray(tokens[r * S:(r + 1) * S + 1]))
            del tokens
            global_row += rows

    def _phase(self, ph, index: int, count: int):
        rows = {src: sum(s["rows"] for s in sels) for src, sels in ph["sources"].items()}
        bad = {k: v for k, v in rows.items() if v % count}
        if bad:
            raise ValueError(f"token replay phase {ph['name']} rows must be divisible by "
                             f"world_size * num_workers; shard_count={count}, "
                             f"incompatible={bad}")
        local = {k: v // count for k, v in rows.items()}
        total = sum(local.values())
        srcs = tuple(TextCorpusSource(name=k, weight=v / total, data_files="-")
                     for k, v in local.items())
        its = {k: self._rows(k, index, count, ph["sources"][k]) for k in local}
        counts = {k: 0 for k in local}
        for _ in range(total):
            s = next_source(srcs, counts)
            try:
                item = next(its[s.name])
            except StopIteration as exc:
                raise RuntimeError(f"token replay phase {ph['name']} exhausted {s.name} before "
                                   "its declared row budget") from exc
            counts[s.name] += 1
            yield item

    def _stream(self, index: int, count: int):
        if self.phases is not None:
            for ph in self.phases:
                for _ in range(ph["passes"]):
                    yield from self._phase(ph, index, count)
            return
        bad = {k: v for k, v in self.rows_by_source.items() if v % count}
        if bad:
            raise ValueError("pretokenized source rows must be divisible by world_size * "
                             f"num_workers; shard_count={count}, incompatible={bad}")
        its = {s.name: self._rows(s.name, index, count) for s in self.sources}
        counts = {s.name: 0 for s in self.sources}
        while True:
            s = next_source(self.sources, counts)
            try:
                item = next(its[s.name])
            except StopIteration:
                return
            counts[s.name] += 1
            yield item

    def __iter__(self):
        workers, wid = _shard_slot()
        count, index = self.world_size * workers, self.rank * workers + wid
        skip = self.resume_skip_rows
        for item in self._stream(index, count):
            if skip > 0:
                skip -= 1
                continue
            yield item


def write_token_mixture(root: Union[str, Path], sources: Mapping[str, Tuple[float, np.ndarray]],
                        seq_len: int, rows_per_shard: int) -> Path:
    """Write ``{name: (weight, 1-D token array)}`` as a pretokenized mixture:
    every source cut into rows of ``seq_len + 1`` tokens (sharing boundaries)
    and shards of at most ``rows_per_shard`` rows.  Returns the manifest path."""
    root = Path(root)
    entries = []
    for name, (weight, toks) in sources.items():
        toks = np.asarray(toks)
        if toks.size and (toks.min() < 0 or toks.max() > 65535):
            raise ValueError(f"{name}: token ids must fit uint16")
        n_rows = (toks.size - 1) // seq_len
        if n_rows < 1:
            raise ValueError(f"{name}: fewer than seq_len + 1 tokens")
        d = root / "corpora" / name
        d.mkdir(parents=True, exist_ok=True)
        shards = []
        for k, r0 in enumerate(range(0, n_rows, rows_per_shard)):
            r = min(rows_per_shard, n_rows - r0)
            chunk = toks[r0 * seq_len:(r0 + r) * seq_len + 1].astype(TOKEN_DTYPE)
            f = f"shard-{k:05d}.bin"
            chunk.tofile(d / f)
            shards.append({"file": f, "rows": r, "tokens": int(chunk.size),
                           "bytes": int(chunk.nbytes),
                           "sha256": hashlib.sha256(chunk.tobytes()).hexdigest()})
        sm = {"format": MIXTURE_FORMAT, "dtype": "uint16", "seq_len": seq_len, "rows": n_rows,
              "shards": shards}
        (d / "manifest.json").write_text(json.dumps(sm, indent=1), encoding="utf-8")
        entries.append({"name": name, "weight": float(weight), "rows": n_rows,
                        "manifest": f"corpora/{name}/manifest.json"})
    m = {"format": MIXTURE_FORMAT, "dtype": "uint16", "seq_len": seq_len, "sources": entries}
    path = root / "mixture_manifest.json"
    path.write_text(json.dumps(m, indent=1), encoding="utf-8")
    return path
