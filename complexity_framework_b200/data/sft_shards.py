"""Pre-tokenised SFT shards: writer, reader, supervision contract and relabeling.

Counterparts of complexity/training/sft_shard.py:1-44 (shard-v2 supervision
contract) and complexity/training/sft_relabel.py:1-255 (relabel existing
shards so every assistant turn is supervised, reusing the token content).
The on-disk layout is the reference's, so shards move between the two
frameworks: a partition directory holds

  input_ids.bin   little-endian uint32 tokens of all examples, concatenated
  labels.bin      little-endian int32 causal targets (-100 = no loss), aligned
  examples.jsonl  one object per example: ``offset``, ``num_tokens`` (+ extras)
  sft.idx.json    metadata (``format``, ``assistant_supervision``, ...)

and a dataset root is one partition or a directory of partitions.  Labels are
causal: ``labels[t]`` is the target predicted at position t, i.e.
``input_ids[t + 1]`` inside supervised spans (the final EOS may exist only
as a label).
"""
from __future__ import annotations

import hashlib
import json
import os
import shutil
import tempfile
from pathlib import Path
from typing import Any, Dict, Iterable, List, Mapping, Optional, Sequence, Tuple

import numpy as np
import torch

SHARD_FORMAT_V2 = "complexity-sft-token-shard-v2"
LEGACY_ALL_ASSISTANT_SUPERVISION = "all_assistant_turns"
FINAL_ASSISTANT_SUPERVISION = "final_assistant_only"
MASKED_ASSISTANT_HISTORY = "masked_context"
ALL_ASSISTANT_PROJECTION = "naturalize_card_hand_supervise_all_assistant_turns"
IGNORE = -100


def validate_shard_supervision(metadata: Mapping[str, Any]) -> None:
    """A v2 shard must say how turns map to labels: every assistant turn, or only
    the final one with the earlier assistant turns declared as masked context."""
    if metadata.get("format") != SHARD_FORMAT_V2:
        return
    mode = metadata.get("assistant_supervision")
    if mode == LEGACY_ALL_ASSISTANT_SUPERVISION:
        return
    if mode == FINAL_ASSISTANT_SUPERVISION:
        if metadata.get("history_assistant_turns") != MASKED_ASSISTANT_HISTORY:
            raise ValueError("final-assistant-only SFT shards must declare masked assistant "
                             "history")
        return
    raise ValueError("SFT shard v2 requires all-assistant-turn or final-assistant-only "
                     "supervision")


def write_sft_shard(path, examples: Iterable[Tuple[Sequence[int], Sequence[int]]],
                    metadata: Optional[Mapping[str, Any]] = None) -> Dict[str, int]:
    """Write one partition from (input_ids, causal labels) pairs."""
    d = Path(path)
    d.mkdir(parents=True, exist_ok=True)
    off, n_sup, index = 0, 0, []
    with open(d / "input_ids.bin", "wb") as fi, open(d / "labels.bin", "wb") as fl:
        for ids, lab in examples:
            ids = np.asarray(ids, dtype="<u4")
            lab = np.asarray(lab, dtype="<i4")
            if ids.shape != lab.shape or ids.ndim != 1 or not len(ids):
                raise ValueError("each example needs aligned, non-empty 1-D ids and labels")
            fi.write(ids.tobytes())
            fl.write(lab.tobytes())
            sup = int((lab != IGNORE).sum())
            index.append({"offset": off, "num_tokens": int(len(ids)), "supervised_tokens": sup})
            off += len(ids)
            n_sup += sup
    with open(d / "examples.jsonl", "w", encoding="utf-8") as f:
        for e in index:
            f.write(json.dumps(e) + "\n")
    meta = {"format": SHARD_FORMAT_V2, "assistant_supervision": LEGACY_ALL_ASSISTANT_SUPERVISION,
            "num_examples": len(index), "num_tokens": off, "supervised_tokens": n_sup}
    meta.update(metadata or {})
    validate_shard_supervision(meta)
    (d / "sft.idx.json").write_text(json.dumps(meta, indent=2, sort_keys=True) + "\n")
    return {"examples": len(index), "tokens": off, "supervised_tokens": n_sup}


def shard_partitions(root) -> List[Path]:
    root = Path(root)
    if (root / "sft.idx.json").is_file():
        return [root]
    return sorted(p for p in root.iterdir() if (p / "sft.idx.json").is_file())


class SFTTokenShardDataset(torch.utils.data.Dataset):
    """Examples of every partition under ``root`` as (input_ids, labels) lists
    (memory-mapped; the labels are returned aligned, i.e. ``labels[t] = ids[t]``
    where supervised, the convention of ``training/sft.py``)."""

    def __init__(self, root, max_len: Optional[int] = None):
        self.parts, self.index = [], []
        for pi, p in enumerate(shard_partitions(root)):
            meta = json.loads((p / "sft.idx.json").read_text())
            validate_shard_supervision(meta)
            ids = np.memmap(p / "input_ids.bin", mode="r", dtype="<u4")
            lab = np.memmap(p / "labels.bin", mode="r", dtype="<i4")
            if ids.shape != lab.shape:
                raise ValueError(f"unaligned shard arrays in {p}")
            self.parts.append((ids, lab, meta))
            for line in (p / "examples.jsonl").read_text().splitlines():
                if line.strip():
                    e = json.loads(line)
                    s, n = int(e["offset"]), int(e["num_tokens"])
                    if s < 0 or n <= 0 or s + n > ids.size:
                        raise ValueError(f"invalid example bounds in {p}: {e}")
                    self.index.append((pi, s, n))
        if not self.index:
            raise FileNotFoundError(f"no SFT shard examples under {root}")
        self.max_len = max_len

    def __len__(self) -> int:
        return len(self.index)

    def __getitem__(self, i: int):
        pi, s, n = self.index[i]
        ids, lab, _ = self.parts[pi]
        x = ids[s:s + n].astype(np.int64)
        y = lab[s:s + n].astype(np.int64)
        aligned = np.full(n, IGNORE, dtype=np.int64)   # causal -> aligned labels
        aligned[1:] = y[:-1]
        out_ids, out_lab = x.tolist(), aligned.tolist()
        if self.max_len is not None:
            out_ids, out_lab = out_ids[:self.max_len], out_lab[:self.max_len]
        return out_ids, out_lab


# -------------------------------------------------------------- relabeling
def _find(tokens: np.ndarray, marker: np.ndarray) -> List[int]:
    if marker.size == 0 or tokens.size < marker.size:
        return []
    win = np.lib.stride_tricks.sliding_window_view(tokens, marker.size)
    return np.flatnonzero((win == marker).all(1)).tolist()


def relabel_example(input_ids, labels, *, assistant_marker: Iterable[int],
                    eos_token_id: int) -> Tuple[np.ndarray, int]:
    """Supervise every complete assistant span of one example.

    A span starts at the last token of the assistant marker (which predicts
    the first content token) and runs up to the token before the span's first
    EOS (whose target is that EOS); a final span without an EOS in the inputs
    keeps its existing labels (its EOS exists only as a target).  Checks: some
    label is active, none lies outside an assistant span, active labels equal
    the next input token, and a last active label is the EOS."""
    tok = np.asarray(input_ids, dtype=np.int64)
    old = np.asarray(labels, dtype=np.int64)
    if tok.ndim != 1 or old.shape != tok.shape:
        raise ValueError("input_ids and labels must be aligned one-dimensional arrays")
    marker = np.asarray(tuple(assistant_marker), dtype=np.int64)
    starts = _find(tok, marker)
    if not starts:
        raise ValueError("example contains no Assistant marker")
    new = old.copy()
    allowed = np.zeros(tok.size, dtype=bool)
    for m0 in starts:
        first = m0 + marker.size - 1
        body = m0 + marker.size
        eos = np.flatnonzero(tok[body:] == int(eos_token_id))
        if eos.size:
            end = body + int(eos[0])
            allowed[first:end] = True
            new[first:end] = tok[first + 1:end + 1]
        else:
            allowed[first:] = True
    act = new != IGNORE
    if not act.any():
        raise ValueError("example contains no supervised assistant token")
    if (act & ~allowed).any():
        raise ValueError("active label found outside an assistant response")
    if (new[:-1][act[:-1]] != tok[1:][act[:-1]]).any():
        raise ValueError("active labels are not causally aligned with input_ids")
    if act[-1] and int(new[-1]) != int(eos_token_id):
        raise ValueError("final active label must be the assistant EOS token")
    return new.astype("<i4"), int(act.sum())


def _link_or_copy(src: Path, dst: Path) -> None:
    dst.parent.mkdir(parents=True, exist_ok=True)
    try:
        os.link(src, dst)
    except OSError:
        shutil.copy2(src, dst)


def _sha256(p: Path) -> str:
    h = hashlib.sha256()
    with open(p, "rb") as f:
        for block in iter(lambda: f.read(1 << 23), b""):
            h.update(block)
    return h.hexdigest()


def _relabel_partition(src: Path, dst: Path, marker: List[int], eos: int,
                       skip_verification: bool) -> Dict[str, int]:
    meta = json.loads((src / "sft.idx.json").read_text())
    ids = np.memmap(src / "input_ids.bin", mode="r", dtype="<u4")
    old = np.memmap(src / "labels.bin", mode="r", dtype="<i4")
    if ids.shape != old.shape:
        raise ValueError(f"unaligned shard arrays in {src}")
    ex = [json.loads(x) for x in (src / "examples.jsonl").read_text().splitlines() if x.strip()]
    dst.mkdir(parents=True, exist_ok=True)
    _link_or_copy(src / "input_ids.bin", dst / "input_ids.bin")
    new = np.memmap(dst / "labels.bin", mode="w+", dtype="<i4", shape=old.shape)
    new[:] = old[:]
    sup = changed = 0
    with open(dst / "examples.jsonl", "w", encoding="utf-8") as f:
        for e in ex:
            s, n = int(e["offset"]), int(e["num_tokens"])
            if s < 0 or n <= 0 or s + n > ids.size:
                raise ValueError(f"invalid example bounds in {src}: {e}")
            lab, k = relabel_example(ids[s:s + n], old[s:s + n], assistant_marker=marker,
                                     eos_token_id=eos)
            new[s:s + n] = lab
            changed += int(np.count_nonzero(lab != old[s:s + n]))
            sup += k
            e["supervised_tokens"] = k
            f.write(json.dumps(e, ensure_ascii=False) + "\n")
    new.flush()
    for p in src.iterdir():
        if p.is_file() and p.name not in ("input_ids.bin", "labels.bin", "examples.jsonl",
                                          "sft.idx.json"):
            _link_or_copy(p, dst / p.name)
    if not skip_verification and _sha256(src / "input_ids.bin") != _sha256(dst / "input_ids.bin"):
        raise ValueError(f"reused input_ids changed in {dst}")
    meta.update({"format": SHARD_FORMAT_V2, "parent_format": meta.get("format"),
                 "assistant_supervision": LEGACY_ALL_ASSISTANT_SUPERVISION,
                 "content_reused": True,
                 "content_verification": "skipped_unchanged" if skip_verification else "sha256",
                 "alignment_verification": "causal_labels_and_assistant_spans",
                 "supervised_tokens": sup})
    (dst / "sft.idx.json").write_text(json.dumps(meta, indent=2, sort_keys=True) + "\n")
    return {"examples": len(ex), "tokens": int(ids.size), "supervised_tokens": sup,
            "changed_labels": changed}


def relabel_dataset(source_root, output_root, *, assistant_marker: Sequence[int],
                    eos_token_id: int, skip_content_verification: bool = False
                    ) -> Dict[str, Dict[str, int]]:
    """New dataset at ``output_root`` with every assistant turn supervised; the
    token files are hard-linked (or copied) and verified unchanged; the output
    appears atomically (built in a temporary sibling, then renamed)."""
    src, out = Path(source_root).resolve(), Path(output_root).resolve()
    if not src.is_dir():
        raise FileNotFoundError(src)
    if out.exists():
        raise FileExistsError(f"output already exists: {out}")
    parts = shard_partitions(src)
    if not parts:
        raise FileNotFoundError(f"no SFT partitions found under {src}")
    if not list(assistant_marker):
        raise ValueError("an assistant marker is required")
    out.parent.mkdir(parents=True, exist_ok=True)
    tmp = Path(tempfile.mkdtemp(prefix=f".{out.name}.tmp-", dir=out.parent))
    try:
        own = {"input_ids.bin", "labels.bin", "examples.jsonl", "sft.idx.json",
               "chat_template.json"}
        for p in src.iterdir():
            # partition files are written by _relabel_partition (a hard link of the
            # source labels must never be opened for writing)
            if p.is_file() and p.name not in own:
                _link_or_copy(p, tmp / p.name)
        tpl = src / "chat_template.json"
        if tpl.is_file():
            t = json.loads(tpl.read_text())
            t["training_projection"] = ALL_ASSISTANT_PROJECTION
            (tmp / "chat_template.json").write_text(json.dumps(t, indent=2, sort_keys=True) + "\n")
        res = {}
        for p in parts:
            rel = p.relative_to(src).as_posix() or "."
            res[rel] = _relabel_partition(p, tmp if rel == "." else tmp / rel,
                                          list(assistant_marker), int(eos_token_id),
                                          skip_content_verification)
        tmp.rename(out)
        return res
    except Exception:
        shutil.rmtree(tmp, ignore_errors=True)
        raise
