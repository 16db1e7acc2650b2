"""Sequence packing.

Counterparts: complexity/training/sequence_packing.py and
complexity/data/preprocessing.py:147-262 (``PackedSequenceCollator``).
Documents are packed first-fit into rows of ``seq_len`` tokens by the native
``_io.pack_documents``; the collator returns labels that never cross a
document boundary, per-document position ids (RoPE restarts in each
document) and document ids (for block-diagonal attention masks).
"""
from __future__ import annotations

import math as _math
from dataclasses import dataclass as _dataclass
from typing import Dict, List, Sequence, Tuple

import torch

from .tokenization import IGNORE_INDEX


def pack_documents(docs: Sequence[Sequence[int]], seq_len: int, pad_id: int = 0):
    """Returns ``(tokens [R, seq_len], doc_ids [R, seq_len])`` (-1 = padding)."""
    from .. import _io

    lens = [len(d) for d in docs]
    ids = torch.tensor([t for d in docs for t in d], dtype=torch.long)
    off = torch.zeros(len(docs) + 1, dtype=torch.long)
    if lens:
        off[1:] = torch.cumsum(torch.tensor(lens, dtype=torch.long), 0)
    return _io.pack_documents(ids, off, int(seq_len), int(pad_id))


def packed_labels_and_positions(tokens: torch.Tensor, doc_ids: torch.Tensor) -> Dict[str, torch.Tensor]:
    """Next-token labels masked at document ends and padding; positions restart per document."""
    labels = torch.full_like(tokens, IGNORE_INDEX)
    same = (doc_ids[:, 1:] == doc_ids[:, :-1]) & (doc_ids[:, 1:] >= 0)
    labels[:, :-1] = torch.where(same, tokens[:, 1:], torch.full_like(tokens[:, 1:], IGNORE_INDEX))
    R, S = tokens.shape
    pos = torch.zeros_like(tokens)
    ar = torch.arange(S).expand(R, S)
    start = torch.ones_like(doc_ids, dtype=torch.bool)
    start[:, 1:] = doc_ids[:, 1:] != doc_ids[:, :-1]
    first = torch.where(start, ar, torch.zeros_like(ar)).cummax(dim=1).values
    pos = ar - first
    return {"input_ids": tokens, "labels": labels, "position_ids": pos, "doc_ids": doc_ids}


def document_attention_mask(doc_ids: torch.Tensor) -> torch.Tensor:
    """Boolean ``[R, S, S]`` causal block-diagonal mask (True = attend)."""
    S = doc_ids.shape[1]
    causal = torch.ones(S, S, dtype=torch.bool, device=doc_ids.device).tril()
    same = doc_ids[:, :, None] == doc_ids[:, None, :]
    return same & causal & (doc_ids[:, :, None] >= 0)


class PackedSequenceCollator:
    """Collate a list of token-id documents into packed rows."""

    def __init__(self, seq_len: int, pad_id: int = 0, eos_id: int = None):
        self.seq_len, self.pad_id, self.eos_id = seq_len, pad_id, eos_id

    def __call__(self, docs: List) -> Dict[str, torch.Tensor]:
        seqs = []
        for d in docs:
            d = d["input_ids"] if isinstance(d, dict) else d
            d = list(d.tolist() if isinstance(d, torch.Tensor) else d)
            if self.eos_id is not None:
                d = d + [self.eos_id]
            seqs.append(d)
        tokens, doc_ids = pack_documents(seqs, self.seq_len, self.pad_id)
        return packed_labels_and_positions(tokens, doc_ids)


def packing_efficiency(doc_ids: torch.Tensor) -> float:
    return float((doc_ids >= 0).float().mean())


# ------------------------------------------------ packing plans (no truncation)
# Counterpart of complexity/training/sequence_packing.py:16-158: next-fit packs
# of whole examples (never split or dropped) with a separator budget between
# neighbours, utilisation statistics, and exact data-parallel epoch boundaries.

@_dataclass(frozen=True)
class SequencePackingPlan:
    packs: Tuple[Tuple[int, ...], ...]
    lengths: Tuple[int, ...]
    sequence_length: int
    separator_tokens: int

    @property
    def source_items(self) -> int:
        return len(self.lengths)

    @property
    def packed_items(self) -> int:
        return len(self.packs)

    @property
    def source_tokens(self) -> int:
        return sum(self.lengths)

    @property
    def separator_count(self) -> int:
        return sum(max(0, len(p) - 1) for p in self.packs)

    @property
    def capacity_tokens(self) -> int:
        return self.packed_items * self.sequence_length

    @property
    def payload_utilization(self) -> float:
        return self.source_tokens / max(1, self.capacity_tokens)

    @property
    def occupied_utilization(self) -> float:
        return ((self.source_tokens + self.separator_count * self.separator_tokens)
                / max(1, self.capacity_tokens))

    @property
    def naive_payload_utilization(self) -> float:
        return self.source_tokens / max(1, self.source_items * self.sequence_length)

    @property
    def compression_ratio(self) -> float:
        return self.source_items / max(1, self.packed_items)

    def assert_exact_coverage(self) -> None:
        if sorted(i for p in self.packs for i in p) != list(range(self.source_items)):
            raise ValueError("packing plan must contain every source item exactly once")
        for p in self.packs:
            if (sum(self.lengths[i] for i in p) + max(0, len(p) - 1) * self.separator_tokens
                    > self.sequence_length):
                raise ValueError("packing plan contains an over-capacity sequence")


def pack_example_lengths(lengths, *, sequence_length: int,
                         separator_tokens: int = 1) -> SequencePackingPlan:
    """Stable next-fit: examples stay in order; a pack closes when the next
    example (plus a separator) would overflow the window."""
    L, sep = int(sequence_length), int(separator_tokens)
    if L < 1:
        raise ValueError("sequence_length must be positive")
    if sep < 0:
        raise ValueError("separator_tokens cannot be negative")
    ls = tuple(int(x) for x in lengths)
    if not ls:
        raise ValueError("cannot pack an empty example set")
    if any(x < 1 or x > L for x in ls):
        raise ValueError("every example length must be within the sequence window")
    packs: List[Tuple[int, ...]] = []
    cur: List[int] = []
    used = 0
    for i, n in enumerate(ls):
        need = n + (sep if cur else 0)
        if cur and used + need > L:
            packs.append(tuple(cur))
            cur, used, need = [], 0, n
        cur.append(i)
        used += need
    packs.append(tuple(cur))
    plan = SequencePackingPlan(tuple(packs), ls, L, sep)
    plan.assert_exact_coverage()
    return plan


@_dataclass(frozen=True)
class EpochSchedule:
    items: int
    world_size: int
    batch_size_per_rank: int
    epochs: int
    steps_per_epoch: int
    total_steps: int

    def epoch_steps(self) -> Tuple[int, ...]:
        """Global step count at the end of each epoch."""
        return tuple(self.steps_per_epoch * e for e in range(1, self.epochs + 1))


def resolve_epoch_schedule(*, items: int, world_size: int, batch_size_per_rank: int,
                           epochs: int) -> EpochSchedule:
    """ceil(ceil(items / world) / batch) steps per epoch on every rank."""
    vals = dict(items=int(items), world_size=int(world_size),
                batch_size_per_rank=int(batch_size_per_rank), epochs=int(epochs))
    if any(v < 1 for v in vals.values()):
        raise ValueError("epoch schedule values must all be positive")
    spe = _math.ceil(_math.ceil(vals["items"] / vals["world_size"]) / vals["batch_size_per_rank"])
    return EpochSchedule(**vals, steps_per_epoch=spe, total_steps=spe * vals["epochs"])
