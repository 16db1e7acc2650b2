"""Sequence packing.

Counterparts: complexity/training/sequence_packing.py and
complexity/data/preprocessing.py:147-262 (``PackedSequenceCollator``).
Documents are packed first-fit into rows of ``seq_len`` tokens by the native
``_io.pack_documents``; the collator returns labels that never cross a
document boundary, per-document position ids (RoPE restarts in each
document) and document ids (for block-diagonal attention masks).
"""
from __future__ import annotations

from typing import Dict, List, Sequence

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
