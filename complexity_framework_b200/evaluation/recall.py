"""Synthetic associative-recall and induction probes.

Counterpart of complexity/evaluation/associative_recall.py:12-130: key/value
pairs followed by a query key (the model must emit the paired value), and
induction sequences (a random prefix repeated; the second copy is predictable
from the first).  ``score_target_logits`` gives accuracy and mean target
log-probability.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class RecallBatch:
    input_ids: torch.Tensor   # [B, S]
    target_ids: torch.Tensor  # [B]  expected next token after the last input position


@dataclass
class RecallMetrics:
    accuracy: float
    mean_logprob: float


def build_associative_recall_batch(batch: int, num_pairs: int, key_vocab: range,
                                   value_vocab: range, seed: int = 0) -> RecallBatch:
    g = torch.Generator().manual_seed(seed)
    rows, tgts = [], []
    keys = torch.tensor(list(key_vocab))
    vals = torch.tensor(list(value_vocab))
    for _ in range(batch):
        k = keys[torch.randperm(len(keys), generator=g)[:num_pairs]]
        v = vals[torch.randint(0, len(vals), (num_pairs,), generator=g)]
        q = int(torch.randint(0, num_pairs, (1,), generator=g))
        rows.append(torch.cat([torch.stack([k, v], 1).reshape(-1), k[q:q + 1]]))
        tgts.append(v[q])
    return RecallBatch(torch.stack(rows), torch.stack(tgts))


def build_induction_batch(batch: int, prefix_len: int, vocab: int, seed: int = 0) -> RecallBatch:
    g = torch.Generator().manual_seed(seed)
    pre = torch.randint(0, vocab, (batch, prefix_len), generator=g)
    ids = torch.cat([pre, pre[:, :-1]], 1)
    return RecallBatch(ids, pre[:, -1])


@torch.no_grad()
def score_target_logits(logits: torch.Tensor, target_ids: torch.Tensor) -> RecallMetrics:
    """``logits`` [B, S, V] (uses the last position) or [B, V]."""
    last = logits[:, -1] if logits.dim() == 3 else logits
    lp = torch.log_softmax(last.float(), -1)
    acc = (last.argmax(-1) == target_ids).float().mean()
    return RecallMetrics(float(acc), float(lp.gather(-1, target_ids[:, None]).mean()))
