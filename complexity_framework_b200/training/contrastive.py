"""Contrastive sentence-embedding training: InfoNCE, pair mixtures, stage runner.

Counterparts: complexity/training/info_nce.py:17-76 (in-batch-negative
InfoNCE with optional per-anchor hard negatives), complexity/training/
embedding_pairs.py:20-284 (tokenised anchor/positive pairs, AllNLI and
MS MARCO pair sources, sqrt-count weights, a weighted pair mixture with
hard negatives and token-target replay) and
scripts/train_tr_hash_embedding_100m.py:103-329 (the ~118M bidirectional
TR-Hash encoder and its chained training stages).

There is no network here, so sources are local: JSONL files (one object per
line) or in-memory row iterables.  Rows use the mixture schema
``{"query": str, "document": str, "negative": [str, ...]}``; AllNLI pair
files use ``{"anchor", "positive"}`` and MS MARCO comes as its three tables
(queries, corpus, triplets of ids).  Batches are dicts of
``anchor_input_ids / anchor_attention_mask / positive_* [/ negative_*]``,
which ``Trainer`` passes straight to ``compute_pair_loss``.
"""
from __future__ import annotations

import json
import math
import random
from typing import Callable, Dict, Iterable, Iterator, List, Mapping, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F
from torch.utils.data import IterableDataset, get_worker_info


# ------------------------------------------------------------------- loss
def info_nce_loss(anchor_embeddings: torch.Tensor, positive_embeddings: torch.Tensor, *,
                  temperature: float = 0.05, symmetric: bool = False,
                  hard_negative_embeddings: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Cross-entropy of each anchor against [every positive of the batch | its own
    hard negatives], the matching positive being the target (L2-normalised
    inputs; logits = cosine / temperature).

    ``symmetric`` averages in the positive -> anchor direction over the batch
    (hard negatives belong to one anchor and take no part in it).
    """
    if anchor_embeddings.shape != positive_embeddings.shape:
        raise ValueError(f"anchor/positive shape mismatch: {tuple(anchor_embeddings.shape)} vs "
                         f"{tuple(positive_embeddings.shape)}")
    B = anchor_embeddings.shape[0]
    if B < 2:
        raise ValueError(f"info_nce_loss needs batch_size >= 2 for in-batch negatives, got {B}")
    inv_t = 1.0 / temperature
    sim = (anchor_embeddings @ positive_embeddings.transpose(0, 1)) * inv_t
    target = torch.arange(B, device=sim.device)
    logits = sim
    if hard_negative_embeddings is not None:
        hn = hard_negative_embeddings
        if hn.dim() != 3 or hn.shape[0] != B:
            raise ValueError(f"hard_negative_embeddings must be (batch={B}, num_hard_negatives, "
                             f"dim), got {tuple(hn.shape)}")
        logits = torch.cat((sim, torch.einsum("bd,bkd->bk", anchor_embeddings, hn) * inv_t), 1)
    loss = F.cross_entropy(logits, target)
    if symmetric:
        loss = 0.5 * (loss + F.cross_entropy(sim.transpose(0, 1), target))
    return loss


def sqrt_normalized_weights(counts: Mapping[str, int]) -> Dict[str, float]:
    """sqrt(count_i) / sum_j sqrt(count_j): small sources gain share, large ones lose."""
    if not counts:
        raise ValueError("counts must be non-empty")
    roots = {k: math.sqrt(float(v)) for k, v in counts.items()}
    z = sum(roots.values())
    return {k: r / z for k, r in roots.items()}


# --------------------------------------------------------------- tokenise
def encode_fixed(tokenizer, text: str, max_len: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """(ids [max_len] int64, mask [max_len] float32): truncated, right-padded.

    Accepts a Hugging Face style callable tokenizer (``tokenizer(text, ...)``)
    or any object with ``encode(text) -> List[int]`` (pad id from
    ``pad_token_id``, else 0).
    """
    if hasattr(tokenizer, "encode") and not hasattr(tokenizer, "model_input_names"):
        ids = list(tokenizer.encode(text))[:max_len]
        pad = getattr(tokenizer, "pad_token_id", None)
        pad = 0 if pad is None else int(pad)
        n = len(ids)
        out = torch.full((max_len,), pad, dtype=torch.long)
        out[:n] = torch.tensor(ids, dtype=torch.long)
        mask = torch.zeros(max_len)
        mask[:n] = 1.0
        return out, mask
    enc = tokenizer(text, padding="max_length", truncation=True, max_length=max_len,
                    return_tensors="pt")
    return enc["input_ids"][0], enc["attention_mask"][0].float()


def tokenize_pair(tokenizer, anchor: str, positive: str, max_len: int) -> Dict[str, torch.Tensor]:
    a_ids, a_mask = encode_fixed(tokenizer, anchor, max_len)
    p_ids, p_mask = encode_fixed(tokenizer, positive, max_len)
    return {"anchor_input_ids": a_ids, "anchor_attention_mask": a_mask,
            "positive_input_ids": p_ids, "positive_attention_mask": p_mask}


# ----------------------------------------------------------------- sources
def read_jsonl(path: str) -> Iterator[dict]:
    with open(path, encoding="utf-8") as f:
        for line in f:
            line = line.strip()
            if line:
                yield json.loads(line)


def _shard_index(rank: int, world: int) -> Tuple[int, int]:
    """(index, count) of this (rank, data-loader worker) among all readers."""
    wi = get_worker_info()
    nw, w = (wi.num_workers, wi.id) if wi is not None else (1, 0)
    return rank * nw + w, world * nw


def _strided(rows: Iterable, index: int, count: int) -> Iterator:
    for i, r in enumerate(rows):
        if i % count == index:
            yield r


class AllNLIPairDataset(IterableDataset):
    """Entailment pairs (``anchor`` premise, ``positive`` hypothesis) from a local
    JSONL file, sharded over ranks and loader workers."""

    def __init__(self, tokenizer, path: str, *, max_seq_len: int = 128, rank: int = 0,
                 world_size: int = 1):
        self.tokenizer, self.path, self.max_seq_len = tokenizer, path, max_seq_len
        self.rank, self.world_size = rank, world_size

    def __iter__(self):
        idx, cnt = _shard_index(self.rank, self.world_size)
        for row in _strided(read_jsonl(self.path), idx, cnt):
            a, p = row.get("anchor"), row.get("positive")
            if a and p:
                yield tokenize_pair(self.tokenizer, a, p, self.max_seq_len)


class MSMarcoPairDataset(IterableDataset):
    """Query / relevant-passage pairs joined from MS MARCO's three tables (local
    JSONL: queries ``{query_id, query}``, corpus ``{passage}`` whose row index is
    the passage id, triplets ``{query_id, positive_id, ...}``); only the positive
    passage is used, in-batch negatives supply the rest."""

    def __init__(self, tokenizer, queries_path: str, corpus_path: str, triplets_path: str, *,
                 max_seq_len: int = 128, rank: int = 0, world_size: int = 1):
        self.tokenizer, self.max_seq_len = tokenizer, max_seq_len
        self.paths = (queries_path, corpus_path, triplets_path)
        self.rank, self.world_size = rank, world_size
        self._queries: Optional[Dict] = None
        self._corpus: Optional[List[str]] = None

    def _load(self) -> None:
        if self._queries is None:
            self._queries = {r["query_id"]: r["query"] for r in read_jsonl(self.paths[0])}
            self._corpus = [r.get("passage", "") for r in read_jsonl(self.paths[1])]

    def __iter__(self):
        self._load()
        idx, cnt = _shard_index(self.rank, self.world_size)
        for row in _strided(read_jsonl(self.paths[2]), idx, cnt):
            q = self._queries.get(row["query_id"])
            pid = int(row["positive_id"])
            doc = self._corpus[pid] if 0 <= pid < len(self._corpus) else None
            if q and doc:
                yield tokenize_pair(self.tokenizer, q, doc, self.max_seq_len)


class WeightedPairMixtureDataset(IterableDataset):
    """Interleave pair sources at target weights by weighted fair queuing: the next
    row comes from the active source with the smallest emitted / weight (the first
    listed on ties).  Every source runs to exhaustion (weights shape the order,
    not the total), unless ``target_tokens`` is set: then an exhausted source
    restarts until that many real tokens (anchor + positive + negatives) were
    emitted.  ``num_hard_negatives`` > 0 samples that many of a row's
    ``negative`` texts (with replacement when it has fewer; rows without any are
    skipped).

    Sources: ``streams`` (name -> re-iterable rows) or ``files`` (name -> JSONL
    path); rows are strided over ranks and loader workers.
    """

    def __init__(self, tokenizer, *, split_weights: Mapping[str, float], max_seq_len: int = 128,
                 num_hard_negatives: int = 0, rank: int = 0, world_size: int = 1, seed: int = 0,
                 target_tokens: Optional[int] = None,
                 streams: Optional[Mapping[str, Sequence[dict]]] = None,
                 files: Optional[Mapping[str, str]] = None, dataset_id: Optional[str] = None):
        if not split_weights:
            raise ValueError("split_weights must be non-empty")
        if streams is None and files is None:
            raise ValueError("give the sources as in-memory streams or local JSONL files "
                             "(no network access to fetch them)")
        self.tokenizer, self.split_weights = tokenizer, dict(split_weights)
        self.max_seq_len, self.num_hard_negatives = max_seq_len, num_hard_negatives
        self.rank, self.world_size, self.seed = rank, world_size, seed
        self.target_tokens, self.streams, self.files = target_tokens, streams, files
        self.dataset_id = dataset_id

    def _open(self, name: str) -> Iterator[dict]:
        idx, cnt = _shard_index(self.rank, self.world_size)
        rows = self.streams[name] if self.streams is not None else read_jsonl(self.files[name])
        return _strided(rows, idx, cnt)

    def _negatives(self, row: dict, rng: random.Random) -> Optional[List[str]]:
        negs = list(row.get("negative") or [])
        if not negs:
            return None
        k = self.num_hard_negatives
        return rng.sample(negs, k) if len(negs) >= k else [rng.choice(negs) for _ in range(k)]

    def __iter__(self):
        wi = get_worker_info()
        rng = random.Random(self.seed + self.rank * 1000 + (wi.id if wi is not None else 0))
        names = list(self.split_weights)
        it = {n: self._open(n) for n in names}
        emitted = {n: 0 for n in names}
        done: set = set()
        tokens = 0
        target = self.target_tokens
        while len(done) < len(names):
            if target is not None and tokens >= target:
                return
            src = min((n for n in names if n not in done),
                      key=lambda n: emitted[n] / self.split_weights[n])
            try:
                row = next(it[src])
            except StopIteration:
                if target is not None:
                    it[src] = self._open(src)  # partial replay toward the token target
                else:
                    done.add(src)
                continue
            emitted[src] += 1
            q, d = row.get("query"), row.get("document")
            if not q or not d:
                continue
            ex = tokenize_pair(self.tokenizer, q, d, self.max_seq_len)
            tokens += int(ex["anchor_attention_mask"].sum() + ex["positive_attention_mask"].sum())
            if self.num_hard_negatives > 0:
                negs = self._negatives(row, rng)
                if negs is None:
                    continue
                enc = [encode_fixed(self.tokenizer, t, self.max_seq_len) for t in negs]
                ex["negative_input_ids"] = torch.stack([e[0] for e in enc])
                ex["negative_attention_mask"] = torch.stack([e[1] for e in enc])
                tokens += int(ex["negative_attention_mask"].sum())
            yield ex


# ------------------------------------------------------------ model + loss
def embedding_config(max_seq_len: int, vocab_size: int):
    """The ~118M bidirectional TR-Hash encoder (12 x 768, GQA 12/2, shared 2560 +
    4 experts of 56, top-2 multi-hash, non-causal)."""
    from ..config import ModelConfig

    return ModelConfig(hidden_size=768, num_hidden_layers=12, num_attention_heads=12,
                       num_key_value_heads=2, intermediate_size=224,
                       shared_intermediate_size=2560, vocab_size=vocab_size,
                       max_position_embeddings=max_seq_len, attention_type="gqa",
                       mlp_type="tr_hash_engine", num_experts=4, top_k=2,
                       top_k_primary_weight=0.5, routing_strategy="token_id_multi_hash",
                       route_hash_count=2, shared_expert=True, use_qk_norm=True,
                       tie_word_embeddings=True, is_causal=False)


def compute_pair_loss(model, batch: Dict[str, torch.Tensor], labels=None, *,
                      temperature: float = 0.05) -> torch.Tensor:
    """InfoNCE of one pair batch (hard negatives encoded as one flat batch)."""
    dev = next(model.parameters()).device
    a = model(batch["anchor_input_ids"].to(dev), batch["anchor_attention_mask"].to(dev))
    p = model(batch["positive_input_ids"].to(dev), batch["positive_attention_mask"].to(dev))
    hn = None
    if "negative_input_ids" in batch:
        B, K, L = batch["negative_input_ids"].shape
        flat = model(batch["negative_input_ids"].reshape(B * K, L).to(dev),
                     batch["negative_attention_mask"].reshape(B * K, L).to(dev))
        hn = flat.reshape(B, K, -1)
    return info_nce_loss(a, p, temperature=temperature, hard_negative_embeddings=hn)


def train_embedding_stage(model, batches: Iterable[Dict[str, torch.Tensor]], config, *,
                          temperature: float = 0.05, init_checkpoint: Optional[str] = None,
                          callbacks: Optional[list] = None) -> dict:
    """One training stage of the embedding model with a fresh optimizer; stages
    chain through ``init_checkpoint`` (weights of the previous stage's
    ``save_pretrained`` directory).  Returns the trainer's summary."""
    from .trainer import Trainer

    if init_checkpoint:
        from ..models.builder import ComplexityModel

        src = ComplexityModel.from_pretrained(init_checkpoint, device="cpu")
        model.backbone.load_state_dict(src.state_dict())
    loss_fn: Callable = lambda m, b, labels=None: compute_pair_loss(m, b, temperature=temperature)  # noqa: E731
    trainer = Trainer(model, config, compute_loss=loss_fn, callbacks=callbacks)
    return trainer.train(batches)
