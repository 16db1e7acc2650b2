"""Class-based evaluation front-ends with the reference's names.

Counterparts of complexity/evaluation/metrics.py:20-560 (``RougeScorer``,
``BleuScorer``, ``DiversityMetrics``, ``CoherenceMetrics``) and
complexity/evaluation/evaluator.py:21-600 (``EvalConfig``, ``Evaluator``,
``evaluate_on_dataset``).  The scorers return the reference's result shapes
(per-metric precision / recall / F1 dictionaries, BLEU with its n-gram
precisions); the model-side evaluations use the framework's own perplexity,
choice log-probability and calibration functions.  Without an embedding
model, sentence coherence is the mean Jaccard overlap of consecutive
sentences' word sets (the reference returns a fixed 0.8 placeholder there).
"""
from __future__ import annotations

import math
import re
from collections import Counter
from dataclasses import dataclass
from typing import Any, Dict, Iterable, List, Optional, Sequence

import torch

from .benchmarks import choice_logprobs
from .metrics import (BertScoreEvaluator, compute_perplexity, distinct_n,
                      expected_calibration_error, exact_match, token_f1)


def _grams(tokens: Sequence[str], n: int) -> Counter:
    return Counter(tuple(tokens[i:i + n]) for i in range(len(tokens) - n + 1))


def _prf(overlap: float, p_total: float, r_total: float) -> Dict[str, float]:
    p = overlap / p_total if p_total else 0.0
    r = overlap / r_total if r_total else 0.0
    return {"precision": p, "recall": r, "f1": 2 * p * r / (p + r) if p + r else 0.0}


class RougeScorer:
    """ROUGE-1 / ROUGE-2 (n-gram overlap) and ROUGE-L (longest common subsequence)."""

    def __init__(self, use_stemmer: bool = False):
        self.use_stemmer = use_stemmer

    def _tokens(self, text: str) -> List[str]:
        toks = re.findall(r"\w+", text.lower())
        if self.use_stemmer:  # light suffix stripping (no external stemmer)
            toks = [re.sub(r"(ing|ed|es|s)$", "", t) if len(t) > 4 else t for t in toks]
        return toks

    @staticmethod
    def _lcs(a: Sequence[str], b: Sequence[str]) -> int:
        prev = [0] * (len(b) + 1)
        for x in a:
            cur = [0]
            for j, y in enumerate(b):
                cur.append(prev[j] + 1 if x == y else max(prev[j + 1], cur[j]))
            prev = cur
        return prev[-1]

    def score(self, prediction: str, reference: str) -> Dict[str, Dict[str, float]]:
        p, r = self._tokens(prediction), self._tokens(reference)
        out = {}
        for n in (1, 2):
            pg, rg = _grams(p, n), _grams(r, n)
            out[f"rouge{n}"] = _prf(sum((pg & rg).values()), sum(pg.values()), sum(rg.values()))
        out["rougeL"] = _prf(self._lcs(p, r), len(p), len(r))
        return out

    def score_batch(self, predictions: List[str], references: List[str]):
        scores = [self.score(p, r) for p, r in zip(predictions, references)]
        return {m: {k: sum(s[m][k] for s in scores) / max(1, len(scores))
                    for k in ("precision", "recall", "f1")} for m in ("rouge1", "rouge2", "rougeL")}


class BleuScorer:
    """Sentence BLEU against several references: n-gram precisions clipped by
    the largest count in any reference, geometric mean (zero when any order has
    no match), brevity penalty against the closest reference length (ties to
    the shorter).  ``smooth``: an order for which the prediction has no n-grams
    at all (shorter than n) counts as 1 / (length + 1) instead of 0."""

    def __init__(self, max_n: int = 4, smooth: bool = True):
        self.max_n, self.smooth = max_n, smooth

    @staticmethod
    def _tokens(text: str) -> List[str]:
        return text.lower().split()

    def _stats(self, c: List[str], refs: List[List[str]]):
        clipped, totals = [], []
        for n in range(1, self.max_n + 1):
            cg = _grams(c, n)
            best: Counter = Counter()
            for r in refs:
                best |= _grams(r, n)
            clipped.append(sum((cg & best).values()))
            totals.append(sum(cg.values()))
        ref_len = min((len(r) for r in refs), key=lambda x: (abs(x - len(c)), x))
        return clipped, totals, ref_len

    def _combine(self, clipped, totals, c_len: int, ref_len: int):
        precs = [(1.0 / (c_len + 1)) if (self.smooth and t == 0) else (h / t if t else 0.0)
                 for h, t in zip(clipped, totals)]
        bp = 1.0 if c_len > ref_len else (math.exp(1 - ref_len / c_len) if c_len else 0.0)
        bleu = bp * math.exp(sum(math.log(p) for p in precs) / len(precs)) \
            if all(p > 0 for p in precs) else 0.0
        return {"bleu": bleu, "precisions": precs, "brevity_penalty": bp}

    def score(self, prediction: str, references: List[str]) -> Dict[str, Any]:
        c = self._tokens(prediction)
        if not c:
            return {"bleu": 0.0, "precisions": [0.0] * self.max_n}
        refs = [self._tokens(r) for r in references]
        clipped, totals, ref_len = self._stats(c, refs)
        return self._combine(clipped, totals, len(c), ref_len)

    def score_corpus(self, predictions: List[str], references_list: List[List[str]]):
        """Corpus BLEU: clipped counts, totals and lengths summed before combining."""
        C, T = [0] * self.max_n, [0] * self.max_n
        cl = rl = 0
        for p, refs in zip(predictions, references_list):
            c = self._tokens(p)
            h, t, r = self._stats(c, [self._tokens(x) for x in refs])
            C = [a + b for a, b in zip(C, h)]
            T = [a + b for a, b in zip(T, t)]
            cl, rl = cl + len(c), rl + r
        return self._combine(C, T, cl, rl)

    def score_batch(self, predictions: List[str], references: List[List[str]]) -> Dict[str, float]:
        s = [self.score(p, r)["bleu"] for p, r in zip(predictions, references)]
        return {"bleu": sum(s) / max(1, len(s))}


class DiversityMetrics:
    def __init__(self, max_n: int = 4):
        self.max_n = max_n

    def distinct_n(self, texts: List[str]) -> Dict[str, float]:
        return distinct_n(texts, self.max_n)

    def self_bleu(self, texts: List[str]) -> float:
        sc = BleuScorer(self.max_n)
        vals = [sc.score(t, texts[:i] + texts[i + 1:])["bleu"] for i, t in enumerate(texts)
                if len(texts) > 1]
        return sum(vals) / len(vals) if vals else 0.0

    def entropy(self, texts: List[str]) -> Dict[str, float]:
        def h(counts: Counter) -> float:
            tot = sum(counts.values())
            return -sum(c / tot * math.log2(c / tot) for c in counts.values()) if tot else 0.0
        toks = [t.lower().split() for t in texts]
        uni = Counter(w for ts in toks for w in ts)
        bi = Counter(g for ts in toks for g in zip(ts, ts[1:]))
        return {"unigram_entropy": h(uni), "bigram_entropy": h(bi)}

    def compute_all(self, texts: List[str]) -> Dict[str, float]:
        out = dict(self.distinct_n(texts))
        out["self_bleu"] = self.self_bleu(texts)
        out.update(self.entropy(texts))
        return out


class CoherenceMetrics:
    def repetition_rate(self, text: str, n: int = 3) -> float:
        """1 - unique / total n-grams of the text."""
        g = _grams(text.lower().split(), n)
        tot = sum(g.values())
        return 1 - len(g) / tot if tot else 0.0

    def sentence_coherence(self, text: str, model=None, tokenizer=None) -> float:
        sents = [s.strip() for s in re.split(r"[.!?]+", text) if s.strip()]
        if len(sents) < 2:
            return 1.0
        if model is not None:
            ev = BertScoreEvaluator(model, tokenizer)
            vals = [float(ev.score([a], [b])["f1"]) for a, b in zip(sents, sents[1:])]
        else:
            vals = []
            for a, b in zip(sents, sents[1:]):
                wa, wb = set(a.lower().split()), set(b.lower().split())
                vals.append(len(wa & wb) / max(1, len(wa | wb)))
        return sum(vals) / len(vals)

    def compute_all(self, texts: List[str], model=None, tokenizer=None) -> Dict[str, float]:
        reps = [self.repetition_rate(t) for t in texts]
        coh = [self.sentence_coherence(t, model, tokenizer) for t in texts]
        return {"avg_repetition_rate": sum(reps) / max(1, len(reps)),
                "avg_coherence": sum(coh) / max(1, len(coh))}


# ------------------------------------------------------------- model side
@dataclass
class EvalConfig:
    batch_size: int = 8
    max_length: int = 2048
    stride: int = 512
    num_samples: Optional[int] = None
    verbose: bool = True
    dtype: torch.dtype = torch.bfloat16


def _take(batches: Iterable, n: Optional[int]):
    for i, b in enumerate(batches):
        if n is not None and i >= n:
            return
        yield b


class Evaluator:
    def __init__(self, model, tokenizer=None, config: Optional[EvalConfig] = None):
        self.model, self.tokenizer = model, tokenizer
        self.config = config or EvalConfig()
        self.model.eval()

    def _dev(self):
        return next(self.model.parameters()).device

    @torch.no_grad()
    def perplexity(self, dataloader: Iterable, max_samples: Optional[int] = None) -> float:
        return float(compute_perplexity(self.model, _take(dataloader, max_samples))["perplexity"])

    @torch.no_grad()
    def _next_token_stats(self, batches):
        dev = self._dev()
        for b in batches:
            ids = (b["input_ids"] if isinstance(b, dict) else
                   (b[0] if isinstance(b, (tuple, list)) else b)).to(dev)
            logits = self.model(ids)["logits"][:, :-1].float()
            yield logits, ids[:, 1:]

    def accuracy(self, dataloader: Iterable, max_samples: Optional[int] = None) -> float:
        hit = tot = 0
        for logits, tgt in self._next_token_stats(_take(dataloader, max_samples)):
            hit += int((logits.argmax(-1) == tgt).sum())
            tot += tgt.numel()
        return hit / tot if tot else 0.0

    def multiple_choice_accuracy(self, questions: List[Dict[str, Any]]) -> float:
        ok = 0
        for q in questions:
            lp = choice_logprobs(self.model, self.tokenizer, q["context"], q["choices"])
            ok += int(max(range(len(lp)), key=lp.__getitem__) == int(q["answer"]))
        return ok / len(questions) if questions else 0.0

    @torch.no_grad()
    def generate_and_evaluate(self, prompts: List[str], references: List[str],
                              max_new_tokens: int = 100,
                              metrics: Sequence[str] = ("f1", "exact_match")) -> Dict[str, float]:
        from ..inference.engine import GenerationConfig, InferenceEngine

        eng = InferenceEngine(self.model)
        gen = GenerationConfig(max_new_tokens=max_new_tokens,
                               eos_token_id=getattr(self.tokenizer, "eos_token_id", None))
        outs = eng.generate_tokens([self.tokenizer.encode(p) for p in prompts], gen)
        texts = [self.tokenizer.decode(o) for o in outs]
        res: Dict[str, float] = {}
        if "f1" in metrics:
            res["f1"] = sum(token_f1(t, r) for t, r in zip(texts, references)) / len(texts)
        if "exact_match" in metrics:
            res["exact_match"] = sum(exact_match(t, r) for t, r in zip(texts, references)) / len(texts)
        if "rouge" in metrics:
            res.update({k: v["f1"] for k, v in RougeScorer().score_batch(texts, references).items()})
        if "bleu" in metrics:
            res.update(BleuScorer().score_batch(texts, [[r] for r in references]))
        return res

    def calibration_error(self, dataloader: Iterable, num_bins: int = 10) -> float:
        conf, correct = [], []
        for logits, tgt in self._next_token_stats(dataloader):
            p = logits.softmax(-1)
            c, pred = p.max(-1)
            conf += c.flatten().tolist()
            correct += (pred == tgt).flatten().tolist()
        return expected_calibration_error(conf, correct, num_bins)


def evaluate_on_dataset(model, dataloader, tokenizer=None,
                        metrics: Sequence[str] = ("perplexity", "accuracy")) -> Dict[str, float]:
    batches = list(dataloader)
    ev = Evaluator(model, tokenizer)
    out = {}
    if "perplexity" in metrics:
        out["perplexity"] = ev.perplexity(batches)
    if "accuracy" in metrics:
        out["accuracy"] = ev.accuracy(batches)
    if "calibration" in metrics or "ece" in metrics:
        out["ece"] = ev.calibration_error(batches)
    return out
