"""Text and classification metrics: perplexity, accuracy, F1, exact match,
BLEU, ROUGE-1/2/L, expected calibration error, BERTScore, distinct-n and
self-BLEU diversity.

Counterparts: complexity/evaluation/evaluator.py:31-176, :476-536 and
metrics.py (ROUGE/BLEU).  BLEU follows Papineni et al. (2002): clipped n-gram
precisions up to 4, geometric mean, brevity penalty; ROUGE-N is n-gram
recall/precision F1 and ROUGE-L the LCS F1 (Lin, 2004).
"""
from __future__ import annotations

import math
import re
from collections import Counter
from typing import Dict, Iterable, List, Sequence

import torch


def perplexity_from_loss(mean_nll: float) -> float:
    return math.exp(min(mean_nll, 100.0))


@torch.no_grad()
def compute_perplexity(model, batches: Iterable, ignore_index: int = -100) -> Dict:
    """Token-weighted NLL.  A batch is ``[B, S]`` ids (predict ids[:, 1:]) or a
    dict / pair with ``labels`` already aligned to the inputs (the data
    loaders' convention: ``labels[t]`` is the token after ``input_ids[t]``)."""
    dev = next(model.parameters()).device
    tot, n = 0.0, 0
    for b in batches:
        if isinstance(b, dict):
            ids, labels = b["input_ids"], b.get("labels")
        elif isinstance(b, (tuple, list)):
            ids, labels = b[0], b[1]
        else:
            ids, labels = b, None
        logits = model(ids.to(dev))["logits"].float()
        if labels is None:
            lg, tgt = logits[:, :-1], ids.to(dev)[:, 1:]
        else:
            lg, tgt = logits, labels.to(dev)
        nll = torch.nn.functional.cross_entropy(lg.reshape(-1, lg.shape[-1]), tgt.reshape(-1),
                                                ignore_index=ignore_index, reduction="sum")
        tot += float(nll)
        n += int((tgt != ignore_index).sum())
    mean = tot / max(n, 1)
    return {"loss": mean, "perplexity": perplexity_from_loss(mean), "tokens": n}


def compute_accuracy(preds: Sequence, labels: Sequence) -> float:
    return sum(int(p == l) for p, l in zip(preds, labels)) / max(1, len(labels))


def compute_f1(preds: Sequence, labels: Sequence, average: str = "macro") -> Dict[str, float]:
    classes = sorted(set(labels) | set(preds))
    per = {}
    tp_all = fp_all = fn_all = 0
    for c in classes:
        tp = sum(1 for p, l in zip(preds, labels) if p == c and l == c)
        fp = sum(1 for p, l in zip(preds, labels) if p == c and l != c)
        fn = sum(1 for p, l in zip(preds, labels) if p != c and l == c)
        tp_all, fp_all, fn_all = tp_all + tp, fp_all + fp, fn_all + fn
        pr = tp / (tp + fp) if tp + fp else 0.0
        rc = tp / (tp + fn) if tp + fn else 0.0
        per[c] = 2 * pr * rc / (pr + rc) if pr + rc else 0.0
    if average == "micro":
        pr = tp_all / (tp_all + fp_all) if tp_all + fp_all else 0.0
        rc = tp_all / (tp_all + fn_all) if tp_all + fn_all else 0.0
        f1 = 2 * pr * rc / (pr + rc) if pr + rc else 0.0
    else:
        f1 = sum(per.values()) / max(1, len(per))
    return {"f1": f1, "per_class": per}


def _norm(s: str) -> str:
    s = s.lower()
    s = re.sub(r"\b(a|an|the)\b", " ", s)
    s = re.sub(r"[^\w\s]", " ", s)
    return " ".join(s.split())


def exact_match(pred: str, ref: str) -> float:
    return float(_norm(pred) == _norm(ref))


def token_f1(pred: str, ref: str) -> float:
    p, r = _norm(pred).split(), _norm(ref).split()
    common = Counter(p) & Counter(r)
    same = sum(common.values())
    if same == 0:
        return 0.0
    pr, rc = same / len(p), same / len(r)
    return 2 * pr * rc / (pr + rc)


def _ngrams(toks: List[str], n: int) -> Counter:
    return Counter(tuple(toks[i:i + n]) for i in range(len(toks) - n + 1))


def bleu(candidates: Sequence[str], references: Sequence[Sequence[str]], max_n: int = 4,
         smooth: bool = True) -> float:
    """Corpus BLEU; each candidate has one or more references."""
    clipped = [0] * max_n
    total = [0] * max_n
    c_len = r_len = 0
    for cand, refs in zip(candidates, references):
        c = cand.split()
        rs = [r.split() for r in refs]
        c_len += len(c)
        r_len += min((abs(len(r) - len(c)), len(r)) for r in rs)[1]
        for n in range(1, max_n + 1):
            cn = _ngrams(c, n)
            mx: Counter = Counter()
            for r in rs:
                mx |= _ngrams(r, n)
            clipped[n - 1] += sum(min(v, mx[g]) for g, v in cn.items())
            total[n - 1] += max(0, len(c) - n + 1)
    logp = 0.0
    for n in range(max_n):
        num, den = clipped[n], total[n]
        if smooth:
            num, den = num + (1 if n > 0 else 0), den + (1 if n > 0 else 0)
        if num == 0 or den == 0:
            return 0.0
        logp += math.log(num / den) / max_n
    bp = 1.0 if c_len > r_len else math.exp(1 - r_len / max(c_len, 1))
    return bp * math.exp(logp)


def _lcs(a: List[str], b: List[str]) -> int:
    prev = [0] * (len(b) + 1)
    for x in a:
        cur = [0]
        for j, y in enumerate(b):
            cur.append(prev[j] + 1 if x == y else max(prev[j + 1], cur[j]))
        prev = cur
    return prev[-1]


def rouge(candidate: str, reference: str) -> Dict[str, float]:
    c, r = _norm(candidate).split(), _norm(reference).split()
    out = {}
    for n in (1, 2):
        cn, rn = _ngrams(c, n), _ngrams(r, n)
        ov = sum((cn & rn).values())
        p = ov / max(1, sum(cn.values()))
        rc = ov / max(1, sum(rn.values()))
        out[f"rouge{n}"] = 2 * p * rc / (p + rc) if p + rc else 0.0
    l = _lcs(c, r)
    p, rc = l / max(1, len(c)), l / max(1, len(r))
    out["rougeL"] = 2 * p * rc / (p + rc) if p + rc else 0.0
    return out


def expected_calibration_error(confidences: Sequence[float], correct: Sequence[bool],
                               bins: int = 10) -> float:
    n = len(confidences)
    ece = 0.0
    for b in range(bins):
        lo, hi = b / bins, (b + 1) / bins
        idx = [i for i, c in enumerate(confidences) if lo < c <= hi or (b == 0 and c == 0)]
        if idx:
            acc = sum(correct[i] for i in idx) / len(idx)
            conf = sum(confidences[i] for i in idx) / len(idx)
            ece += len(idx) / n * abs(acc - conf)
    return ece


# ------------------------------------------------------------ embedding / diversity
def _hidden_states(model, ids: List[int], device) -> "torch.Tensor":
    x = torch.tensor([ids], dtype=torch.long, device=device)
    if _accepts(model, "return_hidden_states"):      # ComplexityModel
        out = model(x, return_hidden_states=True, return_logits=False)
    elif _accepts(model, "output_hidden_states"):    # HF models
        out = model(x, output_hidden_states=True)
    else:
        out = model(x)
    if isinstance(out, dict):
        h = next((out[k] for k in ("hidden_states", "last_hidden_state", "logits")
                  if out.get(k) is not None), None)
    elif hasattr(out, "last_hidden_state"):
        h = out.last_hidden_state
    else:
        h = out[0] if isinstance(out, (tuple, list)) else out
    if isinstance(h, (tuple, list)):
        h = h[-1]
    return h[0].float()


def _accepts(model, name: str) -> bool:
    import inspect

    try:
        return name in inspect.signature(model.forward).parameters
    except (TypeError, ValueError):
        return False


class BertScoreEvaluator:
    """BERTScore with any token encoder (greedy cosine matching of contextual
    token embeddings, Zhang et al. 2020): precision averages, over candidate
    tokens, the best cosine to a reference token; recall the reverse; F1 their
    harmonic mean.  ``pooling="mean"`` instead compares mean-pooled sentence
    embeddings, the counterpart's definition.

    Counterpart: complexity/evaluation/metrics.py:290-358.  ``encode`` maps a
    string to token ids (a ``Tokenizer`` of this package, an HF tokenizer, or a
    callable); the model returns hidden states ([1, T, D]) or a dict / output
    object carrying them.
    """

    def __init__(self, model, tokenizer, device=None, pooling: str = "greedy"):
        import torch

        if pooling not in ("greedy", "mean"):
            raise ValueError("pooling must be 'greedy' or 'mean'")
        self.model, self.tokenizer, self.pooling = model, tokenizer, pooling
        if device is None:
            params = list(model.parameters()) if hasattr(model, "parameters") else []
            device = params[0].device if params else torch.device("cpu")
        self.device = device

    def _ids(self, text: str) -> List[int]:
        tok = self.tokenizer
        ids = tok.encode(text) if hasattr(tok, "encode") else tok(text)
        if isinstance(ids, dict):
            ids = ids["input_ids"]
        return list(ids) or [0]

    def _embed(self, text: str):
        import torch

        with torch.no_grad():
            h = _hidden_states(self.model, self._ids(text), self.device)
        return torch.nn.functional.normalize(h, dim=-1)

    def score(self, predictions: Sequence[str], references: Sequence[str]) -> Dict[str, float]:
        if len(predictions) != len(references):
            raise ValueError("predictions and references differ in length")
        P, R, F = [], [], []
        for pred, ref in zip(predictions, references):
            a, b = self._embed(pred), self._embed(ref)
            if self.pooling == "mean":
                import torch

                s = float(torch.nn.functional.cosine_similarity(a.mean(0), b.mean(0), dim=0))
                p = r = s
            else:
                sim = a @ b.T
                p = float(sim.max(1).values.mean())
                r = float(sim.max(0).values.mean())
            P.append(p)
            R.append(r)
            F.append(2 * p * r / (p + r) if p + r > 0 else 0.0)
        n = max(1, len(F))
        return {"precision": sum(P) / n, "recall": sum(R) / n, "f1": sum(F) / n}


def distinct_n(texts: Sequence[str], max_n: int = 4) -> Dict[str, float]:
    """Unique / total n-grams over all texts, per n (higher = more diverse)."""
    out = {}
    for n in range(1, max_n + 1):
        grams = Counter()
        for t in texts:
            grams.update(_ngrams(t.lower().split(), n))
        total = sum(grams.values())
        out[f"distinct_{n}"] = len(grams) / total if total else 0.0
    return out


def self_bleu(texts: Sequence[str], max_n: int = 4) -> float:
    """Mean BLEU of each text against the others (lower = more diverse)."""
    if len(texts) < 2:
        return 0.0
    scores = [bleu([t], [[o for j, o in enumerate(texts) if j != i]], max_n=max_n)
              for i, t in enumerate(texts)]
    return sum(scores) / len(scores)
