"""Text and classification metrics: perplexity, accuracy, F1, exact match,
BLEU, ROUGE-1/2/L, expected calibration error.

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
