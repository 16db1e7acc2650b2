"""Multiple-choice benchmark runners over local JSONL files.

Counterpart of complexity/evaluation/benchmarks.py:31-640 (MMLU, HellaSwag,
Winogrande, ARC, TruthfulQA and ``BenchmarkRunner``).  There is no network
here, so each benchmark reads a local JSONL file in its public dataset's
schema; scoring is the standard log-likelihood of each choice continuation
given the context (optionally length-normalised), computed for all choices
of a question in one padded forward.
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Dict, List, Optional, Sequence, Tuple

import torch


@dataclass
class BenchmarkResult:
    name: str
    accuracy: float
    num_samples: int
    details: List[Dict[str, Any]] = field(default_factory=list)


@torch.no_grad()
def choice_logprobs(model, tokenizer, context: str, choices: Sequence[str],
                    normalize: bool = True) -> List[float]:
    """Sum (or per-token mean) log p(choice | context) for every choice."""
    dev = next(model.parameters()).device
    ctx = tokenizer.encode(context)
    seqs = [ctx + tokenizer.encode(c) for c in choices]
    L = max(len(s) for s in seqs)
    pad = tokenizer.pad_token_id or 0
    ids = torch.full((len(seqs), L), pad, dtype=torch.long)
    for i, s in enumerate(seqs):
        ids[i, :len(s)] = torch.tensor(s)
    logp = torch.log_softmax(model(ids.to(dev))["logits"].float(), -1).cpu()
    out = []
    for i, s in enumerate(seqs):
        n = len(s) - len(ctx)
        tgt = torch.tensor(s[len(ctx):])
        lp = logp[i, len(ctx) - 1:len(s) - 1].gather(-1, tgt[:, None]).sum()
        out.append(float(lp) / (n if normalize and n else 1))
    return out


class Benchmark:
    name = "benchmark"
    normalize = True

    def __init__(self, path: str, limit: Optional[int] = None):
        self.path, self.limit = path, limit

    def load(self) -> List[Dict[str, Any]]:
        rows = [json.loads(l) for l in Path(self.path).read_text().splitlines() if l.strip()]
        return rows[: self.limit] if self.limit else rows

    def to_mc(self, row: Dict[str, Any]) -> Tuple[str, List[str], int]:
        raise NotImplementedError

    def run(self, model, tokenizer) -> BenchmarkResult:
        correct, details = 0, []
        rows = self.load()
        for row in rows:
            ctx, choices, gold = self.to_mc(row)
            scores = choice_logprobs(model, tokenizer, ctx, choices, self.normalize)
            pred = max(range(len(scores)), key=scores.__getitem__)
            correct += int(pred == gold)
            details.append({"pred": pred, "gold": gold, "scores": scores})
        return BenchmarkResult(self.name, correct / max(1, len(rows)), len(rows), details)


class MMLUBenchmark(Benchmark):
    """Rows: {"question", "choices": [4], "answer": int}."""
    name = "mmlu"
    normalize = False

    def to_mc(self, r):
        letters = "ABCD"
        q = r["question"] + "\n" + "\n".join(f"{letters[i]}. {c}" for i, c in
                                              enumerate(r["choices"])) + "\nAnswer:"
        return q, [f" {letters[i]}" for i in range(len(r["choices"]))], int(r["answer"])


class HellaSwagBenchmark(Benchmark):
    """Rows: {"ctx", "endings": [4], "label": int}."""
    name = "hellaswag"

    def to_mc(self, r):
        return r["ctx"], [" " + e for e in r["endings"]], int(r["label"])


class WinograndeBenchmark(Benchmark):
    """Rows: {"sentence" with "_", "option1", "option2", "answer": "1"|"2"}; the
    two filled-in prefixes are scored on the shared suffix."""
    name = "winogrande"

    def run(self, model, tokenizer) -> BenchmarkResult:
        correct, rows = 0, self.load()
        for r in rows:
            pre, suf = r["sentence"].split("_", 1)
            s = [choice_logprobs(model, tokenizer, pre + r[f"option{k}"], [suf])[0] for k in (1, 2)]
            correct += int((0 if s[0] >= s[1] else 1) == int(r["answer"]) - 1)
        return BenchmarkResult(self.name, correct / max(1, len(rows)), len(rows))


class ARCBenchmark(Benchmark):
    """Rows: {"question", "choices": {"text": [...], "label": [...]}, "answerKey"}."""
    name = "arc"

    def to_mc(self, r):
        labels = r["choices"]["label"]
        return ("Question: " + r["question"] + "\nAnswer:",
                [" " + t for t in r["choices"]["text"]], labels.index(r["answerKey"]))


class TruthfulQABenchmark(Benchmark):
    """MC1 rows: {"question", "mc1_targets": {"choices": [...], "labels": [1,0,...]}}."""
    name = "truthfulqa"

    def to_mc(self, r):
        t = r["mc1_targets"]
        return "Q: " + r["question"] + "\nA:", [" " + c for c in t["choices"]], t["labels"].index(1)


class PIQABenchmark(Benchmark):
    """Rows: {"goal", "sol1", "sol2", "label": 0|1}; zero-shot continuation
    log-likelihood of each solution after "Question: <goal>\nAnswer:".
    ``accuracy`` is acc_norm (log-likelihood per byte of the solution);
    ``details[-1]`` carries both acc and acc_norm."""
    name = "piqa"

    def run(self, model, tokenizer) -> BenchmarkResult:
        rows = self.load()
        acc = acc_norm = 0
        for r in rows:
            ctx = "Question: " + r["goal"] + "\nAnswer:"
            sols = [" " + r["sol1"], " " + r["sol2"]]
            lp = choice_logprobs(model, tokenizer, ctx, sols, normalize=False)
            per_byte = [v / max(1, len(c.encode("utf-8"))) for v, c in zip(lp, sols)]
            gold = int(r["label"])
            acc += int(max(range(2), key=lp.__getitem__) == gold)
            acc_norm += int(max(range(2), key=per_byte.__getitem__) == gold)
        n = max(1, len(rows))
        return BenchmarkResult(self.name, acc_norm / n, len(rows),
                               [{"acc": acc / n, "acc_norm": acc_norm / n}])


BENCHMARKS = {"mmlu": MMLUBenchmark, "piqa": PIQABenchmark, "hellaswag": HellaSwagBenchmark,
              "winogrande": WinograndeBenchmark, "arc": ARCBenchmark,
              "truthfulqa": TruthfulQABenchmark}


class BenchmarkRunner:
    def __init__(self, model, tokenizer, data_dir: str, limit: Optional[int] = None):
        self.model, self.tok, self.dir, self.limit = model, tokenizer, Path(data_dir), limit

    def run_benchmark(self, name: str) -> BenchmarkResult:
        return BENCHMARKS[name](str(self.dir / f"{name}.jsonl"), self.limit).run(self.model, self.tok)

    def run_all(self, names: Optional[Sequence[str]] = None) -> Dict[str, BenchmarkResult]:
        names = names or [n for n in BENCHMARKS if (self.dir / f"{n}.jsonl").exists()]
        return {n: self.run_benchmark(n) for n in names}

    @staticmethod
    def summarize(results: Dict[str, BenchmarkResult]) -> str:
        return "\n".join(f"{n:12s} acc={r.accuracy:.4f} (n={r.num_samples})"
                         for n, r in results.items())
