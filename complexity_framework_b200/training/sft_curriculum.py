"""Deterministic SFT curriculum: stages that select examples from a dataset
without rewriting it.

A curriculum is a YAML file::

    seed: 7
    stages:
      - name: warmup
        tasks: [chat, math]            # keep only these tasks (optional)
        exclude_tasks: [code]
        difficulties: [easy]
        max_num_tokens: 2048           # prompt + response
        max_supervised_tokens: 1024
        exclude_response_substrings: ["As an AI"]
        max_examples: 5000             # deterministic subsample
        max_repeats_per_response: 2    # cap identical responses
        task_weights: {chat: 1.0, math: 2.0}   # per-token loss weights

Rows are chat records (``messages``) with optional ``task``, ``difficulty``
and ``mode`` fields.  Selection is a pure function of the rows, the stage and
the seed: every rank selects the same examples in the same order.
Counterpart of complexity/training/sft_curriculum.py (stage filters, response
caps, task weights) with the Parquet metadata side-table left out.
"""
from __future__ import annotations

import hashlib
from collections import Counter
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Dict, List, Optional, Sequence, Tuple

import yaml


def _strings(v: Any, what: str) -> Tuple[str, ...]:
    if v is None:
        return ()
    if not isinstance(v, list) or not all(isinstance(x, str) for x in v):
        raise ValueError(f"curriculum {what} must be a list of strings")
    return tuple(v)


@dataclass(frozen=True)
class CurriculumStage:
    name: str
    tasks: Tuple[str, ...] = ()
    exclude_tasks: Tuple[str, ...] = ()
    difficulties: Tuple[str, ...] = ()
    modes: Tuple[str, ...] = ()
    max_num_tokens: Optional[int] = None
    max_supervised_tokens: Optional[int] = None
    exclude_response_substrings: Tuple[str, ...] = ()
    max_examples: Optional[int] = None
    max_repeats_per_response: Optional[int] = None
    task_weights: Tuple[Tuple[str, float], ...] = ()

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "CurriculumStage":
        name = str(d.get("name", "")).strip()
        if not name:
            raise ValueError("every curriculum stage needs a name")
        known = set(cls.__dataclass_fields__)
        unknown = set(d) - known
        if unknown:
            raise ValueError(f"stage {name}: unknown keys {sorted(unknown)}")
        weights = d.get("task_weights") or {}
        if not isinstance(weights, dict) or any(
                not isinstance(w, (int, float)) or w <= 0 for w in weights.values()):
            raise ValueError(f"stage {name}: task_weights must map tasks to positive numbers")
        for key in ("max_num_tokens", "max_supervised_tokens", "max_examples",
                    "max_repeats_per_response"):
            v = d.get(key)
            if v is not None and (not isinstance(v, int) or v <= 0):
                raise ValueError(f"stage {name}: {key} must be a positive integer")
        return cls(name=name, tasks=_strings(d.get("tasks"), "tasks"),
                   exclude_tasks=_strings(d.get("exclude_tasks"), "exclude_tasks"),
                   difficulties=_strings(d.get("difficulties"), "difficulties"),
                   modes=_strings(d.get("modes"), "modes"),
                   max_num_tokens=d.get("max_num_tokens"),
                   max_supervised_tokens=d.get("max_supervised_tokens"),
                   exclude_response_substrings=_strings(d.get("exclude_response_substrings"),
                                                        "exclude_response_substrings"),
                   max_examples=d.get("max_examples"),
                   max_repeats_per_response=d.get("max_repeats_per_response"),
                   task_weights=tuple(sorted((str(k), float(v)) for k, v in weights.items())))

    def task_weight(self, task: Optional[str]) -> float:
        for t, w in self.task_weights:
            if t == task:
                return w
        return 1.0


@dataclass(frozen=True)
class Curriculum:
    stages: Tuple[CurriculumStage, ...]
    seed: int = 0

    def stage(self, name: str) -> CurriculumStage:
        for s in self.stages:
            if s.name == name:
                return s
        raise KeyError(f"curriculum has no stage {name!r}; stages: "
                       f"{[s.name for s in self.stages]}")


def load_curriculum(path: str) -> Curriculum:
    data = yaml.safe_load(Path(path).read_text())
    if not isinstance(data, dict) or not isinstance(data.get("stages"), list) or not data["stages"]:
        raise ValueError("a curriculum needs a non-empty 'stages' list")
    stages = tuple(CurriculumStage.from_dict(s) for s in data["stages"])
    names = [s.name for s in stages]
    if len(set(names)) != len(names):
        raise ValueError(f"duplicate stage names in {names}")
    return Curriculum(stages=stages, seed=int(data.get("seed", 0)))


def _response_text(row: Dict[str, Any]) -> str:
    return "\n".join(m.get("content", "") for m in row.get("messages", [])
                     if m.get("role") == "assistant")


def _stable_key(seed: int, i: int, row: Dict[str, Any]) -> str:
    h = hashlib.sha256(f"{seed}:{i}:".encode())
    h.update(_response_text(row).encode())
    return h.hexdigest()


def select_examples(rows: Sequence[Dict[str, Any]], stage: CurriculumStage, *, seed: int = 0,
                    token_counts: Optional[Sequence[Tuple[int, int]]] = None) -> List[int]:
    """Indices of ``rows`` kept by ``stage``, in dataset order.

    ``token_counts[i] = (num_tokens, supervised_tokens)`` enables the length
    filters.  Subsampling (``max_examples``) keeps the examples with the smallest
    seeded hash, so the selection is stable when unrelated rows change.
    """
    keep: List[int] = []
    seen: Counter = Counter()
    for i, row in enumerate(rows):
        task = row.get("task")
        if stage.tasks and task not in stage.tasks:
            continue
        if task in stage.exclude_tasks:
            continue
        if stage.difficulties and row.get("difficulty") not in stage.difficulties:
            continue
        if stage.modes and row.get("mode") not in stage.modes:
            continue
        if token_counts is not None:
            n, sup = token_counts[i]
            if stage.max_num_tokens is not None and n > stage.max_num_tokens:
                continue
            if stage.max_supervised_tokens is not None and sup > stage.max_supervised_tokens:
                continue
        resp = _response_text(row)
        if any(s in resp for s in stage.exclude_response_substrings):
            continue
        if stage.max_repeats_per_response is not None:
            key = hashlib.sha256(resp.strip().encode()).hexdigest()
            if seen[key] >= stage.max_repeats_per_response:
                continue
            seen[key] += 1
        keep.append(i)
    if stage.max_examples is not None and len(keep) > stage.max_examples:
        ranked = sorted(keep, key=lambda i: _stable_key(seed, i, rows[i]))
        keep = sorted(ranked[:stage.max_examples])
    return keep
