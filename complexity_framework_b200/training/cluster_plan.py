"""Run planning arithmetic: tokens per step, steps, Chinchilla multiple.

Counterpart of complexity/training/cluster_plan.py:20-180 and plan_run.py
(the ``cf-plan-cluster`` entry): same quantities and YAML keys.
"""
from __future__ import annotations

import argparse
import math
import re
from dataclasses import dataclass
from pathlib import Path
from typing import Any, List

_SUFFIX = {"k": 10 ** 3, "m": 10 ** 6, "b": 10 ** 9, "g": 10 ** 9, "t": 10 ** 12}


def parse_tokens(value: Any) -> int:
    """``200B`` / ``1.5t`` / ``70_000_000`` -> integer token count."""
    if isinstance(value, (int, float)):
        return int(value)
    s = str(value).strip().lower().replace("_", "").replace(",", "")
    m = re.fullmatch(r"([0-9]*\.?[0-9]+)([kmbgt]?)", s)
    if not m:
        raise ValueError(f"cannot parse token count {value!r}")
    return int(float(m.group(1)) * _SUFFIX.get(m.group(2), 1))


@dataclass(frozen=True)
class ParallelPlan:
    tp_size: int = 1
    pp_size: int = 1
    dp_size: int = 1
    micro_batch_size: int = 8
    gradient_accumulation: int = 1

    @property
    def world_size(self) -> int:
        return self.tp_size * self.pp_size * self.dp_size

    @property
    def model_replica_gpus(self) -> int:
        return self.tp_size * self.pp_size

    @property
    def batch_per_dp_replica(self) -> int:
        return self.micro_batch_size * self.gradient_accumulation

    @property
    def global_batch(self) -> int:
        return self.dp_size * self.batch_per_dp_replica


@dataclass(frozen=True)
class ClusterRunPlan:
    name: str
    target_tokens: int
    seq_len: int
    params: int
    parallel: ParallelPlan

    @property
    def chinchilla_tokens(self) -> int:
        return 20 * self.params

    @property
    def chinchilla_multiple(self) -> float:
        return self.target_tokens / self.chinchilla_tokens

    @property
    def tokens_per_step(self) -> int:
        return self.parallel.global_batch * self.seq_len

    @property
    def steps(self) -> int:
        return math.ceil(self.target_tokens / self.tokens_per_step)

    @property
    def actual_tokens(self) -> int:
        return self.steps * self.tokens_per_step

    @property
    def overshoot_tokens(self) -> int:
        return self.actual_tokens - self.target_tokens

    def validate(self) -> None:
        for k, v in (("params", self.params), ("target_tokens", self.target_tokens),
                     ("seq_len", self.seq_len), ("tp_size", self.parallel.tp_size),
                     ("pp_size", self.parallel.pp_size), ("dp_size", self.parallel.dp_size),
                     ("micro_batch_size", self.parallel.micro_batch_size),
                     ("gradient_accumulation", self.parallel.gradient_accumulation)):
            if v <= 0:
                raise ValueError(f"{k} must be positive")

    def summary_lines(self) -> List[str]:
        self.validate()
        p = self.parallel
        rows = [("run_name", self.name), ("params", f"{self.params:,}"),
                ("target_tokens", f"{self.target_tokens:,}"),
                ("chinchilla_tokens", f"{self.chinchilla_tokens:,}"),
                ("chinchilla_multiple", f"{self.chinchilla_multiple:.2f}x"),
                ("world_size", f"{p.world_size:,}"),
                ("model_replica_gpus", f"{p.model_replica_gpus:,} (TP={p.tp_size} * PP={p.pp_size})"),
                ("dp_replicas", f"{p.dp_size:,}"), ("micro_batch_size", f"{p.micro_batch_size:,}"),
                ("gradient_accumulation", f"{p.gradient_accumulation:,}"),
                ("batch_per_dp_replica", f"{p.batch_per_dp_replica:,}"),
                ("global_batch", f"{p.global_batch:,}"), ("seq_len", f"{self.seq_len:,}"),
                ("tokens_per_step", f"{self.tokens_per_step:,}"), ("steps", f"{self.steps:,}"),
                ("actual_tokens", f"{self.actual_tokens:,}"),
                ("overshoot_tokens", f"{self.overshoot_tokens:,}")]
        return [f"{k:22s}{v}" for k, v in rows]


def load_cluster_run_plan(path) -> ClusterRunPlan:
    import yaml

    d = yaml.safe_load(Path(path).read_text()) or {}
    par = d.get("parallel", {}) or {}
    plan = ClusterRunPlan(
        name=str(d.get("name", Path(path).stem)), target_tokens=parse_tokens(d["target_tokens"]),
        seq_len=int(d["seq_len"]), params=parse_tokens(d["params"]),
        parallel=ParallelPlan(**{k: int(par[k]) for k in (
            "tp_size", "pp_size", "dp_size", "micro_batch_size", "gradient_accumulation")
            if k in par}))
    plan.validate()
    return plan


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="Plan a cluster training run")
    ap.add_argument("config", nargs="?", help="YAML plan file")
    ap.add_argument("--params", default=None)
    ap.add_argument("--target-tokens", default=None)
    ap.add_argument("--seq-len", type=int, default=2048)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--pp", type=int, default=1)
    ap.add_argument("--dp", type=int, default=8)
    ap.add_argument("--micro-batch", type=int, default=8)
    ap.add_argument("--accum", type=int, default=1)
    a = ap.parse_args(argv)
    if a.config:
        plan = load_cluster_run_plan(a.config)
    else:
        if a.params is None or a.target_tokens is None:
            ap.error("--params and --target-tokens are required without a config file")
        plan = ClusterRunPlan("cli", parse_tokens(a.target_tokens), a.seq_len,
                              parse_tokens(a.params),
                              ParallelPlan(a.tp, a.pp, a.dp, a.micro_batch, a.accum))
    print("\n".join(plan.summary_lines()))


if __name__ == "__main__":
    main()
