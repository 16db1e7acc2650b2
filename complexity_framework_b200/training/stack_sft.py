"""Stacked SFT curricula: weighted per-stage dataset mixes and chained LoRA stages.

Counterpart of complexity/training/stack_sft/ (config.py:12-180: source,
mix, stage and stack configs from YAML; datasets.py:27-171: a JSONL builder
sampling records from file-backed sources; runner.py:13-114: stages run one
after another, each starting from the previous stage's checkpoint).  The YAML
schema, validation messages and the record formats are kept, so a recipe
written for the reference runs here; each stage trains through
``training/sft.py`` (LoRA, merged into a full checkpoint at the end of the
stage so the next stage loads plain weights).

Record formats a source row may use (first match wins):
  * ``messages``: a chat; the prompt is every turn before the last assistant
    turn as ``Role:\\ncontent`` blocks, the completion that assistant turn;
  * ``prompt`` + ``completion``;
  * ``instruction`` (+ optional ``input``) + ``output`` (or ``response``),
    wrapped as ``User:\\n...\\n\\nAssistant:\\n``.
Field names are configurable per source; JSONL and parquet files are read.
"""
from __future__ import annotations

import json
import random
import subprocess
import sys
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Dict, List, Optional, Tuple

import yaml


def _req(data: Dict[str, Any], key: str, what: str):
    if key not in data:
        raise ValueError(f"{what} is missing {key}")
    return data[key]


@dataclass
class SourceConfig:
    """One weighted, file-backed source of a stage's mix."""
    name: str
    weight: float
    kind: Optional[str] = None
    path: Optional[str] = None
    format: Optional[str] = None
    prompt_field: str = "prompt"
    completion_field: str = "completion"
    messages_field: str = "messages"
    instruction_field: str = "instruction"
    input_field: str = "input"
    output_field: str = "output"
    max_records: Optional[int] = None

    @classmethod
    def from_dict(cls, data: Dict[str, Any]) -> "SourceConfig":
        name = str(data.get("name") or data.get("kind") or data.get("path") or "")
        if not name:
            raise ValueError("source is missing name/kind/path")
        if "weight" not in data:
            raise ValueError(f"source {name!r} is missing weight")
        kw = {k: str(data[k]) for k in ("prompt_field", "completion_field", "messages_field",
                                        "instruction_field", "input_field", "output_field")
              if k in data}
        return cls(name=name, weight=float(data["weight"]), kind=data.get("kind"),
                   path=data.get("path"), format=data.get("format"),
                   max_records=data.get("max_records"), **kw)


@dataclass
class DatasetMix:
    sources: List[SourceConfig]
    records: int = 80_000
    seed: int = 42
    out: Optional[str] = None

    @classmethod
    def from_dict(cls, data: Dict[str, Any]) -> "DatasetMix":
        raw = data.get("sources")
        if not isinstance(raw, list):
            raise ValueError("dataset mix sources must be a list of file-backed source configs; "
                             "hardcoded synthetic source mappings are not supported")
        sources = [SourceConfig.from_dict(dict(x)) for x in raw]
        if not sources:
            raise ValueError("dataset mix must contain at least one source")
        return cls(sources=sources, records=int(data.get("records", 80_000)),
                   seed=int(data.get("seed", 42)), out=data.get("out"))


@dataclass
class StageConfig:
    name: str
    steps: int
    lr: float
    mix: DatasetMix
    checkpoint: Optional[str] = None
    batch_size: Optional[int] = None
    seq_len: Optional[int] = None
    save_steps: Optional[int] = None
    save_total_limit: Optional[int] = None
    grad_ckpt: Optional[bool] = None
    loss_chunk_tokens: Optional[int] = None
    extra_args: List[str] = field(default_factory=list)

    @classmethod
    def from_dict(cls, data: Dict[str, Any]) -> "StageConfig":
        name = _req(data, "name", "stage")
        mix = _req(data, "mix", f"stage {name!r}")
        return cls(name=str(name), steps=int(data["steps"]), lr=float(data["lr"]),
                   mix=DatasetMix.from_dict(dict(mix)), checkpoint=data.get("checkpoint"),
                   batch_size=data.get("batch_size"), seq_len=data.get("seq_len"),
                   save_steps=data.get("save_steps"),
                   save_total_limit=data.get("save_total_limit"),
                   grad_ckpt=data.get("grad_ckpt"),
                   loss_chunk_tokens=data.get("loss_chunk_tokens"),
                   extra_args=[str(x) for x in data.get("extra_args", [])])


_STACK_DEFAULTS = dict(tokenizer="./tokenizer-o200k", output_dir="checkpoints",
                       data_dir="data/sft/stack_sft", run_dir="runs", batch_size=128,
                       seq_len=1024, save_steps=250, save_total_limit=2, grad_ckpt=True,
                       bf16=True, use_custom_kernels="auto", loss_chunk_tokens=512,
                       lora_rank=64, lora_alpha=128.0, lora_dropout=0.05,
                       lora_targets="q_proj,v_proj,o_proj,shared_gate,shared_up,shared_down")


@dataclass
class StackSFTConfig:
    name: str
    base_checkpoint: str
    tokenizer: str = _STACK_DEFAULTS["tokenizer"]
    output_dir: str = _STACK_DEFAULTS["output_dir"]
    data_dir: str = _STACK_DEFAULTS["data_dir"]
    run_dir: str = _STACK_DEFAULTS["run_dir"]
    batch_size: int = 128
    seq_len: int = 1024
    save_steps: int = 250
    save_total_limit: int = 2
    grad_ckpt: bool = True
    bf16: bool = True
    use_custom_kernels: str = "auto"
    loss_chunk_tokens: int = 512
    lora_rank: int = 64
    lora_alpha: float = 128.0
    lora_dropout: float = 0.05
    lora_targets: str = _STACK_DEFAULTS["lora_targets"]
    stages: List[StageConfig] = field(default_factory=list)

    @classmethod
    def from_dict(cls, data: Dict[str, Any]) -> "StackSFTConfig":
        stages = [StageConfig.from_dict(s) for s in data.get("stages", [])]
        if not stages:
            raise ValueError("stack config must define at least one stage")
        kw = {}
        for k, default in _STACK_DEFAULTS.items():
            kw[k] = type(default)(data.get(k, default))
        if kw["lora_rank"] <= 0:
            raise ValueError("stack SFT requires a positive LoRA rank")
        return cls(name=str(data["name"]), base_checkpoint=str(data["base_checkpoint"]),
                   stages=stages, **kw)

    @classmethod
    def from_yaml(cls, path) -> "StackSFTConfig":
        data = yaml.safe_load(Path(path).read_text(encoding="utf-8"))
        if not isinstance(data, dict):
            raise ValueError(f"invalid stack config: {path}")
        return cls.from_dict(data)


def chat_prompt(user: str) -> str:
    return f"User:\n{user}\n\nAssistant:\n"


def record_line(prompt: str, completion: str) -> str:
    """One output JSONL record (prompt keeps one trailing newline)."""
    return json.dumps({"prompt": prompt.rstrip() + "\n", "completion": completion.strip()},
                      ensure_ascii=False)


class StackSFTDatasetBuilder:
    """Write a stage's JSONL by sampling records (with replacement) from each
    source in proportion to its weight; the rounding remainder goes to the
    first source; the lines are shuffled with the mix's seed."""

    def __init__(self, seed: int = 42):
        self.seed = seed
        self._cache: Dict[Tuple, List[Dict[str, str]]] = {}

    @staticmethod
    def counts(mix: DatasetMix) -> List[Tuple[SourceConfig, int]]:
        total = sum(max(0.0, s.weight) for s in mix.sources)
        if total <= 0:
            raise ValueError("dataset mix weights must sum to a positive value")
        out = [(s, int(mix.records * max(0.0, s.weight) / total)) for s in mix.sources]
        out[0] = (out[0][0], out[0][1] + mix.records - sum(n for _, n in out))
        return out

    def build(self, mix: DatasetMix, out) -> Path:
        out = Path(out)
        out.parent.mkdir(parents=True, exist_ok=True)
        rng = random.Random(mix.seed + self.seed)
        lines: List[str] = []
        for src, n in self.counts(mix):
            if n <= 0:
                continue
            if not src.path:
                raise ValueError(f"stack SFT source {src.name!r} must define a JSONL/parquet "
                                 "path; hardcoded synthetic sources are not supported")
            recs = self.records(src)
            if not recs:
                raise ValueError(f"file source {src.name!r} produced no usable records")
            for _ in range(n):
                r = rng.choice(recs)
                lines.append(record_line(r["prompt"], r["completion"]))
        rng.shuffle(lines)
        # records are separated by LF only: json.dumps escapes U+2028/U+2029 inside
        # strings, so no record can be split by a Unicode line separator
        out.write_text("\n".join(lines) + "\n", encoding="utf-8")
        return out

    def records(self, src: SourceConfig) -> List[Dict[str, str]]:
        key = (src.path, src.format, src.prompt_field, src.completion_field, src.messages_field,
               src.instruction_field, src.input_field, src.output_field, src.max_records)
        if key in self._cache:
            return self._cache[key]
        path = Path(src.path or "")
        fmt = (src.format or path.suffix.lstrip(".") or "jsonl").lower()
        if fmt in ("jsonl", "json"):
            rows = self._jsonl(path)
        elif fmt == "parquet":
            import pyarrow.parquet as pq

            rows = pq.read_table(path).to_pylist()
        else:
            raise ValueError(f"unsupported stack SFT source format: {fmt}")
        recs: List[Dict[str, str]] = []
        for row in rows:
            r = format_record(row, src)
            if r is not None:
                recs.append(r)
            if src.max_records is not None and len(recs) >= int(src.max_records):
                break
        self._cache[key] = recs
        return recs

    @staticmethod
    def _jsonl(path: Path) -> List[Dict[str, Any]]:
        rows = []
        for no, line in enumerate(path.read_text(encoding="utf-8").split("\n"), 1):
            if not line.strip():
                continue
            try:
                row = json.loads(line)
            except json.JSONDecodeError as exc:
                raise ValueError(f"invalid JSON at {path}:{no}: {exc}") from exc
            if isinstance(row, dict):
                rows.append(row)
        return rows


def format_record(row: Dict[str, Any], src: SourceConfig) -> Optional[Dict[str, str]]:
    if src.messages_field in row:
        return _from_messages(row.get(src.messages_field))
    if src.prompt_field in row and src.completion_field in row:
        p = str(row.get(src.prompt_field) or "").strip()
        c = str(row.get(src.completion_field) or "").strip()
        return {"prompt": p, "completion": c} if p and c else None
    if src.instruction_field in row or src.output_field in row:
        ins = str(row.get(src.instruction_field) or "").strip()
        extra = str(row.get(src.input_field) or "").strip()
        c = str(row.get(src.output_field) or row.get("response") or "").strip()
        if ins and c:
            return {"prompt": chat_prompt(f"{ins}\n\n{extra}" if extra else ins), "completion": c}
    return None


def _from_messages(msgs: Any) -> Optional[Dict[str, str]]:
    if not isinstance(msgs, list) or not msgs:
        return None
    last = next((i for i in range(len(msgs) - 1, -1, -1)
                 if isinstance(msgs[i], dict) and msgs[i].get("role") == "assistant"), None)
    if last is None:
        return None
    parts = []
    for m in msgs[:last]:
        if isinstance(m, dict):
            content = str(m.get("content", "")).strip()
            if content:
                parts.append(f"{str(m.get('role', 'user')).strip().title()}:\n{content}")
    c = str(msgs[last].get("content", "")).strip()
    if not parts or not c:
        return None
    return {"prompt": "\n\n".join(parts) + "\n\nAssistant:\n", "completion": c}


class StackSFTRunner:
    """Build each stage's mix and train the stages in order; a stage starts from
    its own ``checkpoint`` if set, else from the previous stage's output."""

    def __init__(self, config: StackSFTConfig, *, dry_run: bool = False,
                 in_process: bool = True):
        self.config, self.dry_run, self.in_process = config, dry_run, in_process
        self.dataset_builder = StackSFTDatasetBuilder()

    @classmethod
    def from_yaml(cls, path, **kw) -> "StackSFTRunner":
        return cls(StackSFTConfig.from_yaml(path), **kw)

    def run(self, *, start_stage: Optional[str] = None, stop_after: Optional[str] = None) -> str:
        ck = self.config.base_checkpoint
        active = start_stage is None
        for st in self.config.stages:
            active = active or st.name == start_stage
            if not active:
                ck = self.stage_checkpoint(st)
                continue
            ck = self.run_stage(st, ck)
            if st.name == stop_after:
                break
        return ck

    def run_stage(self, stage: StageConfig, input_checkpoint: str) -> str:
        data = self.dataset_builder.build(stage.mix, self.stage_dataset_path(stage))
        argv = self.stage_args(stage, stage.checkpoint or input_checkpoint, data)
        if self.dry_run:
            print(" ".join([sys.executable, "-m", "complexity_framework_b200.training.sft"]
                           + argv))
        elif self.in_process:
            from .sft import main as sft_main

            sft_main(argv)
        else:
            subprocess.run([sys.executable, "-m", "complexity_framework_b200.training.sft"]
                           + argv, check=True)
        return self.stage_checkpoint(stage)

    def stage_dataset_path(self, stage: StageConfig) -> Path:
        if stage.mix.out:
            return Path(stage.mix.out)
        return Path(self.config.data_dir) / self.config.name / f"{stage.name}.jsonl"

    def stage_save_dir(self, stage: StageConfig) -> Path:
        return Path(self.config.output_dir) / f"{self.config.name}-{stage.name}"

    def stage_checkpoint(self, stage: StageConfig) -> str:
        return str(self.stage_save_dir(stage) / "final")

    def stage_args(self, stage: StageConfig, checkpoint: str, data: Path) -> List[str]:
        c = self.config
        args = ["--model", checkpoint, "--data", str(data), "--tokenizer", c.tokenizer,
                "--output", str(self.stage_save_dir(stage)),
                "--max-steps", str(stage.steps), "--epochs", "1",
                "--batch-size", str(stage.batch_size or c.batch_size),
                "--seq-len", str(stage.seq_len or c.seq_len), "--lr", str(stage.lr),
                "--lora-rank", str(c.lora_rank), "--lora-alpha", str(c.lora_alpha),
                "--lora-targets", c.lora_targets, "--merge-lora",
                "--precision", "bf16" if c.bf16 else "fp32"]
        return args + list(stage.extra_args)
