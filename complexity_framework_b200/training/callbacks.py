"""Trainer callbacks and metric sinks.

Counterparts: complexity/training/callbacks.py:14-172 (early stopping, W&B,
tqdm, TensorBoard), metrics.py (``MetricsTracker``) and the per-step
``training_log.csv`` / ``metrics.jsonl`` writers of runner.py:472-527.

Hooks a callback may define (all optional):
``on_train_begin(trainer)``, ``on_step_end(trainer, step, loss)`` (``loss`` is
``None`` on steps whose loss was not read back), ``on_evaluate(trainer, step,
eval_loss)``, ``on_train_end(trainer, summary)``.  Reading the loss is
what forces a device sync, so sinks only see it every ``log_steps`` steps.
"""
from __future__ import annotations

import csv
import json
import math
import time
from pathlib import Path
from typing import Dict, List, Optional


class Callback:
    def on_train_begin(self, trainer) -> None: ...

    def on_step_end(self, trainer, step: int, loss: Optional[float]) -> None: ...

    def on_evaluate(self, trainer, step: int, eval_loss: float) -> None: ...

    def on_train_end(self, trainer, summary: Dict) -> None: ...


def _lr(trainer) -> float:
    try:
        return float(trainer.scheduler.get_last_lr()[0])
    except Exception:  # noqa: BLE001 - scheduler-less trainers
        return float("nan")


class _RateMeter:
    def __init__(self):
        self.t = None
        self.tokens = 0

    def rate(self, trainer) -> float:
        now = time.perf_counter()
        if self.t is None:
            self.t, self.tokens = now, trainer.total_tokens
            return 0.0
        dt, dn = now - self.t, trainer.total_tokens - self.tokens
        self.t, self.tokens = now, trainer.total_tokens
        return dn / dt if dt > 0 else 0.0


class CSVLoggerCallback(Callback):
    """``training_log.csv``: step, loss, lr, tokens, tokens/s (rank 0 only)."""

    FIELDS = ["step", "loss", "lr", "total_tokens", "tokens_per_s", "wall_s"]

    def __init__(self, path: str):
        self.path = Path(path)
        self._t0 = time.perf_counter()
        self._rate = _RateMeter()

    def on_train_begin(self, trainer) -> None:
        if trainer.is_main and not self.path.exists():
            self.path.parent.mkdir(parents=True, exist_ok=True)
            with self.path.open("w", newline="") as f:
                csv.writer(f).writerow(self.FIELDS)

    def on_step_end(self, trainer, step, loss) -> None:
        if loss is None or not trainer.is_main:
            return
        if not self.path.exists():
            self.on_train_begin(trainer)
        with self.path.open("a", newline="") as f:
            csv.writer(f).writerow([step, f"{loss:.6f}", f"{_lr(trainer):.3e}",
                                    trainer.total_tokens, f"{self._rate.rate(trainer):.1f}",
                                    f"{time.perf_counter() - self._t0:.2f}"])


class MetricsJsonlCallback(Callback):
    """``metrics.jsonl``: one JSON object per logged step / evaluation."""

    def __init__(self, path: str, extra: Optional[Dict] = None):
        self.path = Path(path)
        self.extra = extra or {}
        self._rate = _RateMeter()

    def _write(self, trainer, rec: Dict) -> None:
        if not trainer.is_main:
            return
        self.path.parent.mkdir(parents=True, exist_ok=True)
        with self.path.open("a") as f:
            f.write(json.dumps({**self.extra, **rec}) + "\n")

    def on_step_end(self, trainer, step, loss) -> None:
        if loss is not None:
            self._write(trainer, {"type": "train", "step": step, "loss": loss, "lr": _lr(trainer),
                                  "total_tokens": trainer.total_tokens,
                                  "tokens_per_s": self._rate.rate(trainer), "time": time.time()})

    def on_evaluate(self, trainer, step, eval_loss) -> None:
        self._write(trainer, {"type": "eval", "step": step, "eval_loss": eval_loss,
                              "eval_ppl": math.exp(min(eval_loss, 50)), "time": time.time()})


class TqdmCallback(Callback):
    """Progress bar with loss, lr and tokens/s on rank 0."""

    def __init__(self, total: Optional[int] = None):
        self.total = total
        self.bar = None
        self._rate = _RateMeter()

    def on_train_begin(self, trainer) -> None:
        if trainer.is_main:
            from tqdm import tqdm

            self.bar = tqdm(total=self.total or trainer.config.max_steps,
                            initial=trainer.global_step, dynamic_ncols=True)

    def on_step_end(self, trainer, step, loss) -> None:
        if self.bar is None:
            return
        self.bar.update(step - self.bar.n)
        if loss is not None:
            self.bar.set_postfix(loss=f"{loss:.4f}", lr=f"{_lr(trainer):.2e}",
                                 tok_s=f"{self._rate.rate(trainer) / 1e3:.0f}k")

    def on_train_end(self, trainer, summary) -> None:
        if self.bar is not None:
            self.bar.close()


class EarlyStoppingCallback(Callback):
    """Sets ``trainer.should_stop`` after ``patience`` evaluations without improvement."""

    def __init__(self, patience: int = 3, min_delta: float = 0.0):
        self.patience, self.min_delta = patience, min_delta
        self.best = float("inf")
        self.bad = 0

    def on_evaluate(self, trainer, step, eval_loss) -> None:
        if eval_loss < self.best - self.min_delta:
            self.best, self.bad = eval_loss, 0
        else:
            self.bad += 1
            if self.bad >= self.patience:
                trainer.should_stop = True


class TensorBoardCallback(Callback):
    """Scalars to TensorBoard when ``tensorboard`` is installed; otherwise a
    JSONL file of the same scalars in ``log_dir``."""

    def __init__(self, log_dir: str):
        self.log_dir = log_dir
        self.writer = None
        try:
            from torch.utils.tensorboard import SummaryWriter

            self.writer = SummaryWriter(log_dir)
        except Exception:  # noqa: BLE001 - optional dependency
            self.fallback = MetricsJsonlCallback(str(Path(log_dir) / "scalars.jsonl"))

    def on_step_end(self, trainer, step, loss) -> None:
        if loss is None or not trainer.is_main:
            return
        if self.writer is not None:
            self.writer.add_scalar("train/loss", loss, step)
            self.writer.add_scalar("train/lr", _lr(trainer), step)
        else:
            self.fallback.on_step_end(trainer, step, loss)

    def on_evaluate(self, trainer, step, eval_loss) -> None:
        if self.writer is not None and trainer.is_main:
            self.writer.add_scalar("eval/loss", eval_loss, step)
        elif trainer.is_main:
            self.fallback.on_evaluate(trainer, step, eval_loss)


class WandBCallback(Callback):
    """Weights & Biases logging when ``wandb`` is importable (offline mode
    unless configured otherwise); a no-op otherwise."""

    def __init__(self, project: str, config: Optional[Dict] = None, mode: str = "offline"):
        try:
            import wandb  # noqa: F401

            self.wandb = wandb
        except ImportError:
            self.wandb = None
        self.project, self.config, self.mode = project, config or {}, mode
        self.run = None

    def on_train_begin(self, trainer) -> None:
        if self.wandb is not None and trainer.is_main:
            self.run = self.wandb.init(project=self.project, config=self.config, mode=self.mode)

    def on_step_end(self, trainer, step, loss) -> None:
        if self.run is not None and loss is not None:
            self.run.log({"loss": loss, "lr": _lr(trainer)}, step=step)

    def on_train_end(self, trainer, summary) -> None:
        if self.run is not None:
            self.run.finish()


class MetricsTracker:
    """In-memory metric history with JSON save/load and running means."""

    def __init__(self):
        self.history: Dict[str, List] = {}

    def update(self, step: int, **metrics) -> None:
        for k, v in metrics.items():
            self.history.setdefault(k, []).append((step, float(v)))

    def mean(self, key: str, last: int = 100) -> float:
        vals = [v for _, v in self.history.get(key, [])[-last:]]
        return sum(vals) / len(vals) if vals else float("nan")

    def latest(self, key: str) -> Optional[float]:
        h = self.history.get(key)
        return h[-1][1] if h else None

    def save(self, path: str) -> None:
        Path(path).write_text(json.dumps(self.history))

    @classmethod
    def load(cls, path: str) -> "MetricsTracker":
        t = cls()
        t.history = {k: [tuple(x) for x in v] for k, v in json.loads(Path(path).read_text()).items()}
        return t


class TensorBoardMetricWriter:
    """Scalar dictionaries to TensorBoard under ``prefix/name``
    (complexity/training/tensorboard.py:13-58); non-numeric, boolean and
    non-finite values are skipped; without the tensorboard package the writer
    is disabled (``enabled`` is False) and every call is a no-op."""

    def __init__(self, log_dir, *, enabled: bool = True):
        import logging as _logging
        import math as _math

        self._isfinite = _math.isfinite
        self.writer = None
        self.log_dir = Path(log_dir)
        if not enabled:
            return
        try:
            from torch.utils.tensorboard import SummaryWriter
        except Exception:  # noqa: BLE001 - optional dependency
            _logging.getLogger(__name__).warning("TensorBoard logging disabled: tensorboard is "
                                                 "not installed")
            return
        self.log_dir.mkdir(parents=True, exist_ok=True)
        self.writer = SummaryWriter(str(self.log_dir))

    @property
    def enabled(self) -> bool:
        return self.writer is not None

    def add_scalars(self, prefix: str, metrics, step: int) -> None:
        if self.writer is None:
            return
        p = prefix.strip("/")
        for k, v in metrics.items():
            if isinstance(v, bool) or not isinstance(v, (int, float)) or \
                    not self._isfinite(float(v)):
                continue
            self.writer.add_scalar(f"{p}/{k}", float(v), step)

    def flush(self) -> None:
        if self.writer is not None:
            self.writer.flush()

    def close(self) -> None:
        if self.writer is not None:
            self.writer.close()
