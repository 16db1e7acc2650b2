"""Checkpoint save / resume.

Directory layout per checkpoint (reference: complexity/utils/checkpointing.py:127-579):
``checkpoint.pt`` = {"model": full state dict, "scheduler": state}, ``model.safetensors``,
``optimizer_rank{r}.pt`` (each rank's optimizer shard), ``training_state.json``
= {step, epoch, best_loss, total_tokens, learning_rate} written LAST so a
directory without it is incomplete and skipped on resume.  Files are written
to a temporary name and renamed (atomic on POSIX).  ``save_total_limit`` keeps
the newest checkpoints per tag.
"""
from __future__ import annotations

import json
import os
import re
import shutil
from pathlib import Path
from typing import Any, Dict, Optional, Tuple

import torch
import torch.distributed as dist

STATE_FILE = "training_state.json"


def _dist() -> Tuple[bool, int, int]:
    on = dist.is_available() and dist.is_initialized()
    return on, (dist.get_rank() if on else 0), (dist.get_world_size() if on else 1)


def gather_full_state_dict(model: torch.nn.Module) -> Tuple[Dict[str, torch.Tensor], bool]:
    """Full CPU state dict on rank 0 (collective: every rank must call it).

    Parameters here are replicated on every rank (optimizer state is what gets
    sharded), so no parameter gather is needed; DTensor-valued entries from
    other wrappers are materialised with ``full_tensor()`` on all ranks.
    """
    on, rank, _ = _dist()
    if on:
        dist.barrier()
    z3 = getattr(model, "zero3", None)
    if z3 is not None:  # ZeRO-3: gather every unit first (collective)
        with z3.summon_full_params():
            # copies: the gathered buffers are freed when the context exits
            sd = {k: v.detach().to("cpu", copy=True).contiguous()
                  for k, v in model.state_dict().items()}
        return (sd if rank == 0 else {}), rank == 0
    out = {}
    for k, v in model.state_dict().items():
        if hasattr(v, "full_tensor"):
            v = v.full_tensor()
        elif hasattr(v, "to_local"):
            v = v.to_local()
        if rank == 0:
            out[k] = v.detach().cpu().contiguous()
    return out, rank == 0


def _atomic_save(obj: Any, path: Path) -> None:
    tmp = path.with_suffix(path.suffix + ".tmp")
    torch.save(obj, tmp)
    os.replace(tmp, path)


def _atomic_json(obj: Any, path: Path) -> None:
    tmp = path.with_suffix(path.suffix + ".tmp")
    with open(tmp, "w") as fh:
        json.dump(obj, fh, indent=2)
    os.replace(tmp, path)


class CheckpointManager:
    def __init__(self, checkpoint_dir: str, save_total_limit: int = 3):
        self.root = Path(checkpoint_dir)
        self.save_total_limit = save_total_limit

    def path_for(self, step: int, tag: str = "step") -> Path:
        return self.root / f"{tag}-{step}"

    def save(self, model: torch.nn.Module, optimizer: Optional[torch.optim.Optimizer], *,
             step: int, scheduler=None, epoch: int = 0, best_loss: float = float("inf"),
             total_tokens: int = 0, tag: str = "step", extra: Optional[dict] = None) -> Path:
        on, rank, _ = _dist()
        path = self.path_for(step, tag)
        sd, is_main = gather_full_state_dict(model)
        if is_main:
            path.mkdir(parents=True, exist_ok=True)
            _atomic_save({"model": sd,
                          "scheduler": scheduler.state_dict() if scheduler is not None else None,
                          "extra": extra or {}}, path / "checkpoint.pt")
            from safetensors.torch import save_file

            save_file(sd, str(path / "model.safetensors.tmp"))
            os.replace(path / "model.safetensors.tmp", path / "model.safetensors")
            if hasattr(model, "config") and hasattr(model.config, "to_dict"):
                _atomic_json(model.config.to_dict(), path / "config.json")
        if on:
            dist.barrier()
        if optimizer is not None:
            path.mkdir(parents=True, exist_ok=True)
            _atomic_save(optimizer.state_dict(), path / f"optimizer_rank{rank}.pt")
        if on:
            dist.barrier()
        if is_main:
            lr = optimizer.param_groups[0]["lr"] if optimizer is not None else None
            _atomic_json({"step": step, "epoch": epoch, "best_loss": best_loss,
                          "total_tokens": total_tokens, "learning_rate": lr},
                         path / STATE_FILE)
            self._rotate(tag)
        if on:
            dist.barrier()
        return path

    def _rotate(self, tag: str) -> None:
        if self.save_total_limit <= 0:
            return
        done = sorted(self._complete(tag), key=lambda p: p[0])
        for _, p in done[:-self.save_total_limit]:
            shutil.rmtree(p, ignore_errors=True)

    def _complete(self, tag: Optional[str] = None):
        if not self.root.exists():
            return []
        out = []
        for p in self.root.iterdir():
            m = re.fullmatch(r"(.+)-(\d+)", p.name)
            if not m or not p.is_dir() or not (p / STATE_FILE).exists():
                continue
            if tag is not None and m.group(1) != tag:
                continue
            out.append((int(m.group(2)), p))
        return out

    def latest(self) -> Optional[Path]:
        """Newest complete checkpoint across tags (incomplete directories are skipped)."""
        done = self._complete()
        if not done:
            return None
        best = max(done, key=lambda sp: (json.load(open(sp[1] / STATE_FILE))["step"], sp[0]))
        return best[1]

    def load(self, path: Path, model: torch.nn.Module,
             optimizer: Optional[torch.optim.Optimizer] = None, scheduler=None,
             map_location="cpu") -> dict:
        _, rank, _ = _dist()
        path = Path(path)
        ck = torch.load(path / "checkpoint.pt", map_location=map_location, weights_only=False)
        z3 = getattr(model, "zero3", None)
        if z3 is not None:
            z3.load_full_state_dict(ck["model"])
        else:
            model.load_state_dict(ck["model"], strict=False)
        if scheduler is not None and ck.get("scheduler") is not None:
            scheduler.load_state_dict(ck["scheduler"])
        opt_path = path / f"optimizer_rank{rank}.pt"
        if optimizer is not None and opt_path.exists():
            optimizer.load_state_dict(torch.load(opt_path, map_location=map_location,
                                                 weights_only=False))
        with open(path / STATE_FILE) as fh:
            return json.load(fh)


def _foreign_checkpoint_step(p: Path) -> Optional[int]:
    """Step of a reference-layout checkpoint directory ``<name>_<step>``, or
    None when it is not one or was left incomplete: complete means
    ``checkpoint.pt`` (or a distributed ``.metadata``) exists; the step comes
    from ``training_state.json`` when present, else from the name."""
    m = re.fullmatch(r".+_(\d+)", p.name)
    if not m or not p.is_dir():
        return None
    if not ((p / "checkpoint.pt").exists() or (p / ".metadata").exists()):
        return None
    try:
        with open(p / STATE_FILE) as fh:
            return int(json.load(fh)["step"])
    except (OSError, ValueError, KeyError):
        return int(m.group(1))


def peek_latest_checkpoint_step(checkpoint_dir: str) -> Optional[int]:
    """Global step of the newest complete checkpoint under ``checkpoint_dir``
    without loading any state (for a resume-time data skip), or None.

    Reads this framework's ``<tag>-<step>`` directories (complete once their
    training state is written) and the reference's ``<name>_<step>`` ones
    (complexity/utils/checkpointing.py peek_latest_checkpoint_step: complete once
    ``checkpoint.pt`` or ``.metadata`` exists), so a run can resume a
    directory written by either framework."""
    root = Path(checkpoint_dir)
    if not root.is_dir():
        return None
    steps = []
    p = CheckpointManager(checkpoint_dir).latest()
    if p is not None:
        with open(p / STATE_FILE) as fh:
            steps.append(int(json.load(fh)["step"]))
    for d in root.iterdir():
        if re.fullmatch(r"(.+)-(\d+)", d.name):
            continue                      # this framework's layout, handled above
        st = _foreign_checkpoint_step(d)
        if st is not None:
            steps.append(st)
    return max(steps) if steps else None


def load_weights_only(model: torch.nn.Module, path: str) -> None:
    """Initialise weights from a checkpoint directory without optimizer state."""
    p = Path(path)
    if (p / "model.safetensors").exists():
        from safetensors.torch import load_file

        sd = load_file(str(p / "model.safetensors"))
    else:
        sd = torch.load(p / "checkpoint.pt", map_location="cpu", weights_only=False)["model"]
    model.load_state_dict(sd, strict=False)


# ----------------------------------------------- reference helper names
from dataclasses import asdict as _asdict, dataclass as _dataclass  # noqa: E402


@_dataclass
class TrainingState:
    """Scalar training progress (complexity/utils/checkpointing.py:128-142)."""
    step: int = 0
    epoch: int = 0
    best_loss: float = float("inf")
    total_tokens: int = 0
    learning_rate: float = 0.0

    def to_dict(self) -> dict:
        return _asdict(self)

    @classmethod
    def from_dict(cls, data: dict) -> "TrainingState":
        return cls(**{k: v for k, v in data.items() if k in cls.__dataclass_fields__})


def enable_activation_checkpointing(model, checkpoint_layers: bool = True) -> None:
    """Recompute each decoder layer's activations in backward (models that
    expose ``gradient_checkpointing_enable``; otherwise every child of
    ``model.layers`` is wrapped)."""
    if not checkpoint_layers:
        return
    if hasattr(model, "gradient_checkpointing_enable"):
        model.gradient_checkpointing_enable()
        return
    from torch.utils.checkpoint import checkpoint

    for layer in getattr(model, "layers", []):
        fwd = layer.forward

        def wrapped(*a, _f=fwd, **k):
            return checkpoint(_f, *a, use_reentrant=False, **k)
        layer.forward = wrapped


def checkpoint_sequential(functions, input, segments: int = 1, **kwargs):
    """Run ``functions`` in order, recomputing each segment's activations in backward."""
    from torch.utils.checkpoint import checkpoint_sequential as _cs

    return _cs(list(functions), max(1, segments), input, use_reentrant=False, **kwargs)
