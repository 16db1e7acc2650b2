"""Small local checkpoints: ``step_XXXXXX/checkpoint.pt`` with a ``latest`` pointer.

Counterpart of complexity/utils/local_checkpoint.py:16-90 (the same directory
layout, so scripts written against it keep working): the step directory is
written under a temporary name and renamed, ``latest`` names the newest
step, and only the newest ``total_limit`` step directories are kept.
"""
from __future__ import annotations

import shutil
from pathlib import Path
from typing import Any, Dict, List, Tuple

import torch

CHECKPOINT_FILE = "checkpoint.pt"
LATEST_FILE = "latest"


def _steps(root: Path) -> List[Path]:
    return sorted(p for p in root.glob("step_*") if p.is_dir())


def resolve_checkpoint_path(path) -> Path:
    """A step directory, or ``<dir>/latest``: the pointed-to step when it is
    complete, else the newest step directory."""
    p = Path(path)
    if p.name != LATEST_FILE:
        return p
    root = p.parent
    if p.is_file():
        target = p.read_text(encoding="utf-8").strip()
        if target and (root / target / CHECKPOINT_FILE).exists():
            return root / target
    steps = _steps(root)
    if not steps:
        raise FileNotFoundError(f"No checkpoints found in {root}")
    return steps[-1]


def rotate_local_checkpoints(save_dir, *, total_limit: int = 3) -> None:
    steps = _steps(Path(save_dir))
    for old in steps[:max(0, len(steps) - max(1, total_limit))]:
        shutil.rmtree(old)


def save_local_checkpoint(save_dir, *, step: int, state: Dict[str, Any],
                          total_limit: int = 3) -> Path:
    root = Path(save_dir)
    root.mkdir(parents=True, exist_ok=True)
    final, tmp = root / f"step_{step:06d}", root / f".step_{step:06d}.tmp"
    if tmp.exists():
        shutil.rmtree(tmp)
    tmp.mkdir(parents=True)
    torch.save(state, tmp / CHECKPOINT_FILE)
    if final.exists():
        shutil.rmtree(final)
    tmp.rename(final)
    (root / LATEST_FILE).write_text(final.name + "\n", encoding="utf-8")
    rotate_local_checkpoints(root, total_limit=total_limit)
    return final


def load_local_checkpoint(path, map_location="cpu") -> Tuple[Path, Dict[str, Any]]:
    d = resolve_checkpoint_path(path)
    f = d / CHECKPOINT_FILE
    if not f.exists():
        raise FileNotFoundError(f"Checkpoint file not found: {f}")
    return d, torch.load(f, map_location=map_location, weights_only=False)
