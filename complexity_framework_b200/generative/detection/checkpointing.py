"""Exactly resumable detector training state.

Counterpart of complexity/generative/detection/checkpointing.py:14-142: next
to the weights, ``training_state.pt`` carries the optimizer, scheduler, EMA,
cursor (epoch, batch in epoch, step), best scores, running loss sums, the run
shape (total epochs, steps per epoch), the options that must not change
across a resume, the RNG state of every rank and caller extras (such as
the host-side augmentation RNGs).  It is written last, through
a temporary file and an atomic rename, so its presence marks a complete,
resumable checkpoint; loading refuses a different run shape, changed options
or a different world size.
"""
from __future__ import annotations

from pathlib import Path
from typing import Any, Dict, List, Mapping, Optional, Sequence

import torch

TRAINING_STATE_FILENAME = "training_state.pt"
TRAINING_STATE_FORMAT = 1


def mismatched_options(saved: Mapping[str, Any], expected: Mapping[str, Any]) -> List[str]:
    return sorted(k for k in set(saved) | set(expected) if saved.get(k) != expected.get(k))


def save_training_state(checkpoint, optimizer, scheduler, *, epoch: int, batch_in_epoch: int,
                        step: int, best_map50: float, running_losses: Mapping[str, float],
                        running_loss_steps: int, total_epochs: int, steps_per_epoch: int,
                        training_options: Mapping[str, Any], ema=None,
                        best_end_to_end_map50: float = -1.0,
                        distributed_rng_states: Optional[Sequence[Mapping]] = None,
                        extra: Optional[Mapping[str, Any]] = None) -> Path:
    ck = Path(checkpoint)
    ck.mkdir(parents=True, exist_ok=True)
    state = {"format_version": TRAINING_STATE_FORMAT, "optimizer": optimizer.state_dict(),
             "scheduler": scheduler.state_dict(), "epoch": epoch,
             "batch_in_epoch": batch_in_epoch, "step": step, "best_map50": best_map50,
             "best_end_to_end_map50": best_end_to_end_map50,
             "running_losses": dict(running_losses), "running_loss_steps": running_loss_steps,
             "total_epochs": total_epochs, "steps_per_epoch": steps_per_epoch,
             "training_options": dict(training_options),
             "torch_rng_state": torch.get_rng_state(),
             "cuda_rng_state_all": (torch.cuda.get_rng_state_all()
                                    if torch.cuda.is_available() and distributed_rng_states is None
                                    else [])}
    if ema is not None:
        state["ema"] = ema.state_dict()
    if extra is not None:
        state["extra"] = dict(extra)  # e.g. host-side augmentation RNG states per rank
    if distributed_rng_states is not None:
        state["distributed_rng_states"] = list(distributed_rng_states)
        state["world_size"] = len(distributed_rng_states)
    tmp = ck / f".{TRAINING_STATE_FILENAME}.tmp"
    torch.save(state, tmp)
    tmp.replace(ck / TRAINING_STATE_FILENAME)
    return ck / TRAINING_STATE_FILENAME


def load_training_state(checkpoint, optimizer, scheduler, *, total_epochs: int,
                        steps_per_epoch: int, training_options: Mapping[str, Any], ema=None,
                        rank: int = 0, world_size: int = 1,
                        device: Optional[torch.device] = None) -> Dict[str, Any]:
    path = Path(checkpoint) / TRAINING_STATE_FILENAME
    if not path.is_file():
        raise ValueError(f"{checkpoint} is a weights-only checkpoint and cannot be resumed "
                         "exactly; fine-tune from its weights instead")
    st = torch.load(path, map_location="cpu", weights_only=False)
    if st.get("format_version") != TRAINING_STATE_FORMAT:
        raise ValueError(f"unsupported detector training-state format: "
                         f"{st.get('format_version')!r}")
    if st.get("total_epochs") != total_epochs:
        raise ValueError("--epochs is the total run target and must match the resumed run "
                         f"({total_epochs} != {st.get('total_epochs')})")
    if st.get("steps_per_epoch") != steps_per_epoch:
        raise ValueError("training dataset or batch size changed: steps per epoch do not match "
                         f"({steps_per_epoch} != {st.get('steps_per_epoch')})")
    bad = mismatched_options(st.get("training_options", {}), training_options)
    if bad:
        raise ValueError("exact resume requires unchanged training options; mismatched: "
                         + ", ".join(bad))
    saved_world = int(st.get("world_size", 1))
    if saved_world != world_size:
        raise ValueError(f"distributed world size differs from the resumed run "
                         f"({world_size} != {saved_world})")
    optimizer.load_state_dict(st["optimizer"])
    scheduler.load_state_dict(st["scheduler"])
    if ema is not None and "ema" in st:
        ema.load_state_dict(st["ema"])
    per_rank = st.get("distributed_rng_states")
    if per_rank is not None:
        torch.set_rng_state(per_rank[rank]["torch"])
        if "cuda" in per_rank[rank]:
            if device is None or device.type != "cuda":
                raise ValueError("distributed CUDA checkpoint requires a CUDA device")
            torch.cuda.set_rng_state(per_rank[rank]["cuda"], device=device)
    else:
        torch.set_rng_state(st["torch_rng_state"])
        cuda_states = st.get("cuda_rng_state_all", [])
        if cuda_states:
            if not torch.cuda.is_available() or len(cuda_states) != torch.cuda.device_count():
                raise ValueError("CUDA device count differs from the resumed run")
            torch.cuda.set_rng_state_all(cuda_states)
    return st
