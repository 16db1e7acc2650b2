"""Step, accumulation and augmentation schedules of detector training.

Counterparts of complexity/generative/detection/training.py:1227-1472: the
per-step cosine multiplier with linear warmup, the validation cadence, the
checkpoint-selection key, the Mosaic schedule (on until ``close_mosaic_epochs``
before the end; optional packed epochs that divide an epoch's step count),
gradient-accumulation grouping (the last group of an epoch may be short and
is averaged over its own size), weight decay scaled to the realised batch,
and warmup resolved in optimizer steps.
"""
from __future__ import annotations

import math
from typing import Any, Dict, Mapping, Optional, Sequence, Tuple


def cosine_schedule(step: int, *, warmup_steps: int, total_steps: int, min_ratio: float) -> float:
    """Learning-rate multiplier: (step+1)/warmup during warmup, then a cosine from
    1 down to ``min_ratio`` over the remaining steps (flat after the horizon)."""
    if warmup_steps and step < warmup_steps:
        return (step + 1) / warmup_steps
    t = min(max((step - warmup_steps) / max(total_steps - warmup_steps, 1), 0.0), 1.0)
    return min_ratio + (1.0 - min_ratio) * 0.5 * (1.0 + math.cos(math.pi * t))


def should_validate_epoch(epoch: int, total_epochs: int, eval_every: int) -> bool:
    done = epoch + 1
    return done % eval_every == 0 or done == total_epochs


def validation_selection_score(metrics: Mapping[str, Any]) -> Tuple[str, float]:
    """Official COCO mAP50-95 when the metrics carry it, else mAP50."""
    key = "coco_map50_95" if metrics.get("official_coco") else "map50"
    if key not in metrics:
        raise ValueError(f"validation metrics are missing checkpoint selection key: {key}")
    return key, float(metrics[key])


def mosaic_source_images_per_sample(mosaic_probability: float, mosaic_tiles: int = 4) -> float:
    if not 0.0 <= mosaic_probability <= 1.0:
        raise ValueError("mosaic probability must be in [0, 1]")
    if mosaic_tiles < 1:
        raise ValueError("mosaic_tiles must be positive")
    return 1.0 + (mosaic_tiles - 1) * mosaic_probability


def mosaic_is_active_epoch(epoch: int, *, total_epochs: int, close_mosaic_epochs: int,
                           mosaic_probability: float) -> bool:
    if mosaic_probability <= 0.0:
        return False
    if not total_epochs or not close_mosaic_epochs:
        return True
    return epoch < max(total_epochs - close_mosaic_epochs, 0)


def _packed(full: int, active: bool, packed_epochs: int) -> int:
    if packed_epochs < 1:
        raise ValueError("packed_epochs must be positive")
    return max(1, math.ceil(full / packed_epochs)) if active else full


def detector_epoch_steps(full_loader_steps: int, epoch: int, *, total_epochs: int,
                         mosaic_probability: float, close_mosaic_epochs: int,
                         mosaic_packed_epoch: bool, packed_epochs: int = 1) -> int:
    """Microbatches of one epoch: the loader's count, divided by ``packed_epochs``
    in Mosaic epochs when packing is on."""
    active = mosaic_packed_epoch and mosaic_is_active_epoch(
        epoch, total_epochs=total_epochs, close_mosaic_epochs=close_mosaic_epochs,
        mosaic_probability=mosaic_probability)
    return _packed(full_loader_steps, active, packed_epochs)


def detector_step_schedule(full_loader_steps: int, *, total_epochs: int,
                           mosaic_probability: float, close_mosaic_epochs: int,
                           mosaic_packed_epoch: bool, packed_epochs: int = 1) -> Tuple[int, ...]:
    return tuple(detector_epoch_steps(full_loader_steps, e, total_epochs=total_epochs,
                                      mosaic_probability=mosaic_probability,
                                      close_mosaic_epochs=close_mosaic_epochs,
                                      mosaic_packed_epoch=mosaic_packed_epoch,
                                      packed_epochs=packed_epochs)
                 for e in range(total_epochs))


def resolve_accumulation_steps(*, per_device_batch_size: int, world_size: int,
                               nominal_batch_size: int, requested_steps: int = 0) -> int:
    """Explicit count, else round(nominal batch / global batch) (at least 1)."""
    if per_device_batch_size <= 0 or world_size <= 0:
        raise ValueError("batch size and world size must be positive")
    if nominal_batch_size < 0 or requested_steps < 0:
        raise ValueError("nominal batch size and accumulation steps cannot be negative")
    if requested_steps:
        return requested_steps
    if not nominal_batch_size:
        return 1
    return max(round(nominal_batch_size / (per_device_batch_size * world_size)), 1)


def optimizer_step_schedule(microbatch_schedule: Sequence[int],
                            accumulation_steps: int) -> Tuple[int, ...]:
    if accumulation_steps <= 0:
        raise ValueError("accumulation_steps must be positive")
    if any(s <= 0 for s in microbatch_schedule):
        raise ValueError("every epoch must contain at least one microbatch")
    return tuple(-(-s // accumulation_steps) for s in microbatch_schedule)


def accumulation_group(batch_index: int, *, epoch_batches: int,
                       accumulation_steps: int) -> Tuple[int, bool]:
    """(size of the group this microbatch belongs to, whether it ends the group)."""
    if epoch_batches <= 0 or accumulation_steps <= 0:
        raise ValueError("epoch_batches and accumulation_steps must be positive")
    if not 0 <= batch_index < epoch_batches:
        raise ValueError("batch_index is outside the epoch")
    start = batch_index - batch_index % accumulation_steps
    size = min(accumulation_steps, epoch_batches - start)
    last = (batch_index + 1) % accumulation_steps == 0 or batch_index + 1 == epoch_batches
    return size, last


def normalized_weight_decay(weight_decay: float, *, global_batch_size: int,
                            accumulation_steps: int, nominal_batch_size: int) -> float:
    """weight_decay * realised effective batch / nominal batch (unchanged if nominal = 0)."""
    if weight_decay < 0.0:
        raise ValueError("weight_decay cannot be negative")
    if global_batch_size <= 0 or accumulation_steps <= 0:
        raise ValueError("global batch size and accumulation steps must be positive")
    if nominal_batch_size < 0:
        raise ValueError("nominal_batch_size cannot be negative")
    if not nominal_batch_size:
        return weight_decay
    return weight_decay * global_batch_size * accumulation_steps / nominal_batch_size


def resolve_warmup_steps(*, requested_steps: int, warmup_epochs: Optional[float],
                         steps_in_first_epoch: int, total_steps: int,
                         unpacked_total_steps: Optional[int] = None) -> int:
    """Warmup in optimizer steps: from epochs when given, else the raw count
    (rescaled when packing shortened the run), clamped to the run length."""
    if requested_steps < 0 or steps_in_first_epoch <= 0 or total_steps <= 0:
        raise ValueError("invalid warmup or optimizer-step horizon")
    if unpacked_total_steps is not None and unpacked_total_steps <= 0:
        raise ValueError("unpacked_total_steps must be positive")
    if warmup_epochs is not None:
        if warmup_epochs < 0.0:
            raise ValueError("warmup_epochs cannot be negative")
        requested_steps = round(warmup_epochs * steps_in_first_epoch)
    elif unpacked_total_steps and unpacked_total_steps > total_steps:
        requested_steps = round(requested_steps * total_steps / unpacked_total_steps)
    return min(requested_steps, total_steps)


def format_loss_metrics_for_logging(averages: Mapping[str, float]) -> Dict[str, float]:
    """``loss`` becomes the fixed-weight monitoring loss when one is reported and
    the optimised value moves to ``optimization_loss``."""
    m = dict(averages)
    opt = m.pop("loss")
    m["optimization_loss"] = opt
    m["loss"] = m.pop("monitor_loss", opt)
    for head in ("one_to_many", "one_to_one"):
        if f"{head}_monitor_loss" in m:
            m[f"{head}_optimization_loss"] = m.pop(f"{head}_loss")
            m[f"{head}_loss"] = m.pop(f"{head}_monitor_loss")
    return m
