"""Data parallelism front-ends with the reference's names.

The work happens in the flat-buffer optimizer (``training.optim.FusedAdamW``):
``ddp`` all-reduces each flat gradient buffer once per step, ``fsdp`` (ZeRO-2)
reduce-scatters it, updates the fp32 master shard and all-gathers the bf16
parameters; ``FULL_SHARD`` selects ZeRO-3 (``parallel/fsdp.py``: parameters
sharded per block, gathered one block ahead, gradients reduce-scattered
during backward).  These helpers keep the call sites of
complexity/parallel/data_parallel.py:79-271 (``wrap_model_fsdp``,
``simple_ddp``, ``GradientAccumulator``, ``ShardingMode``) working: they tag
the model with its data-parallel mode and broadcast rank 0's weights.
"""
from __future__ import annotations

import contextlib
from enum import Enum

import torch
import torch.distributed as dist
import torch.nn as nn


class ShardingMode(str, Enum):
    FULL_SHARD = "full_shard"
    SHARD_GRAD_OP = "shard_grad_op"
    NO_SHARD = "no_shard"
    HYBRID_SHARD = "hybrid_shard"


class PrecisionMode(str, Enum):
    FP32 = "fp32"
    BF16 = "bf16"
    FP16 = "fp16"


@torch.no_grad()
def broadcast_parameters(model: nn.Module, group=None, src: int = 0) -> None:
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    for t in list(model.parameters()) + [b for b in model.buffers() if b.is_floating_point()]:
        dist.broadcast(t.data, src=src, group=group)


def wrap_model_fsdp(model: nn.Module, sharding_mode: ShardingMode = ShardingMode.FULL_SHARD,
                    precision: PrecisionMode = PrecisionMode.BF16, process_group=None,
                    **unused) -> nn.Module:
    """Mark ``model`` for sharded-optimizer data parallelism and cast to ``precision``."""
    dtype = {PrecisionMode.BF16: torch.bfloat16, PrecisionMode.FP16: torch.float16,
             PrecisionMode.FP32: torch.float32}[PrecisionMode(precision)]
    model = model.to(dtype)
    mode = ShardingMode(sharding_mode)
    # FULL_SHARD: parameters, gradient owners and optimizer state sharded per
    # block (ZeRO-3, parallel/fsdp.py, installed by the Trainer);
    # SHARD_GRAD_OP / HYBRID_SHARD: replicated bf16 parameters with sharded
    # optimizer state (ZeRO-2, the fused NVLink reduce + AdamW path)
    model.dp_mode = {ShardingMode.NO_SHARD: "ddp",
                     ShardingMode.FULL_SHARD: "zero3"}.get(mode, "fsdp")
    model.dp_group = process_group
    broadcast_parameters(model, process_group)
    return model


def simple_ddp(model: nn.Module, process_group=None, **unused) -> nn.Module:
    """Mark ``model`` for all-reduce data parallelism (gradients averaged once per step)."""
    model.dp_mode = "ddp"
    model.dp_group = process_group
    broadcast_parameters(model, process_group)
    return model


class GradientAccumulator:
    """``with acc.accumulate(): loss.backward()`` -- reduction happens once, at the
    optimizer step, so no per-micro-batch synchronisation needs suppressing."""

    def __init__(self, model: nn.Module, steps: int):
        self.model = model
        self.steps = steps
        self.count = 0

    @contextlib.contextmanager
    def accumulate(self):
        self.count += 1
        yield

    @property
    def should_step(self) -> bool:
        return self.count % self.steps == 0
