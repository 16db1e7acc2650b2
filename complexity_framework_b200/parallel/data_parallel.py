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


# ---------------------------------------------- reference configuration names
_MODE_TO_DP = {ShardingMode.FULL_SHARD: "zero3", ShardingMode.SHARD_GRAD_OP: "fsdp",
               ShardingMode.HYBRID_SHARD: "fsdp", ShardingMode.NO_SHARD: "ddp"}


def get_sharding_strategy(mode: ShardingMode) -> str:
    """The data-parallel mode a sharding mode selects here: FULL_SHARD -> ZeRO-3
    (``zero3``), SHARD_GRAD_OP / HYBRID_SHARD -> ZeRO-2 (``fsdp``: sharded
    gradients and optimizer state, replicated bf16 parameters), NO_SHARD ->
    ``ddp`` (complexity/parallel/data_parallel.py:54-62 returns torch FSDP enums)."""
    return _MODE_TO_DP[ShardingMode(mode)]


def get_mixed_precision(mode: PrecisionMode):
    """Compute dtype of a precision mode (None for fp32): parameters run in it,
    the optimizer keeps fp32 masters, gradients reduce in it."""
    mode = PrecisionMode(mode)
    return None if mode == PrecisionMode.FP32 else (
        torch.float16 if mode == PrecisionMode.FP16 else torch.bfloat16)


class DataParallelConfig:
    def __init__(self, sharding_mode: ShardingMode = ShardingMode.FULL_SHARD,
                 precision: PrecisionMode = PrecisionMode.BF16, cpu_offload: bool = False,
                 gradient_accumulation_steps: int = 1, sync_module_states: bool = True):
        if cpu_offload:
            raise ValueError("cpu_offload is not supported: 180 GB of HBM per B200 holds the "
                             "sharded fp32 state of every configuration here")
        self.sharding_mode, self.precision = ShardingMode(sharding_mode), PrecisionMode(precision)
        self.cpu_offload = cpu_offload
        self.gradient_accumulation_steps = int(gradient_accumulation_steps)
        self.sync_module_states = sync_module_states

    @property
    def distributed_mode(self) -> str:
        return get_sharding_strategy(self.sharding_mode)


def resolve_dist_timeout_s(is_multi_node: bool, env=None) -> int:
    """Collective timeout: ``COMPLEXITY_DIST_TIMEOUT_S``, else 1800 s across nodes
    and 600 s on one node."""
    import os

    env = os.environ if env is None else env
    return int(env.get("COMPLEXITY_DIST_TIMEOUT_S", 1800 if is_multi_node else 600))


def cleanup() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()
