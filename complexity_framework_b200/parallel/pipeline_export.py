"""Export-based pipeline parallelism on ``torch.distributed.pipelining``.

The model is traced once (torch.export) and split at layer boundaries into
``pp_size`` stages; each rank then runs its stage under a microbatch schedule
(GPipe or 1F1B) with point-to-point sends of the hidden states.  This is the
counterpart of complexity/parallel/pipeline_export.py:17-98 (split specs,
tensor-output wrapper, tracing) with a stage builder and a schedule runner
added; the hand-written 1F1B of ``pipeline_parallel.py`` remains the path that
needs no tracing.

Tracing uses the PyTorch reference math of every layer (the sm_100a kernels
are opaque to export); the traced stages run wherever the module runs.
"""
from __future__ import annotations

from collections.abc import Mapping
from typing import Any, Callable, Optional

import torch
import torch.nn as nn


def pipeline_split_spec(num_layers: int, pp_size: int, *, layers_prefix: str = "layers",
                        require_even: bool = True) -> dict:
    """Split points at the first layer of every stage after the first.

    32 layers over 8 stages: ``layers.4``, ``layers.8``, ..., ``layers.28``.
    """
    if num_layers <= 0:
        raise ValueError("num_layers must be positive")
    if pp_size <= 0:
        raise ValueError("pp_size must be positive")
    if pp_size > num_layers:
        raise ValueError("pp_size cannot exceed num_layers")
    if require_even and num_layers % pp_size:
        raise ValueError(f"num_layers ({num_layers}) must be divisible by pp_size ({pp_size})")
    from torch.distributed.pipelining import SplitPoint

    return {f"{layers_prefix}.{s * num_layers // pp_size}": SplitPoint.BEGINNING
            for s in range(1, pp_size)}


class LastHiddenStateWrapper(nn.Module):
    """Tensor-in / tensor-out view of ``ComplexityModel`` for tracing: returns the
    final hidden state (the LM head and loss stay outside the pipe, as in the
    fused-loss training path)."""

    def __init__(self, model: nn.Module):
        super().__init__()
        self.model = model

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        # Every TR-Hash layer routes by token id.  Stages after the first take no
        # root inputs, so the ids travel with the hidden state as an activation;
        # activations must be floating point (exact for ids < 2^24) and each
        # block turns them back into integers.
        routing = input_ids.to(torch.float32)
        out = self.model(input_ids, routing_ids=routing, return_logits=False)
        return out["last_hidden_state"] if isinstance(out, Mapping) else out


def enable_pipeline_export_mode(model: nn.Module) -> None:
    """Put every layer on its traceable path: the PyTorch reference math for the
    TR-Hash experts and attention (no custom kernels, no CUDA-graph buckets)."""
    model.config.use_custom_kernels = False
    for module in model.modules():
        cfg = getattr(module, "config", None)
        if cfg is not None and hasattr(cfg, "static_expert_capacity"):
            cfg.static_expert_capacity = True
        if hasattr(module, "use_custom_kernels"):
            module.use_custom_kernels = False
    from ..tr_hash import TRHashBackend, TRHashEngine

    for module in model.modules():
        if isinstance(module, TRHashEngine):
            module.config = type(module.config)(**{**module.config.__dict__,
                                                   "backend": TRHashBackend.PYTORCH})


def trace_pipeline(model: nn.Module, example_input_ids: torch.Tensor, *, pp_size: int,
                   layers_prefix: str = "model.layers", return_last_hidden: bool = True) -> Any:
    """Trace ``model`` into a ``torch.distributed.pipelining.Pipe`` of ``pp_size`` stages."""
    from torch.distributed.pipelining import pipeline

    if pp_size <= 0:
        raise ValueError("pp_size must be positive")
    enable_pipeline_export_mode(model)
    traced = LastHiddenStateWrapper(model) if return_last_hidden else model
    spec = pipeline_split_spec(len(model.layers), pp_size,
                               layers_prefix=layers_prefix if return_last_hidden else "layers")
    return pipeline(traced, mb_args=(example_input_ids,), split_spec=spec)


class ExportPipelineRunner:
    """Run one rank's stage of a traced pipe under a microbatch schedule.

    ``loss_fn(hidden, labels)`` is applied on the last stage; ``step(ids, labels)``
    runs forward and backward over ``n_microbatches`` and returns the mean loss
    on the last stage (None elsewhere).  Gradients land on the stage module's
    parameters (``runner.module``).
    """

    def __init__(self, pipe: Any, stage_index: int, num_stages: int, device: torch.device,
                 n_microbatches: int, loss_fn: Callable, schedule: str = "1f1b",
                 group: Optional[Any] = None):
        from torch.distributed.pipelining import Schedule1F1B, ScheduleGPipe

        self.stage = pipe.build_stage(stage_index, device, group)
        self.module = self.stage.submod
        self.stage_index, self.num_stages = stage_index, num_stages
        self.losses = []

        def loss(out, target):
            val = loss_fn(out, target)
            self.losses.append(val.detach())
            return val

        cls = {"1f1b": Schedule1F1B, "gpipe": ScheduleGPipe}[schedule]
        self.schedule = cls(self.stage, n_microbatches=n_microbatches, loss_fn=loss)

    def step(self, input_ids: Optional[torch.Tensor], labels: Optional[torch.Tensor]):
        self.losses = []
        first, last = self.stage_index == 0, self.stage_index == self.num_stages - 1
        args = (input_ids,) if first else ()
        kwargs = {"target": labels} if last else {}
        self.schedule.step(*args, **kwargs)
        if last:
            return torch.stack(self.losses).mean()
        return None
