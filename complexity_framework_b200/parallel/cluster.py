"""3-D parallel layout: [DP, PP, TP] ranks with TP innermost.

Global rank g = (dp * PP + pp) * TP + tp, so tensor-parallel peers are
adjacent ranks (one NVSwitch domain), then pipeline stages, then data
replicas; the same layout and names as complexity/parallel/cluster.py:58-439
(``ClusterConfig``, ``ProcessGroupManager``, ``ClusterModel``).  Expert
parallelism, when used, spans the data-parallel group.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist
import torch.nn as nn


@dataclass
class ClusterConfig:
    tp_size: int = 1
    pp_size: int = 1
    dp_size: Optional[int] = None
    ep_size: int = 1
    pp_schedule: str = "1f1b"
    micro_batches: int = 1
    sharded_optimizer: bool = True

    def resolve(self, world: int) -> "ClusterConfig":
        if self.dp_size is None:
            if world % (self.tp_size * self.pp_size):
                raise ValueError("world size must be divisible by tp_size * pp_size")
            self.dp_size = world // (self.tp_size * self.pp_size)
        if self.tp_size * self.pp_size * self.dp_size != world:
            raise ValueError(f"tp*pp*dp = {self.tp_size * self.pp_size * self.dp_size} "
                             f"!= world size {world}")
        if self.ep_size not in (1, self.dp_size):
            raise ValueError("ep_size must be 1 or equal to dp_size")
        return self

    @staticmethod
    def estimate(world: int, num_params: int, gpu_mem_gb: float = 180.0,
                 bytes_per_param: int = 16) -> "ClusterConfig":
        """Smallest TP that fits params + optimizer state (16 B/param) in 60% of memory."""
        tp = 1
        while tp < min(world, 8) and num_params * bytes_per_param / tp > 0.6 * gpu_mem_gb * 1e9:
            tp *= 2
        return ClusterConfig(tp_size=tp).resolve(world)


class ProcessGroupManager:
    def __init__(self, config: ClusterConfig):
        world = dist.get_world_size()
        self.rank = dist.get_rank()
        self.config = config.resolve(world)
        T, P, D = config.tp_size, config.pp_size, config.dp_size
        self.tp_rank = self.rank % T
        self.pp_rank = (self.rank // T) % P
        self.dp_rank = self.rank // (T * P)
        self.tp_group = self.pp_group = self.dp_group = None
        # every rank must take part in creating every group
        for d in range(D):
            for p in range(P):
                ranks = [(d * P + p) * T + t for t in range(T)]
                g = dist.new_group(ranks)
                if self.rank in ranks:
                    self.tp_group = g
        for d in range(D):
            for t in range(T):
                ranks = [(d * P + p) * T + t for p in range(P)]
                g = dist.new_group(ranks)
                if self.rank in ranks:
                    self.pp_group = g
        for p in range(P):
            for t in range(T):
                ranks = [(d * P + p) * T + t for d in range(D)]
                g = dist.new_group(ranks)
                if self.rank in ranks:
                    self.dp_group = g

    def ranks_of(self, kind: str) -> List[int]:
        T, P, D = self.config.tp_size, self.config.pp_size, self.config.dp_size
        if kind == "tp":
            base = (self.dp_rank * P + self.pp_rank) * T
            return [base + t for t in range(T)]
        if kind == "pp":
            return [(self.dp_rank * P + p) * T + self.tp_rank for p in range(P)]
        return [(d * P + self.pp_rank) * T + self.tp_rank for d in range(D)]


class ClusterModel(nn.Module):
    """Apply TP, then PP, then EP to a full-weight model; data parallelism is the optimizer's."""

    def __init__(self, model: nn.Module, config: ClusterConfig,
                 groups: Optional[ProcessGroupManager] = None):
        super().__init__()
        from .expert_parallel import make_expert_parallel
        from .pipeline_parallel import PipelineModel
        from .tensor_parallel import make_parallel

        self.groups = groups or ProcessGroupManager(config)
        self.config = self.groups.config
        if self.config.tp_size > 1:
            make_parallel(model, self.groups.tp_group)
        if self.config.ep_size > 1:
            make_expert_parallel(model, self.groups.dp_group)
        self.model = model
        self.pipeline = (PipelineModel(model, self.groups.pp_group,
                                       schedule=self.config.pp_schedule)
                         if self.config.pp_size > 1 else None)

    def parameters_for_optimizer(self):
        if self.pipeline is not None:
            return self.pipeline.stage.parameters()
        return self.model.parameters()

    def train_step(self, input_ids: torch.Tensor) -> Optional[torch.Tensor]:
        """Forward+backward of one batch (split into micro-batches for PP); returns the loss."""
        if self.pipeline is not None:
            mbs = list(input_ids.chunk(self.config.micro_batches))
            return self.pipeline.train_step(mbs)
        loss = self.model.loss(input_ids)
        loss.backward()
        return loss.detach()
