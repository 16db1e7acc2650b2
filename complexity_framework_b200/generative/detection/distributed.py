"""Data-parallel plumbing for detector training and evaluation.

Counterpart of complexity/generative/detection/distributed.py:15-136: an
evaluation sampler that shards without padding or duplicates, and a context
object (rank, world, device) that builds samplers, wraps the model in DDP,
gathers / broadcasts Python objects, averages scalar dictionaries and
collects every rank's RNG state for exact resume.  NCCL on CUDA, gloo on CPU
(so the CPU tests run the multi-rank paths).
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Any, Dict, Iterator, List, Mapping, Optional

import torch
import torch.distributed as dist
from torch.utils.data import Dataset, DistributedSampler, Sampler


class DistributedEvalSampler(Sampler[int]):
    """Rank r evaluates items r, r + W, r + 2W, ...: every item exactly once."""

    def __init__(self, dataset: Dataset, rank: int, world_size: int):
        self.n, self.rank, self.world = len(dataset), rank, world_size

    def __iter__(self) -> Iterator[int]:
        return iter(range(self.rank, self.n, self.world))

    def __len__(self) -> int:
        return max(0, -(-(self.n - self.rank) // self.world))


@dataclass(frozen=True)
class DistributedContext:
    device: torch.device
    rank: int = 0
    world_size: int = 1
    local_rank: int = 0

    @property
    def enabled(self) -> bool:
        return self.world_size > 1

    @property
    def is_main(self) -> bool:
        return self.rank == 0

    @classmethod
    def initialize(cls, device: torch.device) -> "DistributedContext":
        """From torchrun's environment (or an already initialised group)."""
        if dist.is_available() and dist.is_initialized():
            w, r = dist.get_world_size(), dist.get_rank()
            return cls(device=device, rank=r, world_size=w,
                       local_rank=int(os.environ.get("LOCAL_RANK", r)))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        if world == 1:
            return cls(device=device)
        local = int(os.environ.get("LOCAL_RANK", "0"))
        if device.type == "cuda":
            torch.cuda.set_device(local)
            device = torch.device("cuda", local)
        dist.init_process_group("nccl" if device.type == "cuda" else "gloo")
        return cls(device=device, rank=dist.get_rank(), world_size=dist.get_world_size(),
                   local_rank=local)

    def train_sampler(self, dataset: Dataset, seed: int) -> Optional[DistributedSampler]:
        if not self.enabled:
            return None
        return DistributedSampler(dataset, num_replicas=self.world_size, rank=self.rank,
                                  shuffle=True, seed=seed, drop_last=False)

    def eval_sampler(self, dataset: Dataset) -> Optional[DistributedEvalSampler]:
        return DistributedEvalSampler(dataset, self.rank, self.world_size) if self.enabled else None

    def wrap(self, model: torch.nn.Module) -> torch.nn.Module:
        if not self.enabled:
            return model
        ids = [self.device.index] if self.device.type == "cuda" else None
        return torch.nn.parallel.DistributedDataParallel(
            model, device_ids=ids, broadcast_buffers=False, gradient_as_bucket_view=True,
            find_unused_parameters=False)

    def all_gather_objects(self, value: Any) -> List[Any]:
        if not self.enabled:
            return [value]
        out: List[Any] = [None] * self.world_size
        dist.all_gather_object(out, value)
        return out

    def broadcast_object(self, value: Any, *, source: int = 0) -> Any:
        if not self.enabled:
            return value
        box = [value if self.rank == source else None]
        dist.broadcast_object_list(box, src=source)
        return box[0]

    def mean_scalars(self, values: Mapping[str, float]) -> Dict[str, float]:
        if not self.enabled:
            return dict(values)
        names = sorted(values)
        dev = self.device if self.device.type == "cuda" else torch.device("cpu")
        t = torch.tensor([float(values[k]) for k in names], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        return dict(zip(names, (t / self.world_size).cpu().tolist()))

    def rng_state(self) -> Dict[str, torch.Tensor]:
        st = {"torch": torch.get_rng_state()}
        if self.device.type == "cuda":
            st["cuda"] = torch.cuda.get_rng_state(self.device)
        return st

    def gather_rng_states(self) -> Optional[List[Dict[str, torch.Tensor]]]:
        return self.all_gather_objects(self.rng_state()) if self.enabled else None

    def barrier(self) -> None:
        if self.enabled:
            dist.barrier()

    def close(self) -> None:
        if self.enabled and dist.is_initialized():
            dist.destroy_process_group()
