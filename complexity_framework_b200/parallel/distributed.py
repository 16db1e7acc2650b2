"""Process-group bootstrap and teardown (one process per GPU).

``init_distributed`` reads the torchrun environment (RANK, WORLD_SIZE,
LOCAL_RANK, MASTER_ADDR/PORT), binds the local GPU, and creates the default
group with NCCL on CUDA or gloo on CPU.  The collective timeout comes from
``COMPLEXITY_DIST_TIMEOUT_S`` (default 600 s single node), and NCCL async
error handling is enabled, as in complexity/parallel/data_parallel.py:278-370.
``safe_main`` aborts and destroys the process group on any exit path so a
failed rank does not leave peers blocked (complexity/gpu/distributed_cleanup.py).
"""
from __future__ import annotations

import datetime
import functools
import os
import sys
from typing import Callable, Optional

import torch
import torch.distributed as dist


def dist_timeout_s(default: float = 600.0) -> float:
    v = os.environ.get("COMPLEXITY_DIST_TIMEOUT_S")
    try:
        return float(v) if v else default
    except ValueError:
        return default


def configure_nccl(*, p2p: bool = True, ib: Optional[bool] = None,
                   socket_ifname: Optional[str] = None, debug: Optional[str] = None) -> dict:
    """Set NCCL environment knobs (before the first NCCL communicator is created)."""
    env = {"TORCH_NCCL_ASYNC_ERROR_HANDLING": "1"}
    if not p2p:
        env["NCCL_P2P_DISABLE"] = "1"
    if ib is not None:
        env["NCCL_IB_DISABLE"] = "0" if ib else "1"
    if socket_ifname:
        env["NCCL_SOCKET_IFNAME"] = socket_ifname
    if debug:
        env["NCCL_DEBUG"] = debug
    for k, v in env.items():
        os.environ.setdefault(k, v)
    return env


def init_distributed(backend: Optional[str] = None, timeout_s: Optional[float] = None):
    """Initialise the default process group from the environment.

    Returns ``(rank, world_size, local_rank, device)``.  A single process with
    no torchrun environment runs without a process group.
    """
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cuda = torch.cuda.is_available() and backend != "gloo"
    device = torch.device("cuda", local) if cuda else torch.device("cpu")
    if cuda:
        torch.cuda.set_device(device)
    if world > 1 and not dist.is_initialized():
        configure_nccl()
        kwargs = dict(backend=backend or ("nccl" if cuda else "gloo"),
                      timeout=datetime.timedelta(seconds=timeout_s or dist_timeout_s()))
        if cuda:
            kwargs["device_id"] = device
        dist.init_process_group(**kwargs)
    return rank, world, local, device


def is_main_process() -> bool:
    return not dist.is_initialized() or dist.get_rank() == 0


def get_rank() -> int:
    return dist.get_rank() if dist.is_initialized() else 0


def get_world_size() -> int:
    return dist.get_world_size() if dist.is_initialized() else 1


def barrier() -> None:
    if dist.is_initialized():
        dist.barrier()


def cleanup_distributed(abort: bool = False) -> None:
    if not dist.is_initialized():
        return
    try:
        if abort:
            pg = dist.distributed_c10d._get_default_group()
            if hasattr(pg, "abort"):
                pg.abort()
        dist.destroy_process_group()
    except Exception:
        pass


def safe_main(fn: Callable) -> Callable:
    """Run ``fn``; on an exception abort the process group so peers fail fast."""

    @functools.wraps(fn)
    def wrapper(*a, **kw):
        try:
            out = fn(*a, **kw)
        except BaseException:
            cleanup_distributed(abort=True)
            raise
        cleanup_distributed(abort=False)
        return out

    return wrapper
