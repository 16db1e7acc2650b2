"""GPU/runtime helpers: backend configuration, memory, precision, gradient
compression, fused gradient clipping.

Counterpart of complexity/gpu/ (setup_gpu, configure_cuda_backends, memory
helpers, precision helpers, ``GradientCompressor`` and
``clip_grad_norm_fused`` of gradient.py:18-138).  The reference's patch that
rewrites an installed torch file on disk is not reproduced; allocator
settings go through ``PYTORCH_CUDA_ALLOC_CONF`` instead.
"""
from __future__ import annotations

import contextlib
import os
from typing import Dict, Iterable, List, Optional

import torch
import torch.distributed as dist

_DTYPES = {"fp32": torch.float32, "float32": torch.float32, "bf16": torch.bfloat16,
           "bfloat16": torch.bfloat16, "fp16": torch.float16, "float16": torch.float16}


def dtype_from_string(name: str) -> torch.dtype:
    try:
        return _DTYPES[name.lower()]
    except KeyError as e:
        raise ValueError(f"unknown dtype {name!r}") from e


def configure_cuda_backends(tf32: bool = True, cudnn_benchmark: bool = True) -> None:
    torch.backends.cuda.matmul.allow_tf32 = tf32
    torch.backends.cudnn.allow_tf32 = tf32
    torch.backends.cudnn.benchmark = cudnn_benchmark


def set_allocator(expandable_segments: bool = True) -> None:
    """Must run before the first CUDA allocation of the process."""
    if expandable_segments:
        os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")


def setup_gpu(device: Optional[int] = None, **kw) -> torch.device:
    set_allocator()
    if not torch.cuda.is_available():
        return torch.device("cpu")
    dev = torch.device("cuda", device if device is not None else
                       int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    configure_cuda_backends(**kw)
    return dev


def memory_stats(device=None) -> Dict[str, float]:
    if not torch.cuda.is_available():
        return {}
    free, total = torch.cuda.mem_get_info(device)
    return {"allocated_gb": torch.cuda.memory_allocated(device) / 1e9,
            "reserved_gb": torch.cuda.memory_reserved(device) / 1e9,
            "peak_gb": torch.cuda.max_memory_allocated(device) / 1e9,
            "free_gb": free / 1e9, "total_gb": total / 1e9}


def free_memory() -> None:
    import gc

    gc.collect()
    if torch.cuda.is_available():
        torch.cuda.empty_cache()


@contextlib.contextmanager
def autocast(precision: str = "bf16", device_type: str = "cuda"):
    dt = dtype_from_string(precision)
    if dt == torch.float32:
        yield
        return
    with torch.autocast(device_type=device_type, dtype=dt):
        yield


@torch.no_grad()
def clip_grad_norm_fused(params: Iterable[torch.nn.Parameter], max_norm: float) -> torch.Tensor:
    """Global L2 norm with one multi-tensor norm and one multi-tensor scale (no host sync)."""
    grads = [p.grad for p in params if p.grad is not None]
    if not grads:
        return torch.zeros(())
    norms = torch._foreach_norm(grads)
    total = torch.linalg.vector_norm(torch.stack([n.float() for n in norms]))
    coef = (max_norm / (total + 1e-6)).clamp(max=1.0)
    torch._foreach_mul_(grads, coef.to(grads[0].dtype))
    return total


class GradientCompressor:
    """Compressed gradient averaging for bandwidth-limited links.

    ``topk``: each rank keeps the largest ``ratio`` fraction of (gradient +
    error-feedback residual) and all-gathers (indices, values); the dropped
    part is kept as the next residual.  ``quantize``: per-rank int8 with one
    absmax scale per tensor, all-gathered and dequantised before summing.
    ``none``: dense all-reduce.
    """

    def __init__(self, method: str = "none", ratio: float = 0.1, group=None):
        if method not in ("none", "topk", "quantize"):
            raise ValueError("method must be none, topk or quantize")
        self.method, self.ratio, self.group = method, ratio, group
        self._residuals: Dict[str, torch.Tensor] = {}

    @torch.no_grad()
    def compress_and_allreduce(self, model: torch.nn.Module) -> None:
        if not (dist.is_available() and dist.is_initialized()):
            return
        world = dist.get_world_size(self.group)
        for name, p in model.named_parameters():
            if p.grad is None:
                continue
            g = p.grad
            if self.method == "none":
                dist.all_reduce(g, group=self.group)
                g.div_(world)
            elif self.method == "topk":
                self._topk(name, g, world)
            else:
                self._quantized(g, world)

    def _topk(self, name, g, world):
        flat = g.reshape(-1).float()
        if name in self._residuals:
            flat = flat + self._residuals[name]
        k = max(1, int(flat.numel() * self.ratio))
        idx = flat.abs().topk(k).indices
        vals = flat[idx]
        res = flat.clone()
        res[idx] = 0
        self._residuals[name] = res
        all_idx = [torch.empty_like(idx) for _ in range(world)]
        all_val = [torch.empty_like(vals) for _ in range(world)]
        dist.all_gather(all_idx, idx, group=self.group)
        dist.all_gather(all_val, vals, group=self.group)
        dense = torch.zeros_like(flat)
        for i, v in zip(all_idx, all_val):
            dense.index_add_(0, i, v)
        g.copy_((dense / world).view_as(g))

    def _quantized(self, g, world):
        flat = g.reshape(-1).float()
        scale = flat.abs().max().clamp_min(1e-12) / 127
        q = torch.round(flat / scale).clamp(-127, 127).to(torch.int8)
        qs = [torch.empty_like(q) for _ in range(world)]
        ss = [torch.empty_like(scale.reshape(1)) for _ in range(world)]
        dist.all_gather(qs, q, group=self.group)
        dist.all_gather(ss, scale.reshape(1), group=self.group)
        tot = sum(a.float() * s for a, s in zip(qs, ss))
        g.copy_((tot / world).view_as(g))
