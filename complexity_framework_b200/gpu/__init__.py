"""GPU runtime helpers under the reference's ``complexity.gpu`` names.

Counterpart of complexity/gpu/ (compile.py, fused_kernels.py, memory.py,
precision.py, patches.py, nccl_config.py, distributed_cleanup.py,
data_loading.py, profiler.py).  The implementations live where this
framework keeps them (``utils/gpu.py``, ``parallel/distributed.py``,
``data/loader.py``, ``profiling/timing.py``, the native kernels behind
``core/layers.RMSNorm``); this package gathers them and adds the few that
have no other home.  Not built: the reference's patch that rewrites a Triton
heuristics file inside the installed torch package (this framework has no
Triton kernels, and it modifies no installed file) and the ROCm/RCCL
configuration (NVIDIA-only target); both entry points report that.
"""
from __future__ import annotations

import gc
import logging
import os
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

from ..core.layers import RMSNorm
from ..data.loader import BackgroundTokenizer, CUDAPrefetcher
from ..parallel.distributed import (cleanup_distributed, configure_nccl, dist_timeout_s,
                                    safe_main)
from ..profiling.timing import StepTimer
from ..utils.gpu import (GradientCompressor, clip_grad_norm_fused, configure_cuda_backends,
                         free_memory, memory_stats, set_allocator, setup_gpu)

logger = logging.getLogger(__name__)


# ------------------------------------------------------------------ compile
def set_compile_env(cache_dir: Optional[str] = None, max_autotune: bool = False) -> None:
    """Environment for ``torch.compile`` users (inductor cache location, autotune)."""
    if cache_dir:
        os.environ["TORCHINDUCTOR_CACHE_DIR"] = cache_dir
        os.environ["TRITON_CACHE_DIR"] = os.path.join(cache_dir, "triton")
    if max_autotune:
        os.environ["TORCHINDUCTOR_MAX_AUTOTUNE"] = "1"


def compile_model(model: torch.nn.Module, mode: str = "default", fullgraph: bool = False,
                  dynamic: bool = False, enabled: bool = True) -> torch.nn.Module:
    """Opt-in ``torch.compile`` of a module for experiments.  The framework's
    training and decode paths do not use it: they run the native kernels and
    replay whole steps from CUDA graphs (``TrainingConfig.cuda_graph``,
    ``InferenceEngine.warmup_decode_graphs``)."""
    if not enabled:
        return model
    return torch.compile(model, mode=mode, fullgraph=fullgraph, dynamic=dynamic)


# ------------------------------------------------------------ fused kernels
class FusedRMSNorm(RMSNorm):
    """RMSNorm on the native ring kernels (bf16 CUDA), PyTorch elsewhere."""

    def __init__(self, hidden_size: int, eps: float = 1e-6):
        super().__init__(hidden_size, eps)


def fused_swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up.  In the models SwiGLU is fused into the gate|up GEMM's
    epilogue; this stand-alone form is the PyTorch expression."""
    return F.silu(gate) * up


def fused_residual_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                           eps: float = 1e-6) -> Tuple[torch.Tensor, torch.Tensor]:
    """(rmsnorm(x + residual) * weight, x + residual)."""
    r = x + residual
    if r.is_cuda and r.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16 \
            and r.shape[-1] % 8 == 0:
        from ..ops import available

        if available():
            from ..ops.fused import rmsnorm

            return rmsnorm(r, weight, eps), r
    rf = r.float()
    y = rf * torch.rsqrt(rf.pow(2).mean(-1, keepdim=True) + eps)
    return (weight * y.to(r.dtype)), r


# ------------------------------------------------------------------ memory
def clear_gpu_cache() -> None:
    gc.collect()
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats()


def log_memory_usage(prefix: str = "", device: int = 0) -> dict:
    if not torch.cuda.is_available():
        return {}
    alloc = torch.cuda.memory_allocated(device) / 1e9
    reserved = torch.cuda.memory_reserved(device) / 1e9
    total = torch.cuda.get_device_properties(device).total_memory / 1e9
    st = {"allocated_gb": round(alloc, 2), "reserved_gb": round(reserved, 2),
          "total_gb": round(total, 2), "free_gb": round(total - alloc, 2),
          "utilization_pct": round(100 * alloc / total, 1)}
    logger.info("[gpu] %sMemory: %.1fGB / %.1fGB (%.1f%%) reserved=%.1fGB", prefix, alloc, total,
                st["utilization_pct"], reserved)
    return st


def estimate_max_batch_size(model: torch.nn.Module, seq_len: int = 2048, vocab_size: int = 32000,
                            device: int = 0, safety_margin: float = 0.85,
                            total_memory_bytes: Optional[int] = None) -> int:
    """Largest power-of-two micro-batch whose estimated footprint fits:
    18 bytes per parameter (bf16 weights + fp32 master and AdamW moments +
    bf16 gradient), plus per sequence the saved activations (about 34 bf16
    values per token per layer and hidden unit for this block design) and the
    bf16 logits chunk of the fused cross-entropy."""
    if total_memory_bytes is None:
        if not torch.cuda.is_available():
            return 32
        total_memory_bytes = torch.cuda.get_device_properties(device).total_memory
    usable = total_memory_bytes * safety_margin
    params = sum(p.numel() for p in model.parameters())
    left = usable - 18 * params
    cfg = getattr(model, "config", None)
    H = getattr(cfg, "hidden_size", 1024)
    L = getattr(cfg, "num_hidden_layers", 24)
    per_seq = seq_len * (34 * H * L * 2 + vocab_size * 2)
    if left <= per_seq:
        return 1
    b = 1
    while 2 * b * per_seq <= left:
        b *= 2
    return b


# --------------------------------------------------------------- precision
def configure_mixed_precision(matmul_bf16: bool = True, conv_bf16: bool = True,
                              rnn_bf16: bool = False, softmax_fp32: bool = True,
                              layernorm_fp32: bool = True, cross_entropy_fp32: bool = True) -> dict:
    """Records the precision policy.  The native paths already compute in bf16
    with fp32 accumulation and keep softmax, norms and cross-entropy statistics
    in fp32; PyTorch autocast keeps the same ops in fp32 by default."""
    policy = dict(matmul_bf16=matmul_bf16, conv_bf16=conv_bf16, rnn_bf16=rnn_bf16,
                  softmax_fp32=softmax_fp32, layernorm_fp32=layernorm_fp32,
                  cross_entropy_fp32=cross_entropy_fp32)
    if torch.cuda.is_available():
        torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    logger.info("[gpu] mixed precision policy: %s", policy)
    return policy


class BF16Autocast:
    """``with BF16Autocast(): ...`` or ``@BF16Autocast.wrap`` (no-op without CUDA)."""

    def __init__(self, enabled: bool = True, cache_enabled: bool = True):
        self.enabled = enabled and torch.cuda.is_available()
        self.cache_enabled = cache_enabled
        self._ctx = None

    def __enter__(self):
        if self.enabled:
            self._ctx = torch.autocast("cuda", dtype=torch.bfloat16,
                                       cache_enabled=self.cache_enabled)
            return self._ctx.__enter__()
        return self

    def __exit__(self, *exc):
        if self._ctx is not None:
            return self._ctx.__exit__(*exc)
        return False

    @staticmethod
    def wrap(fn):
        def run(*a, **k):
            with BF16Autocast():
                return fn(*a, **k)
        return run


def upcast_softmax(attn_weights: torch.Tensor) -> torch.Tensor:
    """Softmax in fp32, cast back to the input dtype."""
    return torch.softmax(attn_weights.float(), dim=-1).to(attn_weights.dtype)


# ----------------------------------------------------------------- patches
def patch_expandable_segments() -> None:
    """Expandable allocator segments (must precede the first CUDA allocation)."""
    set_allocator(expandable_segments=True)


def patch_nccl_timeouts(timeout_s: Optional[float] = None) -> None:
    """Asynchronous NCCL error handling and the collective timeout
    (``COMPLEXITY_DIST_TIMEOUT_S``) for process groups created afterwards."""
    os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "1")
    os.environ["COMPLEXITY_DIST_TIMEOUT_S"] = str(int(timeout_s or dist_timeout_s()))


def patch_triton_heuristics() -> bool:
    """Not built: the reference edits a file of the installed torch package; this
    framework runs no Triton kernels and modifies no installed file."""
    logger.info("[gpu] triton heuristics patch: not applicable (no Triton kernels; installed "
                "files are never modified)")
    return False


def apply_gpu_patches(expandable_segments: bool = True, nccl_timeouts: bool = True,
                      triton_heuristics: bool = False) -> dict:
    done = {}
    if expandable_segments:
        patch_expandable_segments()
        done["expandable_segments"] = True
    if nccl_timeouts:
        patch_nccl_timeouts()
        done["nccl_timeouts"] = True
    done["triton_heuristics"] = patch_triton_heuristics() if triton_heuristics else False
    return done


def configure_rccl(*args, **kwargs):
    raise RuntimeError("RCCL (AMD) is not a target of this framework; use configure_nccl")


__all__ = ["setup_gpu", "set_allocator", "configure_cuda_backends", "memory_stats", "free_memory",
           "clip_grad_norm_fused", "GradientCompressor", "configure_nccl", "configure_rccl",
           "safe_main", "cleanup_distributed", "StepTimer", "CUDAPrefetcher", "BackgroundTokenizer",
           "set_compile_env", "compile_model", "FusedRMSNorm", "fused_swiglu",
           "fused_residual_rmsnorm", "clear_gpu_cache", "log_memory_usage",
           "estimate_max_batch_size", "configure_mixed_precision", "BF16Autocast",
           "upcast_softmax", "patch_expandable_segments", "patch_nccl_timeouts",
           "patch_triton_heuristics", "apply_gpu_patches"]
