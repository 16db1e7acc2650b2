"""Profiling entry points with the reference's names.

Counterparts of complexity/profiling/flops_counter.py:38-98 (``count_flops``,
``estimate_macs``, ``get_model_complexity``), latency_profiler.py:20-468
(``ProfileResult``, ``benchmark_inference``, ``benchmark_training``,
``find_optimal_batch_size``) and memory_profiler.py:20-200 (``MemoryStats``,
``memory_snapshot``, ``get_memory_stats``, ``clear_memory``,
``MemoryTracker``, ``estimate_model_memory``, ``ActivationMemoryProfiler``).

Differences in method: latencies are CUDA-event times of each call (not host
time around unsynchronised launches), the training benchmark runs the
framework's ``Trainer`` (fused kernels, flat AdamW) rather than a plain
optimizer loop, and the batch-size search doubles then bisects on measured
peak memory, treating an out-of-memory error as "does not fit".
"""
from __future__ import annotations

import gc
import math
import statistics
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn as nn

from .flops import FLOPSCounter, ModelComplexity


# ----------------------------------------------------------------- FLOPs
def _dummy_ids(model: nn.Module, input_shape: Tuple[int, ...], device) -> torch.Tensor:
    vocab = int(getattr(getattr(model, "config", None), "vocab_size", 1000) or 1000)
    return torch.randint(0, vocab, tuple(input_shape), device=device)


def _dev(model: nn.Module, device) -> torch.device:
    if device is not None:
        return torch.device(device)
    p = next(model.parameters(), None)
    return p.device if p is not None else torch.device("cpu")


def get_model_complexity(model: nn.Module, input_shape: Tuple[int, ...],
                         device=None) -> ModelComplexity:
    """Forward FLOPs of one call on token ids of ``input_shape`` (matmuls and
    routed-expert GEMMs at their active width) plus the parameter count."""
    return FLOPSCounter().count(model, _dummy_ids(model, input_shape, _dev(model, device)))


def count_flops(model: nn.Module, input_shape: Tuple[int, ...], device=None) -> int:
    return get_model_complexity(model, input_shape, device).flops


def estimate_macs(model: nn.Module, input_shape: Tuple[int, ...]) -> int:
    return count_flops(model, input_shape) // 2


# --------------------------------------------------------------- latency
@dataclass
class ProfileResult:
    mean_latency_ms: float = 0.0
    std_latency_ms: float = 0.0
    min_latency_ms: float = 0.0
    max_latency_ms: float = 0.0
    p50_latency_ms: float = 0.0
    p90_latency_ms: float = 0.0
    p99_latency_ms: float = 0.0
    throughput: float = 0.0        # samples per second
    num_runs: int = 0
    warmup_runs: int = 0

    def __str__(self) -> str:
        return (f"Latency: {self.mean_latency_ms:.2f} +- {self.std_latency_ms:.2f} ms "
                f"(min {self.min_latency_ms:.2f}, p50 {self.p50_latency_ms:.2f}, p90 "
                f"{self.p90_latency_ms:.2f}, p99 {self.p99_latency_ms:.2f}, max "
                f"{self.max_latency_ms:.2f}); throughput {self.throughput:.2f} samples/s")


def _pct(xs: Sequence[float], q: float) -> float:
    s = sorted(xs)
    if not s:
        return 0.0
    i = min(len(s) - 1, max(0, math.ceil(q * len(s)) - 1))
    return s[i]


def time_calls(fn: Callable[[], object], num_runs: int, warmup_runs: int,
               device: torch.device) -> List[float]:
    """Milliseconds per call: CUDA events around each call on CUDA, else a
    host clock (CPU work is synchronous)."""
    for _ in range(warmup_runs):
        fn()
    out = []
    if device.type == "cuda":
        torch.cuda.synchronize(device)
        for _ in range(num_runs):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            e.synchronize()
            out.append(s.elapsed_time(e))
    else:
        import time

        for _ in range(num_runs):
            t = time.perf_counter()
            fn()
            out.append((time.perf_counter() - t) * 1e3)
    return out


def profile_result(times_ms: List[float], samples_per_call: int, warmup: int) -> ProfileResult:
    mean = statistics.fmean(times_ms)
    return ProfileResult(mean, statistics.pstdev(times_ms) if len(times_ms) > 1 else 0.0,
                         min(times_ms), max(times_ms), _pct(times_ms, 0.5), _pct(times_ms, 0.9),
                         _pct(times_ms, 0.99), samples_per_call / (mean / 1e3), len(times_ms),
                         warmup)


@torch.no_grad()
def benchmark_inference(model: nn.Module, input_shape: Tuple[int, ...], num_runs: int = 100,
                        warmup_runs: int = 10, device=None) -> ProfileResult:
    dev = _dev(model, device)
    x = _dummy_ids(model, input_shape, dev)
    model.eval()
    t = time_calls(lambda: model(x), num_runs, warmup_runs, dev)
    return profile_result(t, int(input_shape[0]), warmup_runs)


def benchmark_training(model: nn.Module, batch_size: int, seq_length: int, num_steps: int = 100,
                       learning_rate: float = 1e-4, device=None,
                       warmup_steps: int = 3) -> Dict[str, float]:
    """Optimizer steps of the framework's Trainer on random token batches:
    ms per step and tokens per second (CUDA events on GPU)."""
    from ..training import Trainer, TrainingConfig

    dev = _dev(model, device)
    cfg = TrainingConfig(learning_rate=learning_rate, warmup_steps=0, lr_scheduler="constant",
                         precision="bf16" if dev.type == "cuda" else "fp32",
                         max_steps=10 ** 9, skip_param_update_check=True,
                         distributed_mode="none")
    tr = Trainer(model, cfg, device=dev)
    ids = _dummy_ids(model, (batch_size, seq_length), dev)
    t = time_calls(lambda: tr.train_step(ids, sync=False), num_steps, warmup_steps, dev)
    ms = statistics.fmean(t)
    return {"ms_per_step": ms, "tokens_per_s": batch_size * seq_length / (ms / 1e3),
            "samples_per_s": batch_size / (ms / 1e3), "steps": num_steps}


def find_optimal_batch_size(model: nn.Module, seq_length: int, start_batch: int = 1,
                            max_batch: int = 256, target_memory_fraction: float = 0.9,
                            step: Optional[Callable[[int], object]] = None) -> int:
    """Largest batch in [start_batch, max_batch] whose forward (or ``step(b)``)
    peaks below ``target_memory_fraction`` of the GPU: doubling, then bisection."""
    if not torch.cuda.is_available():
        return start_batch
    dev = _dev(model, None)
    limit = torch.cuda.get_device_properties(dev).total_memory * target_memory_fraction

    def fits(b: int) -> bool:
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats(dev)
        try:
            if step is not None:
                step(b)
            else:
                with torch.no_grad():
                    model(_dummy_ids(model, (b, seq_length), dev))
            torch.cuda.synchronize(dev)
            return torch.cuda.max_memory_allocated(dev) <= limit
        except torch.cuda.OutOfMemoryError:
            torch.cuda.empty_cache()
            return False

    if not fits(start_batch):
        return start_batch
    lo, hi = start_batch, start_batch
    while hi < max_batch and fits(min(2 * hi, max_batch)):
        lo = hi = min(2 * hi, max_batch)
    if hi == max_batch:
        return max_batch
    hi = min(2 * hi, max_batch)
    while hi - lo > 1:
        mid = (lo + hi) // 2
        lo, hi = (mid, hi) if fits(mid) else (lo, mid)
    return lo


# ---------------------------------------------------------------- memory
@dataclass
class MemoryStats:
    allocated_gb: float = 0.0
    reserved_gb: float = 0.0
    peak_allocated_gb: float = 0.0
    free_gb: float = 0.0
    total_gb: float = 0.0

    def __str__(self) -> str:
        return (f"allocated {self.allocated_gb:.2f} GB, reserved {self.reserved_gb:.2f} GB, "
                f"peak {self.peak_allocated_gb:.2f} GB, free {self.free_gb:.2f} / "
                f"{self.total_gb:.2f} GB")


def memory_snapshot(device=None) -> MemoryStats:
    if not torch.cuda.is_available():
        return MemoryStats()
    free, total = torch.cuda.mem_get_info(device)
    g = 2 ** 30
    return MemoryStats(torch.cuda.memory_allocated(device) / g,
                       torch.cuda.memory_reserved(device) / g,
                       torch.cuda.max_memory_allocated(device) / g, free / g, total / g)


def get_memory_stats(device=None) -> Dict[str, float]:
    s = memory_snapshot(device)
    return {"allocated_gb": s.allocated_gb, "reserved_gb": s.reserved_gb,
            "peak_allocated_gb": s.peak_allocated_gb, "free_gb": s.free_gb,
            "total_gb": s.total_gb}


def clear_memory() -> None:
    gc.collect()
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats()


class MemoryTracker:
    """Allocated / peak device memory between ``start()`` and ``stop()``."""

    def __init__(self, device=None):
        self.device = device
        self.reset()

    def reset(self) -> None:
        self._start = self._end = self._peak = 0

    def start(self) -> None:
        if torch.cuda.is_available():
            torch.cuda.synchronize(self.device)
            torch.cuda.reset_peak_memory_stats(self.device)
            self._start = torch.cuda.memory_allocated(self.device)

    def stop(self) -> None:
        if torch.cuda.is_available():
            torch.cuda.synchronize(self.device)
            self._end = torch.cuda.memory_allocated(self.device)
            self._peak = torch.cuda.max_memory_allocated(self.device)

    def __enter__(self):
        self.start()
        return self

    def __exit__(self, *exc):
        self.stop()
        return False

    @property
    def allocated_memory(self) -> int:
        return self._end - self._start

    @property
    def allocated_memory_gb(self) -> float:
        return self.allocated_memory / 2 ** 30

    @property
    def peak_memory(self) -> int:
        return max(0, self._peak - self._start)

    @property
    def peak_memory_gb(self) -> float:
        return self.peak_memory / 2 ** 30


def estimate_model_memory(model: nn.Module, *, optimizer: str = "adamw",
                          compute_dtype: torch.dtype = torch.bfloat16,
                          master_fp32: bool = True, shards: int = 1) -> Dict[str, float]:
    """Bytes (as GB) of weights, gradients and optimizer state; ``shards`` >
    1 divides the fp32 state (and, for ZeRO-3 callers, may divide all of it)."""
    n = sum(p.numel() for p in model.parameters())
    e = torch.empty(0, dtype=compute_dtype).element_size()
    weights, grads = n * e, n * e
    moments = {"adamw": 2, "adam": 2, "sgd": 0, "lion": 1}.get(optimizer.lower(), 2)
    state = n * 4 * (moments + (1 if master_fp32 else 0)) / shards
    g = 2 ** 30
    return {"parameters": n, "weights_gb": weights / g, "gradients_gb": grads / g,
            "optimizer_gb": state / g, "total_gb": (weights + grads + state) / g}


class ActivationMemoryProfiler:
    """Per-module output sizes of one forward (what autograd keeps alive) and
    the device memory allocated across the forward."""

    def __init__(self, model: nn.Module):
        self.model = model
        self.sizes: Dict[str, int] = {}

    def profile(self, *args, **kwargs) -> Dict[str, float]:
        self.sizes = {}
        hooks = []

        def hook(name):
            def fn(_m, _i, out):
                ts = out if isinstance(out, (tuple, list)) else (out,)
                n = sum(t.numel() * t.element_size() for t in ts if torch.is_tensor(t))
                self.sizes[name] = self.sizes.get(name, 0) + n
            return fn

        for name, m in self.model.named_modules():
            if name and not list(m.children()):
                hooks.append(m.register_forward_hook(hook(name)))
        tr = MemoryTracker()
        try:
            with tr:
                self.model(*args, **kwargs)
        finally:
            for h in hooks:
                h.remove()
        return {"module_outputs_gb": sum(self.sizes.values()) / 2 ** 30,
                "allocated_gb": tr.allocated_memory_gb, "peak_gb": tr.peak_memory_gb}

    def top(self, k: int = 10) -> List[Tuple[str, int]]:
        return sorted(self.sizes.items(), key=lambda kv: -kv[1])[:k]
