"""Device timing, throughput/MFU, latency and memory profilers, NVTX ranges."""
from __future__ import annotations

import contextlib
import json
import os
import statistics
import subprocess
import tempfile
import time
from pathlib import Path
from typing import Callable, Dict, List, Optional

import torch
import torch.distributed as dist

_B200_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_measured_peaks(path: Optional[str] = None) -> Dict[str, float]:
    """Measured copy bandwidth / cuBLAS bf16 throughput of this GPU pool
    (``MEASURED_PEAKS.json`` at the repository root, else earlier B200
    measurements)."""
    cands = [path] if path else [os.environ.get("CFB_MEASURED_PEAKS"),
                                 str(Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json")]
    for c in cands:
        if c and Path(c).exists():
            try:
                d = json.loads(Path(c).read_text())
                out = dict(_B200_FALLBACK)
                for k in out:
                    v = d.get(k)
                    if isinstance(v, dict):
                        v = v.get("value")
                    if isinstance(v, (int, float)):
                        out[k] = float(v)
                out["source"] = c
                return out
            except (OSError, ValueError):
                pass
    return dict(_B200_FALLBACK, source="fallback")


def roofline(flops: float = 0.0, bytes_moved: float = 0.0, seconds: float = 1.0,
             peaks: Optional[Dict] = None, sustained: bool = False) -> Dict[str, float]:
    """Achieved TFLOP/s and GB/s and their fractions of the measured peaks."""
    pk = peaks or load_measured_peaks()
    tf = flops / seconds / 1e12
    gb = bytes_moved / seconds / 1e9
    peak_tf = pk["bf16_tflops_sustained" if sustained else "bf16_tflops"]
    return {"tflops": tf, "gbs": gb, "tensor_frac": tf / peak_tf, "hbm_frac": gb / pk["hbm_gbs"]}


def max_over_ranks(value: float, group=None) -> float:
    if not (dist.is_available() and dist.is_initialized()):
        return value
    dev = torch.device("cuda", torch.cuda.current_device()) if (
        dist.get_backend(group) == "nccl") else torch.device("cpu")
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t)


def cuda_time(fn: Callable, iters: int = 10, warmup: int = 3) -> float:
    """Mean milliseconds of ``fn`` by CUDA events on the current stream."""
    for _ in range(warmup):
        fn()
    if not torch.cuda.is_available():
        t0 = time.perf_counter()
        for _ in range(iters):
            fn()
        return (time.perf_counter() - t0) * 1e3 / iters
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def cuda_graph_time(fn: Callable, iters: int = 10, calls_per_graph: int = 10,
                    warmup: int = 3) -> float:
    """Mean device milliseconds of one ``fn()`` call with ``calls_per_graph``
    calls captured in one CUDA graph and the graph replayed ``iters`` times.

    For kernels of a few microseconds, eager timing measures the host's launch
    cost instead of the GPU; serving replays such kernels from graphs, and this
    times them the same way.  Falls back to ``cuda_time`` on CPU."""
    if not torch.cuda.is_available():
        return cuda_time(fn, iters, warmup)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(calls_per_graph):
            fn()
    g.replay()
    return cuda_time(g.replay, iters, warmup) / calls_per_graph


class StepTimer:
    """Per-step device time via CUDA events (host clock on CPU); tokens/s and MFU."""

    def __init__(self, seq_len: int = 2048, batch_size: int = 1, world_size: int = 1,
                 accum: int = 1, flops_per_token: Optional[float] = None, window: int = 100):
        self.tokens_per_step = seq_len * batch_size * world_size * accum
        self.world_size = world_size
        self.flops_per_token = flops_per_token
        self.window = window
        self.times: List[float] = []
        self._ev = None
        self._t0 = None

    def start(self) -> None:
        if torch.cuda.is_available():
            self._ev = torch.cuda.Event(enable_timing=True)
            self._ev.record()
        else:
            self._t0 = time.perf_counter()

    def stop(self) -> float:
        if self._ev is not None:
            end = torch.cuda.Event(enable_timing=True)
            end.record()
            end.synchronize()
            dt = self._ev.elapsed_time(end) / 1e3
        else:
            dt = time.perf_counter() - self._t0
        self.times.append(dt)
        return dt

    @property
    def avg_step_time(self) -> float:
        w = self.times[-self.window:]
        return sum(w) / len(w) if w else 0.0

    @property
    def tokens_per_second(self) -> float:
        a = self.avg_step_time
        return self.tokens_per_step / a if a > 0 else 0.0

    def mfu(self, flops_per_token: Optional[float] = None, peak_tflops: Optional[float] = None) -> float:
        fpt = flops_per_token or self.flops_per_token
        if not fpt:
            return 0.0
        peak = (peak_tflops or load_measured_peaks()["bf16_tflops_sustained"]) * 1e12
        return self.tokens_per_second * fpt / (peak * self.world_size)

    def reset(self) -> None:
        self.times.clear()


class LatencyProfiler:
    """Named sections timed with CUDA events; ``summary`` gives mean/median/p90 ms."""

    def __init__(self):
        self.samples: Dict[str, List[float]] = {}

    @contextlib.contextmanager
    def section(self, name: str):
        if torch.cuda.is_available():
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            yield
            e.record()
            e.synchronize()
            ms = s.elapsed_time(e)
        else:
            t0 = time.perf_counter()
            yield
            ms = (time.perf_counter() - t0) * 1e3
        self.samples.setdefault(name, []).append(ms)

    def summary(self) -> Dict[str, Dict[str, float]]:
        out = {}
        for k, v in self.samples.items():
            sv = sorted(v)
            out[k] = {"mean_ms": statistics.fmean(v), "median_ms": statistics.median(v),
                      "p90_ms": sv[min(len(sv) - 1, int(0.9 * len(sv)))], "n": len(v)}
        return out


class ThroughputBenchmark:
    """Tokens/s of a callable that processes ``tokens_per_call`` tokens."""

    def __init__(self, fn: Callable, tokens_per_call: int):
        self.fn, self.tokens = fn, tokens_per_call

    def run(self, iters: int = 10, warmup: int = 3) -> Dict[str, float]:
        ms = cuda_time(self.fn, iters, warmup)
        return {"ms_per_call": ms, "tokens_per_s": self.tokens / (ms / 1e3)}


class MemoryProfiler:
    """Peak / current device memory around a region."""

    def __init__(self, device=None):
        self.device = device
        self.records: Dict[str, Dict[str, float]] = {}

    @contextlib.contextmanager
    def track(self, name: str):
        if not torch.cuda.is_available():
            yield
            return
        torch.cuda.synchronize(self.device)
        torch.cuda.reset_peak_memory_stats(self.device)
        before = torch.cuda.memory_allocated(self.device)
        yield
        torch.cuda.synchronize(self.device)
        self.records[name] = {"before_gb": before / 1e9,
                              "after_gb": torch.cuda.memory_allocated(self.device) / 1e9,
                              "peak_gb": torch.cuda.max_memory_allocated(self.device) / 1e9}


@contextlib.contextmanager
def nvtx_range(name: str):
    if torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


class ProfilerContext:
    """``torch.profiler`` wrapper writing a chrome trace (off the timed path)."""

    def __init__(self, out_dir: str = "profiles_trace", active: int = 3, warmup: int = 1):
        self.out_dir, self.active, self.warmup = out_dir, active, warmup
        self.prof = None

    def __enter__(self):
        acts = [torch.profiler.ProfilerActivity.CPU]
        if torch.cuda.is_available():
            acts.append(torch.profiler.ProfilerActivity.CUDA)
        self.prof = torch.profiler.profile(
            activities=acts, schedule=torch.profiler.schedule(wait=0, warmup=self.warmup,
                                                              active=self.active),
            on_trace_ready=torch.profiler.tensorboard_trace_handler(self.out_dir))
        self.prof.__enter__()
        return self

    def step(self):
        self.prof.step()

    def __exit__(self, *exc):
        return self.prof.__exit__(*exc)


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a timed region
    (``start()`` before it, ``stop()`` after: median SM MHz, max MHz, the throttle
    reasons seen).  Reads settings only; changes none."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.idx = device_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.fh,
                stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}
