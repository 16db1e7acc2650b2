"""Profiling: FLOP estimates and counters, device-timed step timer with MFU
against measured peaks, latency / throughput / memory profilers, NVTX ranges.

Counterparts: complexity/profiling/{flops_counter,latency_profiler,
memory_profiler}.py and complexity/gpu/profiler.py:15-95 (``StepTimer``,
``profile_model_flops``).  Timing here uses CUDA events on the launching
stream (never host wall-clock around unsynchronised work) and reduces
multi-rank timings as the max over ranks.
"""
from .flops import (FLOPSCounter, ModelComplexity, count_parameters, estimate_transformer_flops,
                    model_flops_per_token, parameter_breakdown, profile_model_flops)
from .bench import (ActivationMemoryProfiler, MemoryStats, MemoryTracker, ProfileResult,
                    benchmark_inference, benchmark_training, clear_memory, count_flops,
                    estimate_macs, estimate_model_memory, find_optimal_batch_size,
                    get_memory_stats, get_model_complexity, memory_snapshot)
from .timing import (LatencyProfiler, MemoryProfiler, ProfilerContext, StepTimer,
                     ThroughputBenchmark, cuda_graph_time, cuda_time, load_measured_peaks, max_over_ranks, nvtx_range,
                     roofline)

__all__ = ["FLOPSCounter", "LatencyProfiler", "MemoryProfiler", "ModelComplexity",
           "ProfilerContext", "StepTimer", "ThroughputBenchmark", "count_parameters", "cuda_graph_time", "cuda_time",
           "estimate_transformer_flops", "load_measured_peaks", "max_over_ranks",
           "model_flops_per_token", "nvtx_range", "parameter_breakdown", "profile_model_flops",
           "roofline", "ActivationMemoryProfiler", "MemoryStats", "MemoryTracker", "ProfileResult",
           "benchmark_inference", "benchmark_training", "clear_memory", "count_flops",
           "estimate_macs", "estimate_model_memory", "find_optimal_batch_size",
           "get_memory_stats", "get_model_complexity", "memory_snapshot"]
