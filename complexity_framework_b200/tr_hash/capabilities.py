"""Backend resolution for a TR-Hash layer.

Decision contract as in the reference (complexity/tr_hash/capabilities.py:68-175):
quantised precisions raise, explicit requests are honoured or raise, ``auto``
picks the fastest available path and records why others were skipped.

Backends here:
  * ``fused_cuda`` - the sm_100a path: shared SwiGLU and all routed experts
    run as two tcgen05 GEMMs (gate|up with a routed-SwiGLU epilogue, down with
    a residual epilogue); routes enter as per-token expert scales.  Used when
    the routed width is a small fraction of the layer (dense-masked experts).
  * ``cggr`` - the grouped path for wide experts: tokens are planned into
    expert-contiguous order and each expert runs on its own rows.
  * ``pytorch`` - the authoritative eager reference math (CPU and CUDA).
  * ``cuda_graph`` - inference-only captured replay of the eager path.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch

from .config import TRHashBackend, TRHashEngineConfig, TRHashPhase, TRHashPrecision


@dataclass(frozen=True)
class BackendDecision:
    requested: TRHashBackend
    selected: TRHashBackend
    reasons: Tuple[str, ...]
    graph_safe: bool
    quantized: bool


def has_pair_metadata(config: TRHashEngineConfig) -> bool:
    """Whether the persisted compact top-2 pair buffers are populated.

    This rule is part of the checkpoint format (non-empty ``fused_route_codes``
    exactly for top-2 with two to eight experts).
    """
    return config.top_k == 2 and 2 <= config.num_experts <= 8


def supports_fused_cuda(config: TRHashEngineConfig) -> bool:
    """Shapes the sm_100a dense-masked expert path can execute."""
    return (config.expert_width % 32 == 0 and config.shared_width % 32 == 0
            and (config.shared_width + config.stored_routed_width) % 128 == 0
            and config.num_experts <= 16)


def dense_masked_profitable(config: TRHashEngineConfig) -> bool:
    """Dense-masked experts cost E/k times the routed FLOPs; use it when cheap.

    The extra work is (E - k) * expert_width columns per token; it is accepted
    while it stays under a quarter of the shared width (e.g. the 200M model:
    2*64 extra vs 3072 shared).
    """
    extra = (config.num_experts - config.top_k) * config.expert_width
    return extra <= max(config.shared_width, 1) // 4


def _extension_available() -> bool:
    from ..ops import available

    return available()


def select_backend(config: TRHashEngineConfig, *, device_type: str,
                   cggr_available: Optional[bool] = None,
                   fused_cuda_available: Optional[bool] = None) -> BackendDecision:
    if fused_cuda_available is None:
        fused_cuda_available = device_type == "cuda" and _extension_available()
    if cggr_available is None:
        cggr_available = device_type == "cuda"
    if config.precision in (TRHashPrecision.FP8, TRHashPrecision.INT8):
        raise NotImplementedError(
            f"{config.precision.value} is reserved by the TR-Hash API but needs the "
            "quantized grouped-GEMM kernel")

    def decide(sel, reasons=(), graph_safe=False):
        return BackendDecision(config.backend, sel, tuple(reasons), graph_safe, False)

    req = config.backend
    if req is TRHashBackend.PYTORCH:
        return decide(TRHashBackend.PYTORCH)
    if req is TRHashBackend.CUDA_GRAPH:
        if device_type != "cuda":
            raise RuntimeError("CUDA Graph backend requires a CUDA device")
        if config.phase is not TRHashPhase.INFERENCE:
            raise RuntimeError("CUDA Graph backend is inference-only")
        return decide(TRHashBackend.CUDA_GRAPH, graph_safe=True)
    if req is TRHashBackend.FUSED_CUDA:
        if device_type != "cuda":
            raise RuntimeError("fused CUDA backend requires a CUDA device")
        if not supports_fused_cuda(config):
            raise RuntimeError("fused CUDA backend needs widths that are multiples of 32 and "
                               "a total MLP width that is a multiple of 128")
        if not fused_cuda_available:
            raise RuntimeError("fused CUDA backend requested but the sm_100a extension is "
                               "not built")
        return decide(TRHashBackend.FUSED_CUDA)
    if req is TRHashBackend.CGGR:
        if device_type != "cuda":
            raise RuntimeError("CGGR backend requires a CUDA device")
        if not cggr_available:
            raise RuntimeError("CGGR backend requested but unavailable")
        return decide(TRHashBackend.CGGR)

    reasons = []
    if device_type != "cuda":
        reasons.extend(("fused CUDA requires CUDA", "CGGR requires CUDA"))
        return decide(TRHashBackend.PYTORCH, reasons)
    if not fused_cuda_available:
        reasons.append("sm_100a extension is not built")
        return decide(TRHashBackend.PYTORCH, reasons)
    if supports_fused_cuda(config) and dense_masked_profitable(config):
        return decide(TRHashBackend.FUSED_CUDA)
    if cggr_available:
        if not supports_fused_cuda(config):
            reasons.append("widths not eligible for the dense-masked fused path")
        else:
            reasons.append("routed width too large for dense-masked experts")
        return decide(TRHashBackend.CGGR, reasons)
    reasons.append("no grouped path available")
    return decide(TRHashBackend.PYTORCH, reasons)


def precision_to_torch_dtype(precision: TRHashPrecision) -> torch.dtype:
    table = {TRHashPrecision.FP32: torch.float32, TRHashPrecision.BF16: torch.bfloat16,
             TRHashPrecision.FP16: torch.float16}
    if precision not in table:
        raise NotImplementedError(f"{precision.value} needs the quantized TR-Hash backend")
    return table[precision]
