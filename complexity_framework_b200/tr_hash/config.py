"""Shape, routing and runtime contract of one TR-Hash layer.

Enum values, field names, defaults and validation match the reference
(complexity/tr_hash/config.py:9-202) because they appear in checkpoints,
``capability_summary`` manifests and user code.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum
from typing import Iterable, Tuple

SUPPORTED_EXPERT_COUNTS = (1, 2, 4, 8, 16)
SUPPORTED_TOP_K = (1, 2, 4)


class TRHashBackend(str, Enum):
    AUTO = "auto"
    PYTORCH = "pytorch"
    CGGR = "cggr"
    FUSED_CUDA = "fused_cuda"
    CUDA_GRAPH = "cuda_graph"


class TRHashPrecision(str, Enum):
    FP32 = "fp32"
    BF16 = "bf16"
    FP16 = "fp16"
    FP8 = "fp8"
    INT8 = "int8"


class TRHashPhase(str, Enum):
    TRAINING = "training"
    INFERENCE = "inference"


class AttentionBackbone(str, Enum):
    GQA = "gqa"
    MHA = "mha"


class TRHashStrategy(str, Enum):
    MODULO_CYCLIC = "modulo_cyclic"
    BALANCED_HASH = "token_id_balanced_hash"
    AFFINE_HASH = "token_id_affine_hash"
    MULTI_HASH = "token_id_multi_hash"
    HIERARCHICAL_HASH = "token_id_hierarchical_hash"


@dataclass(frozen=True)
class GraphBucket:
    """A static (batch, sequence) shape that inference inputs are padded to."""

    batch_size: int
    sequence_length: int

    def __post_init__(self) -> None:
        if self.batch_size <= 0:
            raise ValueError("graph bucket batch_size must be positive")
        if self.sequence_length <= 0:
            raise ValueError("graph bucket sequence_length must be positive")

    @property
    def token_capacity(self) -> int:
        return self.batch_size * self.sequence_length


def _sorted_unique_buckets(values: Iterable[GraphBucket]) -> Tuple[GraphBucket, ...]:
    keys = sorted({(int(b.batch_size), int(b.sequence_length)) for b in values},
                  key=lambda bs: (bs[0] * bs[1], bs[0], bs[1]))
    return tuple(GraphBucket(b, s) for b, s in keys)


@dataclass(frozen=True)
class TRHashEngineConfig:
    hidden_size: int
    vocab_size: int
    num_experts: int = 4
    top_k: int = 2
    shared_width: int = 128
    expert_width: int = 48
    initializer_range: float = 0.02
    routing_strategy: TRHashStrategy = TRHashStrategy.BALANCED_HASH
    layer_index: int = 0
    route_seed: int = 0x71D5A17
    route_hash_count: int = 2
    route_weights: Tuple[float, ...] = ()
    shared_output_scale: float = 1.0
    routed_output_scale: float = 1.0
    attention_backbone: AttentionBackbone = AttentionBackbone.GQA
    phase: TRHashPhase = TRHashPhase.TRAINING
    precision: TRHashPrecision = TRHashPrecision.BF16
    backend: TRHashBackend = TRHashBackend.AUTO
    world_size: int = 1
    graph_buckets: Tuple[GraphBucket, ...] = field(default_factory=tuple)

    def __post_init__(self) -> None:
        setattr_ = object.__setattr__
        setattr_(self, "routing_strategy", TRHashStrategy(self.routing_strategy))
        setattr_(self, "attention_backbone", AttentionBackbone(self.attention_backbone))
        setattr_(self, "phase", TRHashPhase(self.phase))
        setattr_(self, "precision", TRHashPrecision(self.precision))
        setattr_(self, "backend", TRHashBackend(self.backend))
        setattr_(self, "graph_buckets", _sorted_unique_buckets(self.graph_buckets))

        checks = (
            (self.hidden_size > 0, "hidden_size must be positive"),
            (self.vocab_size > 0, "vocab_size must be positive"),
            (self.num_experts in SUPPORTED_EXPERT_COUNTS,
             f"num_experts must be one of {SUPPORTED_EXPERT_COUNTS}, got {self.num_experts}"),
            (self.top_k in SUPPORTED_TOP_K,
             f"top_k must be one of {SUPPORTED_TOP_K}, got {self.top_k}"),
            (self.top_k <= self.num_experts, "top_k cannot exceed num_experts"),
            (self.shared_width >= 0, "shared_width must be non-negative"),
            (self.expert_width > 0, "expert_width must be positive"),
            (self.initializer_range > 0, "initializer_range must be positive"),
            (self.layer_index >= 0, "layer_index must be non-negative"),
            (2 <= self.route_hash_count <= 8, "route_hash_count must be between 2 and 8"),
            (self.shared_output_scale >= 0, "shared_output_scale must be non-negative"),
            (self.routed_output_scale >= 0, "routed_output_scale must be non-negative"),
            (self.world_size > 0, "world_size must be positive"),
        )
        for ok, msg in checks:
            if not ok:
                raise ValueError(msg)

        weights = tuple(float(w) for w in self.route_weights)
        if not weights:
            weights = tuple(1.0 / self.top_k for _ in range(self.top_k))
        setattr_(self, "route_weights", weights)
        if len(weights) != self.top_k:
            raise ValueError("route_weights must contain exactly top_k values")
        if any(w < 0 for w in weights):
            raise ValueError("route_weights must be non-negative")
        if abs(sum(weights) - 1.0) > 1e-6:
            raise ValueError("route_weights must sum to 1")
        if self.backend is TRHashBackend.CUDA_GRAPH:
            if self.phase is not TRHashPhase.INFERENCE:
                raise ValueError("CUDA Graph execution is inference-only")
            if not self.graph_buckets:
                raise ValueError("CUDA Graph execution requires at least one graph bucket")

    @property
    def stored_routed_width(self) -> int:
        return self.num_experts * self.expert_width

    @property
    def active_routed_width(self) -> int:
        return self.top_k * self.expert_width

    @property
    def stored_mlp_width(self) -> int:
        return self.shared_width + self.stored_routed_width

    @property
    def active_mlp_width(self) -> int:
        return self.shared_width + self.active_routed_width

    @property
    def active_width_fraction(self) -> float:
        return self.active_mlp_width / self.stored_mlp_width
