"""Model architecture configuration.

Field names, defaults, validation rules, ``to_dict``/``from_dict`` behaviour
and presets follow the reference's public contract
(complexity/config/model_config.py:15-610) so that ``config.json`` files and
checkpoints move between the two frameworks unchanged.  Experimental fields
that only feed attention/MLP variants outside TR-GQA/TR-MHA are accepted and
round-tripped but do not change the TR-Hash model built here.
"""
from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass, field
from typing import Any, Dict, Optional

import torch

_ROUTING_STRATEGIES = frozenset(
    {
        "zipf",
        "modulo",
        "modulo_cyclic",
        "modulo_balanced_secondary",
        "modulo_frequency_balanced_secondary",
        "token_id_balanced_hash",
        "token_id_pair_coverage_hash",
        "token_id_multi_hash",
        "token_id_hierarchical_hash",
        "round_robin",
        "random",
        "lsh_hidden",
    }
)

_REMOVED_MLP = frozenset(
    {
        "standard", "gelu", "swiglu", "silu", "llama", "geglu", "mixtral", "learned_router",
        "standard_moe", "i64_swiglu", "integer_swiglu", "i64_token_routed", "integer_moe",
        "token_routed", "sort_split", "sort_split_moe", "deterministic_moe", "complexity",
    }
)
_TOKEN_ROUTED_MLP = frozenset(
    {"token_routed", "sort_split", "sort_split_moe", "deterministic_moe", "complexity"}
)
_MHA_TYPES = frozenset({"mha", "tr_mha", "token_routed_mha", "tr_mha_v2", "token_routed_mha_v2"})


@dataclass
class ModelConfig:
    """Architecture of a TR-GQA / TR-MHA decoder with the TR-Hash MoE FFN."""

    # architecture
    hidden_size: int = 768
    num_hidden_layers: int = 12
    intermediate_size: Optional[int] = None
    vocab_size: int = 32000
    # attention
    num_attention_heads: int = 12
    num_key_value_heads: Optional[int] = None
    attention_type: str = "gqa"
    attention_dropout: float = 0.0
    use_qk_norm: bool = True
    sliding_window: Optional[int] = None
    causal_conv_kernel_size: int = 4
    causal_conv_dilation_cycle: int = 8
    causal_state_rank: int = 16
    causal_context_gate_init: float = 1.0
    causal_contextual_mix_init: float = 0.0
    causal_context_fusion_size: int = 0
    causal_stable_delta: bool = False
    causal_delta_chunk_size: int = 512
    causal_delta_timescales: int = 1
    causal_delta_collision_normalized: bool = False
    causal_delta_lexical_values: bool = False
    causal_delta_lexical_forge: bool = False
    causal_delta_occurrence_address: bool = False
    tr_mha_num_experts: int = 4
    tr_mha_adapter_rank: int = 8
    tr_mha_top_k: int = 2
    tr_mha_adapter_gate_init: float = 0.1
    tr_mha_id_primary_logit: float = 2.0
    tr_mha_id_secondary_logit: float = 1.0
    tr_mha_id_other_logit: float = -2.0
    tr_mha_verifier_gate_init: float = 0.1
    tr_mha_verifier_temperature: float = 1.0
    tr_mha_targets: str = "qv"
    # positions
    max_position_embeddings: int = 2048
    rope_theta: float = 10000.0
    rope_type: str = "standard"
    rope_fraction: float = 1.0
    # MLP
    mlp_type: str = "tr_hash_engine"
    hidden_act: str = "silu"
    # TR-Hash MoE
    num_experts: int = 1
    expert_initialization: str = "gpt_normal"
    token_frequencies: Optional[torch.Tensor] = None
    routing_strategy: str = "modulo_cyclic"
    route_hash_count: int = 2
    lsh_routing: bool = False
    lsh_bits: int = 0
    lsh_from_layer: int = 0
    lsh_threshold_mode: str = "zero"
    shared_expert: bool = True
    shared_intermediate_size: Optional[int] = None
    shared_expert_chunk_tokens: int = 0
    use_shared_routed_gates: bool = False
    shared_gate_init: float = 1.0
    routed_gate_init: float = 1.0
    shared_output_scale: float = 1.0
    routed_output_scale: float = 1.0
    shared_output_scale_first_layer: Optional[float] = None
    shared_output_scale_last_layer: Optional[float] = None
    routed_output_scale_first_layer: Optional[float] = None
    routed_output_scale_last_layer: Optional[float] = None
    top_k: int = 1
    top_k_primary_weight: Optional[float] = None
    learn_hash_pair_gates: bool = False
    hash_pair_gate_init: float = 0.5
    learn_hash_channel_modulation: bool = False
    hash_channel_scale_init: float = 0.0
    static_expert_capacity: bool = False
    use_custom_kernels: Any = "auto"
    collect_moe_telemetry: bool = False
    use_cggr: Any = "auto"
    active_num_experts: Optional[int] = None
    active_expert_width: Optional[int] = None
    # lexical variants (accepted for config compatibility)
    lexical_object_rank: int = 16
    lexical_object_gate_init: float = 0.1
    tie_lexical_object_embeddings: bool = False
    micro_num_experts: int = 4
    micro_expert_width: int = 16
    micro_expert_gate_init: float = 0.1
    lexical_gqa_rank: int = 16
    lexical_gqa_gate_init: float = 0.0
    lexical_gqa_use_token_code: bool = True
    lexical_key_gate_init: float = 0.05
    lexical_zipf_path: Optional[str] = None
    lexical_zipf_mode: str = "uniform"
    lexical_zipf_alpha: float = 0.25
    lexical_zipf_floor: float = 0.1
    lexical_zipf_permutation_seed: int = 1729
    # normalisation
    norm_type: str = "rmsnorm"
    norm_eps: float = 1e-6
    # embeddings
    tie_word_embeddings: bool = True
    # runtime
    use_sdpa: bool = True
    use_cache: bool = True
    is_causal: bool = True
    initializer_range: float = 0.02
    # muP
    use_mup_init: bool = False
    use_mup_attn_scale: bool = False
    use_mup_output_mult: bool = False
    mup_base_width: int = 256
    extra_config: Dict[str, Any] = field(default_factory=dict)

    def __post_init__(self) -> None:
        if self.mlp_type in _REMOVED_MLP:
            if self.mlp_type in _TOKEN_ROUTED_MLP:
                raise ValueError(
                    f"mlp_type={self.mlp_type!r} was removed; convert token_routed checkpoints "
                    "with complexity_framework_b200.utils.conversion."
                    "convert_token_routed_state_dict and use 'tr_hash_engine'."
                )
            raise ValueError(
                f"mlp_type={self.mlp_type!r} was removed: only the TR-Hash MoE FFN "
                "('tr_hash_engine' or 'tr_hash_moe') is supported."
            )
        if self.intermediate_size is None:
            if self.mlp_type in ("tr_hash_engine", "tr_hash_moe"):
                width = int(self.hidden_size * 8 / 3)
                self.intermediate_size = (width + 255) // 256 * 256
            else:
                self.intermediate_size = 4 * self.hidden_size
        if self.num_key_value_heads is None:
            if self.attention_type == "mqa":
                self.num_key_value_heads = 1
            elif self.attention_type in _MHA_TYPES:
                self.num_key_value_heads = self.num_attention_heads
            else:
                self.num_key_value_heads = max(1, self.num_attention_heads // 4)
        self._validate()

    # ------------------------------------------------------------------ checks
    def _validate(self) -> None:
        def need(cond: bool, msg: str) -> None:
            if not cond:
                raise ValueError(msg)

        need(self.hidden_size > 0, "hidden_size must be positive")
        need(self.num_hidden_layers > 0, "num_hidden_layers must be positive")
        need(self.intermediate_size is not None and self.intermediate_size > 0,
             "intermediate_size must be positive")
        need(self.vocab_size > 0, "vocab_size must be positive")
        need(self.num_attention_heads > 0, "num_attention_heads must be positive")
        need(self.shared_output_scale >= 0.0, "shared_output_scale must be non-negative")
        need(self.routed_output_scale >= 0.0, "routed_output_scale must be non-negative")
        for name in ("shared_output_scale_first_layer", "shared_output_scale_last_layer",
                     "routed_output_scale_first_layer", "routed_output_scale_last_layer"):
            value = getattr(self, name)
            need(value is None or value >= 0.0, f"{name} must be non-negative")
        need(self.num_key_value_heads is not None and self.num_key_value_heads > 0,
             "num_key_value_heads must be positive")
        need(self.hidden_size % self.num_attention_heads == 0,
             f"hidden_size ({self.hidden_size}) must be divisible by "
             f"num_attention_heads ({self.num_attention_heads})")
        need(self.num_attention_heads % self.num_key_value_heads == 0,
             f"num_attention_heads ({self.num_attention_heads}) must be divisible by "
             f"num_key_value_heads ({self.num_key_value_heads})")
        if self.attention_type in _MHA_TYPES - {"mha"}:
            need(self.num_key_value_heads == self.num_attention_heads,
                 "TR-MHA requires one K/V head per query head")
        need(0.0 <= self.attention_dropout < 1.0, "attention_dropout must be in [0, 1)")
        need(0.0 < self.rope_fraction <= 1.0, "rope_fraction must be in (0, 1]")
        need(self.sliding_window is None or self.sliding_window > 0,
             "sliding_window must be positive when set")
        need(self.causal_conv_kernel_size > 0, "causal_conv_kernel_size must be positive")
        need(self.causal_conv_dilation_cycle > 0, "causal_conv_dilation_cycle must be positive")
        need(self.causal_state_rank > 0, "causal_state_rank must be positive")
        need(self.num_experts > 0, "num_experts must be positive")
        need(self.expert_initialization in ("gpt_normal", "legacy_kaiming"),
             "expert_initialization must be 'gpt_normal' or 'legacy_kaiming'")
        need(self.top_k > 0, "top_k must be positive")
        need(self.top_k <= self.num_experts, "top_k cannot exceed num_experts")
        need(self.top_k_primary_weight is None or 0.0 <= self.top_k_primary_weight <= 1.0,
             "top_k_primary_weight must be in [0, 1]")
        need(0.0 < self.hash_pair_gate_init < 1.0,
             "hash_pair_gate_init must be strictly between 0 and 1")
        need(abs(self.hash_channel_scale_init) <= 1.0, "hash_channel_scale_init must be in [-1, 1]")
        need(self.routing_strategy in _ROUTING_STRATEGIES,
             f"unknown routing_strategy {self.routing_strategy!r}")
        need(self.lsh_threshold_mode in ("batch_median", "zero"),
             "lsh_threshold_mode must be 'batch_median' or 'zero'")
        need(2 <= self.route_hash_count <= 8, "route_hash_count must be between 2 and 8")
        need(self.shared_intermediate_size is None or self.shared_intermediate_size > 0,
             "shared_intermediate_size must be positive when set")
        need(self.shared_expert_chunk_tokens >= 0, "shared_expert_chunk_tokens must be non-negative")
        need(self.lexical_object_rank > 0, "lexical_object_rank must be positive")
        need(self.micro_num_experts > 0, "micro_num_experts must be positive")
        need(self.micro_expert_width > 0, "micro_expert_width must be positive")
        need(self.tr_mha_num_experts > 0, "tr_mha_num_experts must be positive")
        need(self.tr_mha_adapter_rank > 0, "tr_mha_adapter_rank must be positive")
        need(0 < self.tr_mha_top_k <= self.tr_mha_num_experts,
             "tr_mha_top_k must be between 1 and tr_mha_num_experts")
        need(0.0 < self.tr_mha_verifier_gate_init < 1.0, "tr_mha_verifier_gate_init must be in (0, 1)")
        need(self.tr_mha_verifier_temperature > 0.0, "tr_mha_verifier_temperature must be positive")
        need(self.tr_mha_targets in ("q", "v", "qv"), "tr_mha_targets must be one of: q, v, qv")
        need(self.mup_base_width > 0, "mup_base_width must be positive")
        if self.token_frequencies is not None:
            need(isinstance(self.token_frequencies, torch.Tensor),
                 "token_frequencies must be a torch.Tensor")
            need(self.token_frequencies.ndim == 1, "token_frequencies must be a 1D tensor")
            need(self.token_frequencies.numel() == self.vocab_size,
                 "token_frequencies length must match vocab_size")

    # -------------------------------------------------------------- properties
    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @property
    def num_kv_groups(self) -> int:
        return self.num_attention_heads // self.num_key_value_heads

    @property
    def mup_width_mult(self) -> float:
        if not self.use_mup_init:
            return 1.0
        return float(self.hidden_size) / float(self.mup_base_width)

    # ------------------------------------------------------------ (de)serialise
    def to_dict(self) -> Dict[str, Any]:
        """Public fields as a JSON-serialisable dict (tensors are skipped)."""
        out: Dict[str, Any] = {}
        for key, value in self.__dict__.items():
            if key.startswith("_") or isinstance(value, torch.Tensor):
                continue
            out[key] = value
        return out

    def save(self, path: str) -> None:
        data = self.to_dict()
        with open(path, "w") as fh:
            if path.endswith((".yaml", ".yml")):
                import yaml

                yaml.safe_dump(data, fh, default_flow_style=False)
            else:
                json.dump(data, fh, indent=2)

    @classmethod
    def from_dict(cls, data: Dict[str, Any]) -> "ModelConfig":
        """Build from a dict; unknown keys are dropped, unknown routing -> modulo_cyclic."""
        names = {f.name for f in dataclasses.fields(cls)}
        kept = {k: v for k, v in data.items() if k in names}
        if kept.get("routing_strategy") is not None and kept["routing_strategy"] not in _ROUTING_STRATEGIES:
            kept["routing_strategy"] = "modulo_cyclic"
        return cls(**kept)

    @classmethod
    def load(cls, path: str) -> "ModelConfig":
        with open(path) as fh:
            if path.endswith((".yaml", ".yml")):
                import yaml

                data = yaml.safe_load(fh)
            else:
                data = json.load(fh)
        return cls.from_dict(data)

    def __repr__(self) -> str:
        items = ", ".join(f"{k}={v}" for k, v in self.to_dict().items() if v is not None)
        return f"ModelConfig({items})"


# ---------------------------------------------------------------------- presets
def _preset(**kw) -> ModelConfig:
    base = dict(attention_type="gqa", mlp_type="tr_hash_engine", num_experts=4,
                norm_type="rmsnorm", use_qk_norm=True, vocab_size=32000,
                max_position_embeddings=2048)
    base.update(kw)
    return ModelConfig(**base)


def complexity_tiny_config() -> ModelConfig:
    return _preset(hidden_size=256, num_hidden_layers=6, num_attention_heads=4,
                   num_key_value_heads=2, intermediate_size=704)


def complexity_small_config() -> ModelConfig:
    return _preset(hidden_size=512, num_hidden_layers=8, num_attention_heads=8,
                   num_key_value_heads=4, intermediate_size=1408)


def complexity_base_config() -> ModelConfig:
    return _preset(hidden_size=768, num_hidden_layers=12, num_attention_heads=12,
                   num_key_value_heads=4, intermediate_size=2048)


def complexity_large_config() -> ModelConfig:
    return _preset(hidden_size=1024, num_hidden_layers=24, num_attention_heads=16,
                   num_key_value_heads=4, intermediate_size=2816, max_position_embeddings=4096)


def complexity_xl_config() -> ModelConfig:
    return _preset(hidden_size=2048, num_hidden_layers=24, num_attention_heads=16,
                   num_key_value_heads=4, intermediate_size=5632, max_position_embeddings=4096)


def complexity_7b_config() -> ModelConfig:
    return _preset(hidden_size=4096, num_hidden_layers=32, num_attention_heads=32,
                   num_key_value_heads=8, intermediate_size=11008, vocab_size=100000,
                   max_position_embeddings=8192)


def tr_hash_200m_config(**overrides) -> ModelConfig:
    """The released 200M TR-GQA / TR-Hash architecture (201,194,368 parameters).

    Mirrors ``make_config`` of scripts/train_tr_hash_200m_200b.py:107-131.
    """
    kw = dict(hidden_size=896, num_hidden_layers=16, num_attention_heads=14,
              num_key_value_heads=2, intermediate_size=256, shared_intermediate_size=3072,
              vocab_size=32000, num_experts=4, top_k=2, top_k_primary_weight=0.5,
              routing_strategy="token_id_multi_hash", route_hash_count=2, shared_expert=True,
              shared_output_scale=1.0, routed_output_scale=2.0, attention_type="gqa",
              max_position_embeddings=2048, use_qk_norm=True, tie_word_embeddings=True)
    kw.update(overrides)
    return ModelConfig(**kw)


PRESET_CONFIGS = {
    "complexity-tiny": complexity_tiny_config,
    "complexity-small": complexity_small_config,
    "complexity-base": complexity_base_config,
    "complexity-large": complexity_large_config,
    "complexity-xl": complexity_xl_config,
    "complexity-7b": complexity_7b_config,
    "tr-hash-200m": tr_hash_200m_config,
    "tiny": complexity_tiny_config,
    "small": complexity_small_config,
    "base": complexity_base_config,
    "large": complexity_large_config,
    "xl": complexity_xl_config,
}


def get_preset(name: str) -> ModelConfig:
    if name not in PRESET_CONFIGS:
        raise ValueError(f"Unknown preset: {name}. Available: {list(PRESET_CONFIGS)}")
    return PRESET_CONFIGS[name]()
