"""TR-Hash MoE feed-forward block adapter (``tr_hash_engine`` / ``tr_hash_moe``).

Maps the model-level MLP settings to a ``TRHashEngine`` the way
complexity/core/mlp/tr_hash_engine.py:25-158 does: ``intermediate_size`` is
the TOTAL routed width (expert width = intermediate_size // num_experts), the
shared width is ``shared_intermediate_size or intermediate_size`` when a
shared expert is enabled, and route weights are ``(p, (1-p)/(k-1), ...)``.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, Optional

import torch.nn.functional as F
import torch.nn as nn

from ..tr_hash import (AttentionBackbone, TRHashBackend, TRHashEngine, TRHashEngineConfig,
                       TRHashPhase, TRHashPrecision, TRHashStrategy)
from .registry import register_mlp


@dataclass
class MLPConfig:
    hidden_size: int = 768
    intermediate_size: int = 2048
    hidden_act: str = "silu"
    num_experts: int = 1
    expert_initialization: str = "gpt_normal"
    initializer_range: float = 0.02
    vocab_size: int = 32000
    routing_strategy: str = "modulo_cyclic"
    route_hash_count: int = 2
    shared_expert: bool = False
    shared_intermediate_size: Optional[int] = None
    shared_output_scale: float = 1.0
    routed_output_scale: float = 1.0
    top_k: int = 1
    top_k_primary_weight: Optional[float] = None
    layer_idx: int = 0
    use_custom_kernels: Any = "auto"
    use_cggr: Any = "auto"
    active_num_experts: Optional[int] = None
    active_expert_width: Optional[int] = None
    attention_type: str = "gqa"
    # lexical MLPs
    lexical_object_rank: int = 16
    lexical_object_gate_init: float = 0.1
    micro_num_experts: int = 4
    micro_expert_width: int = 16
    micro_expert_gate_init: float = 0.1
    bias: bool = False
    extra: Dict[str, Any] = field(default_factory=dict)


def route_weights_for(top_k: int, primary: Optional[float]):
    if top_k == 1:
        return (1.0,)
    p = 1.0 / top_k if primary is None else float(primary)
    p = min(1.0, max(0.0, p))
    rest = (1.0 - p) / (top_k - 1)
    return (p,) + tuple(rest for _ in range(top_k - 1))


_STRATEGY_ALIASES = {
    "modulo": TRHashStrategy.MODULO_CYCLIC,
    "modulo_cyclic": TRHashStrategy.MODULO_CYCLIC,
    "token_id_balanced_hash": TRHashStrategy.BALANCED_HASH,
    "token_id_multi_hash": TRHashStrategy.MULTI_HASH,
    "token_id_hierarchical_hash": TRHashStrategy.HIERARCHICAL_HASH,
    "token_id_affine_hash": TRHashStrategy.AFFINE_HASH,
}


def strategy_for(name: str) -> TRHashStrategy:
    key = str(name).lower()
    if key not in _STRATEGY_ALIASES:
        raise ValueError("tr_hash_engine supports modulo_cyclic, token_id_balanced_hash, "
                         "token_id_multi_hash, token_id_affine_hash or "
                         f"token_id_hierarchical_hash; got {name!r}")
    return _STRATEGY_ALIASES[key]


def backend_for(use_custom_kernels, use_cggr) -> TRHashBackend:
    def norm(v):
        return v.strip().lower() if isinstance(v, str) else v

    k, c = norm(use_custom_kernels), norm(use_cggr)
    if k in (False, "false"):
        return TRHashBackend.PYTORCH
    if c in (True, "true"):
        return TRHashBackend.CGGR
    return TRHashBackend.AUTO


@register_mlp("tr_hash_engine")
@register_mlp("tr_hash_moe")
class TRHashEngineMLP(nn.Module):
    def __init__(self, config: MLPConfig):
        super().__init__()
        self.config = config
        if config.intermediate_size % config.num_experts:
            raise ValueError("TR-Hash routed width must be divisible by num_experts")
        shared = 0
        if config.shared_expert:
            shared = int(config.shared_intermediate_size if config.shared_intermediate_size
                         is not None else config.intermediate_size)
        self.top_k = int(config.top_k)
        self._primary_weight = (1.0 if self.top_k == 1 else float(
            1.0 / self.top_k if config.top_k_primary_weight is None
            else config.top_k_primary_weight))
        backbone = AttentionBackbone.MHA if config.attention_type == "mha" else AttentionBackbone.GQA
        self.engine = TRHashEngine(TRHashEngineConfig(
            hidden_size=config.hidden_size, vocab_size=config.vocab_size,
            num_experts=config.num_experts, top_k=self.top_k, shared_width=shared,
            expert_width=config.intermediate_size // config.num_experts,
            initializer_range=float(config.initializer_range),
            routing_strategy=strategy_for(config.routing_strategy),
            layer_index=int(config.layer_idx), route_hash_count=int(config.route_hash_count),
            route_weights=route_weights_for(self.top_k, config.top_k_primary_weight),
            shared_output_scale=float(config.shared_output_scale),
            routed_output_scale=float(config.routed_output_scale),
            attention_backbone=backbone, phase=TRHashPhase.TRAINING,
            precision=TRHashPrecision.BF16,
            backend=backend_for(config.use_custom_kernels, config.use_cggr)))
        if config.active_num_experts is not None or config.active_expert_width is not None:
            self.engine.set_active_capacity(num_experts=config.active_num_experts,
                                            expert_width=config.active_expert_width)

    def forward(self, hidden_states, token_ids=None, residual=None, **kwargs):
        if token_ids is None:
            raise ValueError("tr_hash_engine requires token_ids")
        return self.engine(hidden_states, token_ids, residual=residual)

    def forward_sp(self, h_shard, token_ids, residual, ws, name: str):
        """Fused sequence-parallel TP: [T/P, H] -> [T/P, H] (+ residual); routes use
        the token ids of all T tokens."""
        from ..ops import fused
        from ..parallel.tp_fused import TPMLPFn

        eng = self.engine
        cfg = eng.config
        scales = fused.route_scales(token_ids, eng._active_route_table, eng._route_weights,
                                    cfg.num_experts, cfg.routed_output_scale)
        sw = cfg.shared_width
        wg, wu, wd = eng._shared_weights()
        if wg is not None and wg.shape[0] % 128:
            # a TP shard of the shared width that is not a whole number of the
            # epilogue's 128-column gate|up blocks (11008 / 8 = 1376): zero rows
            # of gate/up and zero columns of down pad it, so the padded
            # activations are silu(0) * 0 = 0 and add nothing
            pad = -wg.shape[0] % 128
            wg, wu = F.pad(wg, (0, 0, 0, pad)), F.pad(wu, (0, 0, 0, pad))
            wd = F.pad(wd, (0, pad))
            sw = wg.shape[0]
            w_gu = fused.pack_gate_up(wg, wu, eng.expert_gate, eng.expert_up)
            w_down = fused.pack_down(wd, eng.expert_down)
        else:
            sw = wg.shape[0] if wg is not None else 0
            w_gu, w_down = eng.packed_weights()
        return TPMLPFn.apply(h_shard, w_gu, w_down, scales, residual, ws, name, sw,
                             cfg.expert_width, cfg.num_experts, cfg.shared_output_scale)

    def set_top_k_primary_weight(self, weight: float) -> None:
        """Re-blend route slots; unlike the reference, every backend sees the new weights."""
        if self.top_k == 1:
            self._primary_weight = 1.0
            return
        self._primary_weight = min(1.0, max(0.0, float(weight)))
        self.engine.set_route_weights(route_weights_for(self.top_k, self._primary_weight))

    def set_active_experts(self, num_experts: int) -> None:
        self.engine.set_active_capacity(num_experts=num_experts)

    def set_active_expert_width(self, width: int) -> None:
        self.engine.set_active_capacity(expert_width=width)

    def training_control_capabilities(self) -> frozenset:
        return frozenset({"topk_primary_weight", "active_num_experts", "active_expert_width"})

    def training_telemetry(self) -> dict:
        return {"topk_w": float(self._primary_weight),
                "active_num_experts": float(self.engine.active_num_experts),
                "active_expert_width": float(self.engine.active_expert_width)}

    def capability_summary(self, device_type: str = "cpu") -> dict:
        return self.engine.capability_summary(device_type)
