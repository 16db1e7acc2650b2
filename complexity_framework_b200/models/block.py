"""Pre-norm decoder block: ``x += attn(norm1(x)); x += mlp(norm2(x), token_ids)``.

Module names (``input_layernorm``, ``self_attn``, ``post_attention_layernorm``,
``mlp``) and the per-layer interpolation of the shared/routed output scales
follow complexity/models/block.py:20-280.  On the fused path both residual
adds happen inside GEMM epilogues (o_proj and MLP down projection).
"""
from __future__ import annotations

from typing import Any, Optional, Tuple

import torch
import torch.nn as nn

from ..config.model_config import ModelConfig
from ..core.attention import AttentionConfig
from ..core.mlp import MLPConfig
from ..core.registry import ATTENTION_REGISTRY, MLP_REGISTRY, NORMALIZATION_REGISTRY


def layer_scale(base: float, first: Optional[float], last: Optional[float], layer_idx: int,
                num_layers: int) -> float:
    """Linear interpolation of an output scale from the first to the last layer."""
    if first is None and last is None:
        return float(base)
    start = float(base if first is None else first)
    end = float(start if last is None else last)
    ratio = min(1.0, max(0.0, layer_idx / max(1, num_layers - 1)))
    return start + (end - start) * ratio


class TransformerBlock(nn.Module):
    def __init__(self, config: ModelConfig, layer_idx: int = 0):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.hidden_size = config.hidden_size
        self.input_layernorm = NORMALIZATION_REGISTRY.build(config.norm_type, config.hidden_size,
                                                            eps=config.norm_eps)
        attn_cfg = AttentionConfig(
            hidden_size=config.hidden_size, num_attention_heads=config.num_attention_heads,
            num_key_value_heads=config.num_key_value_heads,
            max_position_embeddings=config.max_position_embeddings,
            rope_theta=config.rope_theta, attention_dropout=config.attention_dropout,
            use_qk_norm=config.use_qk_norm, sliding_window=config.sliding_window,
            use_sdpa=config.use_sdpa, is_causal=config.is_causal, rope_type=config.rope_type,
            rope_fraction=config.rope_fraction, use_mup_attn_scale=config.use_mup_attn_scale,
            layer_idx=layer_idx, vocab_size=config.vocab_size,
            extra={k: getattr(config, k) for k in (
                "tr_mha_num_experts", "tr_mha_adapter_rank", "tr_mha_top_k", "tr_mha_targets",
                "causal_conv_kernel_size", "causal_state_rank", "lexical_object_rank",
                "lexical_gqa_rank", "lexical_gqa_gate_init", "lexical_gqa_use_token_code",
                "lexical_key_gate_init", "causal_stable_delta", "causal_contextual_mix_init",
                "causal_context_gate_init", "causal_delta_chunk_size") if hasattr(config, k)})
        from ..core import attention_variants  # noqa: F401  (registers experimental types)
        attn_type = config.attention_type
        if attn_type not in ATTENTION_REGISTRY:
            raise ValueError(f"attention_type {attn_type!r} is not available; supported: "
                             f"{ATTENTION_REGISTRY.names()}")
        self.self_attn = ATTENTION_REGISTRY.build(attn_type, attn_cfg)
        self.post_attention_layernorm = NORMALIZATION_REGISTRY.build(
            config.norm_type, config.hidden_size, eps=config.norm_eps)
        n = config.num_hidden_layers
        mlp_cfg = MLPConfig(
            hidden_size=config.hidden_size, intermediate_size=config.intermediate_size,
            hidden_act=config.hidden_act, num_experts=config.num_experts,
            expert_initialization=config.expert_initialization,
            initializer_range=config.initializer_range, vocab_size=config.vocab_size,
            routing_strategy=config.routing_strategy, route_hash_count=config.route_hash_count,
            shared_expert=config.shared_expert,
            shared_intermediate_size=config.shared_intermediate_size,
            shared_output_scale=layer_scale(config.shared_output_scale,
                                            config.shared_output_scale_first_layer,
                                            config.shared_output_scale_last_layer, layer_idx, n),
            routed_output_scale=layer_scale(config.routed_output_scale,
                                            config.routed_output_scale_first_layer,
                                            config.routed_output_scale_last_layer, layer_idx, n),
            top_k=config.top_k, top_k_primary_weight=config.top_k_primary_weight,
            layer_idx=layer_idx, use_custom_kernels=config.use_custom_kernels,
            use_cggr=config.use_cggr, active_num_experts=config.active_num_experts,
            active_expert_width=config.active_expert_width, attention_type=attn_type,
            lexical_object_rank=config.lexical_object_rank,
            lexical_object_gate_init=config.lexical_object_gate_init,
            micro_num_experts=config.micro_num_experts,
            micro_expert_width=config.micro_expert_width,
            micro_expert_gate_init=config.micro_expert_gate_init)
        from ..core import dense_mlp, lexical_mlp  # noqa: F401  (registers MLP types)
        self.mlp = MLP_REGISTRY.build(config.mlp_type, mlp_cfg)

    def forward(self, hidden_states: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                past_key_value: Optional[Any] = None, use_cache: bool = False,
                token_ids: Optional[torch.Tensor] = None, **unused
                ) -> Tuple[torch.Tensor, Optional[Any], None]:
        if token_ids is not None and token_ids.is_floating_point():
            # routing ids carried as float between pipeline stages: the integer
            # ids route; a zero-valued term gives the carried ids the (zero)
            # gradient the pipeline runtime sends back to the previous stage
            ids_f = token_ids
            token_ids = ids_f.long()
            hidden_states = hidden_states + (ids_f * 0).unsqueeze(-1).to(hidden_states.dtype)
        h, hidden_states = self._norm_skip(self.input_layernorm, hidden_states)
        if token_ids is not None and hasattr(self.self_attn, "set_token_ids"):
            self.self_attn.set_token_ids(token_ids)
        x, new_kv = self.self_attn(h, attention_mask=attention_mask,
                                   past_key_value=past_key_value, use_cache=use_cache,
                                   residual=hidden_states)
        h, x = self._norm_skip(self.post_attention_layernorm, x)
        x = self.mlp(h, token_ids=token_ids, residual=x)
        return x, new_kv, None

    def forward_sp(self, x_shard: torch.Tensor, token_ids: torch.Tensor, B: int, S: int, ws):
        """Fused sequence-parallel block on a [T/P, H] token shard."""
        name = f"layer{self.layer_idx}"
        h, x = self._norm_skip(self.input_layernorm, x_shard)
        x = self.self_attn.forward_sp(h, x, B, S, ws, name + ".attn")
        h, x = self._norm_skip(self.post_attention_layernorm, x)
        return self.mlp.forward_sp(h, token_ids, x, ws, name + ".mlp")

    @staticmethod
    def _norm_skip(norm, x):
        """Norm output plus the residual stream routed through the norm, so the
        two gradients of ``x`` meet in the norm's backward kernel."""
        if hasattr(norm, "forward_with_skip") and torch.is_grad_enabled() and x.requires_grad:
            return norm.forward_with_skip(x)
        return norm(x), x

    def forward_paged(self, hidden_states: torch.Tensor, cache, token_ids: torch.Tensor):
        h = self.input_layernorm(hidden_states)
        if hasattr(self.self_attn, "set_token_ids"):
            self.self_attn.set_token_ids(token_ids)
        x = self.self_attn.forward_paged(h, cache, self.layer_idx, residual=hidden_states)
        h = self.post_attention_layernorm(x)
        return self.mlp(h, token_ids=token_ids, residual=x)
