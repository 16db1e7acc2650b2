"""Layers and registries (attention, MLP, normalisation, position, losses)."""
from .attention import (AttentionConfig, GroupedQueryAttention, MultiHeadAttention,
                        MultiQueryAttention)
from .layers import (DynamicNTKRotaryEmbedding, IdentityNorm, LayerNorm, RMSNorm,
                     RotaryEmbedding, YaRNRotaryEmbedding, apply_rotary_pos_emb, rotate_half)
from .losses import (CausalLMLossMetrics, causal_lm_loss, causal_lm_loss_from_hidden,
                     fused_linear_causal_lm_loss)
from .mlp import MLPConfig, TRHashEngineMLP
from .registry import (ATTENTION_REGISTRY, MLP_REGISTRY, MODEL_REGISTRY, NORMALIZATION_REGISTRY,
                       POSITION_REGISTRY, register_attention, register_mlp, register_model,
                       register_normalization, register_position)
