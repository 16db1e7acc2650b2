"""Building-block factories: attention, MLP, position, normalisation, blocks,
attention variants and the registries.

Same facade names and call shapes as complexity/api/core/ (``Attention.gqa``,
``MLP.moe``, ``Position.rope``, ``Norm.rms``, ``Block.moe``, ``CUDA.flash``,
``register``); every factory builds this framework's own module (sm_100a
kernels on CUDA bf16).  Attention modules returned by the factories are
called as ``attn(hidden_states) -> hidden_states`` (the KV tuple of the
underlying layer is dropped), like the reference's wrappers.
"""
from __future__ import annotations

from typing import Optional, Type

import torch.nn as nn

from ..config.model_config import ModelConfig
from ..core.attention import AttentionConfig, GroupedQueryAttention
from ..core.layers import (DynamicNTKRotaryEmbedding, IdentityNorm, LayerNorm, RMSNorm,
                           RotaryEmbedding, YaRNRotaryEmbedding, apply_rotary_pos_emb,
                           rotate_half)
from ..core.mlp import MLPConfig
from ..core.positions import ALiBiPositionalBias, LearnedPositionalEmbedding
from ..core.registry import (ATTENTION_REGISTRY, MLP_REGISTRY, MODEL_REGISTRY,
                             NORMALIZATION_REGISTRY, POSITION_REGISTRY, Registry,
                             register_attention, register_mlp, register_model,
                             register_normalization, register_position)
from ..models.block import TransformerBlock
from ..core import attention_variants, dense_mlp, lexical_mlp, positions  # noqa: F401,E402  (register)

_REGISTRIES = {"attention": ATTENTION_REGISTRY, "mlp": MLP_REGISTRY,
               "normalization": NORMALIZATION_REGISTRY, "norm": NORMALIZATION_REGISTRY,
               "position": POSITION_REGISTRY, "model": MODEL_REGISTRY}


def register(component_type: str, name: str):
    """``@register("attention", "my_attn")`` -- decorator into the named registry."""
    key = component_type.lower()
    if key not in _REGISTRIES:
        raise ValueError(f"unknown component type {component_type!r}; "
                         f"one of {sorted(set(_REGISTRIES))}")
    return _REGISTRIES[key].register(name)


class _OutputOnly(nn.Module):
    """``attn(x) -> out`` view of an attention layer that returns ``(out, kv)``."""

    def __init__(self, inner: nn.Module):
        super().__init__()
        self.inner = inner

    def forward(self, *args, **kwargs):
        out = self.inner(*args, **kwargs)
        return out[0] if isinstance(out, tuple) else out


class Attention:
    """``Attention.create("gqa", hidden_size=..., num_heads=..., kv_heads=...)``."""

    @classmethod
    def _config(cls, hidden_size: int = 768, num_heads: int = 12, kv_heads: Optional[int] = None,
                **kw) -> AttentionConfig:
        known = set(AttentionConfig.__dataclass_fields__)
        extra = {k: v for k, v in kw.items() if k not in known}
        cfg = {k: v for k, v in kw.items() if k in known}
        return AttentionConfig(hidden_size=hidden_size, num_attention_heads=num_heads,
                               num_key_value_heads=kv_heads, extra=extra, **cfg)

    @classmethod
    def create(cls, attention_type: str = "gqa", **kwargs) -> nn.Module:
        return _OutputOnly(ATTENTION_REGISTRY.build(attention_type, cls._config(**kwargs)))

    @classmethod
    def gqa(cls, hidden_size: int, num_heads: int, kv_heads: Optional[int] = None,
            **kwargs) -> nn.Module:
        return cls.create("gqa", hidden_size=hidden_size, num_heads=num_heads,
                          kv_heads=kv_heads or max(1, num_heads // 4), **kwargs)

    @classmethod
    def mha(cls, hidden_size: int, num_heads: int, **kwargs) -> nn.Module:
        return cls.create("mha", hidden_size=hidden_size, num_heads=num_heads,
                          kv_heads=num_heads, **kwargs)

    @classmethod
    def mqa(cls, hidden_size: int, num_heads: int, **kwargs) -> nn.Module:
        return cls.create("mqa", hidden_size=hidden_size, num_heads=num_heads, kv_heads=1,
                          **kwargs)

    @classmethod
    def register(cls, name: str, attention_cls: Type) -> Type:
        return ATTENTION_REGISTRY.register(name)(attention_cls)

    @staticmethod
    def available():
        return ATTENTION_REGISTRY.names()


class MLP:
    """``MLP.create("moe", hidden_size=..., num_experts=...)``; "moe" is the TR-Hash
    engine (deterministic token-id routes, shared SwiGLU + routed experts)."""

    _ALIASES = {"moe": "tr_hash_engine", "token_routed": "tr_hash_engine",
                "swiglu": "dense", "mlp": "dense"}

    @classmethod
    def create(cls, mlp_type: str = "moe", **kwargs) -> nn.Module:
        name = cls._ALIASES.get(mlp_type, mlp_type)
        known = set(MLPConfig.__dataclass_fields__)
        cfg = MLPConfig(**{k: v for k, v in kwargs.items() if k in known},
                        extra={k: v for k, v in kwargs.items() if k not in known})
        return MLP_REGISTRY.build(name, cfg)

    @classmethod
    def moe(cls, hidden_size: int, num_experts: int = 8, **kwargs) -> nn.Module:
        kwargs.setdefault("intermediate_size", 4 * hidden_size)
        kwargs.setdefault("top_k", 2 if num_experts >= 2 else 1)
        kwargs.setdefault("shared_expert", True)
        return cls.create("moe", hidden_size=hidden_size, num_experts=num_experts, **kwargs)

    @classmethod
    def register(cls, name: str, mlp_cls: Type) -> Type:
        return MLP_REGISTRY.register(name)(mlp_cls)

    @staticmethod
    def available():
        return MLP_REGISTRY.names()


class Position:
    @classmethod
    def create(cls, pos_type: str = "rope", **kwargs) -> nn.Module:
        return getattr(cls, {"rope": "rope", "standard": "rope", "yarn": "yarn",
                             "dynamic_ntk": "ntk", "ntk": "ntk", "alibi": "alibi",
                             "learned": "learned"}[pos_type])(**kwargs)

    @classmethod
    def rope(cls, dim: int, max_seq_len: int = 8192, base: float = 10000.0,
             **kwargs) -> nn.Module:
        return RotaryEmbedding(dim, max_seq_len=max_seq_len, theta=base)

    @classmethod
    def yarn(cls, dim: int, max_seq_len: int = 8192, scale: float = 4.0, **kwargs) -> nn.Module:
        return YaRNRotaryEmbedding(dim, max_seq_len=max_seq_len, scale=scale,
                                   **{k: v for k, v in kwargs.items()
                                      if k in ("theta", "original_max_position", "beta_fast",
                                               "beta_slow")})

    @classmethod
    def ntk(cls, dim: int, max_seq_len: int = 8192, **kwargs) -> nn.Module:
        return DynamicNTKRotaryEmbedding(dim, max_seq_len=max_seq_len,
                                         **{k: v for k, v in kwargs.items() if k in ("theta",)})

    @classmethod
    def alibi(cls, num_heads: int, **kwargs) -> nn.Module:
        return ALiBiPositionalBias(0, num_heads=num_heads)

    @classmethod
    def learned(cls, max_seq_len: int, hidden_size: int, **kwargs) -> nn.Module:
        return LearnedPositionalEmbedding(max_seq_len, hidden_size)


class Norm:
    @classmethod
    def create(cls, norm_type: str = "rmsnorm", hidden_size: Optional[int] = None,
               **kwargs) -> nn.Module:
        if hidden_size is None:
            raise ValueError("hidden_size is required")
        return NORMALIZATION_REGISTRY.build(norm_type, hidden_size, **kwargs)

    @classmethod
    def rms(cls, hidden_size: int, eps: float = 1e-6, **kwargs) -> nn.Module:
        return RMSNorm(hidden_size, eps=eps)

    @classmethod
    def layer(cls, hidden_size: int, eps: float = 1e-5, **kwargs) -> nn.Module:
        return LayerNorm(hidden_size, eps=eps)


class Block:
    """One decoder block (attention + TR-Hash FFN) from ``ModelConfig`` fields."""

    @classmethod
    def create(cls, layer_idx: int = 0, **kwargs) -> nn.Module:
        return TransformerBlock(ModelConfig(**kwargs), layer_idx)

    @classmethod
    def moe(cls, hidden_size: int, num_heads: int, num_experts: int = 8, top_k: int = 2,
            **kwargs) -> nn.Module:
        kwargs.setdefault("num_key_value_heads", max(1, num_heads // 4))
        kwargs.setdefault("intermediate_size", 4 * hidden_size)
        return cls.create(hidden_size=hidden_size, num_attention_heads=num_heads,
                          num_experts=num_experts, top_k=top_k, **kwargs)


class CUDA:
    """Attention variants by name (``flash``, ``sliding_window``, ``sparse``,
    ``linear``, ``multiscale``); CUDA bf16 runs them on this framework's
    sm_100a kernels where the variant has one."""

    @classmethod
    def create(cls, attention_type: str = "flash", hidden_size: int = 768, num_heads: int = 12,
               kv_heads: Optional[int] = None, **kwargs) -> nn.Module:
        return Attention.create(attention_type, hidden_size=hidden_size, num_heads=num_heads,
                                kv_heads=kv_heads, **kwargs)

    @classmethod
    def flash(cls, hidden_size: int = 768, num_heads: int = 12, **kwargs) -> nn.Module:
        return cls.create("flash", hidden_size, num_heads, **kwargs)

    @classmethod
    def sliding_window(cls, hidden_size: int = 768, num_heads: int = 12, window_size: int = 4096,
                       **kwargs) -> nn.Module:
        return cls.create("sliding_window", hidden_size, num_heads, sliding_window=window_size,
                          **kwargs)

    local = sliding = sliding_window

    @classmethod
    def sparse(cls, hidden_size: int = 768, num_heads: int = 12, **kwargs) -> nn.Module:
        return cls.create("sparse", hidden_size, num_heads, **kwargs)

    @classmethod
    def linear(cls, hidden_size: int = 768, num_heads: int = 12, **kwargs) -> nn.Module:
        return cls.create("linear", hidden_size, num_heads, **kwargs)

    @classmethod
    def multiscale(cls, hidden_size: int = 768, num_heads: int = 12, **kwargs) -> nn.Module:
        return cls.create("multiscale", hidden_size, num_heads, **kwargs)

    @staticmethod
    def kernels_available() -> bool:
        """Whether the sm_100a extension is built and loadable here."""
        from ..ops import available

        return available()


__all__ = ["ATTENTION_REGISTRY", "MLP_REGISTRY", "MODEL_REGISTRY", "NORMALIZATION_REGISTRY",
           "POSITION_REGISTRY", "Registry", "register", "register_attention", "register_mlp",
           "register_model", "register_normalization", "register_position", "Attention", "MLP",
           "Position", "Norm", "Block", "CUDA", "GroupedQueryAttention", "RMSNorm", "LayerNorm",
           "IdentityNorm", "RotaryEmbedding", "YaRNRotaryEmbedding",
           "DynamicNTKRotaryEmbedding", "ALiBiPositionalBias", "LearnedPositionalEmbedding",
           "rotate_half", "apply_rotary_pos_emb", "AttentionConfig", "MLPConfig",
           "TransformerBlock"]
