"""Bidirectional sentence-embedding model on the TR-Hash backbone.

Counterpart of complexity/models/embedding.py:1-85: a ``ComplexityModel``
built with ``is_causal=False`` runs as an encoder; a sentence embedding is
the mean of the last hidden states over real (non-padding) tokens,
L2-normalised.  Pooling has no parameters, so checkpoints are the backbone's
(``save_pretrained`` / ``from_pretrained`` delegate to it).  Registered as
model type ``bidirectional_encoder``.
"""
from __future__ import annotations

from pathlib import Path
from typing import Optional, Union

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..config import ModelConfig
from ..core.registry import register_model
from .builder import ComplexityModel


def padding_bias(padding_mask: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """[B, S] (1 real, 0 pad) -> additive [B, 1, 1, S] key bias: 0 for real keys,
    the dtype's most negative finite value for padding (finite, so a fully
    padded row cannot turn into NaN through -inf * 0)."""
    return (1.0 - padding_mask[:, None, None, :].to(dtype)) * torch.finfo(dtype).min


def masked_mean(hidden: torch.Tensor, padding_mask: torch.Tensor) -> torch.Tensor:
    """Mean of ``hidden`` [B, S, H] over the positions where ``padding_mask`` is 1."""
    m = padding_mask.to(hidden.dtype)[..., None]
    return (hidden * m).sum(1) / m.sum(1).clamp_min(1e-9)


# reference names of the two helpers
build_extended_attention_mask = padding_bias
mean_pool = masked_mean


@register_model("bidirectional_encoder")
class BidirectionalEmbeddingModel(nn.Module):
    """``forward(input_ids, attention_mask)`` -> L2-normalised [B, hidden] embeddings."""

    def __init__(self, config: ModelConfig, backbone: Optional[ComplexityModel] = None):
        super().__init__()
        if getattr(config, "is_causal", True):
            raise ValueError("BidirectionalEmbeddingModel requires config.is_causal=False: a "
                             "causal backbone would hide every later token from each position")
        self.config = config
        self.backbone = backbone if backbone is not None else ComplexityModel(config)

    def forward(self, input_ids: torch.Tensor, attention_mask: torch.Tensor) -> torch.Tensor:
        bias = padding_bias(attention_mask, self.backbone.embed_tokens.weight.dtype)
        out = self.backbone(input_ids, attention_mask=bias, return_logits=False)
        return F.normalize(masked_mean(out["last_hidden_state"], attention_mask), p=2, dim=-1)

    def num_parameters(self, trainable_only: bool = True) -> int:
        return self.backbone.num_parameters(trainable_only=trainable_only)

    def save_pretrained(self, save_directory: Union[str, Path], safe_serialization: bool = True):
        return self.backbone.save_pretrained(save_directory, safe_serialization=safe_serialization)

    @classmethod
    def from_pretrained(cls, path: Union[str, Path], **kwargs) -> "BidirectionalEmbeddingModel":
        backbone = ComplexityModel.from_pretrained(path, **kwargs)
        return cls(backbone.config, backbone=backbone)
