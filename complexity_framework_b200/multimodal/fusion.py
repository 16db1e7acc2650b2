"""Modality fusion and a vision-language model on top of ``ComplexityModel``.

Counterpart of complexity/multimodal/fusion.py:24-560 (cross-attention,
gated fusion, concat projection, Perceiver resampler,
``VisionLanguageConnector``).  ``VisionLanguageModel`` projects encoder tokens
into the decoder's embedding space and prepends them to the text embeddings
(``inputs_embeds``), so the decoder (and its fused kernels) is unchanged;
image positions are excluded from the language-model loss.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F


class VisionLanguageConnector(nn.Module):
    """Two-layer MLP projector from encoder width to decoder width."""

    def __init__(self, in_dim: int, out_dim: int):
        super().__init__()
        self.net = nn.Sequential(nn.Linear(in_dim, out_dim), nn.GELU(), nn.Linear(out_dim, out_dim))

    def forward(self, x):
        return self.net(x)


class PerceiverResampler(nn.Module):
    """Fixed number of learned latents attend to a variable number of inputs."""

    def __init__(self, dim: int, num_latents: int = 64, heads: int = 8, layers: int = 2):
        super().__init__()
        self.latents = nn.Parameter(torch.randn(num_latents, dim) * 0.02)
        self.attn = nn.ModuleList(nn.MultiheadAttention(dim, heads, batch_first=True)
                                  for _ in range(layers))
        self.ff = nn.ModuleList(nn.Sequential(nn.LayerNorm(dim), nn.Linear(dim, 4 * dim),
                                              nn.GELU(), nn.Linear(4 * dim, dim))
                                for _ in range(layers))

    def forward(self, x):
        lat = self.latents[None].expand(x.shape[0], -1, -1)
        for a, f in zip(self.attn, self.ff):
            kv = torch.cat([x, lat], 1)
            lat = lat + a(lat, kv, kv, need_weights=False)[0]
            lat = lat + f(lat)
        return lat


class CrossAttentionFusion(nn.Module):
    """Text tokens attend to modality tokens (gated residual, tanh gate starts at 0)."""

    def __init__(self, dim: int, heads: int = 8):
        super().__init__()
        self.norm = nn.LayerNorm(dim)
        self.attn = nn.MultiheadAttention(dim, heads, batch_first=True)
        self.gate = nn.Parameter(torch.zeros(1))

    def forward(self, text, other):
        return text + torch.tanh(self.gate) * self.attn(self.norm(text), other, other,
                                                         need_weights=False)[0]


class GatedFusion(nn.Module):
    def __init__(self, dim: int):
        super().__init__()
        self.gate = nn.Linear(2 * dim, dim)

    def forward(self, a, b):
        g = torch.sigmoid(self.gate(torch.cat([a, b], -1)))
        return g * a + (1 - g) * b


class ConcatProjection(nn.Module):
    def __init__(self, dims, out_dim: int):
        super().__init__()
        self.proj = nn.Linear(sum(dims), out_dim)

    def forward(self, *xs):
        return self.proj(torch.cat(xs, -1))


class VisionLanguageModel(nn.Module):
    def __init__(self, language_model, vision_encoder, resampler_latents: Optional[int] = 64):
        super().__init__()
        self.lm = language_model
        self.vision = vision_encoder
        vd = vision_encoder.cfg.hidden_size
        ld = language_model.config.hidden_size
        self.resampler = PerceiverResampler(vd, resampler_latents) if resampler_latents else None
        self.connector = VisionLanguageConnector(vd, ld)

    def image_tokens(self, images):
        v = self.vision(images)
        if self.resampler is not None:
            v = self.resampler(v)
        return self.connector(v)

    def forward(self, input_ids, images):
        img = self.image_tokens(images)
        txt = self.lm.embed_tokens(input_ids)
        emb = torch.cat([img.to(txt.dtype), txt], 1)
        n_img = img.shape[1]
        routing = torch.cat([torch.zeros(input_ids.shape[0], n_img, dtype=input_ids.dtype,
                                         device=input_ids.device), input_ids], 1)
        out = self.lm(inputs_embeds=emb, routing_ids=routing)
        out["num_image_tokens"] = n_img
        return out

    def loss(self, input_ids, images):
        out = self.forward(input_ids, images)
        n = out["num_image_tokens"]
        logits = out["logits"][:, n:-1].float()
        return F.cross_entropy(logits.reshape(-1, logits.shape[-1]), input_ids[:, 1:].reshape(-1))
