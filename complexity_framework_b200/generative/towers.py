"""TR-Hash vision and video towers: transformer encoders whose feed-forward is
the deterministic token-routed MoE engine, with patches (and frame x patch
positions) as the routing "tokens".

Counterparts: complexity/generative/vision_language/vision_tower.py
(``TRHashVisionTowerConfig``, ``TRHashVisionBlock``, ``TRHashVisionTower``,
``TRHashVisionClassifier``) and complexity/generative/video/tower.py
(``TRHashVideoTowerConfig``, ``TRHashVideoBlock``, ``TRHashVideoTower``,
``TRHashVideoClassifier``).  Route ids are patch positions (video: frame-major
position of each tubelet), so expert assignment is fixed per location, as the
text model fixes it per token id.  The feed-forward runs through
``TRHashEngine``, i.e. the fused sm_100a SwiGLU GEMMs on CUDA bf16 inputs.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..tr_hash.config import TRHashEngineConfig
from ..tr_hash.engine import TRHashEngine


@dataclass
class TRHashVisionTowerConfig:
    image_size: int = 224
    patch_size: int = 16
    num_channels: int = 3
    hidden_size: int = 384
    num_layers: int = 6
    num_heads: int = 6
    num_experts: int = 4
    top_k: int = 2
    shared_width: int = 768
    expert_width: int = 128
    dropout: float = 0.0
    route_seed: int = 0x71D5A17
    use_cls_token: bool = True

    def __post_init__(self):
        if self.image_size % self.patch_size:
            raise ValueError("image_size must be a multiple of patch_size")
        if self.hidden_size % self.num_heads:
            raise ValueError("hidden_size must be divisible by num_heads")

    @property
    def grid(self) -> int:
        return self.image_size // self.patch_size

    @property
    def num_patches(self) -> int:
        return self.grid * self.grid

    @property
    def route_vocab_size(self) -> int:
        # one route id per patch position, plus one for the class token
        return self.num_patches + 1


def _engine(hidden: int, vocab: int, experts: int, top_k: int, shared: int, width: int,
            layer: int, seed: int) -> TRHashEngine:
    return TRHashEngine(TRHashEngineConfig(
        hidden_size=hidden, vocab_size=vocab, num_experts=experts, top_k=top_k,
        shared_width=shared, expert_width=width, layer_index=layer, route_seed=seed))


def ffn_input(h: torch.Tensor) -> torch.Tensor:
    """Under CUDA bf16 autocast, LayerNorm returns fp32; the TR-Hash engine runs
    its fused sm_100a GEMMs only on bf16 inputs, so cast to the autocast dtype."""
    if h.is_cuda and torch.is_autocast_enabled("cuda") and h.dtype == torch.float32:
        return h.to(torch.get_autocast_dtype("cuda"))
    return h


class SelfAttention(nn.Module):
    """Bidirectional multi-head attention on PyTorch SDPA (cuDNN flash on B200)."""

    def __init__(self, hidden: int, heads: int, dropout: float = 0.0):
        super().__init__()
        self.heads = heads
        self.qkv = nn.Linear(hidden, 3 * hidden)
        self.proj = nn.Linear(hidden, hidden)
        self.dropout = dropout

    def forward(self, x: torch.Tensor, mask: Optional[torch.Tensor] = None,
                causal: bool = False) -> torch.Tensor:
        B, N, H = x.shape
        q, k, v = self.qkv(x).view(B, N, 3, self.heads, H // self.heads).permute(2, 0, 3, 1, 4)
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, is_causal=causal,
                                           dropout_p=self.dropout if self.training else 0.0)
        return self.proj(o.transpose(1, 2).reshape(B, N, H))


class TRHashVisionBlock(nn.Module):
    """Pre-norm block: attention, then the TR-Hash routed FFN keyed on route ids."""

    def __init__(self, config, layer_index: int, route_vocab: Optional[int] = None):
        super().__init__()
        H = config.hidden_size
        self.norm1 = nn.LayerNorm(H)
        self.norm2 = nn.LayerNorm(H)
        self.attn = SelfAttention(H, config.num_heads, config.dropout)
        self.mlp = _engine(H, route_vocab or config.route_vocab_size, config.num_experts,
                           config.top_k, config.shared_width, config.expert_width, layer_index,
                           config.route_seed)

    def forward(self, x: torch.Tensor, route_ids: torch.Tensor,
                mask: Optional[torch.Tensor] = None, causal: bool = False) -> torch.Tensor:
        x = x + self.attn(self.norm1(x), mask, causal)
        return x + self.mlp(ffn_input(self.norm2(x)), route_ids)


class TRHashVisionTower(nn.Module):
    """[B, C, H, W] images -> [B, (1 +) patches, hidden] contextual patch embeddings."""

    def __init__(self, config: TRHashVisionTowerConfig):
        super().__init__()
        self.config = config
        H = config.hidden_size
        self.patch = nn.Conv2d(config.num_channels, H, config.patch_size, config.patch_size)
        n = config.num_patches + (1 if config.use_cls_token else 0)
        self.cls = nn.Parameter(torch.zeros(1, 1, H)) if config.use_cls_token else None
        self.pos = nn.Parameter(torch.randn(1, n, H) * 0.02)
        self.blocks = nn.ModuleList(TRHashVisionBlock(config, i) for i in range(config.num_layers))
        self.norm = nn.LayerNorm(H)
        # route id of each position: patches 0..P-1, the class token P
        ids = torch.arange(config.num_patches)
        if config.use_cls_token:
            ids = torch.cat([torch.tensor([config.num_patches]), ids])
        self.register_buffer("route_ids", ids, persistent=True)

    def patch_grid(self) -> int:
        return self.config.grid

    def forward(self, pixel_values: torch.Tensor) -> torch.Tensor:
        x = self.patch(pixel_values).flatten(2).transpose(1, 2)
        if self.cls is not None:
            x = torch.cat([self.cls.expand(x.shape[0], -1, -1).to(x.dtype), x], 1)
        x = x + self.pos.to(x.dtype)
        ids = self.route_ids.unsqueeze(0).expand(x.shape[0], -1)
        for block in self.blocks:
            x = block(x, ids)
        return self.norm(x)

    def patch_features(self, pixel_values: torch.Tensor) -> torch.Tensor:
        """[B, hidden, grid, grid] feature map (class token dropped)."""
        x = self.forward(pixel_values)
        if self.cls is not None:
            x = x[:, 1:]
        g = self.config.grid
        return x.transpose(1, 2).reshape(x.shape[0], -1, g, g)


class TRHashVisionClassifier(nn.Module):
    """Image classification head on the tower (class token, or mean of patches)."""

    def __init__(self, config: TRHashVisionTowerConfig, num_classes: int):
        super().__init__()
        self.tower = TRHashVisionTower(config)
        self.head = nn.Linear(config.hidden_size, num_classes)

    def forward(self, pixel_values: torch.Tensor, labels: Optional[torch.Tensor] = None) -> dict:
        x = self.tower(pixel_values)
        pooled = x[:, 0] if self.tower.cls is not None else x.mean(1)
        logits = self.head(pooled)
        out = {"logits": logits}
        if labels is not None:
            out["loss"] = F.cross_entropy(logits.float(), labels)
        return out


# ----------------------------------------------------------------- video
@dataclass
class TRHashVideoTowerConfig:
    image_size: int = 112
    patch_size: int = 16
    num_frames: int = 8
    tubelet_size: int = 2
    num_channels: int = 3
    hidden_size: int = 384
    num_layers: int = 6
    num_heads: int = 6
    num_experts: int = 4
    top_k: int = 2
    shared_width: int = 768
    expert_width: int = 128
    dropout: float = 0.0
    route_seed: int = 0x7D1E0
    divided_attention: bool = True  # time attention then space attention per block

    def __post_init__(self):
        if self.image_size % self.patch_size or self.num_frames % self.tubelet_size:
            raise ValueError("image_size / num_frames must divide by patch / tubelet size")

    @property
    def grid(self) -> int:
        return self.image_size // self.patch_size

    @property
    def time_steps(self) -> int:
        return self.num_frames // self.tubelet_size

    @property
    def num_tokens(self) -> int:
        return self.time_steps * self.grid * self.grid

    @property
    def route_vocab_size(self) -> int:
        return self.num_tokens


class TRHashVideoBlock(nn.Module):
    """Divided space-time block: attention over time per patch, then over space per
    time step, then the routed FFN (route id = frame-major tubelet position)."""

    def __init__(self, config: TRHashVideoTowerConfig, layer_index: int):
        super().__init__()
        H = config.hidden_size
        self.cfg = config
        self.norm_t = nn.LayerNorm(H) if config.divided_attention else None
        self.attn_t = SelfAttention(H, config.num_heads) if config.divided_attention else None
        self.norm_s = nn.LayerNorm(H)
        self.attn_s = SelfAttention(H, config.num_heads)
        self.norm_m = nn.LayerNorm(H)
        self.mlp = _engine(H, config.route_vocab_size, config.num_experts, config.top_k,
                           config.shared_width, config.expert_width, layer_index,
                           config.route_seed)

    def forward(self, x: torch.Tensor, route_ids: torch.Tensor) -> torch.Tensor:
        B, N, H = x.shape
        T, P = self.cfg.time_steps, self.cfg.grid ** 2
        if self.attn_t is not None:
            xt = x.view(B, T, P, H).transpose(1, 2).reshape(B * P, T, H)
            xt = xt + self.attn_t(self.norm_t(xt))
            x = xt.view(B, P, T, H).transpose(1, 2).reshape(B, N, H)
            xs = x.view(B * T, P, H)
            x = (xs + self.attn_s(self.norm_s(xs))).view(B, N, H)
        else:
            x = x + self.attn_s(self.norm_s(x))
        return x + self.mlp(ffn_input(self.norm_m(x)), route_ids)


class TRHashVideoTower(nn.Module):
    """[B, C, T, H, W] clips -> [B, T/tubelet * grid^2, hidden]."""

    def __init__(self, config: TRHashVideoTowerConfig):
        super().__init__()
        self.config = config
        H = config.hidden_size
        k = (config.tubelet_size, config.patch_size, config.patch_size)
        self.embed = nn.Conv3d(config.num_channels, H, k, k)
        self.pos = nn.Parameter(torch.randn(1, config.num_tokens, H) * 0.02)
        self.blocks = nn.ModuleList(TRHashVideoBlock(config, i) for i in range(config.num_layers))
        self.norm = nn.LayerNorm(H)
        self.register_buffer("route_ids", torch.arange(config.num_tokens), persistent=True)

    def forward(self, video: torch.Tensor) -> torch.Tensor:
        x = self.embed(video).flatten(2).transpose(1, 2) + self.pos.to(video.dtype)
        ids = self.route_ids.unsqueeze(0).expand(x.shape[0], -1)
        for block in self.blocks:
            x = block(x, ids)
        return self.norm(x)


class TRHashVideoClassifier(nn.Module):
    def __init__(self, config: TRHashVideoTowerConfig, num_classes: int):
        super().__init__()
        self.tower = TRHashVideoTower(config)
        self.head = nn.Linear(config.hidden_size, num_classes)

    def forward(self, video: torch.Tensor, labels: Optional[torch.Tensor] = None) -> dict:
        logits = self.head(self.tower(video).mean(1))
        out = {"logits": logits}
        if labels is not None:
            out["loss"] = F.cross_entropy(logits.float(), labels)
        return out
