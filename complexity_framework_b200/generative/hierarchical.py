"""Hierarchical TR-Hash vision tower: real features at strides 4/8/16/32.

Counterpart: complexity/generative/detection/hierarchical_tower.py (and the
``HierarchicalTRHashVisionClassifier`` the reference image classifier builds
on).  Design here: a convolutional stem to stride 4, then stages joined by
2x2 patch merging (concatenate a 2x2 neighbourhood, LayerNorm, linear to the
next width).  High-resolution stages use windowed self-attention (window w,
every other block shifted by w/2 with a mask that keeps attention inside the
original image regions, plus a learned relative-position bias per window
offset); the last stage attends globally.  Every block's feed-forward is the
TR-Hash engine routed by the token's position in its stage grid, so expert
choice is fixed per location as in the plain tower.  Per-stage 2-D position
grids are interpolated to the actual input size.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .towers import _engine, ffn_input


@dataclass
class HierarchicalTowerConfig:
    image_size: int = 256          # reference resolution of the position grids
    num_channels: int = 3
    dims: Tuple[int, ...] = (64, 128, 256, 384)
    depths: Tuple[int, ...] = (1, 1, 2, 1)
    heads: Tuple[int, ...] = (2, 4, 8, 12)
    window_size: int = 8
    global_last_stage: bool = True
    num_experts: int = 4
    top_k: int = 2
    mlp_ratio: float = 2.0         # shared width = ratio * dim; expert width = dim / 4
    route_seed: int = 0x4E5A

    def stage_grid(self, i: int) -> int:
        return self.image_size // (4 * 2 ** i)


def _rel_index(w: int) -> torch.Tensor:
    ys, xs = torch.meshgrid(torch.arange(w), torch.arange(w), indexing="ij")
    c = torch.stack([ys.flatten(), xs.flatten()])            # 2, N
    d = c[:, :, None] - c[:, None, :] + (w - 1)                # 2, N, N in [0, 2w-2]
    return d[0] * (2 * w - 1) + d[1]


class WindowAttention(nn.Module):
    def __init__(self, dim: int, heads: int, window: int):
        super().__init__()
        self.h, self.w = heads, window
        self.qkv = nn.Linear(dim, 3 * dim)
        self.proj = nn.Linear(dim, dim)
        if window > 0:
            self.bias = nn.Parameter(torch.zeros(heads, (2 * window - 1) ** 2))
            self.register_buffer("rel", _rel_index(window), persistent=False)

    def forward(self, x: torch.Tensor, mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x [B', N, C]; mask [nW, N, N] additive (B' = B * nW) or None."""
        Bp, N, C = x.shape
        q, k, v = self.qkv(x).view(Bp, N, 3, self.h, C // self.h).permute(2, 0, 3, 1, 4)
        bias = None
        if self.w > 0 and N == self.w * self.w:
            bias = self.bias[:, self.rel].to(q.dtype)[None]  # 1, h, N, N
            if mask is not None:
                nw = mask.shape[0]
                bias = (bias.view(1, 1, self.h, N, N) + mask[None, :, None].to(q.dtype)).view(
                    nw, self.h, N, N).repeat(Bp // nw, 1, 1, 1)
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=bias)
        return self.proj(o.transpose(1, 2).reshape(Bp, N, C))


class HierarchicalBlock(nn.Module):
    def __init__(self, dim: int, heads: int, window: int, shift: bool, cfg: HierarchicalTowerConfig,
                 route_vocab: int, layer: int):
        super().__init__()
        self.w, self.shift = window, (window // 2 if shift and window > 0 else 0)
        self.n1, self.n2 = nn.LayerNorm(dim), nn.LayerNorm(dim)
        self.attn = WindowAttention(dim, heads, window)
        self.vocab = route_vocab
        self.mlp = _engine(dim, route_vocab, cfg.num_experts, cfg.top_k,
                           max(128, int(cfg.mlp_ratio * dim) // 128 * 128), max(16, dim // 4),
                           layer, cfg.route_seed)

    def _windows(self, x, H, W):
        B, _, C = x.shape
        w, s = self.w, self.shift
        g = x.view(B, H, W, C)
        Hp, Wp = -(-H // w) * w, -(-W // w) * w
        g = F.pad(g, (0, 0, 0, Wp - W, 0, Hp - H))
        mask = None
        padded = Hp != H or Wp != W
        if s or padded:
            # region ids keep shifted windows from mixing image areas that the
            # cyclic roll brought together; padding positions never act as keys
            region = torch.zeros(Hp, Wp, device=x.device)
            valid = torch.zeros(Hp, Wp, device=x.device)
            valid[:H, :W] = 1
            if s:
                cnt = 0
                for hs in (slice(0, Hp - w), slice(Hp - w, Hp - s), slice(Hp - s, Hp)):
                    for ws in (slice(0, Wp - w), slice(Wp - w, Wp - s), slice(Wp - s, Wp)):
                        region[hs, ws] = cnt
                        cnt += 1
                g = torch.roll(g, (-s, -s), (1, 2))
                valid = torch.roll(valid, (-s, -s), (0, 1))
            r = region.view(Hp // w, w, Wp // w, w).permute(0, 2, 1, 3).reshape(-1, w * w)
            v = valid.view(Hp // w, w, Wp // w, w).permute(0, 2, 1, 3).reshape(-1, w * w)
            bad = (r[:, :, None] != r[:, None, :]) | (v[:, None, :] == 0)
            mask = bad.float() * -1e4
        win = g.view(B, Hp // w, w, Wp // w, w, C).permute(0, 1, 3, 2, 4, 5).reshape(-1, w * w, C)
        return win, mask, Hp, Wp

    def _unwindows(self, win, B, H, W, Hp, Wp):
        w, s = self.w, self.shift
        C = win.shape[-1]
        g = win.view(B, Hp // w, Wp // w, w, w, C).permute(0, 1, 3, 2, 4, 5).reshape(B, Hp, Wp, C)
        if s:
            g = torch.roll(g, (s, s), (1, 2))
        return g[:, :H, :W].reshape(B, H * W, C)

    def forward(self, x: torch.Tensor, H: int, W: int) -> torch.Tensor:
        B = x.shape[0]
        h = self.n1(x)
        if self.w > 0:
            win, mask, Hp, Wp = self._windows(h, H, W)
            h = self._unwindows(self.attn(win, mask), B, H, W, Hp, Wp)
        else:
            h = self.attn(h)
        x = x + h
        ids = (torch.arange(H * W, device=x.device) % self.vocab).unsqueeze(0).expand(B, -1)
        return x + self.mlp(ffn_input(self.n2(x)), ids)


class PatchMerging(nn.Module):
    def __init__(self, dim: int, out: int):
        super().__init__()
        self.norm = nn.LayerNorm(4 * dim)
        self.proj = nn.Linear(4 * dim, out, bias=False)

    def forward(self, x, H, W):
        B, _, C = x.shape
        g = x.view(B, H, W, C)
        g = F.pad(g, (0, 0, 0, W % 2, 0, H % 2))
        g = torch.cat([g[:, 0::2, 0::2], g[:, 1::2, 0::2], g[:, 0::2, 1::2], g[:, 1::2, 1::2]], -1)
        H2, W2 = g.shape[1], g.shape[2]
        return self.proj(self.norm(g.reshape(B, H2 * W2, 4 * C))), H2, W2


class HierarchicalTRHashVisionTower(nn.Module):
    """[B, C, H, W] -> list of [B, dim_i, H / (4 * 2^i), W / (4 * 2^i)] stage maps."""

    def __init__(self, config: HierarchicalTowerConfig):
        super().__init__()
        self.config = c = config
        d0 = c.dims[0]
        self.stem = nn.Sequential(nn.Conv2d(c.num_channels, d0 // 2, 3, 2, 1), nn.GELU(),
                                  nn.Conv2d(d0 // 2, d0, 3, 2, 1))
        self.pos = nn.ParameterList()
        self.stages = nn.ModuleList()
        self.merges = nn.ModuleList()
        self.norms = nn.ModuleList()
        layer = 0
        for i, (d, depth, h) in enumerate(zip(c.dims, c.depths, c.heads)):
            g = c.stage_grid(i)
            last = i == len(c.dims) - 1
            win = 0 if (last and c.global_last_stage) else c.window_size
            self.pos.append(nn.Parameter(torch.randn(1, d, g, g) * 0.02))
            blocks = nn.ModuleList()
            for j in range(depth):
                blocks.append(HierarchicalBlock(d, h, win, shift=j % 2 == 1, cfg=c,
                                                route_vocab=g * g, layer=layer))
                layer += 1
            self.stages.append(blocks)
            self.norms.append(nn.LayerNorm(d))
            if not last:
                self.merges.append(PatchMerging(d, c.dims[i + 1]))

    def forward(self, images: torch.Tensor) -> List[torch.Tensor]:
        x = self.stem(images)
        B, C, H, W = x.shape
        outs = []
        x = x.flatten(2).transpose(1, 2)
        for i, blocks in enumerate(self.stages):
            pos = self.pos[i]
            if pos.shape[-2:] != (H, W):
                pos = F.interpolate(pos, size=(H, W), mode="bicubic", align_corners=False)
            x = x + pos.flatten(2).transpose(1, 2).to(x.dtype)
            for blk in blocks:
                x = blk(x, H, W)
            y = self.norms[i](x)
            outs.append(y.transpose(1, 2).reshape(B, -1, H, W))
            if i < len(self.merges):
                x, H, W = self.merges[i](x, H, W)
        return outs


class HierarchicalTRHashVisionClassifier(nn.Module):
    def __init__(self, config: HierarchicalTowerConfig, num_classes: int):
        super().__init__()
        self.tower = HierarchicalTRHashVisionTower(config)
        self.head = nn.Linear(config.dims[-1], num_classes)

    def forward(self, pixel_values, labels=None) -> dict:
        logits = self.head(self.tower(pixel_values)[-1].mean((2, 3)))
        out = {"logits": logits}
        if labels is not None:
            out["loss"] = F.cross_entropy(logits.float(), labels)
        return out
