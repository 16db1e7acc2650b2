"""Vision, audio and video encoders.

Counterparts: complexity/multimodal/vision.py:25-520 (patch embedding, ViT
blocks with an optional token-routed MLP, ``VisionEncoder``), audio.py:24-520
(log-mel front end, conv stack, ``AudioEncoder``) and video.py:44-450
(tubelet embedding, spatio-temporal blocks, ``VideoEncoder``).

All encoders are pre-norm transformer stacks; attention uses PyTorch SDPA
(cuDNN flash kernels on B200), and the MLP can be the TR-Hash routed MLP with
routes keyed by patch/frame position, mirroring the text model.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class EncoderConfig:
    hidden_size: int = 768
    num_layers: int = 12
    num_heads: int = 12
    mlp_ratio: float = 4.0
    num_experts: int = 1        # > 1: position-routed experts in every block
    dropout: float = 0.0


class _Attention(nn.Module):
    def __init__(self, H: int, heads: int):
        super().__init__()
        self.h = heads
        self.qkv = nn.Linear(H, 3 * H)
        self.proj = nn.Linear(H, H)

    def forward(self, x, mask=None, causal=False):
        B, N, H = x.shape
        q, k, v = self.qkv(x).view(B, N, 3, self.h, H // self.h).permute(2, 0, 3, 1, 4)
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, is_causal=causal)
        return self.proj(o.transpose(1, 2).reshape(B, N, H))


class _RoutedMLP(nn.Module):
    """Experts chosen by token position (deterministic routing, like TR-Hash by id)."""

    def __init__(self, H: int, hidden: int, experts: int):
        super().__init__()
        self.E = experts
        self.fc1 = nn.Parameter(torch.randn(experts, H, hidden) * 0.02)
        self.fc2 = nn.Parameter(torch.randn(experts, hidden, H) * 0.02)

    def forward(self, x):
        B, N, H = x.shape
        e = torch.arange(N, device=x.device) % self.E
        h = F.gelu(torch.einsum("bnh,nhk->bnk", x, self.fc1[e]))
        return torch.einsum("bnk,nkh->bnh", h, self.fc2[e])


class _Block(nn.Module):
    def __init__(self, cfg: EncoderConfig):
        super().__init__()
        H = cfg.hidden_size
        hid = int(H * cfg.mlp_ratio)
        self.n1, self.n2 = nn.LayerNorm(H), nn.LayerNorm(H)
        self.attn = _Attention(H, cfg.num_heads)
        self.mlp = (_RoutedMLP(H, hid // max(1, cfg.num_experts), cfg.num_experts)
                    if cfg.num_experts > 1 else nn.Sequential(nn.Linear(H, hid), nn.GELU(),
                                                              nn.Linear(hid, H)))

    def forward(self, x, mask=None):
        x = x + self.attn(self.n1(x), mask)
        return x + self.mlp(self.n2(x))


class PatchEmbedding(nn.Module):
    def __init__(self, image_size: int = 224, patch_size: int = 16, channels: int = 3,
                 hidden: int = 768):
        super().__init__()
        self.proj = nn.Conv2d(channels, hidden, patch_size, patch_size)
        self.num_patches = (image_size // patch_size) ** 2
        self.cls = nn.Parameter(torch.zeros(1, 1, hidden))
        self.pos = nn.Parameter(torch.randn(1, self.num_patches + 1, hidden) * 0.02)

    def forward(self, img):
        x = self.proj(img).flatten(2).transpose(1, 2)
        x = torch.cat([self.cls.expand(x.shape[0], -1, -1), x], 1)
        return x + self.pos[:, :x.shape[1]]


class VisionEncoder(nn.Module):
    """ViT: [B, C, H, W] -> [B, 1 + patches, hidden]."""

    def __init__(self, cfg: Optional[EncoderConfig] = None, image_size: int = 224,
                 patch_size: int = 16, channels: int = 3):
        super().__init__()
        self.cfg = cfg or EncoderConfig()
        self.embed = PatchEmbedding(image_size, patch_size, channels, self.cfg.hidden_size)
        self.blocks = nn.ModuleList(_Block(self.cfg) for _ in range(self.cfg.num_layers))
        self.norm = nn.LayerNorm(self.cfg.hidden_size)

    def forward(self, images):
        x = self.embed(images)
        for b in self.blocks:
            x = b(x)
        return self.norm(x)


def log_mel_spectrogram(audio: torch.Tensor, sample_rate: int = 16000, n_fft: int = 400,
                        hop: int = 160, n_mels: int = 80) -> torch.Tensor:
    """[B, samples] -> [B, n_mels, frames] log-mel features (triangular mel filter bank)."""
    win = torch.hann_window(n_fft, device=audio.device)
    spec = torch.stft(audio, n_fft, hop, window=win, return_complex=True).abs() ** 2
    n_freq = spec.shape[1]

    def hz_to_mel(f):
        return 2595.0 * math.log10(1.0 + f / 700.0)

    mels = torch.linspace(hz_to_mel(0.0), hz_to_mel(sample_rate / 2), n_mels + 2)
    hz = 700.0 * (10 ** (mels / 2595.0) - 1.0)
    bins = torch.floor((n_fft + 1) * hz / sample_rate).long().clamp(max=n_freq - 1)
    fb = torch.zeros(n_mels, n_freq)
    for m in range(1, n_mels + 1):
        l, c, r = bins[m - 1], bins[m], bins[m + 1]
        for k in range(l, c):
            fb[m - 1, k] = (k - l) / max(1, c - l)
        for k in range(c, r):
            fb[m - 1, k] = (r - k) / max(1, r - c)
    mel = fb.to(audio.device) @ spec
    return torch.log10(mel.clamp_min(1e-10))


class AudioEncoder(nn.Module):
    """Log-mel -> 2 strided convs -> transformer: [B, samples] -> [B, frames/2, hidden]."""

    def __init__(self, cfg: Optional[EncoderConfig] = None, n_mels: int = 80,
                 max_frames: int = 3000):
        super().__init__()
        self.cfg = cfg or EncoderConfig()
        H = self.cfg.hidden_size
        self.n_mels = n_mels
        self.conv1 = nn.Conv1d(n_mels, H, 3, padding=1)
        self.conv2 = nn.Conv1d(H, H, 3, stride=2, padding=1)
        self.pos = nn.Parameter(torch.randn(1, max_frames // 2 + 1, H) * 0.02)
        self.blocks = nn.ModuleList(_Block(self.cfg) for _ in range(self.cfg.num_layers))
        self.norm = nn.LayerNorm(H)

    def forward(self, audio=None, mel=None):
        if mel is None:
            mel = log_mel_spectrogram(audio, n_mels=self.n_mels)
        x = F.gelu(self.conv2(F.gelu(self.conv1(mel)))).transpose(1, 2)
        x = x + self.pos[:, :x.shape[1]]
        for b in self.blocks:
            x = b(x)
        return self.norm(x)


class VideoEncoder(nn.Module):
    """Tubelet embedding (t x p x p) + space-time transformer: [B, C, T, H, W] -> tokens."""

    def __init__(self, cfg: Optional[EncoderConfig] = None, frames: int = 8, image_size: int = 224,
                 patch_size: int = 16, tubelet: int = 2, channels: int = 3):
        super().__init__()
        self.cfg = cfg or EncoderConfig()
        H = self.cfg.hidden_size
        self.embed = nn.Conv3d(channels, H, (tubelet, patch_size, patch_size),
                               (tubelet, patch_size, patch_size))
        n = (frames // tubelet) * (image_size // patch_size) ** 2
        self.pos = nn.Parameter(torch.randn(1, n, H) * 0.02)
        self.blocks = nn.ModuleList(_Block(self.cfg) for _ in range(self.cfg.num_layers))
        self.norm = nn.LayerNorm(H)

    def forward(self, video):
        x = self.embed(video).flatten(2).transpose(1, 2)
        x = x + self.pos[:, :x.shape[1]]
        for b in self.blocks:
            x = b(x)
        return self.norm(x)
