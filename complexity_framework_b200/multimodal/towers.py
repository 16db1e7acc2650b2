"""Vision, audio and video encoder towers and multimodal fusion modules.

Counterparts of complexity/multimodal/vision.py:25-538 (``VisionConfig``,
``PatchEmbedding``, ``VisionTransformer`` with class token and learned
positions, ``VisionEncoder``, ``CLIPVisionEncoder``, ``SigLIPEncoder`` with
its sigmoid loss), audio.py:24-558 (``AudioConfig``, ``AudioConvStack``,
``MelSpectrogramEncoder``, ``WhisperEncoder`` with sinusoidal positions,
``AudioEncoder``, ``AudioPreprocessor``), video.py:44-456 (``VideoConfig``,
``TubeletEmbedding``, factorised ``SpatioTemporalBlock``, ``VideoTransformer``,
``VideoEncoder``) and fusion.py:24-575 (``FusionConfig``, cross-attention
blocks, ``CrossAttentionFusion``, ``GatedFusion``, ``ConcatProjection``,
``PerceiverResampler``, ``MultimodalFusion``, ``VisionLanguageConnector``).
Constructor arguments, output dictionaries and parameter names are kept, so
state dicts load in both directions.

Differences in how the work is done:
  * attention runs through ``F.scaled_dot_product_attention`` (flash kernels
    on GPU) with the same additive-mask convention;
  * the position-routed MLP (expert = position mod E, plus a shared SwiGLU)
    computes every expert's gate|up for a token with ONE matmul against the
    stacked expert weights and selects the token's expert, then runs the down
    projection as one matmul over a one-hot expanded activation -- the cost
    of a dense MLP of the total routed width, no per-token weight gather
    ([B*N, H, 2I] copies) and no host synchronisation.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F


# =================================================================== shared
class PositionRoutedMLP(nn.Module):
    """Shared SwiGLU plus one routed SwiGLU expert per token, chosen by position.

    ``gate_up_proj`` [E, H, 2I] (gate columns first, then up), ``down_proj``
    [E, I, H]; ``expert_ids`` [N] gives each position's expert (default:
    position mod E).
    """

    def __init__(self, hidden_size: int, expert_intermediate: int, shared_intermediate: int,
                 num_experts: int, what: str = "routed"):
        super().__init__()
        if shared_intermediate <= expert_intermediate:
            raise ValueError(f"{what} shared MLP must be wider than each routed expert")
        self.hidden_size, self.num_experts = hidden_size, num_experts
        self.expert_intermediate_size = expert_intermediate
        self.shared_intermediate_size = shared_intermediate
        self.shared_gate_up_proj = nn.Linear(hidden_size, 2 * shared_intermediate, bias=False)
        self.shared_down_proj = nn.Linear(shared_intermediate, hidden_size, bias=False)
        self.gate_up_proj = nn.Parameter(
            torch.randn(num_experts, hidden_size, 2 * expert_intermediate) * 0.02)
        self.down_proj = nn.Parameter(
            torch.randn(num_experts, expert_intermediate, hidden_size) * 0.02)

    def forward(self, x: torch.Tensor, expert_ids: Optional[torch.Tensor] = None) -> torch.Tensor:
        B, N, H = x.shape
        E, I = self.num_experts, self.expert_intermediate_size
        if expert_ids is None:
            expert_ids = torch.arange(N, device=x.device) % E
        g, u = self.shared_gate_up_proj(x).chunk(2, -1)
        shared = self.shared_down_proj(F.silu(g) * u)
        w_gu = self.gate_up_proj.permute(1, 0, 2).reshape(H, E * 2 * I)
        gu_all = (x @ w_gu).view(B, N, E, 2 * I)
        sel = expert_ids.view(1, N, 1, 1).expand(B, N, 1, 2 * I)
        gu = gu_all.gather(2, sel).squeeze(2)
        inter = F.silu(gu[..., :I]) * gu[..., I:]
        onehot = F.one_hot(expert_ids, E).to(inter.dtype)                   # [N, E]
        spread = (inter[:, :, None, :] * onehot[None, :, :, None]).reshape(B, N, E * I)
        return shared + spread @ self.down_proj.reshape(E * I, H)


def _attend(q, k, v, heads: int, mask: Optional[torch.Tensor], dropout: float, training: bool):
    B, Nq, H = q.shape
    Nk = k.shape[1]
    d = H // heads
    q = q.view(B, Nq, heads, d).transpose(1, 2)
    k = k.view(B, Nk, heads, d).transpose(1, 2)
    v = v.view(B, Nk, heads, d).transpose(1, 2)
    o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask,
                                       dropout_p=dropout if training else 0.0)
    return o.transpose(1, 2).reshape(B, Nq, H)


class _FusedQKVAttention(nn.Module):
    """Self-attention with one ``qkv`` projection and an output ``proj``."""

    def __init__(self, hidden_size: int, heads: int, dropout: float = 0.0):
        super().__init__()
        self.num_heads, self.head_dim = heads, hidden_size // heads
        self.scale = self.head_dim ** -0.5
        self.qkv = nn.Linear(hidden_size, 3 * hidden_size)
        self.proj = nn.Linear(hidden_size, hidden_size)
        self.p = dropout

    def forward(self, x: torch.Tensor, attention_mask: Optional[torch.Tensor] = None):
        q, k, v = self.qkv(x).chunk(3, -1)
        return self.proj(_attend(q, k, v, self.num_heads, attention_mask, self.p, self.training))


class _SplitQKVAttention(nn.Module):
    """Attention with separate q/k/v/out projections (self- or cross-attention)."""

    def __init__(self, hidden_size: int, heads: int, dropout: float = 0.0):
        super().__init__()
        self.num_heads, self.head_dim = heads, hidden_size // heads
        self.scale = self.head_dim ** -0.5
        self.q_proj = nn.Linear(hidden_size, hidden_size)
        self.k_proj = nn.Linear(hidden_size, hidden_size)
        self.v_proj = nn.Linear(hidden_size, hidden_size)
        self.out_proj = nn.Linear(hidden_size, hidden_size)
        self.p = dropout

    def forward(self, x: torch.Tensor, kv: Optional[torch.Tensor] = None,
                attention_mask: Optional[torch.Tensor] = None):
        if kv is not None and not torch.is_tensor(kv):
            raise TypeError("key/value source must be a tensor")
        src = x if kv is None else kv
        o = _attend(self.q_proj(x), self.k_proj(src), self.v_proj(src), self.num_heads,
                    attention_mask, self.p, self.training)
        return self.out_proj(o)


class _GeluMLP(nn.Module):
    def __init__(self, hidden_size: int, intermediate: int, dropout: float = 0.0):
        super().__init__()
        self.fc1 = nn.Linear(hidden_size, intermediate)
        self.act = nn.GELU()
        self.fc2 = nn.Linear(intermediate, hidden_size)
        self.dropout = nn.Dropout(dropout)

    def forward(self, x, _expert_ids=None):
        return self.dropout(self.fc2(self.dropout(self.act(self.fc1(x)))))


def _routed_or_dense(cfg, intermediate: int, dropout: float, what: str) -> nn.Module:
    if cfg.num_experts > 1:
        shared = intermediate if cfg.shared_intermediate_size is None else cfg.shared_intermediate_size
        return PositionRoutedMLP(cfg.hidden_size, intermediate // cfg.num_experts, shared,
                                 cfg.num_experts, what)
    return _GeluMLP(cfg.hidden_size, intermediate, dropout)


# =================================================================== vision
@dataclass
class VisionConfig:
    image_size: int = 224
    patch_size: int = 16
    hidden_size: int = 768
    num_hidden_layers: int = 12
    num_attention_heads: int = 12
    intermediate_size: int = 3072
    shared_intermediate_size: Optional[int] = None
    hidden_dropout_prob: float = 0.0
    attention_dropout_prob: float = 0.0
    num_channels: int = 3
    layer_norm_eps: float = 1e-6
    use_class_token: bool = True
    use_2d_pos_embed: bool = True
    num_experts: int = 4                   # 1 = dense GELU MLP


class PatchEmbedding(nn.Module):
    """[B, C, H, W] -> [B, (H/p)(W/p), hidden] by a stride-p convolution."""

    def __init__(self, image_size: int = 224, patch_size: int = 16, num_channels: int = 3,
                 hidden_size: int = 768):
        super().__init__()
        self.image_size, self.patch_size = image_size, patch_size
        self.num_patches = (image_size // patch_size) ** 2
        self.projection = nn.Conv2d(num_channels, hidden_size, patch_size, patch_size)

    def forward(self, pixel_values: torch.Tensor) -> torch.Tensor:
        return self.projection(pixel_values).flatten(2).transpose(1, 2)


class VisionTokenRoutedMLP(PositionRoutedMLP):
    def __init__(self, config: VisionConfig):
        shared = (config.intermediate_size if config.shared_intermediate_size is None
                  else config.shared_intermediate_size)
        super().__init__(config.hidden_size, config.intermediate_size // config.num_experts,
                         shared, config.num_experts, "vision")


class VisionTransformerBlock(nn.Module):
    def __init__(self, config: VisionConfig):
        super().__init__()
        self.attention = _FusedQKVAttention(config.hidden_size, config.num_attention_heads,
                                            config.attention_dropout_prob)
        self.mlp = _routed_or_dense(config, config.intermediate_size,
                                    config.hidden_dropout_prob, "vision")
        self.norm1 = nn.LayerNorm(config.hidden_size, eps=config.layer_norm_eps)
        self.norm2 = nn.LayerNorm(config.hidden_size, eps=config.layer_norm_eps)

    def forward(self, x, expert_ids, attention_mask=None):
        x = x + self.attention(self.norm1(x), attention_mask)
        return x + self.mlp(self.norm2(x), expert_ids)


class VisionTransformer(nn.Module):
    """ViT: patches (+ class token) + learned positions, pre-norm blocks whose
    routed MLP picks expert = patch index mod E (the class token uses expert 0).
    Returns ``last_hidden_state``, ``pooler_output`` (class token, else the
    mean) and optionally ``hidden_states``."""

    def __init__(self, config: VisionConfig):
        super().__init__()
        self.config = config
        self.patch_embed = PatchEmbedding(config.image_size, config.patch_size,
                                          config.num_channels, config.hidden_size)
        n = self.patch_embed.num_patches
        if config.use_class_token:
            self.cls_token = nn.Parameter(torch.zeros(1, 1, config.hidden_size))
            nn.init.trunc_normal_(self.cls_token, std=0.02)
        self.position_embedding = nn.Parameter(
            torch.zeros(1, n + int(config.use_class_token), config.hidden_size))
        nn.init.trunc_normal_(self.position_embedding, std=0.02)
        self.dropout = nn.Dropout(config.hidden_dropout_prob)
        self.blocks = nn.ModuleList(VisionTransformerBlock(config)
                                    for _ in range(config.num_hidden_layers))
        self.norm = nn.LayerNorm(config.hidden_size, eps=config.layer_norm_eps)
        ids = torch.arange(n) % config.num_experts
        if config.use_class_token:
            ids = torch.cat((torch.zeros(1, dtype=torch.long), ids))
        self.register_buffer("expert_ids", ids)

    def forward(self, pixel_values, attention_mask=None, output_hidden_states: bool = False):
        x = self.patch_embed(pixel_values)
        if self.config.use_class_token:
            x = torch.cat((self.cls_token.expand(x.shape[0], -1, -1), x), 1)
        x = self.dropout(x + self.position_embedding)
        hs: List[torch.Tensor] = []
        for blk in self.blocks:
            if output_hidden_states:
                hs.append(x)
            x = blk(x, self.expert_ids, attention_mask)
        x = self.norm(x)
        out = {"last_hidden_state": x,
               "pooler_output": x[:, 0] if self.config.use_class_token else x.mean(1)}
        if output_hidden_states:
            out["hidden_states"] = hs + [x]
        return out


class _ProjectedEncoder(nn.Module):
    def _finish(self, out: dict, return_all_features: bool):
        f = out["last_hidden_state"] if return_all_features else out["pooler_output"]
        return self.proj(f) if self.proj is not None else f


class VisionEncoder(_ProjectedEncoder):
    def __init__(self, image_size: int = 224, patch_size: int = 16, hidden_size: int = 768,
                 num_layers: int = 12, num_heads: int = 12, num_experts: int = 4,
                 output_dim: Optional[int] = None):
        super().__init__()
        self.encoder = VisionTransformer(VisionConfig(
            image_size=image_size, patch_size=patch_size, hidden_size=hidden_size,
            num_hidden_layers=num_layers, num_attention_heads=num_heads,
            num_experts=num_experts))
        self.proj = (nn.Linear(hidden_size, output_dim)
                     if output_dim is not None and output_dim != hidden_size else None)

    def forward(self, pixel_values, return_all_features: bool = False):
        return self._finish(self.encoder(pixel_values), return_all_features)


class CLIPVisionEncoder(nn.Module):
    """ViT + bias-free projection, L2-normalised; ``get_logit_scale`` =
    exp(logit_scale) clamped to 100 (initialised to 1/0.07)."""

    def __init__(self, image_size: int = 224, patch_size: int = 14, hidden_size: int = 1024,
                 num_layers: int = 24, num_heads: int = 16, output_dim: int = 768,
                 num_experts: int = 4):
        super().__init__()
        self.encoder = VisionTransformer(VisionConfig(
            image_size=image_size, patch_size=patch_size, hidden_size=hidden_size,
            num_hidden_layers=num_layers, num_attention_heads=num_heads,
            intermediate_size=4 * hidden_size, num_experts=num_experts))
        self.proj = nn.Linear(hidden_size, output_dim, bias=False)
        self.logit_scale = nn.Parameter(torch.tensor(math.log(1 / 0.07)))

    def forward(self, pixel_values, normalize: bool = True):
        f = self.proj(self.encoder(pixel_values)["pooler_output"])
        return F.normalize(f, dim=-1) if normalize else f

    def get_logit_scale(self) -> torch.Tensor:
        return self.logit_scale.exp().clamp(max=100)


class SigLIPEncoder(nn.Module):
    """ViT without class token (mean pooled), optional projection; the sigmoid
    pair loss -mean(logsigmoid(y * (s <img, txt> + b))), y = +1 on the diagonal,
    -1 elsewhere (s initialised to 10, b to 0)."""

    def __init__(self, image_size: int = 384, patch_size: int = 14, hidden_size: int = 1152,
                 num_layers: int = 27, num_heads: int = 16, output_dim: int = 1152,
                 num_experts: int = 4):
        super().__init__()
        self.encoder = VisionTransformer(VisionConfig(
            image_size=image_size, patch_size=patch_size, hidden_size=hidden_size,
            num_hidden_layers=num_layers, num_attention_heads=num_heads,
            intermediate_size=4 * hidden_size, use_class_token=False, num_experts=num_experts))
        self.proj = nn.Linear(hidden_size, output_dim) if output_dim != hidden_size else None
        self.bias = nn.Parameter(torch.zeros(()))
        self.scale = nn.Parameter(torch.ones(()) * 10)

    def forward(self, pixel_values, normalize: bool = True):
        f = self.encoder(pixel_values)["pooler_output"]
        if self.proj is not None:
            f = self.proj(f)
        return F.normalize(f, dim=-1) if normalize else f

    def compute_loss(self, image_features, text_features):
        logits = image_features @ text_features.transpose(0, 1) * self.scale + self.bias
        n = image_features.shape[0]
        y = 2 * torch.eye(n, device=logits.device, dtype=logits.dtype) - 1
        return -F.logsigmoid(y * logits).mean()


# ==================================================================== audio
@dataclass
class AudioConfig:
    n_mels: int = 80
    n_fft: int = 400
    hop_length: int = 160
    sample_rate: int = 16000
    hidden_size: int = 768
    num_hidden_layers: int = 12
    num_attention_heads: int = 12
    intermediate_size: int = 3072
    shared_intermediate_size: Optional[int] = None
    dropout: float = 0.0
    max_length: int = 3000
    layer_norm_eps: float = 1e-5
    num_experts: int = 4


class AudioConvStack(nn.Module):
    """[B, n_mels, T] -> [B, ceil(T/2), hidden]: conv3 + GELU, stride-2 conv3 + GELU."""

    def __init__(self, n_mels: int = 80, hidden_size: int = 768):
        super().__init__()
        self.conv1 = nn.Conv1d(n_mels, hidden_size, 3, padding=1)
        self.conv2 = nn.Conv1d(hidden_size, hidden_size, 3, stride=2, padding=1)
        self.gelu = nn.GELU()

    def forward(self, mel_spectrogram):
        return self.gelu(self.conv2(self.gelu(self.conv1(mel_spectrogram)))).transpose(1, 2)


class AudioTokenRoutedMLP(PositionRoutedMLP):
    def __init__(self, config: AudioConfig):
        shared = (config.intermediate_size if config.shared_intermediate_size is None
                  else config.shared_intermediate_size)
        super().__init__(config.hidden_size, config.intermediate_size // config.num_experts,
                         shared, config.num_experts, "audio")


class AudioTransformerBlock(nn.Module):
    def __init__(self, config: AudioConfig):
        super().__init__()
        self.self_attn = _SplitQKVAttention(config.hidden_size, config.num_attention_heads,
                                            config.dropout)
        self.mlp = _routed_or_dense(config, config.intermediate_size, config.dropout, "audio")
        self.norm1 = nn.LayerNorm(config.hidden_size, eps=config.layer_norm_eps)
        self.norm2 = nn.LayerNorm(config.hidden_size, eps=config.layer_norm_eps)

    def forward(self, x, expert_ids, attention_mask=None):
        x = x + self.self_attn(self.norm1(x), None, attention_mask)
        return x + self.mlp(self.norm2(x), expert_ids)


def _frames_check(n: int, table: torch.Tensor, max_length: int):
    if n > table.numel():
        raise ValueError(f"mel spectrogram produced {n} encoder frames after downsampling, "
                         f"exceeding max_length={max_length} ({table.numel()} frames); truncate "
                         "the input or construct this encoder with a larger max_length")


class MelSpectrogramEncoder(nn.Module):
    """Conv stack, learned positions, routed blocks (expert = frame mod E)."""

    def __init__(self, config: AudioConfig):
        super().__init__()
        self.config = config
        self.conv_stack = AudioConvStack(config.n_mels, config.hidden_size)
        self.position_embedding = nn.Embedding(config.max_length, config.hidden_size)
        self.blocks = nn.ModuleList(AudioTransformerBlock(config)
                                    for _ in range(config.num_hidden_layers))
        self.norm = nn.LayerNorm(config.hidden_size, eps=config.layer_norm_eps)
        self.register_buffer("expert_ids_table",
                             torch.arange(config.max_length // 2) % config.num_experts)

    def forward(self, mel_spectrogram, attention_mask=None):
        x = self.conv_stack(mel_spectrogram)
        n = x.shape[1]
        _frames_check(n, self.expert_ids_table, self.config.max_length)
        x = x + self.position_embedding(torch.arange(n, device=x.device))
        ids = self.expert_ids_table[:n]
        for blk in self.blocks:
            x = blk(x, ids, attention_mask)
        x = self.norm(x)
        return {"last_hidden_state": x, "pooler_output": x.mean(1)}


def sinusoidal_positions(n: int, dim: int) -> torch.Tensor:
    """[n, dim]: sin at even, cos at odd channels, frequencies 10000^(-2i/dim)."""
    pos = torch.arange(n, dtype=torch.float32)[:, None]
    freq = torch.exp(torch.arange(0, dim, 2, dtype=torch.float32) * (-math.log(10000.0) / dim))
    pe = torch.zeros(n, dim)
    pe[:, 0::2] = torch.sin(pos * freq)
    pe[:, 1::2] = torch.cos(pos * freq)
    return pe


class WhisperEncoder(nn.Module):
    """Two convolutions (second stride 2), fixed sinusoidal positions, routed
    blocks, final LayerNorm."""

    def __init__(self, n_mels: int = 80, hidden_size: int = 768, num_layers: int = 12,
                 num_heads: int = 12, max_length: int = 1500, num_experts: int = 4):
        super().__init__()
        cfg = AudioConfig(n_mels=n_mels, hidden_size=hidden_size, num_hidden_layers=num_layers,
                          num_attention_heads=num_heads, intermediate_size=4 * hidden_size,
                          max_length=max_length, num_experts=num_experts)
        self.max_length = max_length
        self.conv1 = nn.Conv1d(n_mels, hidden_size, 3, padding=1)
        self.conv2 = nn.Conv1d(hidden_size, hidden_size, 3, stride=2, padding=1)
        self.register_buffer("positional_embedding", sinusoidal_positions(max_length, hidden_size))
        self.blocks = nn.ModuleList(AudioTransformerBlock(cfg) for _ in range(num_layers))
        self.norm = nn.LayerNorm(hidden_size)
        self.register_buffer("expert_ids_table", torch.arange(max_length) % num_experts)

    def forward(self, mel_spectrogram, attention_mask=None):
        x = F.gelu(self.conv2(F.gelu(self.conv1(mel_spectrogram)))).transpose(1, 2)
        n = x.shape[1]
        _frames_check(n, self.expert_ids_table, self.max_length)
        x = x + self.positional_embedding[:n]
        ids = self.expert_ids_table[:n]
        for blk in self.blocks:
            x = blk(x, ids, attention_mask)
        x = self.norm(x)
        return {"last_hidden_state": x, "pooler_output": x.mean(1)}


class AudioEncoder(_ProjectedEncoder):
    def __init__(self, n_mels: int = 80, hidden_size: int = 768, num_layers: int = 12,
                 num_heads: int = 12, output_dim: Optional[int] = None,
                 encoder_type: str = "whisper", num_experts: int = 4):
        super().__init__()
        if encoder_type == "whisper":
            self.encoder = WhisperEncoder(n_mels, hidden_size, num_layers, num_heads,
                                          num_experts=num_experts)
        else:
            self.encoder = MelSpectrogramEncoder(AudioConfig(
                n_mels=n_mels, hidden_size=hidden_size, num_hidden_layers=num_layers,
                num_attention_heads=num_heads, num_experts=num_experts))
        self.proj = (nn.Linear(hidden_size, output_dim)
                     if output_dim is not None and output_dim != hidden_size else None)

    def forward(self, mel_spectrogram, return_all_features: bool = False):
        return self._finish(self.encoder(mel_spectrogram), return_all_features)


class AudioPreprocessor(nn.Module):
    """Waveform [B, T] (or [B, 1, T]) -> log-mel spectrogram [B, n_mels, frames]:
    Hann-window STFT power through a triangular mel filterbank (HTK mel scale),
    natural log (floored at 1e-10) and, with ``normalize``, standardised over
    the whole batch to zero mean and unit variance."""

    def __init__(self, sample_rate: int = 16000, n_mels: int = 80, n_fft: int = 400,
                 hop_length: int = 160, normalize: bool = True):
        super().__init__()
        self.sample_rate, self.n_mels, self.n_fft, self.hop_length = (sample_rate, n_mels, n_fft,
                                                                      hop_length)
        self.normalize = normalize
        self.register_buffer("mel_filters", mel_filterbank(sample_rate, n_fft, n_mels))

    def forward(self, waveform):
        if waveform.dim() == 3:
            waveform = waveform.squeeze(1)
        spec = torch.stft(waveform, self.n_fft, self.hop_length,
                          window=torch.hann_window(self.n_fft, device=waveform.device),
                          return_complex=True)
        log = torch.log((self.mel_filters.to(waveform.device) @ spec.abs().square())
                        .clamp_min(1e-10))
        if self.normalize:
            log = (log - log.mean()) / (log.std() + 1e-8)
        return log


def mel_filterbank(sample_rate: int, n_fft: int, n_mels: int) -> torch.Tensor:
    """[n_mels, n_fft/2 + 1] triangular filters evenly spaced on the HTK mel scale."""
    def mel(f):
        return 2595.0 * torch.log10(1.0 + f / 700.0)

    def hz(m):
        return 700.0 * (10.0 ** (m / 2595.0) - 1.0)

    pts = hz(torch.linspace(0.0, float(mel(torch.tensor(sample_rate / 2.0))), n_mels + 2))
    f = torch.linspace(0.0, sample_rate / 2.0, n_fft // 2 + 1)
    lo, mid, hi = pts[:-2, None], pts[1:-1, None], pts[2:, None]
    up = (f[None] - lo) / (mid - lo)
    down = (hi - f[None]) / (hi - mid)
    return torch.clamp(torch.minimum(up, down), min=0.0)


# ==================================================================== video
@dataclass
class VideoConfig:
    image_size: int = 224
    patch_size: int = 16
    num_frames: int = 16
    temporal_patch_size: int = 2
    hidden_size: int = 768
    num_hidden_layers: int = 12
    num_attention_heads: int = 12
    intermediate_size: int = 3072
    shared_intermediate_size: Optional[int] = None
    hidden_dropout_prob: float = 0.0
    attention_dropout_prob: float = 0.0
    num_channels: int = 3
    layer_norm_eps: float = 1e-6
    num_experts: int = 4

    @property
    def num_spatial_patches(self) -> int:
        return (self.image_size // self.patch_size) ** 2

    @property
    def num_temporal_patches(self) -> int:
        return self.num_frames // self.temporal_patch_size

    @property
    def num_patches(self) -> int:
        return self.num_spatial_patches * self.num_temporal_patches


class TubeletEmbedding(nn.Module):
    """[B, C, T, H, W] -> [B, T_p * S_p, hidden] (time-major) by a strided Conv3d."""

    def __init__(self, config: VideoConfig):
        super().__init__()
        self.T, self.S = config.num_temporal_patches, config.num_spatial_patches
        k = (config.temporal_patch_size, config.patch_size, config.patch_size)
        self.projection = nn.Conv3d(config.num_channels, config.hidden_size, k, k)

    def forward(self, video):
        x = self.projection(video)                       # [B, H, T_p, h, w]
        return x.flatten(2).transpose(1, 2)              # [B, T_p*h*w, H]


class VideoTokenRoutedMLP(PositionRoutedMLP):
    def __init__(self, config: VideoConfig):
        shared = (config.intermediate_size if config.shared_intermediate_size is None
                  else config.shared_intermediate_size)
        super().__init__(config.hidden_size, config.intermediate_size // config.num_experts,
                         shared, config.num_experts, "video")


class SpatioTemporalBlock(nn.Module):
    """Factorised block: attention over the patches of each frame, then over the
    frames at each spatial position, then the (routed) MLP; pre-norm residuals."""

    def __init__(self, config: VideoConfig):
        super().__init__()
        h, p = config.num_attention_heads, config.attention_dropout_prob
        self.spatial_attn = _FusedQKVAttention(config.hidden_size, h, p)
        self.temporal_attn = _FusedQKVAttention(config.hidden_size, h, p)
        self.mlp = _routed_or_dense(config, config.intermediate_size,
                                    config.hidden_dropout_prob, "video")
        eps = config.layer_norm_eps
        self.norm_spatial = nn.LayerNorm(config.hidden_size, eps=eps)
        self.norm_temporal = nn.LayerNorm(config.hidden_size, eps=eps)
        self.norm_mlp = nn.LayerNorm(config.hidden_size, eps=eps)

    def forward(self, x, T: int, S: int, expert_ids):
        B, _, H = x.shape
        x = x + self.spatial_attn(self.norm_spatial(x).reshape(B * T, S, H)).reshape(B, T * S, H)
        t = self.norm_temporal(x).reshape(B, T, S, H).transpose(1, 2).reshape(B * S, T, H)
        x = x + self.temporal_attn(t).reshape(B, S, T, H).transpose(1, 2).reshape(B, T * S, H)
        return x + self.mlp(self.norm_mlp(x), expert_ids)


class VideoTransformer(nn.Module):
    """Tubelets + factorised (spatial + temporal) learned positions, factorised
    blocks (expert = spatial patch index mod E); mean-pooled output."""

    def __init__(self, config: VideoConfig):
        super().__init__()
        self.config = config
        self.T, self.S = config.num_temporal_patches, config.num_spatial_patches
        self.tubelet_embed = TubeletEmbedding(config)
        self.spatial_pos_embed = nn.Parameter(torch.zeros(1, 1, self.S, config.hidden_size))
        self.temporal_pos_embed = nn.Parameter(torch.zeros(1, self.T, 1, config.hidden_size))
        nn.init.trunc_normal_(self.spatial_pos_embed, std=0.02)
        nn.init.trunc_normal_(self.temporal_pos_embed, std=0.02)
        self.dropout = nn.Dropout(config.hidden_dropout_prob)
        self.blocks = nn.ModuleList(SpatioTemporalBlock(config)
                                    for _ in range(config.num_hidden_layers))
        self.norm = nn.LayerNorm(config.hidden_size, eps=config.layer_norm_eps)
        self.register_buffer("expert_ids",
                             (torch.arange(self.S) % config.num_experts).repeat(self.T))

    def forward(self, video, output_hidden_states: bool = False):
        x = self.tubelet_embed(video)
        pos = (self.spatial_pos_embed + self.temporal_pos_embed).reshape(1, self.T * self.S, -1)
        x = self.dropout(x + pos)
        hs: List[torch.Tensor] = []
        for blk in self.blocks:
            if output_hidden_states:
                hs.append(x)
            x = blk(x, self.T, self.S, self.expert_ids)
        x = self.norm(x)
        out = {"last_hidden_state": x, "pooler_output": x.mean(1)}
        if output_hidden_states:
            out["hidden_states"] = hs + [x]
        return out


class VideoEncoder(_ProjectedEncoder):
    def __init__(self, image_size: int = 224, patch_size: int = 16, num_frames: int = 16,
                 temporal_patch_size: int = 2, hidden_size: int = 768, num_layers: int = 12,
                 num_heads: int = 12, num_experts: int = 4, output_dim: Optional[int] = None):
        super().__init__()
        self.encoder = VideoTransformer(VideoConfig(
            image_size=image_size, patch_size=patch_size, num_frames=num_frames,
            temporal_patch_size=temporal_patch_size, hidden_size=hidden_size,
            num_hidden_layers=num_layers, num_attention_heads=num_heads,
            num_experts=num_experts))
        self.proj = (nn.Linear(hidden_size, output_dim)
                     if output_dim is not None and output_dim != hidden_size else None)

    def forward(self, video, return_all_features: bool = False):
        return self._finish(self.encoder(video), return_all_features)


# =================================================================== fusion
@dataclass
class FusionConfig:
    hidden_size: int = 768
    num_attention_heads: int = 12
    num_layers: int = 2
    dropout: float = 0.1
    num_latents: int = 64
    layer_norm_eps: float = 1e-6
    num_experts: int = 4
    shared_intermediate_size: Optional[int] = None


class FusionTokenRoutedMLP(PositionRoutedMLP):
    """Routed MLP of query tokens (expert = query position mod E); experts of
    width 4H / E, shared SwiGLU 4H unless set."""

    def __init__(self, config: FusionConfig):
        shared = (4 * config.hidden_size if config.shared_intermediate_size is None
                  else config.shared_intermediate_size)
        super().__init__(config.hidden_size, 4 * config.hidden_size // config.num_experts,
                         shared, config.num_experts, "fusion")


class FusionPlainMLP(nn.Module):
    def __init__(self, config: FusionConfig):
        super().__init__()
        H, p = config.hidden_size, config.dropout
        self.net = nn.Sequential(nn.Linear(H, 4 * H), nn.GELU(), nn.Dropout(p),
                                 nn.Linear(4 * H, H), nn.Dropout(p))

    def forward(self, x, _expert_ids=None):
        return self.net(x)


class CrossAttention(_SplitQKVAttention):
    """Queries from one modality, keys/values from another."""

    def __init__(self, hidden_size: int, num_heads: int, dropout: float = 0.0):
        super().__init__(hidden_size, num_heads, dropout)

    def forward(self, query, key_value, attention_mask=None):
        return super().forward(query, key_value, attention_mask)


class CrossAttentionBlock(nn.Module):
    def __init__(self, config: FusionConfig):
        super().__init__()
        self.cross_attn = CrossAttention(config.hidden_size, config.num_attention_heads,
                                         config.dropout)
        self.norm1 = nn.LayerNorm(config.hidden_size, eps=config.layer_norm_eps)
        self.norm2 = nn.LayerNorm(config.hidden_size, eps=config.layer_norm_eps)
        self.mlp = (FusionTokenRoutedMLP(config) if config.num_experts > 1
                    else FusionPlainMLP(config))

    def forward(self, query, key_value, attention_mask=None, expert_ids=None):
        query = query + self.cross_attn(self.norm1(query), key_value, attention_mask)
        return query + self.mlp(self.norm2(query), expert_ids)


class CrossAttentionFusion(nn.Module):
    """Text queries attend to another modality through ``num_layers`` blocks."""

    def __init__(self, hidden_size: int = 768, num_heads: int = 12, num_layers: int = 2,
                 dropout: float = 0.1, num_experts: int = 4):
        super().__init__()
        cfg = FusionConfig(hidden_size=hidden_size, num_attention_heads=num_heads,
                           num_layers=num_layers, dropout=dropout, num_experts=num_experts)
        self.layers = nn.ModuleList(CrossAttentionBlock(cfg) for _ in range(num_layers))
        self.norm = nn.LayerNorm(hidden_size)

    def forward(self, text_features, other_features, attention_mask=None):
        x = text_features
        for layer in self.layers:
            x = layer(x, other_features, attention_mask)
        return self.norm(x)


class GatedFusion(nn.Module):
    """Per-modality sigmoid gates computed from all modalities; projection of the
    gated concatenation.  Every modality must be present (use zeros for a
    missing one)."""

    def __init__(self, hidden_size: int = 768, num_modalities: int = 2):
        super().__init__()
        self.num_modalities = num_modalities
        cat = hidden_size * num_modalities
        self.gates = nn.ModuleList(nn.Sequential(nn.Linear(cat, hidden_size), nn.Sigmoid())
                                   for _ in range(num_modalities))
        self.proj = nn.Linear(cat, hidden_size)

    def forward(self, *features):
        if len(features) != self.num_modalities:
            raise ValueError(f"GatedFusion configured for {self.num_modalities} modalities, got "
                             f"{len(features)}; a missing modality must be represented "
                             "explicitly (e.g. a zero tensor)")
        cat = torch.cat(features, -1)
        return self.proj(torch.cat([g(cat) * f for f, g in zip(features, self.gates)], -1))


class ConcatProjection(nn.Module):
    """Mean-pool each modality (if [B, N, H]), concatenate, 2-layer GELU projection."""

    def __init__(self, hidden_size: int = 768, num_modalities: int = 2, dropout: float = 0.1):
        super().__init__()
        self.proj = nn.Sequential(nn.Linear(hidden_size * num_modalities, 2 * hidden_size),
                                  nn.GELU(), nn.Dropout(dropout),
                                  nn.Linear(2 * hidden_size, hidden_size))

    def forward(self, *features):
        return self.proj(torch.cat([f.mean(1) if f.dim() == 3 else f for f in features], -1))


class PerceiverResampler(nn.Module):
    """``num_latents`` learned queries cross-attend to the features
    (latent i uses expert i mod E): [B, N, H] -> [B, num_latents, H]."""

    def __init__(self, hidden_size: int = 768, num_latents: int = 64, num_heads: int = 12,
                 num_layers: int = 2, dropout: float = 0.1, num_experts: int = 4):
        super().__init__()
        self.num_latents = num_latents
        self.latents = nn.Parameter(torch.randn(num_latents, hidden_size) * 0.02)
        cfg = FusionConfig(hidden_size=hidden_size, num_attention_heads=num_heads,
                           num_layers=num_layers, dropout=dropout, num_latents=num_latents,
                           num_experts=num_experts)
        self.layers = nn.ModuleList(CrossAttentionBlock(cfg) for _ in range(num_layers))
        self.norm = nn.LayerNorm(hidden_size)
        self.register_buffer("expert_ids", torch.arange(num_latents) % num_experts)

    def forward(self, features, attention_mask=None):
        x = self.latents[None].expand(features.shape[0], -1, -1)
        for layer in self.layers:
            x = layer(x, features, attention_mask, self.expert_ids)
        return self.norm(x)


class MultimodalFusion(nn.Module):
    """One of cross_attention | gated | concat | perceiver behind one call
    ``(text_features, other_features, attention_mask)``."""

    def __init__(self, hidden_size: int = 768, num_heads: int = 12, num_layers: int = 2,
                 fusion_type: str = "cross_attention", num_latents: int = 64,
                 dropout: float = 0.1, num_experts: int = 4):
        super().__init__()
        self.fusion_type = fusion_type
        if fusion_type == "cross_attention":
            self.fusion = CrossAttentionFusion(hidden_size, num_heads, num_layers, dropout,
                                               num_experts)
        elif fusion_type == "gated":
            self.fusion = GatedFusion(hidden_size)
        elif fusion_type == "concat":
            self.fusion = ConcatProjection(hidden_size, dropout=dropout)
        elif fusion_type == "perceiver":
            self.fusion = PerceiverResampler(hidden_size, num_latents, num_heads, num_layers,
                                             dropout, num_experts)
        else:
            raise ValueError(f"Unknown fusion type: {fusion_type}")

    def forward(self, text_features, other_features, attention_mask=None):
        t = self.fusion_type
        if t == "cross_attention":
            return self.fusion(text_features, other_features, attention_mask)
        if t == "gated":
            def pool(f):
                return f.mean(1, keepdim=True) if f.dim() == 3 else f[:, None]
            return self.fusion(pool(text_features), pool(other_features)).squeeze(1)
        if t == "concat":
            return self.fusion(text_features, other_features)
        return self.fusion(other_features, attention_mask)


class VisionLanguageConnector(nn.Module):
    """Vision features -> language width: a 2-layer GELU MLP, or a Perceiver
    resampler (64 latents) followed by a projection."""

    def __init__(self, vision_hidden_size: int = 1024, language_hidden_size: int = 4096,
                 num_tokens: int = 576, connector_type: str = "mlp"):
        super().__init__()
        self.num_tokens, self.connector_type = num_tokens, connector_type
        if connector_type == "mlp":
            self.connector = nn.Sequential(nn.Linear(vision_hidden_size, language_hidden_size),
                                           nn.GELU(),
                                           nn.Linear(language_hidden_size, language_hidden_size))
        elif connector_type == "resampler":
            self.connector = PerceiverResampler(vision_hidden_size, 64, 16, 2)
            self.proj = nn.Linear(vision_hidden_size, language_hidden_size)
        else:
            raise ValueError(f"Unknown connector type: {connector_type}")

    def forward(self, vision_features):
        out = self.connector(vision_features)
        return out if self.connector_type == "mlp" else self.proj(out)
