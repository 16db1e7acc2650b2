"""Text-to-image generation and instruction-based image editing in latent space.

Counterparts: complexity/generative/image/ (codec.py ``FrozenAutoencoderKL``,
config.py ``TRHashImageConfig``, model.py ``TRHashTextToImage``, editing.py
``TRHashImageEditConfig`` / ``TRHashImageEditor``, data.py / edit_data.py tar
datasets, training.py / edit_training.py).

* codec: a convolutional KL autoencoder (8x downsampling, Gaussian latent),
  trained with reconstruction + KL, frozen while the generator trains;
* generator: a transformer over 2x2 latent patches; every block has adaptive
  LayerNorm scale/shift/gate from the flow time, cross-attention to text
  tokens, and the TR-Hash FFN keyed by latent patch position;
* objective: rectified flow (x_t = (1 - t) x_0 + t noise, predict
  noise - x_0) sampled with Euler steps from t = 1 to 0 and classifier-free
  guidance (text dropped to a learned null sequence during training);
* editing: the source image's latent is concatenated to the noisy latent
  channels, so the model learns target = f(source, instruction).
"""
from __future__ import annotations

import io
import math
import tarfile
from dataclasses import dataclass
from typing import Dict, Optional, Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from .towers import SelfAttention, _engine, ffn_input


# ------------------------------------------------------------------ codec
class _Res(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.b = nn.Sequential(nn.GroupNorm(8, c), nn.SiLU(), nn.Conv2d(c, c, 3, 1, 1),
                               nn.GroupNorm(8, c), nn.SiLU(), nn.Conv2d(c, c, 3, 1, 1))

    def forward(self, x):
        return x + self.b(x)


class FrozenAutoencoderKL(nn.Module):
    """[B, 3, S, S] in [-1, 1] <-> [B, latent_channels, S/8, S/8] (scaled latents)."""

    def __init__(self, channels: int = 64, latent_channels: int = 4, scale: float = 1.0,
                 frozen: bool = True):
        super().__init__()
        c = channels
        enc = [nn.Conv2d(3, c, 3, 1, 1)]
        for _ in range(3):
            enc += [_Res(c), nn.Conv2d(c, c, 4, 2, 1)]
        enc += [_Res(c), nn.GroupNorm(8, c), nn.SiLU(), nn.Conv2d(c, 2 * latent_channels, 3, 1, 1)]
        self.encoder = nn.Sequential(*enc)
        dec = [nn.Conv2d(latent_channels, c, 3, 1, 1), _Res(c)]
        for _ in range(3):
            dec += [nn.Upsample(scale_factor=2.0, mode="nearest"), nn.Conv2d(c, c, 3, 1, 1), _Res(c)]
        dec += [nn.GroupNorm(8, c), nn.SiLU(), nn.Conv2d(c, 3, 3, 1, 1)]
        self.decoder = nn.Sequential(*dec)
        self.latent_channels, self.scale = latent_channels, scale
        self.set_frozen(frozen)

    def set_frozen(self, frozen: bool) -> None:
        self.frozen = frozen
        for p in self.parameters():
            p.requires_grad_(not frozen)

    def encode_dist(self, images):
        mean, logvar = self.encoder(images).chunk(2, 1)
        return mean, logvar.clamp(-20, 10)

    def encode(self, images: torch.Tensor, sample: bool = False) -> torch.Tensor:
        mean, logvar = self.encode_dist(images)
        z = mean + torch.randn_like(mean) * torch.exp(0.5 * logvar) if sample else mean
        return z * self.scale

    def decode(self, latents: torch.Tensor) -> torch.Tensor:
        return self.decoder(latents / self.scale)

    def loss(self, images: torch.Tensor, kl_weight: float = 1e-6) -> Dict[str, torch.Tensor]:
        mean, logvar = self.encode_dist(images)
        z = mean + torch.randn_like(mean) * torch.exp(0.5 * logvar)
        rec = self.decoder(z)
        l_rec = F.l1_loss(rec, images) + F.mse_loss(rec, images)
        kl = 0.5 * (mean ** 2 + logvar.exp() - 1 - logvar).mean()
        return {"loss": l_rec + kl_weight * kl, "loss_rec": l_rec, "loss_kl": kl}


# -------------------------------------------------------------- generator
@dataclass
class TRHashImageConfig:
    image_size: int = 256
    latent_channels: int = 4
    latent_downsample: int = 8
    patch_size: int = 2
    hidden_size: int = 384
    num_layers: int = 8
    num_heads: int = 6
    num_experts: int = 4
    top_k: int = 2
    shared_width: int = 768
    expert_width: int = 128
    text_vocab_size: int = 32000
    text_dim: int = 384           # width of the conditioning text tokens
    max_text_len: int = 77
    cond_drop_prob: float = 0.1   # classifier-free guidance training
    route_seed: int = 0x1A6E
    dropout: float = 0.0
    in_channels_extra: int = 0    # editing: source latent channels

    @property
    def latent_size(self) -> int:
        return self.image_size // self.latent_downsample

    @property
    def grid(self) -> int:
        return self.latent_size // self.patch_size

    @property
    def route_vocab_size(self) -> int:
        return self.grid * self.grid


def timestep_embedding(t: torch.Tensor, dim: int, max_period: float = 10000.0) -> torch.Tensor:
    """Sinusoidal features of t in [0, 1] (scaled by 1000)."""
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, device=t.device) / half)
    a = 1000.0 * t.float()[:, None] * freqs[None]
    return torch.cat([a.cos(), a.sin()], -1)


class _CrossAttention(nn.Module):
    def __init__(self, dim: int, ctx_dim: int, heads: int):
        super().__init__()
        self.h = heads
        self.q = nn.Linear(dim, dim)
        self.kv = nn.Linear(ctx_dim, 2 * dim)
        self.o = nn.Linear(dim, dim)

    def forward(self, x, ctx, mask=None):
        B, N, D = x.shape
        q = self.q(x).view(B, N, self.h, D // self.h).transpose(1, 2)
        k, v = self.kv(ctx).view(B, ctx.shape[1], 2, self.h, D // self.h).permute(2, 0, 3, 1, 4)
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
        return self.o(o.transpose(1, 2).reshape(B, N, D))


class TRHashDiTBlock(nn.Module):
    def __init__(self, cfg: TRHashImageConfig, layer: int):
        super().__init__()
        H = cfg.hidden_size
        self.n1 = nn.LayerNorm(H, elementwise_affine=False)
        self.n2 = nn.LayerNorm(H)
        self.n3 = nn.LayerNorm(H, elementwise_affine=False)
        self.attn = SelfAttention(H, cfg.num_heads)
        self.cross = _CrossAttention(H, cfg.text_dim, cfg.num_heads)
        self.mlp = _engine(H, cfg.route_vocab_size, cfg.num_experts, cfg.top_k,
                           cfg.shared_width, cfg.expert_width, layer, cfg.route_seed)
        self.ada = nn.Linear(H, 6 * H)
        nn.init.zeros_(self.ada.weight)
        nn.init.zeros_(self.ada.bias)

    def forward(self, x, c, ctx, ctx_mask, route_ids):
        s1, b1, g1, s2, b2, g2 = self.ada(F.silu(c))[:, None].chunk(6, -1)
        x = x + g1 * self.attn(self.n1(x) * (1 + s1) + b1)
        x = x + self.cross(self.n2(x), ctx, ctx_mask)
        return x + g2 * self.mlp(ffn_input(self.n3(x) * (1 + s2) + b2), route_ids)


class TRHashTextToImage(nn.Module):
    """Latent rectified-flow transformer conditioned on text tokens.

    Text conditioning: ``text_ids`` embedded by a learned table (``text_dim``
    wide), or ``text_states`` [B, L, text_dim] from an external text encoder
    (e.g. a frozen decoder's hidden states)."""

    def __init__(self, config: TRHashImageConfig, codec: Optional[FrozenAutoencoderKL] = None):
        super().__init__()
        self.config = c = config
        self.codec = codec
        p, H = c.patch_size, c.hidden_size
        cin = (c.latent_channels + c.in_channels_extra) * p * p
        self.patch_in = nn.Linear(cin, H)
        self.pos = nn.Parameter(torch.randn(1, c.grid * c.grid, H) * 0.02)
        self.t_mlp = nn.Sequential(nn.Linear(256, H), nn.SiLU(), nn.Linear(H, H))
        self.text_embed = nn.Embedding(c.text_vocab_size, c.text_dim)
        self.null_text = nn.Parameter(torch.zeros(1, 1, c.text_dim))
        self.blocks = nn.ModuleList(TRHashDiTBlock(c, i) for i in range(c.num_layers))
        self.n_out = nn.LayerNorm(H, elementwise_affine=False)
        self.ada_out = nn.Linear(H, 2 * H)
        self.out = nn.Linear(H, c.latent_channels * p * p)
        nn.init.zeros_(self.out.weight)
        nn.init.zeros_(self.out.bias)
        self.register_buffer("route_ids", torch.arange(c.grid * c.grid), persistent=False)

    # ------------------------------------------------------------ pieces
    def _patchify(self, z):
        B, C, S, _ = z.shape
        p, g = self.config.patch_size, S // self.config.patch_size
        return z.view(B, C, g, p, g, p).permute(0, 2, 4, 1, 3, 5).reshape(B, g * g, C * p * p)

    def _unpatchify(self, x):
        B = x.shape[0]
        p, g, C = self.config.patch_size, self.config.grid, self.config.latent_channels
        return x.view(B, g, g, C, p, p).permute(0, 3, 1, 4, 2, 5).reshape(B, C, g * p, g * p)

    def text_context(self, text_ids=None, text_states=None, drop: Optional[torch.Tensor] = None):
        ctx = text_states if text_states is not None else self.text_embed(text_ids)
        if drop is not None:  # per-sample classifier-free-guidance dropout
            ctx = torch.where(drop[:, None, None], self.null_text.expand_as(ctx).to(ctx.dtype), ctx)
        return ctx

    def velocity(self, z_t, t, ctx, extra=None):
        x = z_t if extra is None else torch.cat([z_t, extra], 1)
        h = self.patch_in(self._patchify(x)) + self.pos.to(x.dtype)
        c = self.t_mlp(timestep_embedding(t, 256).to(h.dtype))
        ids = self.route_ids.unsqueeze(0).expand(h.shape[0], -1)
        for blk in self.blocks:
            h = blk(h, c, ctx, None, ids)
        s, b = self.ada_out(F.silu(c))[:, None].chunk(2, -1)
        return self._unpatchify(self.out(self.n_out(h) * (1 + s) + b))

    # --------------------------------------------------------- training
    def flow_loss(self, latents, ctx, extra=None) -> torch.Tensor:
        B = latents.shape[0]
        t = torch.rand(B, device=latents.device)
        noise = torch.randn_like(latents)
        z_t = (1 - t)[:, None, None, None] * latents + t[:, None, None, None] * noise
        v = self.velocity(z_t, t, ctx, extra)
        return F.mse_loss(v.float(), (noise - latents).float())

    def forward(self, images=None, text_ids=None, text_states=None, latents=None) -> dict:
        if latents is None:
            with torch.no_grad():
                latents = self.codec.encode(images)
        B = latents.shape[0]
        drop = torch.rand(B, device=latents.device) < self.config.cond_drop_prob
        ctx = self.text_context(text_ids, text_states, drop if self.training else None)
        return {"loss": self.flow_loss(latents, ctx)}

    # ---------------------------------------------------------- sampling
    @torch.no_grad()
    def sample_latents(self, ctx, steps: int = 30, guidance: float = 4.0, extra=None,
                       generator: Optional[torch.Generator] = None) -> torch.Tensor:
        c = self.config
        B = ctx.shape[0]
        z = torch.randn(B, c.latent_channels, c.latent_size, c.latent_size, generator=generator,
                        device=ctx.device if generator is None else "cpu").to(ctx.device)
        null = self.null_text.expand_as(ctx).to(ctx.dtype)
        ts = torch.linspace(1.0, 0.0, steps + 1, device=ctx.device)
        for i in range(steps):
            t = ts[i].expand(B)
            v = self.velocity(z, t, ctx, extra)
            if guidance != 1.0:
                vu = self.velocity(z, t, null, extra)
                v = vu + guidance * (v - vu)
            z = z + (ts[i + 1] - ts[i]) * v
        return z

    @torch.no_grad()
    def generate(self, text_ids=None, text_states=None, steps: int = 30, guidance: float = 4.0,
                 generator=None) -> torch.Tensor:
        z = self.sample_latents(self.text_context(text_ids, text_states), steps, guidance,
                                generator=generator)
        return self.codec.decode(z).clamp(-1, 1) if self.codec is not None else z


def sample_edit_condition_dropout(batch: int, *, caption_dropout: float, source_dropout: float,
                                  device, generator: Optional[torch.Generator] = None):
    """(drop_text, drop_source) masks for classifier-free-guidance training of
    edits.  An instruction means nothing without its source image, so dropping
    the source drops the text too (the unconditional branch); dropping only the
    text keeps the image-only branch."""
    dt = torch.rand(batch, device=device, generator=generator) < caption_dropout
    ds = torch.rand(batch, device=device, generator=generator) < source_dropout
    return dt | ds, ds


@dataclass
class TRHashImageEditConfig(TRHashImageConfig):
    in_channels_extra: int = 4
    source_drop_prob: float = 0.0    # > 0: also train the unconditional (no source) branch


class TRHashImageEditor(TRHashTextToImage):
    """Instruction-based editing: source latent concatenated to the noisy latent."""

    def __init__(self, config: TRHashImageEditConfig, codec=None):
        if config.in_channels_extra != config.latent_channels:
            raise ValueError("in_channels_extra must equal latent_channels for editing")
        super().__init__(config, codec)

    def forward(self, source=None, target=None, text_ids=None, text_states=None,
                source_latents=None, target_latents=None) -> dict:
        with torch.no_grad():
            if source_latents is None:
                source_latents = self.codec.encode(source)
            if target_latents is None:
                target_latents = self.codec.encode(target)
        B = target_latents.shape[0]
        drop_text = drop_src = None
        if self.training:
            drop_text, drop_src = sample_edit_condition_dropout(
                B, caption_dropout=self.config.cond_drop_prob,
                source_dropout=getattr(self.config, "source_drop_prob", 0.0),
                device=target_latents.device)
            # a dropped source is an all-zero latent (the null image condition)
            source_latents = source_latents * (~drop_src).to(source_latents.dtype)[:, None, None, None]
        ctx = self.text_context(text_ids, text_states, drop_text)
        return {"loss": self.flow_loss(target_latents, ctx, extra=source_latents)}

    @torch.no_grad()
    def edit(self, source=None, text_ids=None, text_states=None, source_latents=None,
             steps: int = 30, guidance: float = 3.0, generator=None) -> torch.Tensor:
        if source_latents is None:
            source_latents = self.codec.encode(source)
        z = self.sample_latents(self.text_context(text_ids, text_states), steps, guidance,
                                extra=source_latents, generator=generator)
        return self.codec.decode(z).clamp(-1, 1) if self.codec is not None else z


# ---------------------------------------------------------------- datasets
def _read_tar_groups(path: str):
    groups: Dict[str, Dict[str, tarfile.TarInfo]] = {}
    with tarfile.open(path) as tf:
        for m in tf.getmembers():
            if m.isfile() and "." in m.name:
                key, ext = m.name.split(".", 1)
                groups.setdefault(key, {})[ext.lower()] = m
    return groups


def _load_image(tf, member, size):
    from PIL import Image
    import torchvision.transforms.functional as TF

    img = Image.open(io.BytesIO(tf.extractfile(member).read())).convert("RGB")
    return TF.to_tensor(img.resize((size, size))) * 2 - 1


class AtlasImageTarDataset(torch.utils.data.Dataset):
    """Tar shard of ``<key>.jpg|png`` + ``<key>.txt`` (caption): images in [-1, 1]."""

    def __init__(self, tar_path: str, tokenizer, image_size: int = 256, max_text: int = 77):
        self.path, self.tok, self.size, self.max_text = tar_path, tokenizer, image_size, max_text
        g = _read_tar_groups(tar_path)
        self.items = [(k, v) for k, v in sorted(g.items())
                      if "txt" in v and any(e in v for e in ("jpg", "jpeg", "png"))]
        self._tf = None

    def __len__(self):
        return len(self.items)

    def __getitem__(self, i):
        if self._tf is None:
            self._tf = tarfile.open(self.path)
        _, g = self.items[i]
        img = _load_image(self._tf, next(g[e] for e in ("jpg", "jpeg", "png") if e in g), self.size)
        ids = self.tok.encode(self._tf.extractfile(g["txt"]).read().decode("utf-8"))
        return img, torch.tensor(ids[: self.max_text], dtype=torch.long)


class AtlasImageEditTarDataset(torch.utils.data.Dataset):
    """Tar shard of ``<key>.src.png``, ``<key>.tgt.png`` and ``<key>.txt`` (instruction)."""

    def __init__(self, tar_path: str, tokenizer, image_size: int = 256, max_text: int = 77):
        self.path, self.tok, self.size, self.max_text = tar_path, tokenizer, image_size, max_text
        g = _read_tar_groups(tar_path)
        self.items = [(k, v) for k, v in sorted(g.items())
                      if {"src.png", "tgt.png", "txt"} <= set(v)]
        self._tf = None

    def __len__(self):
        return len(self.items)

    def __getitem__(self, i):
        if self._tf is None:
            self._tf = tarfile.open(self.path)
        _, g = self.items[i]
        src = _load_image(self._tf, g["src.png"], self.size)
        tgt = _load_image(self._tf, g["tgt.png"], self.size)
        ids = self.tok.encode(self._tf.extractfile(g["txt"]).read().decode("utf-8"))
        return src, tgt, torch.tensor(ids[: self.max_text], dtype=torch.long)


def _pad(seqs: Sequence[torch.Tensor], pad_id: int = 0) -> torch.Tensor:
    T = max(1, max(len(s) for s in seqs))
    out = torch.full((len(seqs), T), pad_id, dtype=torch.long)
    for i, s in enumerate(seqs):
        out[i, :len(s)] = s
    return out


def collate_atlas_images(batch, pad_id: int = 0):
    return torch.stack([b[0] for b in batch]), _pad([b[1] for b in batch], pad_id)


def collate_atlas_image_edits(batch, pad_id: int = 0):
    return (torch.stack([b[0] for b in batch]), torch.stack([b[1] for b in batch]),
            _pad([b[2] for b in batch], pad_id))
