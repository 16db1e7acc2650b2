"""Image-text-to-text on the TR-Hash vision tower and decoder.

Counterparts: complexity/generative/vision_language/ (config.py
``TRHashVisionLanguageConfig``, model.py ``TRHashImageTextToText`` /
``VisualTokenResampler``, data.py ``VisionLanguageTarDataset`` /
``collate_vision_language``, pretraining.py / training.py).  Patch embeddings
are resampled to a fixed number of visual tokens, projected to the decoder
width and prefixed to the text (``PrefixLM``).  Pretraining (captioning) and
instruction tuning are the same loss with different text.
"""
from __future__ import annotations

import io
import tarfile
from dataclasses import dataclass, field
from typing import Dict, Optional, Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from .prefix_lm import PrefixLM, TokenResampler
from .towers import TRHashVisionTower, TRHashVisionTowerConfig

VisualTokenResampler = TokenResampler


@dataclass
class TRHashVisionLanguageConfig:
    vision: TRHashVisionTowerConfig = field(default_factory=TRHashVisionTowerConfig)
    num_visual_tokens: int = 64
    freeze_vision: bool = False


class TRHashImageTextToText(nn.Module):
    def __init__(self, config: TRHashVisionLanguageConfig, decoder):
        super().__init__()
        self.config = config
        self.vision = TRHashVisionTower(config.vision)
        self.resampler = TokenResampler(config.vision.hidden_size, decoder.config.hidden_size,
                                        config.num_visual_tokens,
                                        max(1, config.vision.num_heads // 2))
        self.lm = PrefixLM(decoder)
        if config.freeze_vision:
            for p in self.vision.parameters():
                p.requires_grad_(False)

    def prefix(self, pixel_values: torch.Tensor) -> torch.Tensor:
        return self.resampler(self.vision(pixel_values))

    def forward(self, pixel_values: torch.Tensor, input_ids: torch.Tensor,
                labels: Optional[torch.Tensor] = None) -> Dict[str, torch.Tensor]:
        return {"loss": self.lm.loss(self.prefix(pixel_values), input_ids, labels)}

    @torch.no_grad()
    def generate(self, pixel_values: torch.Tensor, prompt_ids: torch.Tensor,
                 max_new_tokens: int = 32, eos_id: Optional[int] = None) -> torch.Tensor:
        return self.lm.generate(self.prefix(pixel_values), prompt_ids, max_new_tokens, eos_id)


class VisionLanguageTarDataset(torch.utils.data.Dataset):
    """Webdataset-style tar shard: ``<key>.jpg|png`` with ``<key>.txt`` captions.
    Images are resized to ``image_size``; text is tokenized by ``tokenizer.encode``."""

    def __init__(self, tar_path: str, tokenizer, image_size: int = 224, max_text: int = 128):
        self.tar_path, self.tok, self.size, self.max_text = tar_path, tokenizer, image_size, max_text
        groups: Dict[str, Dict[str, tarfile.TarInfo]] = {}
        with tarfile.open(tar_path) as tf:
            for m in tf.getmembers():
                if not m.isfile() or "." not in m.name:
                    continue
                key, ext = m.name.rsplit(".", 1)
                groups.setdefault(key, {})[ext.lower()] = m
        self.items = [(k, g) for k, g in sorted(groups.items())
                      if "txt" in g and any(e in g for e in ("jpg", "jpeg", "png"))]
        self._tf = None

    def __len__(self) -> int:
        return len(self.items)

    def __getitem__(self, i: int):
        from PIL import Image
        import torchvision.transforms.functional as TF

        if self._tf is None:
            self._tf = tarfile.open(self.tar_path)
        key, g = self.items[i]
        img_m = next(g[e] for e in ("jpg", "jpeg", "png") if e in g)
        img = Image.open(io.BytesIO(self._tf.extractfile(img_m).read())).convert("RGB")
        img = TF.to_tensor(img.resize((self.size, self.size)))
        text = self._tf.extractfile(g["txt"]).read().decode("utf-8").strip()
        ids = self.tok.encode(text)[: self.max_text]
        return img, torch.tensor(ids, dtype=torch.long)


def collate_vision_language(batch: Sequence, pad_id: int = 0):
    """-> (images [B, 3, S, S], input_ids [B, T] padded, labels with -100 on padding)."""
    images = torch.stack([b[0] for b in batch])
    T = max(len(b[1]) for b in batch)
    ids = torch.full((len(batch), T), pad_id, dtype=torch.long)
    labels = torch.full((len(batch), T), -100, dtype=torch.long)
    for i, (_, t) in enumerate(batch):
        ids[i, :len(t)] = t
        labels[i, :len(t)] = t
    return images, ids, labels
