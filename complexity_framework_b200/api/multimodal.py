"""Multimodal factories: vision, audio, video, fusion, robotics and omni.

Facade names follow complexity/api/multimodal.py (``Vision``, ``Audio``,
``Video``, ``Fusion``, ``Robot``, ``Omni`` and their config classes); each
builds this framework's encoders (``multimodal/``), fusion modules and
TR-Hash towers (``generative/``).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.nn as nn

from ..generative.sensor_fusion import (SENSOR_MODALITIES, TRHashSensorFusionClassifier,
                                        TRHashSensorFusionConfig)
from ..generative.towers import TRHashVisionTowerConfig
from ..generative.vision_language import TRHashImageTextToText, TRHashVisionLanguageConfig
from ..multimodal.encoders import (AudioEncoder, EncoderConfig, PatchEmbedding, VideoEncoder,
                                   VisionEncoder, log_mel_spectrogram)
from ..multimodal.fusion import (ConcatProjection, CrossAttentionFusion, GatedFusion,
                                 PerceiverResampler, VisionLanguageConnector,
                                 VisionLanguageModel)


@dataclass
class VisionConfig:
    image_size: int = 224
    patch_size: int = 16
    channels: int = 3
    hidden_size: int = 768
    num_layers: int = 12
    num_heads: int = 12
    num_experts: int = 1


@dataclass
class AudioConfig:
    n_mels: int = 80
    max_frames: int = 3000
    hidden_size: int = 768
    num_layers: int = 12
    num_heads: int = 12


@dataclass
class FusionConfig:
    hidden_size: int = 768
    num_heads: int = 8
    num_latents: int = 64


def _enc(hidden_size: int, num_layers: int, num_heads: int, num_experts: int = 1) -> EncoderConfig:
    return EncoderConfig(hidden_size=hidden_size, num_layers=num_layers, num_heads=num_heads,
                         num_experts=num_experts)


class Vision:
    @classmethod
    def create(cls, vision_type: str = "vit", **kwargs) -> nn.Module:
        return {"vit": cls.encoder, "clip": cls.clip, "siglip": cls.siglip,
                "patches": cls.patches}[vision_type](**kwargs)

    @classmethod
    def encoder(cls, image_size: int = 224, patch_size: int = 16, hidden_size: int = 768,
                num_layers: int = 12, num_heads: int = 12, channels: int = 3,
                num_experts: int = 1, **kwargs) -> nn.Module:
        return VisionEncoder(_enc(hidden_size, num_layers, num_heads, num_experts), image_size,
                             patch_size, channels)

    @classmethod
    def clip(cls, hidden_size: int = 768, **kwargs) -> nn.Module:
        kwargs.setdefault("patch_size", 14)
        return cls.encoder(hidden_size=hidden_size, **kwargs)

    @classmethod
    def siglip(cls, hidden_size: int = 768, **kwargs) -> nn.Module:
        kwargs.setdefault("patch_size", 16)
        return cls.encoder(hidden_size=hidden_size, **kwargs)

    @classmethod
    def patches(cls, image_size: int = 224, patch_size: int = 16, channels: int = 3,
                hidden_size: int = 768) -> nn.Module:
        return PatchEmbedding(image_size, patch_size, channels, hidden_size)

    @classmethod
    def from_config(cls, config: VisionConfig) -> nn.Module:
        return cls.encoder(**config.__dict__)


class Audio:
    @classmethod
    def create(cls, audio_type: str = "standard", **kwargs) -> nn.Module:
        return {"standard": cls.encoder, "whisper": cls.whisper, "mel": cls.mel}[audio_type](**kwargs)

    @classmethod
    def encoder(cls, n_mels: int = 80, hidden_size: int = 768, num_layers: int = 12,
                num_heads: int = 12, max_frames: int = 3000, **kwargs) -> nn.Module:
        return AudioEncoder(_enc(hidden_size, num_layers, num_heads), n_mels, max_frames)

    @classmethod
    def whisper(cls, hidden_size: int = 768, n_mels: int = 80, **kwargs) -> nn.Module:
        return cls.encoder(n_mels=n_mels, hidden_size=hidden_size, **kwargs)

    @classmethod
    def mel(cls, n_mels: int = 80, hidden_size: int = 768, **kwargs) -> nn.Module:
        return cls.encoder(n_mels=n_mels, hidden_size=hidden_size, num_layers=2, num_heads=4)

    conv_stack = mel

    @staticmethod
    def spectrogram(audio, sample_rate: int = 16000, n_mels: int = 80):
        return log_mel_spectrogram(audio, sample_rate=sample_rate, n_mels=n_mels)


class Video:
    @classmethod
    def encoder(cls, frames: int = 8, image_size: int = 224, patch_size: int = 16,
                tubelet: int = 2, hidden_size: int = 768, num_layers: int = 12,
                num_heads: int = 12, channels: int = 3, **kwargs) -> nn.Module:
        return VideoEncoder(_enc(hidden_size, num_layers, num_heads), frames, image_size,
                            patch_size, tubelet, channels)

    @classmethod
    def create(cls, **kwargs) -> nn.Module:
        return cls.encoder(**kwargs)

    tubelets = encoder


class Fusion:
    @classmethod
    def create(cls, fusion_type: str = "cross_attention", **kwargs) -> nn.Module:
        return {"cross_attention": cls.cross_attention, "gated": cls.gated,
                "concat": cls.concat, "perceiver": cls.perceiver,
                "multimodal": cls.multimodal}[fusion_type](**kwargs)

    @classmethod
    def cross_attention(cls, hidden_size: int = 768, num_heads: int = 8, **kwargs) -> nn.Module:
        return CrossAttentionFusion(hidden_size, num_heads)

    @classmethod
    def gated(cls, hidden_size: int = 768, **kwargs) -> nn.Module:
        return GatedFusion(hidden_size)

    @classmethod
    def concat(cls, hidden_sizes: List[int], output_size: int, **kwargs) -> nn.Module:
        return ConcatProjection(hidden_sizes, output_size)

    @classmethod
    def perceiver(cls, hidden_size: int = 768, num_latents: int = 64, num_heads: int = 8,
                  num_layers: int = 2, **kwargs) -> nn.Module:
        return PerceiverResampler(hidden_size, num_latents, num_heads, num_layers)

    @classmethod
    def multimodal(cls, hidden_size: int = 768, in_size: Optional[int] = None,
                   **kwargs) -> nn.Module:
        """Projection of encoder features into the language model's width."""
        return VisionLanguageConnector(in_size or hidden_size, hidden_size)

    @classmethod
    def vision_language(cls, language_model, vision_encoder, resampler_latents: int = 64):
        return VisionLanguageModel(language_model, vision_encoder, resampler_latents)


class Robot:
    """TR-Hash sensor fusion (IMU, radar, skeleton, depth / IR / thermal frames).

    Follows complexity/api Robot: visual clips are [batch, channels, time,
    height, width] unless ``visual_layout`` says otherwise, and the model is
    cast to the config's ``precision``."""

    MODALITIES = SENSOR_MODALITIES

    @classmethod
    def config(cls, **kwargs) -> TRHashSensorFusionConfig:
        kwargs.setdefault("visual_layout", "bcthw")
        return TRHashSensorFusionConfig(**kwargs)

    @classmethod
    def from_config(cls, config: TRHashSensorFusionConfig) -> nn.Module:
        dtype = {"fp32": torch.float32, "bf16": torch.bfloat16,
                 "fp16": torch.float16}[config.precision]
        return TRHashSensorFusionClassifier(config).to(dtype)

    @classmethod
    def model(cls, **kwargs) -> nn.Module:
        return cls.from_config(cls.config(**kwargs))


class Omni:
    """Image-text-to-text: TR-Hash vision tower + resampler prefix + a decoder."""

    @classmethod
    def config(cls, **kwargs) -> TRHashVisionLanguageConfig:
        vis = {k[len("vision_"):]: kwargs.pop(k) for k in list(kwargs) if k.startswith("vision_")}
        return TRHashVisionLanguageConfig(vision=TRHashVisionTowerConfig(**vis), **kwargs)

    @classmethod
    def from_config(cls, config: TRHashVisionLanguageConfig, decoder=None) -> nn.Module:
        if decoder is None:
            from ..config.model_config import ModelConfig
            from ..models.builder import ComplexityModel

            decoder = ComplexityModel(ModelConfig(hidden_size=512, num_hidden_layers=4,
                                                  num_attention_heads=8, num_key_value_heads=2,
                                                  intermediate_size=512,
                                                  shared_intermediate_size=1024))
        return TRHashImageTextToText(config, decoder)

    @classmethod
    def model(cls, decoder=None, **kwargs) -> nn.Module:
        return cls.from_config(cls.config(**kwargs), decoder)


__all__ = ["Vision", "VisionConfig", "Audio", "AudioConfig", "Video", "Fusion", "FusionConfig",
           "Robot", "Omni", "VisionEncoder", "AudioEncoder", "VideoEncoder", "PatchEmbedding",
           "CrossAttentionFusion", "GatedFusion", "ConcatProjection", "PerceiverResampler",
           "TRHashSensorFusionClassifier", "TRHashSensorFusionConfig"]
