"""Multimodal encoders and fusion on top of the TR-Hash decoder.

The package-level names follow the reference's ``complexity.multimodal`` API
(``towers.py``: ViT / CLIP / SigLIP, Whisper / mel audio, factorised video
towers, cross-attention / gated / concat / Perceiver fusion).  ``encoders`` and
``fusion`` hold the compact config-driven towers and the vision-language model
used by the high-level API.
"""
from .encoders import EncoderConfig, log_mel_spectrogram
from .fusion import VisionLanguageModel
from .towers import (AudioConfig, AudioConvStack, AudioEncoder, AudioPreprocessor,
                     AudioTokenRoutedMLP, CLIPVisionEncoder, ConcatProjection, CrossAttention,
                     CrossAttentionBlock, CrossAttentionFusion, FusionConfig,
                     FusionTokenRoutedMLP, GatedFusion, MelSpectrogramEncoder, MultimodalFusion,
                     PatchEmbedding, PerceiverResampler, PositionRoutedMLP, SigLIPEncoder,
                     SpatioTemporalBlock, TubeletEmbedding, VideoConfig, VideoEncoder,
                     VideoTokenRoutedMLP, VideoTransformer, VisionConfig, VisionEncoder,
                     VisionLanguageConnector, VisionTokenRoutedMLP, VisionTransformer,
                     WhisperEncoder, mel_filterbank)

__all__ = ["VisionEncoder", "VisionConfig", "PatchEmbedding", "VisionTransformer",
           "VisionTokenRoutedMLP", "CLIPVisionEncoder", "SigLIPEncoder", "AudioEncoder",
           "AudioConfig", "MelSpectrogramEncoder", "WhisperEncoder", "AudioConvStack",
           "AudioTokenRoutedMLP", "AudioPreprocessor", "VideoEncoder", "VideoConfig",
           "TubeletEmbedding", "VideoTransformer", "VideoTokenRoutedMLP", "SpatioTemporalBlock",
           "MultimodalFusion", "FusionConfig", "CrossAttentionFusion", "CrossAttention",
           "CrossAttentionBlock", "GatedFusion", "ConcatProjection", "PerceiverResampler",
           "FusionTokenRoutedMLP", "VisionLanguageConnector", "PositionRoutedMLP",
           "EncoderConfig", "VisionLanguageModel", "log_mel_spectrogram", "mel_filterbank"]
