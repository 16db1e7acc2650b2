"""Multimodal encoders and fusion on top of the TR-Hash decoder."""
from .encoders import (AudioEncoder, EncoderConfig, PatchEmbedding, VideoEncoder, VisionEncoder,
                       log_mel_spectrogram)
from .fusion import (ConcatProjection, CrossAttentionFusion, GatedFusion, PerceiverResampler,
                     VisionLanguageConnector, VisionLanguageModel)
