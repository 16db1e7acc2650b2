"""Models beyond text-only autoregression on the TR-Hash engine: vision and
video towers, object detection and other vision tasks, audio (speech-to-text,
text-to-speech), image-text-to-text, text-to-image / image editing and
multimodal sensor fusion.

Counterpart: complexity/generative/ (same public names).  Non-text tokens
(patches, frames, latent patches, sensor samples) route through the experts
by position, as text tokens route by id; on CUDA bf16 the feed-forwards run
on the fused sm_100a TR-Hash GEMMs.
"""
from .audio import (AudioEncoder, AudioEncoderConfig, LogMelSpectrogram, TRHashAudioConfig,
                    TRHashSpeechToText, TRHashSpeechToTextConfig, TRHashTextToSpeech,
                    build_mel_filterbank)
from .detection import TRHashDetectorConfig, TRHashObjectDetector
from .hierarchical import (HierarchicalTowerConfig, HierarchicalTRHashVisionClassifier,
                           HierarchicalTRHashVisionTower)
from .image import (FrozenAutoencoderKL, TRHashImageConfig, TRHashImageEditConfig,
                    TRHashImageEditor, TRHashTextToImage)
from .prefix_lm import PrefixLM, TokenResampler
from .sensor_fusion import (SENSOR_MODALITIES, TRHashSensorFusionBlock,
                            TRHashSensorFusionClassifier, TRHashSensorFusionConfig)
from .sensor_structured import IMUDeviceGraphTokenizer, SkeletonGraphTokenizer, gradient_reverse
from .towers import (TRHashVideoBlock, TRHashVideoClassifier, TRHashVideoTower,
                     TRHashVideoTowerConfig, TRHashVisionBlock, TRHashVisionClassifier,
                     TRHashVisionTower, TRHashVisionTowerConfig)
from .vision_language import (TRHashImageTextToText, TRHashVisionLanguageConfig,
                              VisualTokenResampler)
from .vision_tasks import (SUPPORTED_VISION_TASKS, TRHashDepthEstimator, TRHashImageClassifier,
                           TRHashInstanceSegmenter, TRHashOBBDetector, TRHashPoseEstimator,
                           TRHashSemanticSegmenter, create_vision_model,
                           load_vision_task_checkpoint, save_vision_task_checkpoint)

__all__ = ["IMUDeviceGraphTokenizer", "SkeletonGraphTokenizer", "gradient_reverse",
           
    "TRHashImageTextToText", "TRHashVisionLanguageConfig", "TRHashVisionTower",
    "TRHashVisionTowerConfig", "TRHashVisionBlock", "TRHashVisionClassifier",
    "VisualTokenResampler", "TRHashSpeechToText", "TRHashSpeechToTextConfig",
    "TRHashTextToSpeech", "TRHashAudioConfig", "AudioEncoder", "AudioEncoderConfig",
    "LogMelSpectrogram", "build_mel_filterbank", "TokenResampler", "PrefixLM",
    "TRHashVideoTower", "TRHashVideoTowerConfig", "TRHashVideoBlock", "TRHashVideoClassifier",
    "TRHashObjectDetector", "TRHashDetectorConfig", "TRHashSensorFusionClassifier",
    "TRHashSensorFusionConfig", "TRHashSensorFusionBlock", "SENSOR_MODALITIES",
    "SUPPORTED_VISION_TASKS", "TRHashDepthEstimator", "TRHashImageClassifier",
    "TRHashInstanceSegmenter", "TRHashOBBDetector", "TRHashPoseEstimator",
    "TRHashSemanticSegmenter", "create_vision_model", "load_vision_task_checkpoint",
    "save_vision_task_checkpoint", "FrozenAutoencoderKL", "TRHashImageConfig",
    "TRHashImageEditConfig", "TRHashImageEditor", "TRHashTextToImage",
    "HierarchicalTowerConfig", "HierarchicalTRHashVisionTower", "HierarchicalTRHashVisionClassifier",
]
