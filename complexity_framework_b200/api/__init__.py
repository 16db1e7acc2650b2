"""High-level API: the ``Model`` facade plus the factory namespaces of the
reference's ``complexity.api`` (building blocks, helpers, small-budget tools,
tokenizer / data / trainer / generation facades, multimodal factories).

Counterpart of complexity/api/__init__.py:60-330; the Triton facade has no
counterpart (this framework runs its own sm_100a kernels; ``CUDA`` names the
attention variants and ``CUDA.kernels_available()`` reports the extension).
"""
from .blocks import (ATTENTION_REGISTRY, CUDA, MLP, MLP_REGISTRY, MODEL_REGISTRY,
                     NORMALIZATION_REGISTRY, POSITION_REGISTRY, ALiBiPositionalBias, Attention,
                     AttentionConfig, Block, DynamicNTKRotaryEmbedding, GroupedQueryAttention,
                     IdentityNorm, LayerNorm, LearnedPositionalEmbedding, MLPConfig, Norm,
                     Position, Registry, RMSNorm, RotaryEmbedding, TransformerBlock,
                     YaRNRotaryEmbedding, apply_rotary_pos_emb, register, register_attention,
                     register_mlp, register_model, register_normalization, register_position,
                     rotate_half)
from .efficient import (Efficient, MemoryEfficient, MixedPrecision, QuantConfig, Quantize,
                        QuantizedLinear, SmallModels)
from .helpers import (Checkpointing, Debug, Helpers, Init, KVCache, Mask, Sampling,
                      SlidingWindowCache, Tensors)
from .model import Model, load
from .multimodal import (Audio, AudioConfig, Fusion, FusionConfig, Omni, Robot, Video, Vision,
                         VisionConfig)
from .runtime import (DataConfig, DataPipeline, Dataset, DecodingStrategy, Generate,
                      GenerationConfig, InferenceConfig, InferenceEngine, StreamingDataset,
                      Tokenizer, TokenizerConfig, Trainer, TrainerConfig, create_engine)
from ..config.model_config import ModelConfig
from ..models.builder import ComplexityModel

# reference aliases
StandardRoPE = RoPE = RotaryEmbedding
YaRN = YaRNRoPE = YaRNRotaryEmbedding
DynamicNTKRoPE = DynamicNTKRotaryEmbedding
ALiBi = ALiBiPositionBias = ALiBiPositionalBias
LearnedPositionEmbedding = LearnedPositionalEmbedding
MultiHeadAttention = MultiQueryAttention = GroupedQueryAttention
build_norm = Norm.create


def GQA(hidden_size: int, num_heads: int, kv_heads=None, **kw):  # noqa: N802
    return Attention.gqa(hidden_size, num_heads, kv_heads, **kw)


def MHA(hidden_size: int, num_heads: int, **kw):  # noqa: N802
    return Attention.mha(hidden_size, num_heads, **kw)


def MQA(hidden_size: int, num_heads: int, **kw):  # noqa: N802
    return Attention.mqa(hidden_size, num_heads, **kw)


__all__ = [
    "Model", "load", "ModelConfig", "ComplexityModel",
    "Tokenizer", "TokenizerConfig", "Dataset", "DataConfig", "StreamingDataset", "DataPipeline",
    "Trainer", "TrainerConfig",
    "Attention", "MLP", "Position", "Norm", "Block", "CUDA",
    "GQA", "MHA", "MQA", "GroupedQueryAttention", "MultiHeadAttention", "MultiQueryAttention",
    "AttentionConfig", "MLPConfig",
    "RoPE", "StandardRoPE", "YaRN", "YaRNRoPE", "DynamicNTKRoPE", "ALiBi", "ALiBiPositionBias",
    "LearnedPositionEmbedding", "RotaryEmbedding", "rotate_half", "apply_rotary_pos_emb",
    "RMSNorm", "LayerNorm", "IdentityNorm", "build_norm", "TransformerBlock",
    "Registry", "register", "ATTENTION_REGISTRY", "MLP_REGISTRY", "NORMALIZATION_REGISTRY",
    "POSITION_REGISTRY", "MODEL_REGISTRY", "register_attention", "register_mlp",
    "register_normalization", "register_position", "register_model",
    "Helpers", "Init", "Mask", "KVCache", "SlidingWindowCache", "Sampling", "Tensors", "Debug",
    "Checkpointing",
    "Efficient", "Quantize", "QuantConfig", "QuantizedLinear", "MixedPrecision",
    "MemoryEfficient", "SmallModels",
    "Generate", "GenerationConfig", "InferenceEngine", "InferenceConfig", "DecodingStrategy",
    "create_engine",
    "Vision", "VisionConfig", "Audio", "AudioConfig", "Video", "Fusion", "FusionConfig",
    "Robot", "Omni",
]
