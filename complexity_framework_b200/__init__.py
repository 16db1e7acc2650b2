"""complexity_framework_b200: a Blackwell (sm_100a) framework for TR-GQA / TR-MHA
decoders with the deterministic token-routed TR-Hash MoE feed-forward.

Public API mirrors the ``complexity`` package of Complexity-ML/complexity-framework:
``ModelConfig``, ``ComplexityModel``, ``tr_hash``, ``parallel``, ``training``,
``inference``.
"""
from .config import PRESET_CONFIGS, ModelConfig, get_preset, tr_hash_200m_config
from .models import ComplexityModel, TransformerBlock

__version__ = "0.1.0"
__all__ = ["ComplexityModel", "ModelConfig", "PRESET_CONFIGS", "TransformerBlock", "get_preset",
           "tr_hash_200m_config"]
