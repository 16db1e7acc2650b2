from .model_config import PRESET_CONFIGS, ModelConfig, get_preset, tr_hash_200m_config

__all__ = ["ModelConfig", "PRESET_CONFIGS", "get_preset", "tr_hash_200m_config"]
