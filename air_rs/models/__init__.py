"""Model definitions: configs from GGUF metadata, device weights, the CPU oracle."""
from .config import ModelConfig, ModelVariant, NormType, FfnType, PRESETS

__all__ = ["ModelConfig", "ModelVariant", "NormType", "FfnType", "PRESETS"]
