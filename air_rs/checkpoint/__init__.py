"""Non-GGUF checkpoints: safetensors files (read / write) and Hugging Face model
directories converted to this framework's tensor records."""
from .safetensors import SafetensorsFile, load_safetensors, save_safetensors  # noqa: F401
from .hf import hf_config, hf_records  # noqa: F401
