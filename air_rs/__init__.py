"""air_rs — a B200-native (sm_100a) LLM inference engine with Air.rs's public surface."""
__version__ = "1.3.0"
