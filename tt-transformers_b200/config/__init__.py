"""Typed configurations: the model's (from config.json) and the engine's."""

from .base import ConfigError, read_config_json
from .engine import EngineConfig
from .llama import LlamaConfig, RopeScaling

__all__ = ["ConfigError", "EngineConfig", "LlamaConfig", "RopeScaling", "read_config_json"]
