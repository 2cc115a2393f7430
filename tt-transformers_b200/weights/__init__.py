"""Reading checkpoints by tensor name, and making random ones."""

from .loader import WeightError, check_tensors, read_safetensors
from .random_init import random_tensors, write_model_folder

__all__ = ["WeightError", "check_tensors", "read_safetensors", "random_tensors", "write_model_folder"]
