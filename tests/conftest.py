"""Test set-up: the `gpu` marker, the repository on the import path, and the two tiny
configurations that differ in every size and option."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.dirname(os.path.abspath(__file__))):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (run with -m gpu on a B200)")


TINY_A = {
    "architectures": ["LlamaForCausalLM"],
    "hidden_size": 64, "num_hidden_layers": 2, "num_attention_heads": 4, "num_key_value_heads": 2,
    "intermediate_size": 128, "vocab_size": 256, "rms_norm_eps": 1e-5, "max_position_embeddings": 128,
    "rope_theta": 10000.0, "rope_scaling": None, "tie_word_embeddings": True,
}

TINY_B = {
    "architectures": ["LlamaForCausalLM"],
    "hidden_size": 96, "num_hidden_layers": 3, "num_attention_heads": 3, "num_key_value_heads": 1,
    "head_dim": 32, "intermediate_size": 320, "vocab_size": 384, "rms_norm_eps": 1e-6,
    "max_position_embeddings": 256, "rope_theta": 500000.0,
    "rope_scaling": {"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                     "original_max_position_embeddings": 64},
    "tie_word_embeddings": False,
}

# A third shape for longer sequences: sizes that are no power of two, five heads in groups of five.
TINY_C = {
    "architectures": ["LlamaForCausalLM"],
    "hidden_size": 80, "num_hidden_layers": 2, "num_attention_heads": 5, "num_key_value_heads": 5,
    "head_dim": 48, "intermediate_size": 200, "vocab_size": 1000, "rms_norm_eps": 1e-5,
    "max_position_embeddings": 2048, "rope_theta": 10000.0, "tie_word_embeddings": False,
}


# Head sizes that the tensor-core attention kernel takes: 64 with groups of four, 128 with groups of three.
TINY_D = {
    "architectures": ["LlamaForCausalLM"],
    "hidden_size": 128, "num_hidden_layers": 2, "num_attention_heads": 8, "num_key_value_heads": 2,
    "head_dim": 64, "intermediate_size": 256, "vocab_size": 512, "rms_norm_eps": 1e-5,
    "max_position_embeddings": 4096, "rope_theta": 500000.0,
    "rope_scaling": {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                     "original_max_position_embeddings": 256},
    "tie_word_embeddings": True,
}
TINY_E = {
    "architectures": ["LlamaForCausalLM"],
    "hidden_size": 72, "num_hidden_layers": 2, "num_attention_heads": 3, "num_key_value_heads": 1,
    "head_dim": 128, "intermediate_size": 136, "vocab_size": 300, "rms_norm_eps": 1e-6,
    "max_position_embeddings": 1024, "rope_theta": 10000.0, "tie_word_embeddings": False,
}


@pytest.fixture(scope="session")
def tiny_folders(tmp_path_factory):
    """Model folders of the tiny configurations with random weights, made once per session
    in a temporary place. float32 storage keeps the plain implementation and the 32-bit
    engine on the very same numbers."""
    import torch
    from tt_transformers_b200.weights import write_model_folder

    root = tmp_path_factory.mktemp("models")
    out = {}
    for name, cfg, seed, norm_std in (("A", TINY_A, 0, 0.0), ("B", TINY_B, 1, 0.1), ("C", TINY_C, 2, 0.1),
                                      ("D", TINY_D, 3, 0.1), ("E", TINY_E, 4, 0.0)):
        out[name] = write_model_folder(str(root / name), cfg, seed=seed, std=0.02 if name in "AB" else 0.05,
                                       norm_std=norm_std, dtype=torch.float32)
    return out
