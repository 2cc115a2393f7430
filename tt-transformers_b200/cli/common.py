"""What the command lines share: named random models and loading."""

from __future__ import annotations

import tempfile

import torch

LLAMA3_SCALING = {"rope_type": "llama3", "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                  "original_max_position_embeddings": 8192}


def llama_config(hidden, layers, heads, kv_heads, head_dim, inter, factor, tied, vocab=128256):
    return {"architectures": ["LlamaForCausalLM"], "hidden_size": hidden, "num_hidden_layers": layers,
            "num_attention_heads": heads, "num_key_value_heads": kv_heads, "head_dim": head_dim,
            "intermediate_size": inter, "vocab_size": vocab, "rms_norm_eps": 1e-5, "max_position_embeddings": 131072,
            "rope_theta": 500000.0, "rope_scaling": dict(LLAMA3_SCALING, factor=factor), "tie_word_embeddings": tied}


# Layer sizes of the models that the reference ships packages for (src/tt_transformers/models/
# llama32_1b, llama32_3b, llama3_8b), for runs with random weights where no checkpoint is at hand.
RANDOM_MODELS = {
    "llama-3.2-1b": llama_config(2048, 16, 32, 8, 64, 8192, 32.0, True),
    "llama-3.2-3b": llama_config(3072, 28, 24, 8, 128, 8192, 32.0, True),
    "llama-3.1-8b": llama_config(4096, 32, 32, 8, 128, 14336, 8.0, False),
    "tiny": {"architectures": ["LlamaForCausalLM"], "hidden_size": 128, "num_hidden_layers": 2,
             "num_attention_heads": 8, "num_key_value_heads": 2, "head_dim": 64, "intermediate_size": 256,
             "vocab_size": 512, "rms_norm_eps": 1e-5, "max_position_embeddings": 4096, "rope_theta": 10000.0,
             "tie_word_embeddings": True},
}


def load(hf_model, random_model, *, seed=0, **engine_options):
    """An LLM from a model folder, or from a named random model (weights drawn on the GPU)."""
    from ..config.engine import EngineConfig
    from ..engine.llm import LLM, from_pretrained
    from ..engine.step import build_engine
    from ..weights import random_tensors

    if hf_model:
        return from_pretrained(hf_model, **engine_options)
    if random_model not in RANDOM_MODELS:
        raise SystemExit(f"unknown random model {random_model!r}; known: {sorted(RANDOM_MODELS)}")
    cfg = RANDOM_MODELS[random_model]
    n_layers = engine_options.pop("n_layers", None)
    device = engine_options.get("device", "cuda:0")
    tensors = random_tensors(cfg, seed=seed, dtype=torch.bfloat16, device=device)
    engine = build_engine(config_dict=cfg, tensors=tensors, engine_config=EngineConfig(**engine_options),
                          n_layers=n_layers)
    return LLM(engine)
