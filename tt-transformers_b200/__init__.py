"""tt_transformers_b200: a single-GPU inference engine for NVIDIA B200 (sm_100a).

From a model folder (config.json + safetensors) to generated tokens: a typed configuration
and an architecture registry, layers put together from parts, a paged cache manager, one
step function for mixed batches, a scheduler with sampling, and hand-written CUDA kernels.
"""

__version__ = "0.1.0"

_LAZY = {
    "LLM": ("tt_transformers_b200.engine.llm", "LLM"),
    "from_pretrained": ("tt_transformers_b200.engine.llm", "from_pretrained"),
    "SamplingParams": ("tt_transformers_b200.sampling.params", "SamplingParams"),
    "EngineConfig": ("tt_transformers_b200.config.engine", "EngineConfig"),
    "Engine": ("tt_transformers_b200.engine.step", "Engine"),
    "StepEntry": ("tt_transformers_b200.engine.step", "StepEntry"),
    "build_engine": ("tt_transformers_b200.engine.step", "build_engine"),
    "register_architecture": ("tt_transformers_b200.registry", "register_architecture"),
    "register_part": ("tt_transformers_b200.parts.base", "register_part"),
}


def __getattr__(name):
    if name in _LAZY:
        import importlib

        module, attr = _LAZY[name]
        return getattr(importlib.import_module(module), attr)
    raise AttributeError(f"module 'tt_transformers_b200' has no attribute {name!r}")
