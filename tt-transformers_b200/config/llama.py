"""The Llama dense decoder's configuration, read from its own config.json keys.

Which keys the reference reads: hidden_size, num_attention_heads,
num_key_value_heads, intermediate_size, vocab_size, rms_norm_eps
(src/tt_transformers/models/llama32_1b/hf_generator.py:312-323), num_hidden_layers
(:293), tie_word_embeddings (:254), max_position_embeddings (:350), and the rope
keys rope_theta and rope_scaling / rope_parameters with rope_type "llama3"
(src/tt_transformers/models/llama3_8b/hf_generator.py:55-66).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

from .base import ConfigError, require, take


@dataclass(frozen=True)
class RopeScaling:
    """Llama-3 per-frequency scaling of the rotation frequencies."""

    factor: float
    low_freq_factor: float
    high_freq_factor: float
    original_max_position_embeddings: int

    def to_dict(self) -> dict:
        return {
            "rope_type": "llama3",
            "factor": self.factor,
            "low_freq_factor": self.low_freq_factor,
            "high_freq_factor": self.high_freq_factor,
            "original_max_position_embeddings": self.original_max_position_embeddings,
        }


@dataclass(frozen=True)
class LlamaConfig:
    architecture: str
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    intermediate_size: int
    vocab_size: int
    rms_norm_eps: float
    max_position_embeddings: int
    rope_theta: float
    rope_scaling: Optional[RopeScaling]
    tie_word_embeddings: bool
    eos_token_ids: tuple = ()
    bos_token_id: Optional[int] = None

    @classmethod
    def from_dict(cls, data: dict) -> "LlamaConfig":
        archs = data.get("architectures")
        require(isinstance(archs, list) and len(archs) >= 1 and isinstance(archs[0], str),
                "config.json: 'architectures' must be a list holding the model class name")
        hidden = take(data, "hidden_size", int)
        heads = take(data, "num_attention_heads", int)
        kv_heads = take(data, "num_key_value_heads", int, heads)
        require(heads >= 1 and kv_heads >= 1, "config.json: head counts must be positive")
        require(heads % kv_heads == 0,
                f"config.json: 'num_attention_heads' ({heads}) must be a multiple of "
                f"'num_key_value_heads' ({kv_heads})")
        head_dim = take(data, "head_dim", int, None)
        if head_dim is None:
            require(hidden % heads == 0,
                    f"config.json: 'hidden_size' ({hidden}) is no multiple of "
                    f"'num_attention_heads' ({heads}) and no 'head_dim' is given")
            head_dim = hidden // heads
        require(head_dim >= 2 and head_dim % 2 == 0,
                f"config.json: 'head_dim' ({head_dim}) must be even: rotation pairs element i with i + head_dim/2")
        act = take(data, "hidden_act", str, "silu")
        require(act == "silu", f"config.json: 'hidden_act' {act!r} is not supported (the feed-forward is SwiGLU: 'silu')")
        for key in ("attention_bias", "mlp_bias"):
            require(not take(data, key, bool, False), f"config.json: '{key}' true is not supported")

        rope_parameters = data.get("rope_parameters") or {}
        require(isinstance(rope_parameters, dict), "config.json: 'rope_parameters' must be an object")
        theta = take(data, "rope_theta", float, None)
        if theta is None:
            theta = take(rope_parameters, "rope_theta", float, 10000.0, where="config.json rope_parameters")
        scaling_dict = data.get("rope_scaling")
        if scaling_dict is None and ("rope_type" in rope_parameters or "type" in rope_parameters):
            scaling_dict = rope_parameters
        scaling = None
        if scaling_dict is not None:
            require(isinstance(scaling_dict, dict), "config.json: 'rope_scaling' must be an object or null")
            where = "config.json rope_scaling"
            kind = scaling_dict.get("rope_type", scaling_dict.get("type", "default"))
            if kind == "llama3":
                scaling = RopeScaling(
                    factor=take(scaling_dict, "factor", float, where=where),
                    low_freq_factor=take(scaling_dict, "low_freq_factor", float, where=where),
                    high_freq_factor=take(scaling_dict, "high_freq_factor", float, where=where),
                    original_max_position_embeddings=take(
                        scaling_dict, "original_max_position_embeddings", int, where=where),
                )
                require(scaling.high_freq_factor != scaling.low_freq_factor,
                        f"{where}: 'high_freq_factor' must differ from 'low_freq_factor'")
            elif kind != "default":
                raise ConfigError(f"{where}: rope_type {kind!r} is not supported (known: 'default', 'llama3')")

        eos = data.get("eos_token_id")
        if eos is None:
            eos_ids = ()
        elif isinstance(eos, int):
            eos_ids = (eos,)
        elif isinstance(eos, list) and all(isinstance(e, int) for e in eos):
            eos_ids = tuple(eos)
        else:
            raise ConfigError(f"config.json: 'eos_token_id' must be an integer or a list of integers, got {eos!r}")

        cfg = cls(
            architecture=archs[0],
            hidden_size=hidden,
            num_hidden_layers=take(data, "num_hidden_layers", int),
            num_attention_heads=heads,
            num_key_value_heads=kv_heads,
            head_dim=head_dim,
            intermediate_size=take(data, "intermediate_size", int),
            vocab_size=take(data, "vocab_size", int),
            rms_norm_eps=take(data, "rms_norm_eps", float),
            max_position_embeddings=take(data, "max_position_embeddings", int),
            rope_theta=theta,
            rope_scaling=scaling,
            tie_word_embeddings=take(data, "tie_word_embeddings", bool, False),
            eos_token_ids=eos_ids,
            bos_token_id=take(data, "bos_token_id", int, None),
        )
        for key in ("hidden_size", "num_hidden_layers", "intermediate_size", "vocab_size", "max_position_embeddings"):
            require(getattr(cfg, key) >= 1, f"config.json: '{key}' must be positive")
        require(cfg.rms_norm_eps > 0, "config.json: 'rms_norm_eps' must be positive")
        require(cfg.rope_theta > 0, "config.json: 'rope_theta' must be positive")
        return cfg

    def with_layers(self, n_layers: int) -> "LlamaConfig":
        """The same model cut to its first n_layers blocks (the reference's n_layers
        argument, src/tt_transformers/models/llama32_1b/hf_generator.py:274)."""
        from dataclasses import replace

        require(1 <= n_layers <= self.num_hidden_layers, f"n_layers must be in 1..{self.num_hidden_layers}")
        return replace(self, num_hidden_layers=n_layers)

    def to_dict(self) -> dict:
        out = {
            "architectures": [self.architecture],
            "model_type": "llama",
            "hidden_size": self.hidden_size,
            "num_hidden_layers": self.num_hidden_layers,
            "num_attention_heads": self.num_attention_heads,
            "num_key_value_heads": self.num_key_value_heads,
            "head_dim": self.head_dim,
            "intermediate_size": self.intermediate_size,
            "vocab_size": self.vocab_size,
            "rms_norm_eps": self.rms_norm_eps,
            "max_position_embeddings": self.max_position_embeddings,
            "rope_theta": self.rope_theta,
            "rope_scaling": self.rope_scaling.to_dict() if self.rope_scaling else None,
            "tie_word_embeddings": self.tie_word_embeddings,
            "hidden_act": "silu",
            "attention_bias": False,
            "mlp_bias": False,
        }
        if self.eos_token_ids:
            out["eos_token_id"] = list(self.eos_token_ids) if len(self.eos_token_ids) > 1 else self.eos_token_ids[0]
        if self.bos_token_id is not None:
            out["bos_token_id"] = self.bos_token_id
        return out
