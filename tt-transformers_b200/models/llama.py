"""The Llama dense decoder as a ModelSpec.

Every layer: RMSNorm, grouped-query attention with rotary positions, RMSNorm, SwiGLU,
in a pre-norm block (src/tt_transformers/models/llama32_1b/model.py:113-186); a final
RMSNorm and a head that may be tied to the embedding (:958-995;
src/tt_transformers/models/llama32_1b/hf_generator.py:254-261). Tensor names are the
checkpoint's (hf_generator.py:234-261; weight_utils.py:59-62,96-98).
"""

from __future__ import annotations

from ..config.llama import LlamaConfig
from ..parts import LayerCall, LayerSpec, ModelSpec, PartSpec


def load_config(data: dict) -> LlamaConfig:
    return LlamaConfig.from_dict(data)


def model_spec(cfg: LlamaConfig) -> ModelSpec:
    rotary = PartSpec("rotary", dict(
        rotary_dim=cfg.head_dim, theta=cfg.rope_theta,
        scaling=cfg.rope_scaling.to_dict() if cfg.rope_scaling else None))
    layers = []
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        layers.append(LayerSpec(
            norm1=PartSpec("rmsnorm", dict(width=cfg.hidden_size, eps=cfg.rms_norm_eps,
                                           weight_name=p + "input_layernorm.weight")),
            mixer=PartSpec("attention", dict(width=cfg.hidden_size, heads=cfg.num_attention_heads,
                                             kv_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim,
                                             prefix=p + "self_attn.")),
            position=rotary,
            norm2=PartSpec("rmsnorm", dict(width=cfg.hidden_size, eps=cfg.rms_norm_eps,
                                           weight_name=p + "post_attention_layernorm.weight")),
            feed_forward=PartSpec("swiglu", dict(width=cfg.hidden_size, inter=cfg.intermediate_size,
                                                 prefix=p + "mlp.")),
        ))
    return ModelSpec(
        vocab_size=cfg.vocab_size,
        width=cfg.hidden_size,
        embedding=PartSpec("table", dict(vocab=cfg.vocab_size, width=cfg.hidden_size,
                                         weight_name="model.embed_tokens.weight")),
        layers=tuple(layers),
        order=tuple(LayerCall(i) for i in range(cfg.num_hidden_layers)),
        final_norm=PartSpec("rmsnorm", dict(width=cfg.hidden_size, eps=cfg.rms_norm_eps, weight_name="model.norm.weight")),
        head=PartSpec("linear", dict(vocab=cfg.vocab_size, width=cfg.hidden_size,
                                     weight_name=None if cfg.tie_word_embeddings else "lm_head.weight")),
        max_positions=cfg.max_position_embeddings,
    )


# Tensors that a checkpoint may carry without the model using them.
def ignorable(cfg: LlamaConfig, name: str) -> bool:
    if name.endswith("rotary_emb.inv_freq"):
        return True
    return cfg.tie_word_embeddings and name == "lm_head.weight"
