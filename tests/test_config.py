"""Configuration and registry (no GPU)."""

import copy

import pytest

from conftest import TINY_A, TINY_B
from tt_transformers_b200.config import ConfigError, EngineConfig, LlamaConfig
from tt_transformers_b200.registry import (UnknownArchitecture, architecture_of, get_architecture,
                                           known_architectures, register_architecture)


def test_reads_every_size_from_its_own_keys():
    a, b = LlamaConfig.from_dict(TINY_A), LlamaConfig.from_dict(TINY_B)
    assert (a.hidden_size, a.num_hidden_layers, a.num_attention_heads, a.num_key_value_heads) == (64, 2, 4, 2)
    assert a.head_dim == 16 and a.rope_scaling is None and a.tie_word_embeddings and a.rms_norm_eps == 1e-5
    assert (b.head_dim, b.intermediate_size, b.vocab_size, b.rope_theta) == (32, 320, 384, 500000.0)
    assert b.rope_scaling.factor == 32.0 and b.rope_scaling.original_max_position_embeddings == 64
    assert not b.tie_word_embeddings and b.rms_norm_eps == 1e-6


def test_round_trip_through_a_dictionary():
    for cfg in (TINY_A, TINY_B):
        c = LlamaConfig.from_dict(cfg)
        assert LlamaConfig.from_dict(c.to_dict()) == c


def test_defaults_and_other_spellings():
    d = copy.deepcopy(TINY_A)
    del d["num_key_value_heads"], d["rope_theta"], d["rope_scaling"], d["tie_word_embeddings"]
    c = LlamaConfig.from_dict(d)
    assert c.num_key_value_heads == 4 and c.rope_theta == 10000.0 and not c.tie_word_embeddings
    d = copy.deepcopy(TINY_B)
    scaling = d.pop("rope_scaling")
    d.pop("rope_theta")
    d["rope_parameters"] = dict(scaling, rope_theta=12345.0)
    c = LlamaConfig.from_dict(d)
    assert c.rope_theta == 12345.0 and c.rope_scaling.high_freq_factor == 4.0
    d["rope_parameters"] = {"rope_type": "default", "rope_theta": 777.0}
    assert LlamaConfig.from_dict(d).rope_scaling is None
    d = dict(TINY_A, eos_token_id=[5, 6], bos_token_id=1)
    c = LlamaConfig.from_dict(d)
    assert c.eos_token_ids == (5, 6) and c.bos_token_id == 1


@pytest.mark.parametrize("key", ["hidden_size", "num_hidden_layers", "num_attention_heads", "intermediate_size",
                                 "vocab_size", "rms_norm_eps", "max_position_embeddings"])
def test_a_missing_key_is_named(key):
    d = copy.deepcopy(TINY_A)
    del d[key]
    with pytest.raises(ConfigError, match=key):
        LlamaConfig.from_dict(d)


@pytest.mark.parametrize("change,match", [
    ({"hidden_size": "64"}, "hidden_size"),
    ({"num_key_value_heads": 3}, "num_key_value_heads"),
    ({"hidden_act": "gelu"}, "hidden_act"),
    ({"attention_bias": True}, "attention_bias"),
    ({"mlp_bias": True}, "mlp_bias"),
    ({"rope_scaling": {"rope_type": "yarn", "factor": 2.0}}, "yarn"),
    ({"rope_scaling": {"rope_type": "llama3", "factor": 2.0}}, "low_freq_factor"),
    ({"head_dim": 15}, "head_dim"),
    ({"tie_word_embeddings": "yes"}, "tie_word_embeddings"),
    ({"rms_norm_eps": 0}, "rms_norm_eps"),
    ({"architectures": []}, "architectures"),
    ({"hidden_size": 66, "head_dim": None}, "hidden_size"),
])
def test_unsupported_values_are_refused(change, match):
    d = copy.deepcopy(TINY_A)
    d.update(change)
    with pytest.raises(ConfigError, match=match):
        LlamaConfig.from_dict(d)


def test_with_layers():
    c = LlamaConfig.from_dict(TINY_B)
    assert c.with_layers(2).num_hidden_layers == 2
    with pytest.raises(ConfigError):
        c.with_layers(4)


def test_registry():
    assert "LlamaForCausalLM" in known_architectures()
    arch = get_architecture("LlamaForCausalLM")
    spec = arch.model_spec(arch.load_config(TINY_B))
    assert len(spec.layers) == 3 and spec.head.params["weight_name"] == "lm_head.weight" and spec.vocab_size == 384
    assert arch.model_spec(arch.load_config(TINY_A)).head.params["weight_name"] is None
    with pytest.raises(UnknownArchitecture, match="LlamaForCausalLM"):
        get_architecture("NoSuchModelForCausalLM")
    assert architecture_of(TINY_A) == "LlamaForCausalLM"
    with pytest.raises(ConfigError):
        architecture_of({})
    register_architecture("ToyForTests", arch.load_config, arch.model_spec)
    assert get_architecture("ToyForTests").model_spec is arch.model_spec


def test_engine_config():
    c = EngineConfig(page_size=8, max_batch_size=3, max_seq_len=100)
    assert c.pages_per_request == 13 and c.resolved_num_pages() == 39
    assert EngineConfig(num_pages=7).resolved_num_pages() == 7
    for bad in (dict(dtype="float16"), dict(page_size=0), dict(num_pages=0), dict(max_step_tokens=-1)):
        with pytest.raises(ConfigError):
            EngineConfig(**bad)


def test_engine_config_options():
    from tt_transformers_b200.config import EngineConfig
    from tt_transformers_b200.config.base import ConfigError

    c = EngineConfig(graph_batch_sizes=[1, 2, 6], gpu_memory_fraction=0.5, admission="conservative")
    assert c.graph_batch_sizes == (1, 2, 6)
    for bad in (dict(graph_batch_sizes=(4, 2)), dict(graph_batch_sizes=()), dict(gpu_memory_fraction=0.0),
                dict(gpu_memory_fraction=1.5), dict(admission="greedy")):
        with pytest.raises(ConfigError):
            EngineConfig(**bad)


def test_bytes_per_page():
    import torch

    from tt_transformers_b200.cache import CacheManager
    from tt_transformers_b200.parts import PagedKV, SlotState

    requests = [PagedKV(2, 16), PagedKV(2, 16), None, 0, PagedKV(1, 8, window=4), SlotState((3,))]
    # two units of K and V pages of 2 x 4 x 16 bfloat16, one unit of 1 x 4 x 8
    assert CacheManager.bytes_per_page(requests, 4, torch.bfloat16) == 2 * 2 * (2 * 4 * 16) * 2 + 2 * (4 * 8) * 2
