"""Weight reading, checking and random initialisation (no GPU)."""

import json
import os

import pytest
import torch
from safetensors.torch import load_file, save_file

from conftest import TINY_A, TINY_B
from tt_transformers_b200.parts import DecoderModel
from tt_transformers_b200.registry import get_architecture
from tt_transformers_b200.weights import (WeightError, check_tensors, random_tensors, read_safetensors,
                                          write_model_folder)


def specs_of(cfg):
    arch = get_architecture("LlamaForCausalLM")
    return DecoderModel(arch.model_spec(arch.load_config(cfg))).tensor_specs()


def test_random_folder_reads_back(tmp_path):
    folder = write_model_folder(str(tmp_path / "m"), TINY_B, seed=1, norm_std=0.1)
    assert sorted(os.listdir(folder)) == ["config.json", "model.safetensors"]
    with open(os.path.join(folder, "config.json")) as f:
        assert json.load(f)["hidden_size"] == 96
    tensors = read_safetensors(folder)
    check_tensors(tensors, specs_of(TINY_B))
    assert tensors["model.layers.2.self_attn.k_proj.weight"].shape == (32, 96)
    assert tensors["lm_head.weight"].dtype == torch.bfloat16
    assert "lm_head.weight" not in read_safetensors(write_model_folder(str(tmp_path / "a"), TINY_A, seed=0))


def test_same_seed_same_weights_other_seed_other_weights():
    a, b, c = random_tensors(TINY_A, 3), random_tensors(TINY_A, 3), random_tensors(TINY_A, 4)
    assert all(torch.equal(a[k], b[k]) for k in a)
    assert not torch.equal(a["model.embed_tokens.weight"], c["model.embed_tokens.weight"])
    assert torch.equal(a["model.norm.weight"], torch.ones(64, dtype=torch.bfloat16))
    assert float(random_tensors(TINY_A, 3, norm_std=0.1)["model.norm.weight"].float().std()) > 0.01


def test_stored_precision(tmp_path):
    tensors = random_tensors(TINY_A, 0, dtype=torch.float32)
    tensors["model.norm.weight"] = tensors["model.norm.weight"].to(torch.float16)
    tensors["model.layers.0.input_layernorm.weight"] = tensors["model.layers.0.input_layernorm.weight"].to(torch.bfloat16)
    tensors["extra.table"] = torch.arange(6, dtype=torch.int64).reshape(2, 3)
    os.makedirs(tmp_path / "m")
    save_file(tensors, str(tmp_path / "m" / "model.safetensors"))
    got = read_safetensors(str(tmp_path / "m"))
    assert got["model.embed_tokens.weight"].dtype == torch.float32        # stored in 32-bit: stays so
    assert got["model.norm.weight"].dtype == torch.bfloat16               # 16-bit floats are kept as bfloat16
    assert got["model.layers.0.input_layernorm.weight"].dtype == torch.bfloat16
    assert got["extra.table"].dtype == torch.int32                        # integer tables
    # for an engine that computes in float32, float16 keeps every bit of its mantissa
    wide = read_safetensors(str(tmp_path / "m"), widen_float16=True)
    assert wide["model.norm.weight"].dtype == torch.float32
    assert torch.equal(wide["model.norm.weight"], tensors["model.norm.weight"].float())
    assert wide["model.layers.0.input_layernorm.weight"].dtype == torch.bfloat16


def test_one_error_lists_everything(tmp_path):
    tensors = random_tensors(TINY_B, 1)
    del tensors["model.layers.1.mlp.up_proj.weight"]
    del tensors["model.norm.weight"]
    tensors["model.layers.0.self_attn.q_proj.weight"] = torch.zeros(96, 95, dtype=torch.bfloat16)
    tensors["model.layers.7.mlp.gate_proj.weight"] = torch.zeros(2, 2, dtype=torch.bfloat16)
    tensors["model.layers.0.input_layernorm.weight"] = torch.zeros(96, dtype=torch.int32)
    with pytest.raises(WeightError) as e:
        check_tensors(tensors, specs_of(TINY_B))
    text = str(e.value)
    assert "missing tensors (2)" in text and "model.layers.1.mlp.up_proj.weight [320, 96]" in text
    assert "model.norm.weight" in text
    assert "unexpected tensors (1)" in text and "model.layers.7.mlp.gate_proj.weight" in text
    assert "wrong shapes or kinds (2)" in text and "shape [96, 95], expected [96, 96]" in text
    assert "expected floating-point" in text


def test_tied_head_in_the_checkpoint_may_go_unused(tmp_path):
    arch = get_architecture("LlamaForCausalLM")
    cfg = arch.load_config(TINY_A)
    tensors = random_tensors(TINY_A, 0)
    tensors["lm_head.weight"] = tensors["model.embed_tokens.weight"].clone()
    tensors["model.layers.0.self_attn.rotary_emb.inv_freq"] = torch.zeros(8)
    check_tensors(tensors, specs_of(TINY_A), ignorable=lambda n: arch.ignorable(cfg, n))
    with pytest.raises(WeightError, match="unexpected"):
        check_tensors(tensors, specs_of(TINY_A))
    untied = random_tensors(TINY_B, 0)
    del untied["lm_head.weight"]
    with pytest.raises(WeightError, match="lm_head.weight"):
        check_tensors(untied, specs_of(TINY_B))


def test_sharded_checkpoint(tmp_path):
    tensors = random_tensors(TINY_A, 0)
    names = sorted(tensors)
    folder = tmp_path / "m"
    os.makedirs(folder)
    half = len(names) // 2
    parts = {"model-00001-of-00002.safetensors": names[:half], "model-00002-of-00002.safetensors": names[half:]}
    weight_map = {}
    for fname, keys in parts.items():
        save_file({k: tensors[k] for k in keys}, str(folder / fname))
        weight_map.update({k: fname for k in keys})
    with open(folder / "model.safetensors.index.json", "w") as f:
        json.dump({"weight_map": weight_map}, f)
    got = read_safetensors(str(folder))
    check_tensors(got, specs_of(TINY_A))
    assert torch.equal(got[names[0]], tensors[names[0]])
    with pytest.raises(WeightError, match="no .safetensors"):
        os.makedirs(tmp_path / "empty")
        read_safetensors(str(tmp_path / "empty"))


def test_reading_only_what_is_wanted(tmp_path):
    folder = write_model_folder(str(tmp_path / "m"), TINY_B, seed=1)
    got = read_safetensors(folder, wanted=["model.norm.weight"])
    assert set(got) == {"model.norm.weight", "__unread__"}
    assert got["__unread__"]["lm_head.weight"] == (384, 96)
    assert load_file(os.path.join(folder, "model.safetensors"))["model.norm.weight"].shape == (96,)
