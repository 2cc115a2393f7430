"""Plain, slow Llama forward pass: the oracle that the engine is compared with.

Whole sequences, no cache, no paging, 32-bit floats on the CPU, one function per
part. It shares no code with the package: it reads config.json and the safetensors
file by itself.

The reference's own model code cannot run here (every forward op is a call into
its accelerator library, which is not installed), so this file rests on the
formulas that the reference's code, tests and notes pin down; each function cites
the file and line (paths relative to the reference project's root).
"""

from __future__ import annotations

import json
import math
import os

import torch
from safetensors import safe_open


def read_model_folder(folder):
    """config.json as a dict and every tensor of model.safetensors as float32."""
    with open(os.path.join(folder, "config.json")) as f:
        config = json.load(f)
    tensors = {}
    with safe_open(os.path.join(folder, "model.safetensors"), framework="pt", device="cpu") as f:
        for name in f.keys():
            tensors[name] = f.get_tensor(name).to(torch.float32)
    return config, tensors


def head_dim_of(config):
    # src/tt_transformers/models/llama32_1b/hf_generator.py:312-318 derives
    # head_dim = hidden_size // num_attention_heads; a "head_dim" key, where the
    # checkpoint has one, is the same number spelled out.
    return int(config.get("head_dim") or config["hidden_size"] // config["num_attention_heads"])


def rope_settings(config):
    """(theta, scaling dict or None) from either spelling of the rope keys.

    tests/models/llama32_1b/test_hf_adaptor.py:20-27 (rope_scaling / rope_parameters
    with rope_type "llama3").
    """
    params = config.get("rope_parameters") or {}
    theta = config.get("rope_theta", params.get("rope_theta", 10000.0))
    scaling = config.get("rope_scaling") or (params if params.get("rope_type") else None)
    if scaling is not None:
        kind = scaling.get("rope_type", scaling.get("type", "default"))
        if kind == "default":
            scaling = None
        elif kind != "llama3":
            raise ValueError(f"plain implementation knows only llama3 rope scaling, not {kind}")
    return float(theta), scaling


def rope_inverse_frequencies(head_dim, theta, scaling):
    """theta_i = theta^(-2i/hd), then the llama3 per-frequency scaling.

    src/tt_transformers/models/llama3_8b/hf_generator.py:88-103 (scaling) and
    :106-120 (base frequencies); tests/modules/rope/test_rope_1d.py:49-66.
    """
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))
    if scaling is None:
        return inv_freq
    factor = float(scaling["factor"])
    low = float(scaling["low_freq_factor"])
    high = float(scaling["high_freq_factor"])
    original = float(scaling["original_max_position_embeddings"])
    wavelen = 2 * math.pi / inv_freq
    smooth = (original / wavelen - low) / (high - low)
    blended = (1 - smooth) * inv_freq / factor + smooth * inv_freq
    scaled = torch.where(wavelen > original / low, inv_freq / factor, blended)
    return torch.where(wavelen < original / high, inv_freq, scaled)


def rope_rotate(x, positions, inv_freq):
    """Rotate [T, heads, hd] by the angles positions x inv_freq.

    tests/modules/attention/low_pcc_notes.md:5-16 gives the pair rotation
    (x_2i, x_2i+1) -> (x_2i cos - x_2i+1 sin, x_2i+1 cos + x_2i sin) on the
    interleaved layout that src/tt_transformers/models/llama32_1b/weight_utils.py:23-25
    permutes the checkpoint's rows into. On the checkpoint's own row order the pair
    (2i, 2i+1) is (i, i + hd/2), which is what is rotated here.
    """
    half = x.shape[-1] // 2
    angles = torch.outer(positions.to(torch.float32), inv_freq)  # [T, hd/2]
    cos = torch.cos(angles)[:, None, :]
    sin = torch.sin(angles)[:, None, :]
    first, second = x[..., :half], x[..., half:]
    return torch.cat([first * cos - second * sin, second * cos + first * sin], dim=-1)


def rms_norm(x, weight, eps):
    """y = x / sqrt(mean(x^2) + eps) * w, no unit offset.

    src/tt_transformers/modules/rmsnorm/rmsnorm_1d.py:208-215;
    tests/modules/rmsnorm/test_rmsnorm_1d.py:748,872.
    """
    variance = x.pow(2).mean(dim=-1, keepdim=True)
    return x * torch.rsqrt(variance + eps) * weight


def causal_attention(q, k, v, window=None):
    """softmax(q k^T / sqrt(hd), causal) v with grouped KV heads.

    q [T, H, hd], k and v [T, G, hd]. Head h reads KV head h // (H/G).
    src/tt_transformers/modules/attention/attention_1d.py:650-659 (causal),
    :1641-1642 (scale = hd^-0.5), :539-545 (head grouping).
    `window`, if given, lets a query see only the last `window` keys up to itself.
    """
    T, H, hd = q.shape
    G = k.shape[1]
    rep = H // G
    k = k.repeat_interleave(rep, dim=1)
    v = v.repeat_interleave(rep, dim=1)
    scores = torch.einsum("thd,shd->hts", q, k) * (hd ** -0.5)
    idx = torch.arange(T)
    visible = idx[None, :] <= idx[:, None]
    if window is not None:
        visible &= idx[None, :] > idx[:, None] - window
    scores = scores.masked_fill(~visible[None], float("-inf"))
    probs = torch.softmax(scores, dim=-1)
    return torch.einsum("hts,shd->thd", probs, v)


def attention_block(x, positions, w, prefix, config, inv_freq):
    """q,k,v projections without bias, rope on q and k, attention, output projection.

    src/tt_transformers/modules/attention/attention_1d.py:507-518 (projection),
    :557-571 (rope on q and k only), :699-706 (output projection).
    """
    T = x.shape[0]
    H = config["num_attention_heads"]
    G = config.get("num_key_value_heads") or H
    hd = head_dim_of(config)
    q = (x @ w[prefix + "q_proj.weight"].T).view(T, H, hd)
    k = (x @ w[prefix + "k_proj.weight"].T).view(T, G, hd)
    v = (x @ w[prefix + "v_proj.weight"].T).view(T, G, hd)
    q = rope_rotate(q, positions, inv_freq)
    k = rope_rotate(k, positions, inv_freq)
    o = causal_attention(q, k, v).reshape(T, H * hd)
    return o @ w[prefix + "o_proj.weight"].T


def swiglu(x, w, prefix):
    """(silu(x W1) * (x W3)) W2. tests/modules/mlp/test_mlp_1d.py:676;
    src/tt_transformers/modules/mlp/mlp_1d.py:240-294."""
    gate = x @ w[prefix + "gate_proj.weight"].T
    up = x @ w[prefix + "up_proj.weight"].T
    return (torch.nn.functional.silu(gate) * up) @ w[prefix + "down_proj.weight"].T


def forward(config, w, tokens):
    """Logits [T, vocab] of one whole sequence of token ids.

    Block order: src/tt_transformers/models/llama32_1b/model.py:141-186 (norm,
    attention, add, norm, feed-forward, add), final norm and head :958-995, tied
    head src/tt_transformers/models/llama32_1b/hf_generator.py:254-261.
    """
    tokens = torch.as_tensor(tokens, dtype=torch.long)
    positions = torch.arange(tokens.shape[0])
    eps = float(config["rms_norm_eps"])
    theta, scaling = rope_settings(config)
    inv_freq = rope_inverse_frequencies(head_dim_of(config), theta, scaling)
    x = w["model.embed_tokens.weight"][tokens]
    for i in range(config["num_hidden_layers"]):
        p = f"model.layers.{i}."
        h = rms_norm(x, w[p + "input_layernorm.weight"], eps)
        x = x + attention_block(h, positions, w, p + "self_attn.", config, inv_freq)
        h = rms_norm(x, w[p + "post_attention_layernorm.weight"], eps)
        x = x + swiglu(h, w, p + "mlp.")
    x = rms_norm(x, w["model.norm.weight"], eps)
    head = w["model.embed_tokens.weight"] if config.get("tie_word_embeddings", False) else w["lm_head.weight"]
    return x @ head.T


def greedy(config, w, prompt, steps):
    """Greedy continuation by running the whole sequence again for every token."""
    seq = list(prompt)
    for _ in range(steps):
        logits = forward(config, w, seq)
        seq.append(int(torch.argmax(logits[-1])))
    return seq[len(prompt):]


def host_allowed(row, top_k, top_p):
    """Which tokens of one row of (temperature-scaled) scores may be drawn: a boolean mask.
    src/tt_transformers/models/hf_generation.py:138-146."""
    allowed = torch.ones_like(row, dtype=torch.bool)
    if top_k:
        kth = torch.sort(row, descending=True).values[min(top_k, row.numel()) - 1]
        allowed &= row >= kth
    if top_p < 1.0:
        masked = torch.where(allowed, row, torch.full_like(row, float("-inf")))
        order = torch.argsort(masked)  # ascending: the tail comes first
        tail_mass = torch.cumsum(torch.softmax(masked, dim=-1)[order], dim=-1)
        drop = tail_mass <= 1.0 - top_p
        drop[-1] = False
        allowed[order[drop]] = False
    return allowed


def host_select(scores, do_sample, temperature, top_k, top_p, generator=None):
    """Host sampler: which tokens may be drawn, and the draw.

    The rules are those of src/tt_transformers/models/hf_generation.py:125-148:
    without sampling the largest score wins; with it the scores are divided by the
    temperature, everything below the top_k-th largest score is excluded, then the
    low tail whose cumulative probability stays within 1 - top_p is excluded (the
    best token is always kept), and a token is drawn from what is left.
    """
    scores = scores.to(torch.float32)
    if not do_sample:
        return torch.argmax(scores, dim=-1)
    picks = []
    for row in scores / temperature:
        allowed = host_allowed(row, top_k, top_p)
        probs = torch.softmax(torch.where(allowed, row, torch.full_like(row, float("-inf"))), dim=-1)
        picks.append(torch.multinomial(probs, 1, generator=generator)[0])
    return torch.stack(picks)
