"""The plain implementation itself: its parts against closed forms, and against the outputs
of the reference's own pure-PyTorch functions kept under tests/golden/ (no GPU)."""

import math
import os

import pytest
import torch

import plain_llama
from conftest import TINY_A, TINY_B
from tt_transformers_b200.weights import random_tensors

GOLDEN = torch.load(os.path.join(os.path.dirname(__file__), "golden", "reference_parts.pt"))


def weights_of(cfg, seed):
    return {k: v.float() for k, v in random_tensors(cfg, seed, norm_std=0.1, dtype=torch.float32).items()}


def test_llama3_scaling_equals_the_references():
    for case in GOLDEN["llama3_scaling"]:
        scaling = {"factor": case["factor"], "low_freq_factor": case["low"], "high_freq_factor": case["high"],
                   "original_max_position_embeddings": case["original"]}
        ours = plain_llama.rope_inverse_frequencies(case["head_dim"], case["theta"], scaling)
        assert torch.equal(ours, case["scaled"])


def test_the_engines_frequencies_equal_the_references_too():
    from tt_transformers_b200.parts.position import rotary_inverse_frequencies

    for case in GOLDEN["llama3_scaling"]:
        scaling = {"factor": case["factor"], "low_freq_factor": case["low"], "high_freq_factor": case["high"],
                   "original_max_position_embeddings": case["original"]}
        assert torch.equal(rotary_inverse_frequencies(case["head_dim"], case["theta"], scaling), case["scaled"])
    assert torch.equal(rotary_inverse_frequencies(16, 10000.0, None),
                       plain_llama.rope_inverse_frequencies(16, 10000.0, None))


def test_rotation_on_checkpoint_rows_equals_the_references_interleaved_rotation():
    heads, hd = GOLDEN["rope_heads"], GOLDEN["rope_head_dim"]
    q = (GOLDEN["rope_x"] @ GOLDEN["rope_w"].T).view(3, heads, hd)
    ours = plain_llama.rope_rotate(q, GOLDEN["rope_pos"], GOLDEN["rope_inv_freq"])
    interleaved = torch.stack([ours[..., :hd // 2], ours[..., hd // 2:]], dim=-1).flatten(-2)
    assert torch.allclose(interleaved, GOLDEN["rope_rotated_meta"], atol=1e-6)


def test_host_sampler_equals_the_references_where_it_is_deterministic():
    logits = GOLDEN["select_logits"]
    assert torch.equal(plain_llama.host_select(logits, False, 1.0, 0, 1.0), GOLDEN["select_greedy"])
    assert torch.equal(plain_llama.host_select(logits, True, 0.7, 1, 1.0), GOLDEN["select_top_k1"])
    assert torch.equal(plain_llama.host_select(logits, True, 0.7, 0, 1e-4), GOLDEN["select_top_p_small"])


def test_host_sampler_allows_the_tokens_the_reference_allows():
    """For random settings: the set of tokens that may be drawn, and their probabilities, as the reference's
    _select handed them to its draw."""
    logits = GOLDEN["allowed_logits"]
    assert len(GOLDEN["allowed"]) >= 5
    for case in GOLDEN["allowed"]:
        for row in range(logits.shape[0]):
            scaled = logits[row] / case["temperature"]
            mask = plain_llama.host_allowed(scaled, case["top_k"], case["top_p"])
            assert torch.equal(mask, case["mask"][row]), (case["top_k"], case["top_p"], row)
            probs = torch.softmax(torch.where(mask, scaled, torch.full_like(scaled, float("-inf"))), dim=-1)
            assert torch.allclose(probs, case["probs"][row], atol=1e-6)


def test_host_sampler_respects_its_cuts():
    gen = torch.Generator().manual_seed(0)
    logits = torch.tensor([[5.0, 4.0, 3.0, 2.0, 1.0, 0.0]]).repeat(300, 1)
    picks = plain_llama.host_select(logits, True, 1.0, 3, 1.0, generator=gen)
    assert set(picks.tolist()) == {0, 1, 2}
    picks = plain_llama.host_select(logits, True, 1.0, 0, 0.5, generator=gen)   # p = .63, .23, ...: the best alone reaches 0.5
    assert set(picks.tolist()) <= {0, 1}


def test_frequencies_without_scaling_and_scaling_limits():
    f = plain_llama.rope_inverse_frequencies(16, 10000.0, None)
    assert torch.allclose(f, torch.tensor([10000.0 ** (-2 * i / 16) for i in range(8)]))
    scaling = {"factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0, "original_max_position_embeddings": 8192}
    base = plain_llama.rope_inverse_frequencies(128, 500000.0, None)
    scaled = plain_llama.rope_inverse_frequencies(128, 500000.0, scaling)
    wavelen = 2 * math.pi / base
    assert torch.equal(scaled[wavelen < 8192 / 4], base[wavelen < 8192 / 4])
    assert torch.allclose(scaled[wavelen > 8192], base[wavelen > 8192] / 8)
    mid = (wavelen >= 8192 / 4) & (wavelen <= 8192)
    assert mid.any() and bool(((scaled[mid] <= base[mid]) & (scaled[mid] >= base[mid] / 8)).all())


def test_rotation_keeps_lengths_and_depends_on_distance_only():
    g = torch.Generator().manual_seed(1)
    q, k = torch.randn(1, 1, 32, generator=g), torch.randn(1, 1, 32, generator=g)
    f = plain_llama.rope_inverse_frequencies(32, 10000.0, None)
    assert torch.equal(plain_llama.rope_rotate(q, torch.tensor([0]), f), q)
    r = plain_llama.rope_rotate(q, torch.tensor([17]), f)
    assert torch.allclose(r.norm(), q.norm(), rtol=1e-5)
    dots = []
    for p in (0, 5, 40):
        qq = plain_llama.rope_rotate(q, torch.tensor([p + 9]), f)
        kk = plain_llama.rope_rotate(k, torch.tensor([p]), f)
        dots.append(float((qq * kk).sum()))
    assert max(dots) - min(dots) < 1e-4


def test_rms_norm_equals_torchs_and_swiglu_the_references_expression():
    """The reference's module tests take torch.nn.RMSNorm(dim, eps) as what its norm must equal
    (tests/modules/rmsnorm/test_rmsnorm_1d.py:744-748) and the expression (silu(x @ w1) * (x @ w3)) @ w2 as what
    its feed-forward must equal (tests/modules/mlp/test_mlp_1d.py:675-676, weights [in, out] there)."""
    g = torch.Generator().manual_seed(3)
    for width, eps in ((64, 1e-5), (96, 1e-6), (80, 1e-2)):
        x = torch.randn(7, width, generator=g) * 3
        norm = torch.nn.RMSNorm(width, eps=eps)
        with torch.no_grad():
            norm.weight.copy_(1 + 0.3 * torch.randn(width, generator=g))
            want = norm(x)
        assert torch.allclose(plain_llama.rms_norm(x, norm.weight.detach(), eps), want, atol=1e-6, rtol=1e-5)
        assert torch.allclose(plain_llama.rms_norm(x, norm.weight.detach(), eps),
                              torch.nn.functional.rms_norm(x, (width,), norm.weight.detach(), eps), atol=1e-6, rtol=1e-5)
    width, inter = 48, 112
    x = torch.randn(5, width, generator=g)
    w1, w3 = torch.randn(width, inter, generator=g) * 0.2, torch.randn(width, inter, generator=g) * 0.2
    w2 = torch.randn(inter, width, generator=g) * 0.2
    want = (torch.nn.functional.silu(x @ w1) * (x @ w3)) @ w2
    weights = {"gate_proj.weight": w1.T.contiguous(), "up_proj.weight": w3.T.contiguous(),
               "down_proj.weight": w2.T.contiguous()}
    assert torch.allclose(plain_llama.swiglu(x, weights, ""), want, atol=1e-6)


def test_rms_norm_and_swiglu_by_hand():
    x = torch.tensor([[3.0, 4.0]])
    w = torch.tensor([2.0, 0.5])
    assert torch.allclose(plain_llama.rms_norm(x, w, 0.0), torch.tensor([[3 / math.sqrt(12.5) * 2, 4 / math.sqrt(12.5) * 0.5]]))
    weights = {"gate_proj.weight": torch.tensor([[1.0]]), "up_proj.weight": torch.tensor([[2.0]]),
               "down_proj.weight": torch.tensor([[3.0]])}
    out = plain_llama.swiglu(torch.tensor([[1.0]]), weights, "")
    assert torch.allclose(out, torch.tensor([[1 / (1 + math.exp(-1)) * 2 * 3]]))


def test_attention_by_loops():
    g = torch.Generator().manual_seed(2)
    T, H, G, hd = 7, 4, 2, 8
    q, k, v = torch.randn(T, H, hd, generator=g), torch.randn(T, G, hd, generator=g), torch.randn(T, G, hd, generator=g)
    for window in (None, 3):
        got = plain_llama.causal_attention(q, k, v, window)
        for t in range(T):
            for h in range(H):
                lo = 0 if window is None else max(0, t - window + 1)
                s = torch.tensor([float(q[t, h] @ k[j, h // 2]) / math.sqrt(hd) for j in range(lo, t + 1)])
                p = torch.softmax(s, 0)
                want = sum(p[j - lo] * v[j, h // 2] for j in range(lo, t + 1))
                assert torch.allclose(got[t, h], want, atol=1e-5)


@pytest.mark.parametrize("cfg,seed", [(TINY_A, 0), (TINY_B, 1)])
def test_a_position_does_not_see_what_follows(cfg, seed):
    w = weights_of(cfg, seed)
    tokens = torch.randint(0, cfg["vocab_size"], (20,), generator=torch.Generator().manual_seed(seed)).tolist()
    whole = plain_llama.forward(cfg, w, tokens)
    prefix = plain_llama.forward(cfg, w, tokens[:11])
    assert whole.shape == (20, cfg["vocab_size"])
    assert torch.allclose(whole[:11], prefix, atol=1e-5)
    other = plain_llama.forward(cfg, w, tokens[:11] + [(t + 1) % cfg["vocab_size"] for t in tokens[11:]])
    assert torch.allclose(whole[:11], other[:11], atol=1e-5) and not torch.allclose(whole[11:], other[11:], atol=1e-3)


def test_tied_and_untied_heads():
    w = weights_of(TINY_A, 0)
    logits = plain_llama.forward(TINY_A, w, [1, 2, 3])
    w2 = dict(w)
    w2["lm_head.weight"] = torch.zeros_like(w["model.embed_tokens.weight"])
    assert torch.equal(plain_llama.forward(TINY_A, w2, [1, 2, 3]), logits)          # tied: lm_head is not read
    assert float(plain_llama.forward(dict(TINY_A, tie_word_embeddings=False), w2, [1, 2, 3]).abs().max()) == 0


def test_the_kernel_twins_sampler_draws_from_the_references_allowed_sets():
    """tests/torch_kernels.py states the device sampler's rules in plain torch; its draws stay within the sets the
    reference's _select allows, for top_p over the whole vocabulary and top_k beyond the kernel's candidate list."""
    from torch_kernels import TorchKernels

    twin = TorchKernels()
    logits = GOLDEN["allowed_logits"]
    draws = 200
    for case in GOLDEN["allowed"]:
        for row in range(logits.shape[0]):
            rows = logits[row][None].repeat(draws, 1)
            picks = twin.sample(rows, torch.full((draws,), case["temperature"]),
                                torch.full((draws,), case["top_k"], dtype=torch.int32), torch.full((draws,), case["top_p"]),
                                torch.full((draws,), 99 + row, dtype=torch.int64), torch.arange(draws, dtype=torch.int32))
            drawn = torch.zeros(logits.shape[1], dtype=torch.bool)
            drawn[picks.long()] = True
            allowed, probs = case["mask"][row], case["probs"][row]
            assert not bool((drawn & ~allowed).any()), (case["top_k"], case["top_p"], row)
            assert bool(drawn[probs >= 0.08].all())
