"""Makes tests/golden/reference_parts.pt from the reference's own code, where it runs on a CPU.

The reference's forward pass cannot run without its accelerator library, so whole-model
outputs cannot be taken from it. Three of its pure-PyTorch functions can be imported and
were run once, on small inputs, to anchor the plain implementation:
  - the Llama-3 frequency scaling, src/tt_transformers/models/llama3_8b/hf_generator.py:88-103
    (the module imports the accelerator library at the top, so a stand-in object is put in
    sys.modules for the import; the function itself uses only torch and math);
  - the host sampler _select, src/tt_transformers/models/hf_generation.py:125-148 (its choices where they
    are deterministic, and, for random settings, the set of tokens it may draw and their probabilities);
  - the checkpoint-row permutation reverse_permute, src/tt_transformers/models/llama32_1b/weight_utils.py:23-25,
    with the pair-swap matrix of src/tt_transformers/tensor_utils.py:91-112, to show that rotating
    interleaved pairs of permuted rows equals rotating (i, i + d/2) of the checkpoint's rows.
Usage: python tests/golden/make_golden.py /path/to/reference
"""

import os
import sys
from unittest.mock import MagicMock

import torch


def main(reference_root):
    sys.path.insert(0, os.path.join(reference_root, "src"))
    stand_in = MagicMock(TILE_SIZE=32)
    stand_in.__path__ = []                       # lets "import ttnn.x" resolve
    sys.modules.setdefault("ttnn", stand_in)
    for sub in ("ttnn.tools", "ttnn.tools.trace_allocation_tracker"):
        sys.modules.setdefault(sub, MagicMock())
    out = {}

    from tt_transformers.models.llama3_8b import hf_generator as g8

    cases = []
    for head_dim, theta, factor, low, high, original in ((32, 500000.0, 32.0, 1.0, 4.0, 64), (64, 500000.0, 32.0, 1.0, 4.0, 8192),
                                                         (128, 500000.0, 8.0, 1.0, 4.0, 8192), (16, 10000.0, 4.0, 2.0, 8.0, 32)):
        inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))
        scaling = g8.RopeScaling(rope_type="llama3", factor=factor, low_freq_factor=low, high_freq_factor=high,
                                 original_max_position_embeddings=original)
        cases.append(dict(head_dim=head_dim, theta=theta, factor=factor, low=low, high=high, original=original,
                          scaled=g8._llama3_scaled_inv_freq(inv_freq, scaling)))
    out["llama3_scaling"] = cases

    from tt_transformers.models import hf_generation

    gen = torch.Generator().manual_seed(0)
    logits = torch.randn(6, 50, generator=gen) * 2
    active = torch.ones(6, dtype=torch.bool)
    out["select_logits"] = logits
    out["select_greedy"] = hf_generation._select(logits, batch_size=6, vocab_size=50, do_sample=False, temperature=1.0,
                                                 top_k=0, top_p=1.0, active=active)
    # with top_k = 1, or a top_p so small that only the best token stays, sampling is deterministic
    out["select_top_k1"] = hf_generation._select(logits, batch_size=6, vocab_size=50, do_sample=True, temperature=0.7,
                                                 top_k=1, top_p=1.0, active=active)
    out["select_top_p_small"] = hf_generation._select(logits, batch_size=6, vocab_size=50, do_sample=True,
                                                      temperature=0.7, top_k=0, top_p=1e-4, active=active)

    # Which tokens _select may draw, for settings where sampling is random: the probabilities it hands to
    # torch.multinomial are caught on the way (the function itself runs unchanged); a token is allowed where
    # its probability is positive. Logits: 400 values spread so that no cut falls within rounding of a token.
    wide = torch.randn(3, 400, generator=gen) * 2.5
    out["allowed_logits"] = wide
    out["allowed"] = []
    real_multinomial = torch.multinomial
    for temperature, top_k, top_p in ((1.0, 0, 0.9), (0.8, 100, 1.0), (1.3, 50, 0.8), (1.0, 0, 0.5), (0.7, 200, 0.95)):
        caught = []
        torch.multinomial = lambda probs, num_samples, **kw: (caught.append(probs.clone()), real_multinomial(probs, num_samples, **kw))[1]
        try:
            hf_generation._select(wide, batch_size=3, vocab_size=400, do_sample=True, temperature=temperature,
                                  top_k=top_k, top_p=top_p, active=torch.ones(3, dtype=torch.bool))
        finally:
            torch.multinomial = real_multinomial
        out["allowed"].append(dict(temperature=temperature, top_k=top_k, top_p=top_p, mask=caught[0] > 0,
                                   probs=caught[0]))

    from tt_transformers.models.llama32_1b.weight_utils import reverse_permute
    from tt_transformers.tensor_utils import get_rot_transformation_mat

    heads, head_dim, width = 2, 8, 5
    w = torch.randn(heads * head_dim, width, generator=gen)
    x = torch.randn(3, width, generator=gen)
    permuted = reverse_permute(w, heads, heads * head_dim, width)
    T = get_rot_transformation_mat(dhead=head_dim)
    T = T.reshape(T.shape[-2], T.shape[-1])[:head_dim, :head_dim].float()
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, head_dim, 2).float() / head_dim))
    pos = torch.tensor([0.0, 3.0, 11.0])
    ang = torch.outer(pos, inv_freq)
    cos = torch.stack([ang.cos(), ang.cos()], -1).flatten(-2)          # [c0, c0, c1, c1, ...]
    sin = torch.stack([ang.sin(), ang.sin()], -1).flatten(-2)
    q_meta = (x @ permuted.T).view(3, heads, head_dim)
    rotated_meta = q_meta * cos[:, None] + (q_meta @ T) * sin[:, None]
    out["rope_w"], out["rope_x"], out["rope_pos"], out["rope_inv_freq"] = w, x, pos, inv_freq
    out["rope_rotated_meta"] = rotated_meta
    out["rope_heads"], out["rope_head_dim"] = heads, head_dim
    torch.save(out, os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_parts.pt"))
    print("written", {k: (v.shape if hasattr(v, "shape") else type(v).__name__) for k, v in out.items()})


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py /path/to/the/reference/checkout")
    main(sys.argv[1])
