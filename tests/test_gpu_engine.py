"""The engine on the GPU against the plain implementation, under every way of cutting."""

import pytest
import torch

import helpers
from conftest import TINY_A, TINY_B, TINY_C, TINY_D, TINY_E

pytestmark = pytest.mark.gpu

CONFIGS = {"A": TINY_A, "B": TINY_B, "C": TINY_C, "D": TINY_D, "E": TINY_E}
TOL = {"float32": 1e-4, "bfloat16": 4e-2}


def make_engine(folder, dtype, page_size, num_pages, max_seq_len=512):
    from tt_transformers_b200.config import EngineConfig
    from tt_transformers_b200.engine.step import build_engine

    return build_engine(folder, EngineConfig(dtype=dtype, page_size=page_size, num_pages=num_pages, max_batch_size=4,
                                             max_seq_len=max_seq_len, max_step_tokens=4096, device="cuda:0"))


def requests_for(name, lengths, seed=0):
    vocab = CONFIGS[name]["vocab_size"]
    return {f"r{i}": helpers.random_tokens(vocab, n, seed + i) for i, n in enumerate(lengths)}


def check(got, ref, dtype):
    for rid in ref:
        err = helpers.relative_error(got[rid], ref[rid])
        assert err <= TOL[dtype], f"request {rid}: relative error {err}"
        if dtype == "float32":
            assert torch.equal(got[rid].argmax(-1), ref[rid].argmax(-1))


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("name,lengths,page", [("A", (7, 13, 70), 4), ("B", (5, 17, 33, 90), 8), ("C", (150, 40), 16),
                                               ("D", (300, 45, 130, 70, 64), 16), ("E", (100, 37, 65), 8)])
@pytest.mark.parametrize("cut", ["whole", "tail", "portions", "mixed"])
def test_cuttings_match_plain(tiny_folders, dtype, name, lengths, page, cut):
    requests = requests_for(name, lengths)
    ref = helpers.plain_logits(tiny_folders[name], requests)
    steps = {"whole": helpers.steps_whole, "tail": helpers.steps_decode_tail, "portions": helpers.steps_portions,
             "mixed": helpers.steps_mixed}[cut](requests)
    tokens = helpers.max_live_tokens(requests, steps, rounding=page)
    engine = make_engine(tiny_folders[name], dtype, page, num_pages=-(-tokens // page))
    got = helpers.run_steps(engine, steps)
    engine.cache.audit()
    assert engine.cache.free_pages() == engine.cache.num_pages      # everything was given back
    check(got, ref, dtype)
    engine.close()


@pytest.mark.parametrize("name,lengths,page", [("C", (150, 40), 16), ("D", (300, 45, 130, 70, 64), 16), ("B", (5, 17, 33, 90), 8)])
@pytest.mark.parametrize("cut,graphs", [("tail", False), ("tail", True), ("mixed", True)])
def test_sub_layers_that_add_to_the_stream_and_hand_on_a_prepared_norm(tiny_folders, name, lengths, page, cut, graphs):
    """With the fusions of the skinny products switched on (the last product of a sub-layer adds to the residual
    stream and prepares the next norm, the first product of the next finishes it), a decode step runs the norm
    kernel once, after the embedding; portions of prompts take the unfused way. Same tolerance as without."""
    from tt_transformers_b200.config import EngineConfig
    from tt_transformers_b200.engine.step import build_engine

    requests = requests_for(name, lengths)
    ref = helpers.plain_logits(tiny_folders[name], requests)
    steps = {"tail": helpers.steps_decode_tail, "mixed": helpers.steps_mixed}[cut](requests)
    tokens = helpers.max_live_tokens(requests, steps, rounding=page)
    engine = build_engine(tiny_folders[name], EngineConfig(
        dtype="bfloat16", page_size=page, num_pages=-(-tokens // page), max_batch_size=4, max_seq_len=512,
        max_step_tokens=4096, cuda_graph=graphs, device="cuda:0"))
    kernels = engine.kernels
    before = kernels.fuse_norm, kernels.fuse_add
    plain_norm = kernels.add_rmsnorm
    rows_normed = []
    kernels.fuse_norm = kernels.fuse_add = True
    kernels.add_rmsnorm = lambda *a, **kw: (rows_normed.append(a[0].shape[0]), plain_norm(*a, **kw))[1]
    try:
        got = helpers.run_steps(engine, steps)
        check(got, ref, "bfloat16")
        engine.cache.audit()
    finally:
        kernels.add_rmsnorm = plain_norm
        kernels.fuse_norm, kernels.fuse_add = before
        engine.close()
    if not graphs:
        decode_steps = sum(1 for s in steps if s["entries"] and all(len(e["tokens"]) == 1 for e in s["entries"]))
        small = sum(1 for rows in rows_normed if rows <= 16)
        # one per decode step; a prompt portion adds one more for the few rows of its wanted places
        assert 0 < decode_steps <= small <= len(steps)
