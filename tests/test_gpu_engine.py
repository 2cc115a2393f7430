"""The engine on the GPU against the plain implementation, under every way of cutting."""

import pytest
import torch

import helpers
from conftest import TINY_A, TINY_B, TINY_C, TINY_D, TINY_E

pytestmark = pytest.mark.gpu

CONFIGS = {"A": TINY_A, "B": TINY_B, "C": TINY_C, "D": TINY_D, "E": TINY_E}
TOL = {"float32": 1e-4, "bfloat16": 2.5e-2}
BF16_MEAN_TINY = 2.5e-3       # mean |engine - plain| over all logits, relative to the largest |plain| logit


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
    if dtype == "bfloat16":
        # beside the largest error: the mean error, and the best token on rows that the plain logits decide
        # clearly (a wrong page in one layer of several moves these long before it moves the maximum by 4 %)
        stats = helpers.error_stats(got, ref)
        assert stats["mean"] <= BF16_MEAN_TINY, stats
        if stats["clear_rows"] >= 20:
            assert stats["clear_top1"] >= 0.995, stats


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


# ---------------------------------------------------------------------------- many live requests: the captured buckets 16, 32, 64
WIDE = {   # the layer sizes of Llama 3.2 1B, two layers
    "architectures": ["LlamaForCausalLM"],
    "hidden_size": 2048, "num_hidden_layers": 2, "num_attention_heads": 32, "num_key_value_heads": 8,
    "head_dim": 64, "intermediate_size": 8192, "vocab_size": 128256, "rms_norm_eps": 1e-5,
    "max_position_embeddings": 131072, "rope_theta": 500000.0,
    "rope_scaling": {"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                     "original_max_position_embeddings": 8192},
    "tie_word_embeddings": True,
}
_MANY = {}


def many_case(tmp_path_factory, tiny_folders, name, live):
    """Folder, requests, steps and the plain logits at the wanted places; made once per (model, live)."""
    key = (name, live)
    if key not in _MANY:
        import plain_llama

        if name == "wide":
            from tt_transformers_b200.weights import write_model_folder
            if "wide" not in _MANY:
                _MANY["wide"] = write_model_folder(str(tmp_path_factory.mktemp("wide")), WIDE, seed=0, norm_std=0.05)
            folder, vocab = _MANY["wide"], WIDE["vocab_size"]
        else:
            folder, vocab = tiny_folders[name], CONFIGS[name]["vocab_size"]
        count = live + max(3, live // 4)                     # more requests than are live at a time: pages come back
        g = torch.Generator().manual_seed(live)
        lengths = (torch.randint(46, 110, (count,), generator=g)).tolist()
        requests = {f"q{i}": helpers.random_tokens(vocab, n, 500 + i) for i, n in enumerate(lengths)}
        steps = helpers.steps_many(requests, live, tail=44, seed=live)
        places = helpers.wanted_positions(steps)
        config, weights = plain_llama.read_model_folder(folder)
        ref = {rid: plain_llama.forward(config, weights, toks)[places[rid]] for rid, toks in requests.items()}
        _MANY[key] = (folder, requests, steps, ref)
    return _MANY[key]


# bfloat16 against the plain float32 logits: the largest error as everywhere, and, because one wrong page in one
# layer can hide below 4 % of the largest logit, also the mean error and how often the best token is the same on
# rows that the plain logits decide clearly (lead over the runner-up above 2 % of the largest logit)
BF16_MEAN, BF16_CLEAR_TOP1 = 2.5e-3, 0.995


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("name,live", [("D", 9), ("D", 17), ("D", 33), ("D", 64), ("wide", 17), ("wide", 64)])
def test_many_live_requests_through_captured_steps(tmp_path_factory, tiny_folders, dtype, name, live):
    """9 to 64 requests live at a time, of unequal lengths: prompts in portions beside decoded tokens, then at
    least 44 decode steps each through the captured graphs of 16, 32 and 64 rows, requests ending on the way and
    later ones taking over their pages; against the plain implementation."""
    from tt_transformers_b200.config import EngineConfig
    from tt_transformers_b200.engine.step import build_engine

    folder, requests, steps, ref = many_case(tmp_path_factory, tiny_folders, name, live)
    page = 16
    pages = -(-helpers.max_live_tokens(requests, steps, rounding=page) // page)
    engine = build_engine(folder, EngineConfig(dtype=dtype, page_size=page, num_pages=pages, max_batch_size=64,
                                               max_seq_len=128, max_step_tokens=4096, device="cuda:0"))
    for g in engine.cache.groups:
        for tensor in g.storage.values():
            tensor.fill_(float("nan"))
    got = helpers.run_steps(engine, steps)
    engine.cache.audit()
    assert engine.cache.free_pages() == pages
    buckets = engine.graphs.captured_sizes()
    assert engine.graphs.replays >= 44 and max(buckets) >= min(64, 1 << (live - 1).bit_length()), buckets
    stats = helpers.error_stats(got, ref)
    print(f"\\n{name} live={live} {dtype}: {stats} buckets={buckets} replays={engine.graphs.replays}")
    assert stats["max"] <= TOL[dtype], stats
    if dtype == "float32":
        assert stats["top1"] == 1.0, stats
    else:
        assert stats["mean"] <= BF16_MEAN and stats["clear_top1"] >= BF16_CLEAR_TOP1 and stats["clear_rows"] > 50, stats
    engine.close()


# ---------------------------------------------------------------------------- captured prompt steps
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("name,lengths,page", [("D", (2, 31, 32, 33, 100, 128, 257, 512), 16), ("B", (3, 17, 64, 150), 8),
                                               ("E", (40, 129), 8)])
def test_short_prompts_as_replays_of_a_captured_step(tiny_folders, dtype, name, lengths, page):
    """A lone request's first portion, wanting its last logits, runs as a replay of the step captured for its length
    bucket: the rest of the bucket is a segment on the scratch page (filled with NaN here: nothing of it may reach
    the real rows). The prompt's last logits and three decoded positions against the plain implementation."""
    from tt_transformers_b200.config import EngineConfig
    from tt_transformers_b200.engine.step import build_engine

    requests = {f"s{n}": helpers.random_tokens(CONFIGS[name]["vocab_size"], n + 3, 900 + n) for n in lengths}
    ref = helpers.plain_logits(tiny_folders[name], requests)
    engine = build_engine(tiny_folders[name], EngineConfig(dtype=dtype, page_size=page, max_batch_size=2,
                                                           max_seq_len=1024 if name == "D" else 256, device="cuda:0"))
    assert engine.prompt_graphs is not None
    for g in engine.cache.groups:
        for tensor in g.storage.values():
            tensor.fill_(float("nan"))
    steps = []
    for n in lengths:
        toks = requests[f"s{n}"]
        steps.append({"entries": [{"id": f"s{n}", "tokens": toks[:n], "want": [n - 1]}], "end": []})
        for i in range(n, n + 3):
            steps.append({"entries": [{"id": f"s{n}", "tokens": [toks[i]], "want": [0]}], "end": [f"s{n}"] if i == n + 2 else []})
    got = helpers.run_steps(engine, steps)
    assert engine.prompt_graphs.replays == len(lengths)
    assert len(engine.prompt_graphs._graphs) == len({engine.prompt_graphs._bucket(n) for n in lengths})
    check(got, {rid: ref[rid][len(requests[rid]) - 4:] for rid in requests}, dtype)
    # a portion that wants no logits runs the same way and returns none; one that wants several runs eagerly
    before = engine.prompt_graphs.replays
    assert engine.step([helpers_entry("x", requests[f"s{lengths[-1]}"][:lengths[0] + 7], [])]).shape[0] == 0
    assert engine.prompt_graphs.replays == before + 1
    engine.finish("x")
    assert engine.step([helpers_entry("y", requests[f"s{lengths[-1]}"][:9], [0, 8])]).shape[0] == 2
    assert engine.prompt_graphs.replays == before + 1
    engine.finish("y")
    engine.cache.audit()
    engine.close()


def helpers_entry(rid, tokens, want):
    from tt_transformers_b200.engine.step import StepEntry

    return StepEntry(rid, tokens, want)
