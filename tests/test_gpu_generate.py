"""Generation through the entry point, long decoding, the first tokens of a sequence, the
replay program as a user runs it, and the layer sizes of the real model."""

import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import helpers
import plain_llama
from conftest import ROOT, TINY_A, TINY_B, TINY_D

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_greedy_generation_through_the_entry_point(tiny_folders, dtype):
    from tt_transformers_b200 import from_pretrained

    for name, cfg, page in (("A", TINY_A, 4), ("B", TINY_B, 8), ("D", TINY_D, 16)):
        config, weights = plain_llama.read_model_folder(tiny_folders[name])
        prompts = [helpers.random_tokens(cfg["vocab_size"], n, 50 + n) for n in (7, 13, 33)]
        expect = [plain_llama.greedy(config, weights, p, 8) for p in prompts]
        llm = from_pretrained(tiny_folders[name], dtype=dtype, page_size=page, max_batch_size=4, max_seq_len=64,
                              max_step_tokens=24, max_chunk_tokens=16)
        got = llm.generate(prompts, max_new_tokens=8)
        if dtype == "float32":
            assert got == expect
        else:       # bfloat16 may flip a near tie; most tokens agree, and the first always starts from the same prompt
            agree = sum(a == b for g, e in zip(got, expect) for a, b in zip(g, e))
            assert agree >= 18, (got, expect)
        assert llm.engine.cache.free_pages() == llm.engine.cache.num_pages
        llm.cleanup()


def test_temperature_sampling_is_reproducible_and_independent_of_the_batch(tiny_folders):
    from tt_transformers_b200 import SamplingParams, from_pretrained

    llm = from_pretrained(tiny_folders["B"], dtype="float32", page_size=8, max_batch_size=4, max_seq_len=64)
    prompts = [helpers.random_tokens(384, n, n) for n in (5, 17, 33)]
    params = [SamplingParams(temperature=0.8, seed=1 + i, max_new_tokens=8) for i in range(3)]
    together = [r.output for r in llm.generate_requests(prompts, params)]
    alone = [llm.generate_requests([p], [sp])[0].output for p, sp in zip(prompts, params)]
    assert together == alone
    out = llm.generate(torch.tensor([prompts[0]]), max_new_tokens=5, do_sample=True, temperature=0.8, top_k=20, top_p=0.9, seed=3)
    again = llm.generate(torch.tensor([prompts[0]]), max_new_tokens=5, do_sample=True, temperature=0.8, top_k=20, top_p=0.9, seed=3)
    assert torch.equal(out, again) and out.shape == (1, 10)
    # the reference's host sampler takes any top_k, and top_p without top_k cuts over the whole vocabulary
    # (src/tt_transformers/models/hf_generation.py:138-146): so does generate(), and so do requests
    for top_k, top_p in ((0, 0.9), (100, 1.0), (300, 0.5)):
        a = llm.generate([prompts[1]], max_new_tokens=6, do_sample=True, temperature=1.1, top_k=top_k, top_p=top_p, seed=9)
        b = llm.generate([prompts[1]], max_new_tokens=6, do_sample=True, temperature=1.1, top_k=top_k, top_p=top_p, seed=9)
        assert a == b and len(a[0]) == 6
    wide = llm.generate([prompts[1]], max_new_tokens=12, do_sample=True, temperature=5.0, top_k=0, top_p=1.0, seed=9)
    tight = llm.generate([prompts[1]], max_new_tokens=12, do_sample=True, temperature=5.0, top_k=0, top_p=1e-6, seed=9)
    greedy = llm.generate([prompts[1]], max_new_tokens=12)
    assert tight == greedy and wide != greedy         # a top_p that keeps the best token alone is greedy decoding
    llm.cleanup()


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_decoding_ahead_of_the_host_gives_the_same_tokens(tiny_folders, dtype):
    """The step that is launched while the host still waits for the one before (tokens fed back on
    the device) must produce what the plain one-step-at-a-time loop produces; so must the engine's
    decode loop, and a step ahead that is taken back (a request ends early) must leave no trace."""
    from tt_transformers_b200 import SamplingParams, from_pretrained
    from tt_transformers_b200.engine.step import StepEntry

    llm = from_pretrained(tiny_folders["D"], dtype=dtype, page_size=16, max_batch_size=4, max_seq_len=256)
    prompts = [helpers.random_tokens(512, n, 70 + n) for n in (9, 30, 17)]
    params = [SamplingParams(temperature=0.7 if i else 0.0, seed=5 + i, max_new_tokens=n) for i, n in enumerate((40, 25, 33))]
    llm.look_ahead = False
    plain = [r.output for r in llm.generate_requests(prompts, params)]
    llm.look_ahead = True
    ahead = [r.output for r in llm.generate_requests(prompts, params)]
    assert ahead == plain and [len(o) for o in ahead] == [40, 25, 33]
    stop = plain[0][7]                                       # ends the first request early: a step ahead is taken back
    early = [SamplingParams(temperature=0.0, max_new_tokens=40, eos_token_ids=(stop,)), params[1], params[2]]
    llm.look_ahead = False
    plain_early = [r.output for r in llm.generate_requests(prompts, early)]
    llm.look_ahead = True
    assert [r.output for r in llm.generate_requests(prompts, early)] == plain_early
    assert plain_early[0] == plain[0][:plain[0].index(stop) + 1] and plain_early[1:] == plain[1:]
    llm.engine.cache.audit()
    assert llm.engine.cache.free_pages() == llm.engine.cache.num_pages

    engine = llm.engine
    one_by_one, fed_back = [], None
    for mode in ("host", "device"):
        for i, p in enumerate(prompts):
            engine.step([StepEntry(i, p, [])])
        first = [3, 4, 5]
        if mode == "host":
            cur = first
            for _ in range(20):
                cur = engine.kernels.sample(engine.step([StepEntry(i, [t], [0]) for i, t in enumerate(cur)])).tolist()
                one_by_one.append(cur)
        else:
            fed_back = engine.decode_steps([0, 1, 2], first, 20)
        for i in range(3):
            engine.finish(i)
    assert fed_back == one_by_one


@pytest.mark.parametrize("dtype,tol", [("float32", 1e-4), ("bfloat16", 4e-2)])
def test_long_decoding(tiny_folders, dtype, tol):
    """A short prompt, then hundreds of tokens one by one (captured steps), across many pages."""
    from tt_transformers_b200.config import EngineConfig
    from tt_transformers_b200.engine.step import build_engine

    requests = {"a": helpers.random_tokens(512, 420, 7), "b": helpers.random_tokens(512, 300, 8)}
    ref = helpers.plain_logits(tiny_folders["D"], requests)
    engine = build_engine(tiny_folders["D"], EngineConfig(dtype=dtype, page_size=16, num_pages=48, max_batch_size=2,
                                                          max_seq_len=448, device="cuda:0"))
    engine.graphs.MIN_CONTEXT_BUCKET = 64        # the contexts grow through the buckets 64, 128, 256 and 448
    steps = [{"entries": [{"id": "a", "tokens": requests["a"][:20], "want": [19]},
                          {"id": "b", "tokens": requests["b"][:3], "want": [2]}], "end": []}]
    for i in range(400):
        entries = [{"id": "a", "tokens": [requests["a"][20 + i]], "want": [0]}]
        if 3 + i < 300:
            entries.append({"id": "b", "tokens": [requests["b"][3 + i]], "want": [0]})
        steps.append({"entries": entries, "end": ["b"] if 3 + i == 299 else []})
    got = helpers.run_steps(engine, steps)
    assert engine.graphs is not None and engine.graphs.replays >= 399
    assert sorted({bucket for _, bucket in engine.graphs._graphs}) == [64, 128, 256, 448]
    assert helpers.relative_error(got["a"], ref["a"][19:]) < tol
    assert helpers.relative_error(got["b"], ref["b"][2:]) < tol


@pytest.mark.parametrize("dtype,tol", [("float32", 1e-4), ("bfloat16", 4e-2)])
def test_the_first_tokens_of_a_sequence(tiny_folders, dtype, tol):
    from tt_transformers_b200.config import EngineConfig
    from tt_transformers_b200.engine.step import build_engine

    for name, vocab, page in (("A", 256, 4), ("D", 512, 16)):
        requests = {f"r{n}": helpers.random_tokens(vocab, n, n) for n in (1, 2, 3, 5)}
        ref = helpers.plain_logits(tiny_folders[name], requests)
        engine = build_engine(tiny_folders[name], EngineConfig(dtype=dtype, page_size=page, max_batch_size=4,
                                                               max_seq_len=32, device="cuda:0"))
        whole = helpers.run_steps(engine, [{"entries": [{"id": rid, "tokens": t, "want": list(range(len(t)))}
                                                        for rid, t in requests.items()], "end": list(requests)}])
        one_by_one = helpers.run_steps(engine, helpers.steps_decode_tail(requests, tail=8))
        for rid in requests:
            assert helpers.relative_error(whole[rid], ref[rid]) < tol
            assert helpers.relative_error(one_by_one[rid], ref[rid]) < tol


@pytest.mark.parametrize("eager", [False, True])
@pytest.mark.parametrize("dtype,tol", [("float32", 1e-4), ("bfloat16", 4e-2)])
def test_trace_run_as_a_program(tiny_folders, tmp_path, dtype, tol, eager):
    requests = {f"r{i}": helpers.random_tokens(384, n, 30 + i) for i, n in enumerate((40, 90, 17, 64, 33))}
    ref = helpers.plain_logits(tiny_folders["B"], requests)
    steps = helpers.steps_mixed(requests)
    lines = "".join(json.dumps(dict(s, step=i)) + "\n" for i, s in enumerate(steps))
    out = tmp_path / "out"
    proc = subprocess.run([sys.executable, os.path.join(ROOT, "bin", "trace_run"), "--model", tiny_folders["B"],
                           "--dtype", dtype, "--out", str(out), "--max-tokens",
                           str(helpers.max_live_tokens(requests, steps))] + (["--eager"] if eager else []),
                          input=lines, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stderr[-2000:]
    assert [l for l in proc.stdout.split("\n") if l.startswith("done")] == [f"done {i}" for i in range(len(steps))]
    got = {}
    for i, s in enumerate(steps):
        rows = np.fromfile(out / f"{i}.f32", dtype="<f4").reshape(-1, 384)
        r = 0
        for e in s["entries"]:
            for _ in e["want"]:
                got.setdefault(e["id"], []).append(torch.from_numpy(rows[r].copy()))
                r += 1
        assert r == rows.shape[0]
    for rid in requests:
        assert helpers.relative_error(torch.stack(got[rid]), ref[rid]) < tol


@pytest.mark.parametrize("name,dtype,tol", [("D", "float32", 1e-4), ("D", "bfloat16", 6e-2), ("E", "bfloat16", 6e-2)])
def test_many_requests_arriving_at_random_into_a_scarce_pool(tiny_folders, name, dtype, tol):
    """Two hundred requests of random lengths arrive a few per step; the page pool holds a fraction of what twelve live
    requests may need, so requests give way and are computed again, while steps are decoded ahead of the host and
    replayed from captured graphs. Every token that comes out must be the plain implementation's best token given the
    tokens before it (or within the tolerance of it), and the cache's books must balance all the way."""
    import random

    from tt_transformers_b200 import from_pretrained
    from tt_transformers_b200.sampling import SamplingParams

    rng = random.Random(5)
    config, weights = plain_llama.read_model_folder(tiny_folders[name])
    vocab = config["vocab_size"]
    llm = from_pretrained(tiny_folders[name], dtype=dtype, max_batch_size=12, max_seq_len=448, page_size=16, num_pages=90,
                          max_step_tokens=192, max_chunk_tokens=96)
    todo = []
    for _ in range(200):
        n = min(rng.choice([1, 2, 3, 5, 17, 40, 96, 130, 200, 260]) + rng.randrange(0, 7), 440)
        todo.append(([rng.randrange(vocab) for _ in range(n)], rng.choice([1, 2, 8, 33, 64, 120])))
    live, steps = [], 0
    try:
        while todo or llm.has_unfinished():
            for _ in range(rng.choice([0, 1, 1, 2, 4, 8])):
                if todo:
                    prompt, new = todo.pop()
                    live.append(llm.add_request(prompt, SamplingParams(temperature=0.0, max_new_tokens=new, ignore_eos=True)))
            if llm.has_unfinished():
                llm.step()
                steps += 1
            if steps % 64 == 0:
                llm.engine.cache.audit()
        llm.engine.kernels.check_status()
        gave_way = llm._scheduler.preemptions
    finally:
        llm.cleanup()
    assert gave_way > 10, "the pool was meant to be too small"
    for r in live:
        assert r.finish_reason in ("length", "context") and len(r.output) >= 1
        seq = list(r.prompt) + list(r.output)
        if len(seq) < 2:
            continue
        logits = plain_llama.forward(config, weights, seq[:-1])
        for j, tok in enumerate(r.output):
            row = logits[len(r.prompt) - 1 + j]
            assert float(row.max() - row[tok]) <= tol * max(1.0, float(row.abs().max())), (len(r.prompt), j)


def test_the_demo_as_a_program(tiny_folders):
    """bin/demo with the reference demo's options: a folder without a tokenizer takes token ids and prints token ids,
    the same ones that greedy generation through the plain implementation gives."""
    prompt = helpers.random_tokens(384, 23, 77)
    config, weights = plain_llama.read_model_folder(tiny_folders["B"])
    want = plain_llama.greedy(config, weights, prompt, 12)
    proc = subprocess.run([sys.executable, os.path.join(ROOT, "bin", "demo"), "--hf-model", tiny_folders["B"], "--prompt",
                           ",".join(map(str, prompt)), "--max-new-tokens", "12", "--max-seq-len", "256", "--dtype", "float32"],
                          capture_output=True, text=True)
    assert proc.returncode == 0, proc.stderr[-2000:]
    got = [int(t) for t in proc.stdout.strip().split("\n")[-1].split()]
    assert len(got) == 12 and all(0 <= t < 384 for t in got)
    from tt_transformers_b200 import from_pretrained

    llm = from_pretrained(tiny_folders["B"], dtype="float32", max_batch_size=1, max_seq_len=256)
    try:
        assert llm.generate([prompt], max_new_tokens=12)[0] == got
    finally:
        llm.cleanup()
    assert got == want


MODEL_SIZED = {
    "architectures": ["LlamaForCausalLM"],
    "hidden_size": 2048, "num_hidden_layers": 2, "num_attention_heads": 32, "num_key_value_heads": 8,
    "head_dim": 64, "intermediate_size": 8192, "vocab_size": 128256, "rms_norm_eps": 1e-5,
    "max_position_embeddings": 131072, "rope_theta": 500000.0,
    "rope_scaling": {"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                     "original_max_position_embeddings": 8192},
    "tie_word_embeddings": True,
}


def test_the_real_layer_sizes_in_32_bit_and_bfloat16(tmp_path):
    """Two layers with the sizes of Llama 3.2 1B (width 2048, 32 heads in 8 groups, head size 64,
    feed-forward 8192, vocabulary 128256): whole, tail by tokens and mixed against the plain
    implementation."""
    from tt_transformers_b200.config import EngineConfig
    from tt_transformers_b200.engine.step import build_engine
    from tt_transformers_b200.weights import write_model_folder

    folder = write_model_folder(str(tmp_path / "sized"), MODEL_SIZED, seed=0, norm_std=0.05)
    requests = {"a": helpers.random_tokens(128256, 150, 1), "b": helpers.random_tokens(128256, 70, 2)}
    ref = helpers.plain_logits(folder, requests)
    for dtype, tol in (("float32", 1e-4), ("bfloat16", 4e-2)):
        engine = build_engine(folder, EngineConfig(dtype=dtype, page_size=16, num_pages=20, max_batch_size=2,
                                                   max_seq_len=256, device="cuda:0"))
        for steps in (helpers.steps_whole(requests), helpers.steps_decode_tail(requests, tail=12),
                      helpers.steps_mixed(requests)):
            got = helpers.run_steps(engine, steps)
            for rid in requests:
                assert helpers.relative_error(got[rid], ref[rid]) < tol, (dtype, rid)
        engine.close()
        del engine
        torch.cuda.empty_cache()


def test_token_match_at_full_depth():
    """Llama 3.2 1B with all 16 layers, random weights, float32: the logits of two prompts against the plain
    implementation in the four ways of cutting (the benchmark's token-match case)."""
    from tt_transformers_b200.cli import measure

    result = measure.run_token_match(measure.model_config("1b"), prompt_lengths=(80, 47))
    print(result)
    assert result["layers"] == 16 and set(result["modes"]) == {"whole", "decode_tail", "portions", "mixed"}
    for mode, figures in result["modes"].items():
        assert figures["max_relative_error"] <= 1e-4, (mode, figures)
        assert figures["argmax_agreement"] == 1.0, (mode, figures)


def test_engine_options_memory_share_graph_sizes_and_conservative_admission(tiny_folders):
    """The cache sized by a share of the device's memory, decode steps captured at chosen batch sizes, and requests
    admitted only when everything they may hold fits: the same tokens as with the defaults."""
    from tt_transformers_b200 import from_pretrained

    prompts = [helpers.random_tokens(512, n, 300 + n) for n in (12, 40, 7, 25, 18)]
    plain = from_pretrained(tiny_folders["D"], dtype="float32", max_batch_size=4, max_seq_len=256)
    expect = plain.generate(prompts, max_new_tokens=12)
    plain.cleanup()
    llm = from_pretrained(tiny_folders["D"], dtype="float32", max_batch_size=64, max_seq_len=4096, gpu_memory_fraction=1.0)
    assert llm.engine.cache.num_pages == 64 * 256           # capped by what every slot at full length needs
    free, total = torch.cuda.mem_get_info()
    share = (total - free + (64 << 20)) / total             # what is in use now and 64 MiB more
    small = from_pretrained(tiny_folders["D"], dtype="float32", max_batch_size=64, max_seq_len=4096,
                            gpu_memory_fraction=share, graph_batch_sizes=(1, 3), admission="conservative")
    assert 500 < small.engine.cache.num_pages < 8000, small.engine.cache.num_pages     # 16 KiB a page: about 4,000
    assert small.engine.graphs.sizes == [1, 3, 64]
    got = small.generate(prompts, max_new_tokens=12)
    assert got == expect
    assert 64 in small.engine.graphs.captured_sizes() and set(small.engine.graphs.captured_sizes()) <= {1, 3, 64}
    alone = small.generate(prompts[:3], max_new_tokens=5)               # three rows: the captured size 3
    assert alone == [e[:5] for e in expect[:3]] and 3 in small.engine.graphs.captured_sizes()
    assert small.last_stats["preemptions"] == 0
    small.cleanup()
    llm.cleanup()


def test_greedy_decoding_on_the_device_across_context_buckets(tiny_folders):
    """Decode steps are captured per batch size and context bucket. A greedy loop that feeds every step's own
    argmax to the next one on the device keeps doing so when the contexts grow into the next bucket (another graph
    with buffers of its own): the tokens equal the plain implementation's."""
    from tt_transformers_b200 import from_pretrained

    import plain_llama

    config, weights = plain_llama.read_model_folder(tiny_folders["D"])
    prompts = [helpers.random_tokens(512, n, 640 + n) for n in (11, 27)]
    expect = [plain_llama.greedy(config, weights, p, 60) for p in prompts]
    llm = from_pretrained(tiny_folders["D"], dtype="float32", page_size=16, max_batch_size=2, max_seq_len=256)
    llm.engine.graphs.MIN_CONTEXT_BUCKET = 16
    assert llm.generate(prompts, max_new_tokens=60) == expect
    buckets = sorted({bucket for _, bucket in llm.engine.graphs._graphs})
    assert buckets == [32, 64, 128], buckets
    # and through the engine's own decode loop, from the prompts' last tokens on
    engine = llm.engine
    from tt_transformers_b200.engine.step import StepEntry
    firsts = []
    for i, p in enumerate(prompts):
        logits = engine.step([StepEntry(f"g{i}", p, [len(p) - 1])])
        firsts.append(int(engine.kernels.sample(logits)[0]))
    rest = engine.decode_steps(["g0", "g1"], firsts, 59)
    assert [[firsts[i]] + [row[i] for row in rest] for i in range(2)] == expect
    llm.cleanup()


def test_the_references_benchmark_cases_on_a_tiny_model(tiny_folders):
    """eval-32 (the same prompts rotated through the rows of a 32-request batch give the same outputs) and
    token-accuracy (teacher forcing, bfloat16 against the float32 path) as bin/benchmark runs them."""
    from tt_transformers_b200 import from_pretrained
    from tt_transformers_b200.cli.benchmark import run_eval_32, run_token_accuracy

    llm = from_pretrained(tiny_folders["D"], dtype="bfloat16", max_batch_size=32, max_seq_len=256)
    result = run_eval_32(llm, repeats=3, new_tokens=16)
    llm.cleanup()
    assert result == {"repeats": 3, "prompts": 32, "deterministic": True}
    accuracy = run_token_accuracy(lambda dtype: from_pretrained(tiny_folders["D"], dtype=dtype, max_batch_size=1,
                                                                max_seq_len=512), prompt_len=200, forced=100)
    assert accuracy["positions"] == 101 and accuracy["top5"] >= 0.99 and accuracy["top1"] >= 0.9, accuracy


def test_abort_and_the_references_argument_names(tiny_folders):
    from tt_transformers_b200 import SamplingParams, from_pretrained

    with pytest.raises(TypeError):
        from_pretrained()
    with pytest.raises(ValueError):
        from_pretrained(hf_model=tiny_folders["A"], optimizations="fast")
    llm = from_pretrained(hf_model=tiny_folders["D"], optimizations="accuracy", max_batch_size=4, max_seq_len=128)
    assert llm.engine.runtime.dtype == torch.float32
    prompts = [helpers.random_tokens(512, n, 800 + n) for n in (9, 21, 14)]
    alone = llm.generate([prompts[0], prompts[2]], max_new_tokens=20)
    params = SamplingParams(max_new_tokens=20)
    reqs = [llm.add_request(p, params) for p in prompts]
    for _ in range(6):
        llm.step()
    llm.abort(reqs[1])                                     # in the middle of decoding, a step may be running ahead
    while llm.has_unfinished():
        llm.step()
    assert reqs[1].finish_reason == "aborted" and 0 < len(reqs[1].output) < 20
    assert [reqs[0].output, reqs[2].output] == alone       # the others are not disturbed
    llm.engine.cache.audit()
    assert llm.engine.cache.free_pages() == llm.engine.cache.num_pages
    llm.cleanup()


def test_warmup_captures_every_step_ahead_of_time(tiny_folders):
    from tt_transformers_b200 import from_pretrained

    prompts = [helpers.random_tokens(512, n, 900 + n) for n in (12, 40, 7)]
    plain = from_pretrained(tiny_folders["D"], dtype="float32", max_batch_size=4, max_seq_len=2048)
    expect = plain.generate(prompts, max_new_tokens=10) + plain.generate(prompts[:1], max_new_tokens=10)
    plain.cleanup()
    llm = from_pretrained(tiny_folders["D"], dtype="float32", max_batch_size=4, max_seq_len=2048)
    captured = llm.warmup()
    # batch sizes 1, 2, 4 in the context buckets 1,024 and 2,048; prompt buckets 32 .. 512
    assert captured == 3 * 2 + 5 and llm.engine.cache.free_pages() == llm.engine.cache.num_pages
    assert llm.warmup() == 0
    decode_graphs, prompt_graphs = dict(llm.engine.graphs._graphs), dict(llm.engine.prompt_graphs._graphs)
    got = llm.generate(prompts, max_new_tokens=10) + llm.generate(prompts[:1], max_new_tokens=10)
    assert got == expect
    assert llm.engine.graphs._graphs.keys() == decode_graphs.keys()           # nothing was captured while generating
    assert llm.engine.prompt_graphs._graphs.keys() == prompt_graphs.keys()
    llm.cleanup()
