"""The step function, the cache and the entry point with the plain PyTorch twins of the
kernels in the kernels' place, on the CPU: how requests are cut, batched and paged must not
change the logits. (The CUDA kernels themselves are tested under -m gpu.)"""

import io
import json
import os

import pytest
import torch

import helpers
import plain_llama
from conftest import TINY_A, TINY_B
from torch_kernels import TorchKernels
from tt_transformers_b200.cache import OutOfPages
from tt_transformers_b200.config import EngineConfig
from tt_transformers_b200.engine.llm import from_pretrained
from tt_transformers_b200.engine.step import StepEntry, build_engine
from tt_transformers_b200.engine.trace import run_trace

CONFIGS = {"A": TINY_A, "B": TINY_B}


def cpu_engine(folder, page_size, num_pages, slots=4, max_seq_len=256):
    return build_engine(folder, EngineConfig(dtype="float32", page_size=page_size, num_pages=num_pages,
                                             max_batch_size=slots, max_seq_len=max_seq_len, max_step_tokens=4096,
                                             device="cpu"), kernels=TorchKernels())


@pytest.mark.parametrize("name,lengths,page", [("A", (7, 13, 40), 4), ("B", (5, 17, 33, 50), 8)])
@pytest.mark.parametrize("cut", ["whole", "tail", "portions", "mixed"])
def test_cuttings_match_plain(tiny_folders, name, lengths, page, cut):
    vocab = CONFIGS[name]["vocab_size"]
    requests = {f"r{i}": helpers.random_tokens(vocab, n, i) for i, n in enumerate(lengths)}
    ref = helpers.plain_logits(tiny_folders[name], requests)
    steps = {"whole": helpers.steps_whole, "tail": lambda r: helpers.steps_decode_tail(r, 8),
             "portions": helpers.steps_portions, "mixed": helpers.steps_mixed}[cut](requests)
    tokens = helpers.max_live_tokens(requests, steps, rounding=page)
    engine = cpu_engine(tiny_folders[name], page, -(-tokens // page))
    got = helpers.run_steps(engine, steps)
    engine.cache.audit()
    assert engine.cache.free_pages() == engine.cache.num_pages
    for rid in ref:
        assert helpers.relative_error(got[rid], ref[rid]) < 1e-5


def test_step_refuses_what_it_cannot_run(tiny_folders):
    engine = cpu_engine(tiny_folders["A"], 4, 3, slots=2, max_seq_len=12)
    with pytest.raises(ValueError, match="no tokens"):
        engine.step([StepEntry("a", [], [])])
    with pytest.raises(ValueError, match="twice"):
        engine.step([StepEntry("a", [1], []), StepEntry("a", [2], [])])
    with pytest.raises(ValueError, match="vocabulary"):
        engine.step([StepEntry("a", [256], [])])
    assert not engine.cache.is_live("a")
    with pytest.raises(ValueError, match="outside"):
        engine.step([StepEntry("a", [1, 2], [2])])
    engine.step([StepEntry("a", [1] * 8, [])])
    with pytest.raises(OutOfPages):                       # 3 pages of 4: b's 5 tokens need 2, one is free
        engine.step([StepEntry("a", [1], [0]), StepEntry("b", [1] * 5, [])])
    assert engine.cache.free_pages() == 1 and not engine.cache.is_live("b") and engine.cache.length("a") == 8
    engine.cache.audit()
    assert engine.step([StepEntry("a", [1], [0])]).shape == (1, 256)
    with pytest.raises(ValueError, match="limit"):
        engine.step([StepEntry("a", [1] * 4, [])])
    engine.finish("a")
    assert engine.cache.free_pages() == 3


def test_generate_matches_plain_greedy_under_pressure(tiny_folders):
    config, weights = plain_llama.read_model_folder(tiny_folders["B"])
    prompts = [helpers.random_tokens(384, n, 10 + n) for n in (5, 17, 33)]
    expect = [plain_llama.greedy(config, weights, p, 8) for p in prompts]
    # 9 pages of 8 tokens for 3 requests that end at 13, 25 and 41 tokens: they cannot all stay
    llm = from_pretrained(tiny_folders["B"], dtype="float32", page_size=8, num_pages=9, max_batch_size=3,
                          max_seq_len=128, max_step_tokens=16, max_chunk_tokens=8, device="cpu", kernels=TorchKernels())
    assert llm.generate(prompts, max_new_tokens=8) == expect
    assert llm.last_stats["preemptions"] >= 1
    llm.engine.cache.audit()
    assert llm.engine.cache.free_pages() == 9
    ids = torch.tensor([[0, 0] + prompts[0], prompts[0] + [0, 0]])
    mask = torch.tensor([[0, 0] + [1] * 5, [1] * 5 + [0, 0]])
    out = llm.generate(ids, mask, max_new_tokens=3, pad_token_id=0)
    assert out.shape == (2, 10) and out[0, 7:].tolist() == expect[0][:3] and out[1, 7:].tolist() == expect[0][:3]
    with pytest.raises(TypeError):
        llm.generate(prompts, num_beams=4)
    with pytest.raises(ValueError, match="KV pages"):
        llm.generate([list(range(60))], max_new_tokens=60)


def test_sampled_tokens_do_not_depend_on_the_batch(tiny_folders):
    llm = from_pretrained(tiny_folders["B"], dtype="float32", page_size=8, num_pages=40, max_batch_size=4,
                          max_seq_len=128, device="cpu", kernels=TorchKernels())
    prompts = [helpers.random_tokens(384, n, n) for n in (6, 11, 19)]
    from tt_transformers_b200.sampling import SamplingParams

    params = [SamplingParams(temperature=0.8, seed=100 + i, max_new_tokens=6) for i in range(3)]
    together = [r.output for r in llm.generate_requests(prompts, params)]
    alone = [llm.generate_requests([p], [sp])[0].output for p, sp in zip(prompts, params)]
    assert together == alone
    assert len({tuple(o) for o in together}) == 3


def test_eos_and_padding(tiny_folders):
    config, weights = plain_llama.read_model_folder(tiny_folders["B"])
    prompt = helpers.random_tokens(384, 33, 43)
    expect = plain_llama.greedy(config, weights, prompt, 6)
    stop = next(j for j in range(1, 6) if expect[j] not in expect[:j])     # a token that ends the row at place j
    llm = from_pretrained(tiny_folders["B"], dtype="float32", page_size=4, max_batch_size=2, max_seq_len=64,
                          device="cpu", kernels=TorchKernels())
    out = llm.generate(torch.tensor([prompt, prompt[:20] + [0] * 13]), torch.tensor([[1] * 33, [1] * 20 + [0] * 13]),
                       max_new_tokens=6, eos_token_id=expect[stop], pad_token_id=383)
    assert out.shape[0] == 2 and out[0, 33:33 + stop + 1].tolist() == expect[:stop + 1]
    assert all(t == 383 for t in out[0, 33 + stop + 1:].tolist())          # a finished row is padded
    assert llm.generate([prompt], max_new_tokens=6, eos_token_id=expect[stop], ignore_eos=True)[0] == expect


def test_trace_replay_writes_logits(tiny_folders, tmp_path):
    requests = {"a": helpers.random_tokens(256, 21, 1), "b": helpers.random_tokens(256, 9, 2)}
    ref = helpers.plain_logits(tiny_folders["A"], requests)
    lines = [
        {"step": 0, "entries": [{"id": "a", "tokens": requests["a"][:10], "want": [0, 9]}], "end": []},
        {"step": 1, "entries": [{"id": "a", "tokens": requests["a"][10:12], "want": []},
                                {"id": "b", "tokens": requests["b"], "want": [8]}], "end": ["b"]},
        {"step": 5, "entries": [{"id": "a", "tokens": requests["a"][12:], "want": [8]}], "end": ["a"]},
    ]
    log = io.StringIO()
    run_trace(tiny_folders["A"], "float32", str(tmp_path), 128, [json.dumps(l) for l in lines], log=log,
              device="cpu", kernels=TorchKernels(), page_size=16)
    assert log.getvalue().split() == ["done", "0", "done", "1", "done", "5"]
    assert sorted(os.listdir(tmp_path)) == ["0.f32", "1.f32", "5.f32"]
    import numpy as np

    s0 = np.fromfile(tmp_path / "0.f32", dtype="<f4").reshape(2, 256)
    assert np.allclose(s0, ref["a"][[0, 9]].numpy(), atol=1e-5)
    s1 = np.fromfile(tmp_path / "1.f32", dtype="<f4").reshape(1, 256)
    assert np.allclose(s1, ref["b"][[8]].numpy(), atol=1e-5)
    s5 = np.fromfile(tmp_path / "5.f32", dtype="<f4").reshape(1, 256)
    assert np.allclose(s5, ref["a"][[20]].numpy(), atol=1e-5)
