"""Accuracy and performance cases, named as in the reference's benchmark.

    --case token-accuracy   teacher forcing: 512 prompt tokens, then 511 given tokens one per
                            step; how often the model's best token is the reference's best, and
                            among the reference's five best (examples/common/run_helpers.py:201-289).
                            The reference scores against tokens that a float32 run of the same
                            checkpoint produced on a book text; here the float32 path of this
                            engine produces them, on seeded random token ids.
    --case batch-1          one request: ~100 prompt tokens, 200 decode steps: time to first token,
                            tokens/s/user (examples/llama32_1b/benchmark.py:13-16,202-204)
    --case batch-32         32 requests, max_seq_len 1024, same workload
    --case batch-32-ci      32 requests, max_seq_len 2048, 1,024 decode steps
    --case eval-32          three repeats of a 32-request batch with the prompts rotated through
                            the rows; every prompt's output must be the same in every repeat
                            (examples/llama32_1b/benchmark.py:1026-1094)
    --optimizations         performance: bfloat16; accuracy: float32 (the reference's two
                            precision recipes, src/tt_transformers/models/llama32_1b/model.py:256-290,
                            are block-float formats of its own hardware)
Metrics as the reference computes them: TTFT = prefill time / batch; tokens/s/user = decode
steps / sum of step times without the first; tokens/s = that times the batch
(examples/common/run_helpers.py:86-101).
"""

from __future__ import annotations

import argparse
import json
import os
import time

import torch

EXAMPLE_CASES = ("token-accuracy", "batch-1", "batch-32", "batch-32-ci", "eval-32")


def _prompts(vocab, batch, seed=0, low=90, high=125):
    g = torch.Generator().manual_seed(seed)
    lengths = torch.randint(low, high + 1, (batch,), generator=g).tolist()
    return [torch.randint(0, vocab, (n,), generator=g).tolist() for n in lengths]


def run_perf(llm, batch, decode_steps):
    from ..sampling import SamplingParams

    prompts = _prompts(llm.engine.vocab_size, batch)
    params = SamplingParams(temperature=0.0, max_new_tokens=decode_steps + 1, ignore_eos=True)
    for warm in range(2):                       # the first pass captures the decode graphs
        for p in prompts:
            llm.add_request(p, params)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        while any(not r.output for r in llm._scheduler.running) or llm._scheduler.waiting:
            llm.step()
        torch.cuda.synchronize()
        prefill_s = time.perf_counter() - t0
        times = []
        while llm.has_unfinished():
            t = time.perf_counter()
            llm.step()
            times.append(time.perf_counter() - t)
    steady = times[1:]
    per_user = len(steady) / sum(steady)
    return {"batch": batch, "decode_steps": len(times), "ttft_ms": prefill_s * 1e3 / batch,
            "tokens_per_s_per_user": per_user, "tokens_per_s": per_user * batch}


def run_token_accuracy(load_llm, prompt_len=512, forced=511):
    from ..engine.step import StepEntry

    results = {}
    tokens = None
    for dtype in ("float32", "bfloat16"):
        llm = load_llm(dtype)
        engine = llm.engine
        if tokens is None:
            g = torch.Generator().manual_seed(0)
            tokens = torch.randint(0, engine.vocab_size, (prompt_len + forced,), generator=g).tolist()
        rows = [engine.step([StepEntry("t", tokens[:prompt_len], [prompt_len - 1])])[0].clone()]
        for i in range(prompt_len, prompt_len + forced):
            rows.append(engine.step([StepEntry("t", [tokens[i]], [0])])[0].clone())
        engine.finish("t")
        results[dtype] = torch.stack(rows).float().cpu()
        llm.cleanup()
        del llm
        torch.cuda.empty_cache()
    ref, got = results["float32"], results["bfloat16"]
    best = got.argmax(-1)
    top5 = ref.topk(5, dim=-1).indices
    return {"positions": ref.shape[0], "top1": float((best == ref.argmax(-1)).float().mean()),
            "top5": float((top5 == best[:, None]).any(-1).float().mean())}


def run_eval_32(llm, repeats=3, new_tokens=32):
    prompts = _prompts(llm.engine.vocab_size, 32, seed=1, low=20, high=60)
    outputs = []
    for r in range(repeats):
        order = prompts[r:] + prompts[:r]                  # the prompts move through the rows
        out = llm.generate(order, max_new_tokens=new_tokens, ignore_eos=True)
        outputs.append(out[len(out) - r:] + out[:len(out) - r])
    same = all(outputs[0] == o for o in outputs[1:])
    return {"repeats": repeats, "prompts": 32, "deterministic": same}


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--case", choices=EXAMPLE_CASES, default=EXAMPLE_CASES[0])
    parser.add_argument("--optimizations", choices=("performance", "accuracy"), default="performance")
    parser.add_argument("--hf-model", default=None, help="model folder (default: $HF_MODEL, else --random)")
    parser.add_argument("--random", default="llama-3.2-1b", help="named model with random weights")
    parser.add_argument("--n-layers", type=int, default=None)
    args = parser.parse_args(argv)
    from .common import load

    hf_model = args.hf_model or os.environ.get("HF_MODEL")
    dtype = "bfloat16" if args.optimizations == "performance" else "float32"
    sizes = {"batch-1": (1, 2048, 200), "batch-32": (32, 1024, 200), "batch-32-ci": (32, 2048, 1024)}
    if args.case == "token-accuracy":
        result = run_token_accuracy(lambda d: load(hf_model, args.random, max_batch_size=1, max_seq_len=1024,
                                                   dtype=d, n_layers=args.n_layers))
    elif args.case == "eval-32":
        llm = load(hf_model, args.random, max_batch_size=32, max_seq_len=1024, dtype=dtype, n_layers=args.n_layers)
        result = run_eval_32(llm)
        llm.cleanup()
    else:
        batch, max_seq_len, steps = sizes[args.case]
        llm = load(hf_model, args.random, max_batch_size=batch, max_seq_len=max_seq_len, dtype=dtype,
                   n_layers=args.n_layers, max_step_tokens=4096)
        result = run_perf(llm, batch, steps)
        llm.cleanup()
    result.update(case=args.case, optimizations=args.optimizations, model=hf_model or f"random:{args.random}")
    print(json.dumps(result))
    if args.case == "eval-32" and not result["deterministic"]:
        raise SystemExit(1)


if __name__ == "__main__":
    main()
