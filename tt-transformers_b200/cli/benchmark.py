"""Accuracy and performance cases.

The engine's own cases (one JSON object out; `--json FILE` also writes it to a file):
    --case prefill-2048     one prompt of 2,048 tokens in one step: tokens/s, share of the bf16 peak
    --case decode-b1|b8|b64 decode steps at that batch, every request holding about --context tokens:
                            tokens/s, tokens/s/user, share of the HBM peak that (weights + live cache) per step
                            stands for; decode-b1 also reports the time to first token of a 128-token prompt
    --case mixed-3b         32 requests, prompt lengths uniform in [128, 2048], 256 decoded tokens each, through
                            the scheduler with its token budget (Llama 3.2 3B sizes unless --model says otherwise)
    --case decode-8b-b64    64 requests with 4,096-token prompts, context limit 32,768, decode (Llama 3.1 8B sizes)
    --case token-match      float32 logits against the plain implementation (tests/plain_llama.py) on the same
                            random weights, all layers, in four ways of cutting the prompts into steps
    --case all              every case above, one object holding them all
    --case decode-sweep     decode steps over batch sizes 1, 8, 32, 64 and contexts 2,048, 8,192, 32,768 under ONE engine
                            whose context limit is 32,768 (cache filled with random numbers; combinations whose cache
                            exceeds 90 GB left out): step time and share of the HBM peak for each
    --case prefill-sweep    one prompt of 128, 512, 2,048, 8,192 and 32,768 tokens through the step function in portions of
                            at most 2,048 tokens: time, tokens/s and share of the bf16 peak (products and causal attention)
    --model {1b,3b,8b}      layer sizes (random weights); --n-layers cuts the model short
    --context N --steps K   context held while decoding, timed decode steps

The reference's cases, by its names (examples/llama32_1b/benchmark.py:1100-1121):
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
ENGINE_CASES = ("prefill-2048", "decode-b1", "decode-b8", "decode-b64", "mixed-3b", "decode-8b-b64", "token-match", "all")
EXTRA_CASES = ("decode-sweep", "prefill-sweep")


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
        # every request's first token is on the host now; the decode step that LLM.step has already launched for
        # the tokens after it is not part of the time to first token
        prefill_s = time.perf_counter() - t0
        torch.cuda.synchronize()
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


def run_engine_case(case: str, model: str, context: int, steps: int, warmup: int, n_layers=None, fill="prefill") -> dict:
    """One of the engine's own cases; every figure through tt_transformers_b200.cli.measure."""
    from ..engine.llm import LLM
    from . import measure

    if case == "decode-sweep":
        from . import measure as m

        cfg = m.model_config(model or "1b")
        layers = n_layers or cfg["num_hidden_layers"]
        cfg = dict(cfg, num_hidden_layers=layers)
        per_token = m.cache_bytes_per_token(cfg, layers)
        grid = [(b, c) for c in (2048, 8192, 32768) for b in (1, 8, 32, 64) if b * c * per_token < 90e9]
        engine = m.make_engine(cfg, max_batch=64, context=32768 + 64, pool_tokens=max(b * (c + 64) for b, c in grid))
        rows = []
        for b, c in grid:
            r = m.measure_decode(engine, cfg, layers, m.peaks(), b, c, steps, warmup, how="synthetic")
            rows.append({"batch": b, "context": c, "ms_per_step": r["ms_per_step"], "tokens_per_s": r["tokens_per_s"],
                         "gb_per_step": round(r["roofline"]["bytes_per_step"] / 1e9, 2), "frac": r["roofline"]["frac"]})
        engine.close()
        return {"case": case, "model": m.MODEL_NAMES.get(model or "1b"), "layers": layers, "context_limit": 32768 + 64,
                "peaks": m.peaks()["source"], "rows": rows}
    if case == "prefill-sweep":
        from ..engine.step import StepEntry

        cfg = measure.model_config(model or "1b")
        layers = n_layers or cfg["num_hidden_layers"]
        cfg = dict(cfg, num_hidden_layers=layers)
        pk = measure.peaks()
        portion = measure.PREFILL_TOKENS
        engine = measure.make_engine(cfg, max_batch=1, context=32768 + 64)
        prompts = measure.Prompts(cfg["vocab_size"])
        rows = []
        for n in (128, 512, 2048, 8192, 32768):
            ids = prompts(n)

            def once():
                for at in range(0, n, portion):
                    part = ids[at:at + portion]
                    engine.step([StepEntry("p", part, [len(part) - 1] if at + portion >= n else [])])
                engine.finish("p")

            for _ in range(2):
                once()
            ms = measure.timed(once, 3)
            flops = measure.prefill_flops(cfg, layers, n)
            rows.append({"tokens": n, "ms": round(ms, 3), "tokens_per_s": round(n / ms * 1e3),
                         "frac": round(flops / (ms * 1e-3) / (pk["bf16_tflops"] * 1e12), 3)})
        engine.close()
        return {"case": case, "model": measure.MODEL_NAMES.get(model or "1b"), "layers": layers, "portion": portion,
                "peaks": pk["source"], "rows": rows}
    if case == "all":
        out = {}
        for each in ENGINE_CASES[:-1]:
            out[each] = run_engine_case(each, model, context, steps, warmup, n_layers, fill)
            torch.cuda.empty_cache()
        return out
    if case == "mixed-3b" and model is None:
        model = "3b"
    if case == "decode-8b-b64" and model is None:
        model = "8b"
    model = model or "1b"
    cfg = measure.model_config(model)
    layers = n_layers or cfg["num_hidden_layers"]
    cfg = dict(cfg, num_hidden_layers=layers)
    pk = measure.peaks()
    out = {"case": case, "model": measure.MODEL_NAMES.get(model, model), "layers": layers,
           "layers_full": measure.model_config(model)["num_hidden_layers"], "dtype": "bfloat16"}
    if case == "token-match":
        out.update(measure.run_token_match(cfg, layers=layers), dtype="float32")
        return out
    sampler = measure.ClockSampler()
    try:
        if case == "prefill-2048":
            engine = measure.make_engine(cfg, max_batch=1, context=max(context or 4096, measure.PREFILL_TOKENS + measure.PAGE))
            out.update(measure.measure_prefill(engine, cfg, layers, pk))
        elif case in ("decode-b1", "decode-b8", "decode-b64"):
            batch = int(case.split("-b")[1])
            context = context or 8192
            engine = measure.make_engine(cfg, max_batch=batch, context=context)
            if batch == 1:
                out["ttft"] = measure.measure_ttft(engine, cfg, 128)
            out.update(measure.measure_decode(engine, cfg, layers, pk, batch, context, steps, warmup, sampler=sampler, how=fill))
        elif case == "mixed-3b":
            context = context or 8192
            engine = measure.make_engine(cfg, max_batch=32, context=context, pool_tokens=32 * (2048 + 256 + measure.PAGE))
            out.update(measure.run_mixed(LLM(engine), cfg, layers, pk, sampler=sampler), context=context)
        elif case == "decode-8b-b64":
            context = context or 32768
            prompt = 4096
            engine = measure.make_engine(cfg, max_batch=64, context=context,
                                         pool_tokens=64 * (prompt + steps + warmup + 2 * measure.PAGE))
            # every request holds `prompt` tokens when decoding starts
            out.update(measure.measure_decode(engine, cfg, layers, pk, 64, prompt + steps + warmup + 1, steps, warmup,
                                              sampler=sampler, how=fill), prompt_tokens=prompt, context_limit=context)
        else:
            raise SystemExit(f"unknown case {case!r}")
        engine.close()
    finally:
        sampler.stop()
    return out


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--case", choices=ENGINE_CASES + EXTRA_CASES + EXAMPLE_CASES, default=EXAMPLE_CASES[0])
    parser.add_argument("--optimizations", choices=("performance", "accuracy"), default="performance")
    parser.add_argument("--hf-model", default=None, help="model folder (default: $HF_MODEL, else --random)")
    parser.add_argument("--random", default="llama-3.2-1b", help="named model with random weights (the reference's cases)")
    parser.add_argument("--model", choices=("1b", "3b", "8b"), default=None, help="layer sizes for the engine's own cases")
    parser.add_argument("--context", type=int, default=None, help="tokens every request holds while decoding")
    parser.add_argument("--steps", type=int, default=64, help="timed decode steps")
    parser.add_argument("--warmup", type=int, default=8)
    parser.add_argument("--fill", default="prefill", choices=("prefill", "synthetic"))
    parser.add_argument("--json", default=None, metavar="FILE", help="also write the result object to FILE")
    parser.add_argument("--n-layers", type=int, default=None)
    args = parser.parse_args(argv)
    from .common import load

    if args.case in ENGINE_CASES + EXTRA_CASES:
        result = run_engine_case(args.case, args.model, args.context, args.steps, max(args.warmup, 3), args.n_layers, args.fill)
        text = json.dumps(result)
        print(text)
        if args.json:
            with open(args.json, "w") as f:
                f.write(text + "\n")
        if args.case == "token-match" and not (result["max_relative_error"] <= 1e-4 and result["argmax_agreement"] == 1.0):
            raise SystemExit(1)
        return

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
    text = json.dumps(result)
    print(text)
    if args.json:
        with open(args.json, "w") as f:
            f.write(text + "\n")
    if args.case == "eval-32" and not result["deterministic"]:
        raise SystemExit(1)


if __name__ == "__main__":
    main()
