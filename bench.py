"""bench.py --gpus 1 --steps K --warmup W: decode and prefill throughput of the engine.

The model has the layer sizes of Llama 3.2 1B with random weights. The headline `value` is
decoded tokens per second at batch 8 with every request holding about `context` tokens; a
"step" is one decode step. It prints ONE JSON line. The engine runs on one GPU: for
--gpus N > 1 it prints one line that says so and exits with 2.
"""

from __future__ import annotations

import argparse
import atexit
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

MODEL_1B = {
    "architectures": ["LlamaForCausalLM"],
    "hidden_size": 2048, "num_hidden_layers": 16, "num_attention_heads": 32, "num_key_value_heads": 8,
    "head_dim": 64, "intermediate_size": 8192, "vocab_size": 128256, "rms_norm_eps": 1e-5,
    "max_position_embeddings": 131072, "rope_theta": 500000.0,
    "rope_scaling": {"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                     "original_max_position_embeddings": 8192},
    "tie_word_embeddings": True,
}
FULL_LAYERS = 16
PAGE = 16
PREFILL_TOKENS = 2048
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.isfile(path):
        with open(path) as f:
            data = json.load(f)
        return {"hbm_gbs": float(data["hbm_gbs"]), "bf16_tflops": float(data["bf16_tflops"]), "source": "measured"}
    return {**FALLBACK_PEAKS, "source": "fallback"}


class ClockSampler:
    """nvidia-smi in the background for the whole run (reading only); a timed region keeps the samples that
    arrived while it ran, or, if the region was shorter than the sampling period, the sample nearest to it."""

    QUERY = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, period_ms: int = 50):
        self.samples = []                   # (arrival time, SM MHz, max SM MHz, active reasons)
        self.proc = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", "0", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", str(period_ms)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            return
        atexit.register(self.stop)          # whatever way the run ends, the child does not outlive it
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 6:
                continue
            try:
                clock, max_clock = float(parts[0]), float(parts[1])
            except ValueError:
                continue
            reasons = [n for n, flag in zip(self.NAMES, parts[2:6]) if flag.lower().startswith("active")]
            self.samples.append((time.perf_counter(), clock, max_clock, reasons))

    def wait_for_first_sample(self, timeout_s: float = 5.0):
        end = time.perf_counter() + timeout_s
        while self.proc is not None and not self.samples and time.perf_counter() < end:
            time.sleep(0.01)

    def __enter__(self):
        self.t0 = time.perf_counter()
        return self

    def __exit__(self, *exc):
        t1 = time.perf_counter()
        self.summary = {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}
        if self.proc is None:
            return
        time.sleep(0.03)                    # a sample taken at the region's end may still be on its way
        inside = [x for x in self.samples if self.t0 <= x[0] <= t1 + 0.03]
        if not inside and self.samples:
            inside = [min(self.samples, key=lambda x: min(abs(x[0] - self.t0), abs(x[0] - t1)))]
        if inside:
            self.summary = {"sm_mhz": statistics.median(x[1] for x in inside), "sm_max_mhz": inside[-1][2],
                            "reasons": sorted({r for x in inside for r in x[3]})}

    def stop(self):
        if self.proc is not None and self.proc.poll() is None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()


def decode_bytes(cfg, layers, batch, context, elem=2):
    """Bytes a decode step has to read: every weight it uses once, and the cache of the live requests."""
    d, inter, vocab = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    heads, kv, hd = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
    per_layer = (heads + 2 * kv) * hd * d + heads * hd * d + 3 * inter * d + 2 * d
    weights = (layers * per_layer + vocab * d + d) * elem
    cache = batch * context * layers * 2 * kv * hd * elem
    return weights + cache


def prefill_flops(cfg, layers, tokens):
    d, inter, vocab = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    heads, kv, hd = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
    linear = 2 * tokens * ((heads + 2 * kv) * hd * d + heads * hd * d + 3 * inter * d)
    attention = 2 * 2 * heads * hd * tokens * (tokens + 1) / 2      # causal QK^T and PV
    return layers * (linear + attention) + 2 * vocab * d            # plus one row of logits


def reference_arm() -> dict:
    """The reference's own generation path needs its vendor's accelerator library (ttnn) and a
    Tenstorrent device. If the package under baseline/_ref and that library import, its stock
    loader would be driven here; where they do not, the arm says so in one line."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "tt_transformers")):
        return {"impl": "reference", "unavailable": "baseline/_ref holds no installed tt_transformers package"}
    sys.path.insert(0, ref)
    try:
        import ttnn  # noqa: F401
    except Exception as e:            # not installed here: there is no wheel of it offline and no CUDA backend
        return {"impl": "reference", "unavailable":
                f"tt_transformers is installed under baseline/_ref (--no-deps), but its accelerator library "
                f"cannot be imported ({type(e).__name__}: {e}); every forward op of the reference is a call into it"}
    return {"impl": "reference", "unavailable": "ttnn imported, but no Tenstorrent device is present on a B200 box"}


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=64)
    parser.add_argument("--warmup", type=int, default=8)
    parser.add_argument("--impl", default="ours", choices=("ours", "reference"))
    parser.add_argument("--batch", type=int, default=8)
    parser.add_argument("--context", type=int, default=8192)
    parser.add_argument("--layers", type=int, default=FULL_LAYERS)
    parser.add_argument("--points", default="1,64", help="other decode batch sizes to report, comma separated")
    parser.add_argument("--skip-prefill", action="store_true", help="leave the prefill measurement out (for profiling decode)")
    parser.add_argument("--skip-e2e", action="store_true", help="leave the end-to-end measurement out (for profiling)")
    parser.add_argument("--fill", default="prefill", choices=("prefill", "synthetic"),
                        help="how the cache gets its context before decoding: through the engine's own prefill, "
                             "or filled with random numbers (faster; decode time does not depend on the values)")
    args = parser.parse_args(argv)

    if args.impl == "reference":
        print(json.dumps(reference_arm()))
        return 0
    if args.gpus != 1:
        print(f"bench.py: this engine runs on one GPU; --gpus {args.gpus} is not supported")
        return 2
    warmup = max(args.warmup, 3)

    import torch

    from tt_transformers_b200.config import EngineConfig
    from tt_transformers_b200.engine.llm import LLM
    from tt_transformers_b200.engine.step import StepEntry, build_engine
    from tt_transformers_b200.sampling import SamplingParams
    from tt_transformers_b200.weights import random_tensors

    sampler = ClockSampler()             # runs for the whole measurement; each timed region takes its own samples
    cfg = dict(MODEL_1B, num_hidden_layers=args.layers)
    pk = peaks()
    device = "cuda:0"
    torch.cuda.set_device(0)
    point_batches = [int(x) for x in args.points.split(",") if x]
    max_batch = max([args.batch] + point_batches)
    tensors = random_tensors(cfg, seed=0, dtype=torch.bfloat16, device=device)
    pages_per_request = -(-args.context // PAGE)
    engine = build_engine(config_dict=cfg, tensors=tensors, engine_config=EngineConfig(
        dtype="bfloat16", page_size=PAGE, num_pages=pages_per_request * max_batch, max_batch_size=max_batch,
        max_seq_len=args.context, max_step_tokens=PREFILL_TOKENS, max_chunk_tokens=PREFILL_TOKENS, device=device))
    del tensors
    llm = LLM(engine)
    kernels = engine.kernels
    gen = torch.Generator().manual_seed(0)

    def prompt(n):
        return torch.randint(0, cfg["vocab_size"], (n,), generator=gen).tolist()

    def timed(fn, reps):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record()
        for _ in range(reps):
            fn()
        end.record()
        torch.cuda.synchronize()
        return start.elapsed_time(end) / reps

    # ------------------------------------------------------------------ prefill of 2,048 tokens, one step
    pre_tokens = prompt(PREFILL_TOKENS)

    def prefill_once():
        engine.step([StepEntry("p", pre_tokens, [PREFILL_TOKENS - 1])])
        engine.finish("p")

    prefill_ms = float("nan")
    if not args.skip_prefill:
        for _ in range(3):
            prefill_once()
        # steps back to back, so that the host's part of a step runs under the step before; the median of three
        # such runs, so that one slow run does not decide
        prefill_ms = statistics.median(timed(prefill_once, 5) for _ in range(3))
    flops = prefill_flops(cfg, args.layers, PREFILL_TOKENS)
    prefill = {"value": round(PREFILL_TOKENS / prefill_ms * 1e3, 1), "tokens": PREFILL_TOKENS,
               "ms": round(prefill_ms, 3), "frac": round(flops / (prefill_ms * 1e-3) / (pk["bf16_tflops"] * 1e12), 4)}

    # ------------------------------------------------------------------ decode
    def fill(batch, length):
        """`batch` requests that hold `length` tokens each."""
        ids = [f"d{i}" for i in range(batch)]
        if args.fill == "synthetic":
            for rid in ids:
                engine.cache.admit(rid)
                engine.cache.reserve(rid, length)
                engine.cache.commit(rid, length)
            for g in engine.cache.groups:
                if g.pool is not None:
                    for tensor in g.storage.values():
                        tensor.normal_(0, 1)
            return ids
        for rid in ids:
            toks = prompt(length)
            for i in range(0, length, PREFILL_TOKENS):
                engine.step([StepEntry(rid, toks[i:i + PREFILL_TOKENS], [])])
        return ids

    def decode_run(batch, steps, warm):
        ids = fill(batch, args.context - steps - warm - 1)
        # the engine's decode loop: every step takes its tokens from the sampler's output of the step
        # before, on the device; the sampled ids reach the host behind the steps
        tokens = engine.decode_steps(ids, [1] * batch, warm)[-1]
        before = kernels.launches
        sampler.wait_for_first_sample()
        with sampler as clocks:
            ms = timed(lambda: engine.decode_steps(ids, tokens, steps), 1) / steps
        launches = kernels.launches - before
        for rid in ids:
            engine.finish(rid)
        return ms, launches, clocks.summary

    ms_step, launches, clocks = decode_run(args.batch, args.steps, warmup)
    value = args.batch / ms_step * 1e3
    need = decode_bytes(cfg, args.layers, args.batch, args.context)
    achieved = need / (ms_step * 1e-3) / 1e9
    points = {}
    for b in point_batches:
        ms_b, _, _ = decode_run(b, max(8, args.steps // 2), warmup)
        points[f"decode_b{b}"] = round(b / ms_b * 1e3, 1)

    # ------------------------------------------------------------------ end to end through the Python entry point
    params = SamplingParams(temperature=0.0, max_new_tokens=1 << 30, ignore_eos=True)
    # Requests whose prompts are done decode while the others' prompts are still being computed, one
    # token for every later prompt portion: leave room for that, so that nobody reaches the context
    # limit (and leaves the batch) inside the timed region.
    length = args.context - args.steps - warmup - 2 - args.batch * (args.context // PREFILL_TOKENS + 1)
    if args.skip_e2e:
        e2e = None
    elif args.fill == "synthetic":
        reqs = []
        for i in range(args.batch):       # the prompts' last token goes through the engine; the rest is filled
            r = llm.add_request(prompt(length), params)
            reqs.append(r)
        sched = llm._scheduler
        for r in list(sched.waiting):
            sched.waiting.remove(r)
            engine.cache.admit(r.request_id)
            engine.cache.reserve(r.request_id, length - 1)
            engine.cache.commit(r.request_id, length - 1)
            r.num_computed = length - 1
            sched.running.append(r)
    else:
        for i in range(args.batch):
            llm.add_request(prompt(length), params)
        while any(r.num_computed < len(r.prompt) for r in llm._scheduler.running) or llm._scheduler.waiting:
            llm.step()
    if not args.skip_e2e:
      for _ in range(warmup):
        llm.step()
      torch.cuda.synchronize()
      h2d, d2h = engine.h2d_bytes, llm.d2h_bytes
      t0 = time.perf_counter()
      for _ in range(args.steps):
        llm.step()
      torch.cuda.synchronize()
      e2e_ms = (time.perf_counter() - t0) * 1e3 / args.steps
      e2e = {"value": round(args.batch / e2e_ms * 1e3, 1), "unit": "tokens/s",
             "h2d_bytes_per_step": (engine.h2d_bytes - h2d) // args.steps,
             "d2h_bytes_per_step": (llm.d2h_bytes - d2h) // args.steps}

    line = {
        "metric": "decode tokens/s, Llama 3.2 1B sizes, batch 8", "value": round(value, 1), "unit": "tokens/s",
        "n_gpus": 1, "steps": args.steps, "warmup": warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: random weights N(0, 0.02), uniform-random token ids",
        "config": {"model": "llama-3.2-1b-sizes", "layers": args.layers, "layers_full": FULL_LAYERS,
                   "hidden": cfg["hidden_size"], "heads": cfg["num_attention_heads"],
                   "kv_heads": cfg["num_key_value_heads"], "head_dim": cfg["head_dim"],
                   "intermediate": cfg["intermediate_size"], "vocab": cfg["vocab_size"], "global_batch": args.batch,
                   "seq_len": args.context, "page_size": PAGE, "prefill_tokens": PREFILL_TOKENS,
                   "parallelism": "single-gpu", "cache_fill": args.fill,
                   "l2": "inputs larger than L2 (weights and cache are re-read every step)",
                   "peaks": pk["source"]},
        "clocks": clocks, "e2e": e2e, "gpu_launches": launches, "prefill": prefill,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / pk["hbm_gbs"], 4)},
        "points": points,
    }
    sampler.stop()
    print(json.dumps(line))
    return 0


if __name__ == "__main__":
    sys.exit(main())
