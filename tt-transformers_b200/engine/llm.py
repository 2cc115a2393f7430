"""The Python entry point: from_pretrained() and generate(), in the reference's manner.

The reference: from_pretrained(mesh, hf_model=..., max_batch_size, max_seq_len, n_layers,
dtype, ...) (src/tt_transformers/models/llama32_1b/hf_generator.py:380-394) gives an object
with generate(input_ids, attention_mask, *, max_new_tokens, do_sample, temperature, top_k,
top_p, eos_token_id, pad_token_id) -> prompt + continuation, finished rows padded
(src/tt_transformers/models/hf_generation.py:222-413), and cleanup(). The same names and
meanings are kept here; `model` is a folder on disk, and prompts may also be given as
lists of token ids, which gives lists back.
"""

from __future__ import annotations

import os
from typing import Dict, List, Optional, Sequence, Union

import torch

from ..config.engine import EngineConfig
from ..sampling.params import SamplingParams
from ..sampling.sampler import Sampler
from .graph import OWN_ARGMAX
from .scheduler import Request, Scheduler
from .step import Engine, StepEntry, build_engine

class _Flight:
    """A step that has been launched: which requests its rows belong to, where the sampled ids
    will arrive on the host, and what every request held before it (to take it back)."""

    def __init__(self, ids, tokens_dev, tokens_host, event, lengths_before):
        self.ids, self.tokens_dev, self.tokens_host = ids, tokens_dev, tokens_host
        self.event, self.lengths_before = event, lengths_before

    def result(self) -> List[int]:
        if self.event is not None:
            self.event.synchronize()
        return self.tokens_host.tolist()


_UNSET = object()
# what the reference falls back to when neither the call nor the checkpoint says otherwise
# (src/tt_transformers/models/hf_generation.py:26,277)
_DEFAULTS = {"do_sample": False, "temperature": 1.0, "top_k": 50, "top_p": 1.0, "max_new_tokens": 128}


class LLM:
    def __init__(self, engine: Engine, eos_token_ids: Sequence[int] = (), pad_token_id: Optional[int] = None,
                 tokenizer=None):
        self.engine = engine
        self.config = engine.model_config
        self.sampler = Sampler(engine.kernels, engine.runtime.device)
        self.eos_token_ids = tuple(eos_token_ids)
        self.pad_token_id = pad_token_id
        self.tokenizer = tokenizer
        self._busy = False
        self._ahead: Optional[_Flight] = None
        self.look_ahead = True            # launch the next decode step while the host waits for this one's ids
        self._scheduler: Optional[Scheduler] = None
        self._next_id = 0
        self.steps = 0
        self.d2h_bytes = 0                  # bytes of sampled token ids read back so far
        self.last_stats: Dict[str, float] = {}

    # ------------------------------------------------------------------ generation
    def generate(self, input_ids, attention_mask=None, *, max_new_tokens=_UNSET, do_sample=_UNSET,
                 temperature=_UNSET, top_k=_UNSET, top_p=_UNSET, eos_token_id=_UNSET, pad_token_id=_UNSET,
                 seed: Optional[int] = None, ignore_eos: bool = False, **unknown):
        """Continue every prompt. input_ids: an integer tensor [batch, width] on the CPU with
        an optional attention_mask (padding on either side), giving an int64 tensor
        [batch, width + n] with finished rows padded; or a list of lists of token ids, giving
        the continuations as lists."""
        if unknown:
            raise TypeError(f"generate() got unexpected arguments: {sorted(unknown)}")
        opt = lambda value, key: _DEFAULTS[key] if value is _UNSET else value  # noqa: E731
        max_new_tokens = int(opt(max_new_tokens, "max_new_tokens"))
        do_sample = bool(opt(do_sample, "do_sample"))
        temperature, top_k, top_p = float(opt(temperature, "temperature")), int(opt(top_k, "top_k")), float(opt(top_p, "top_p"))
        if do_sample and temperature <= 0:
            raise ValueError("temperature must be positive when do_sample is true")
        if eos_token_id is _UNSET or eos_token_id is None:
            eos = self.eos_token_ids
        else:
            eos = (eos_token_id,) if isinstance(eos_token_id, int) else tuple(eos_token_id)
        pad = self.pad_token_id if pad_token_id is _UNSET or pad_token_id is None else int(pad_token_id)
        if pad is None:
            pad = eos[0] if eos else 0
        as_tensor = isinstance(input_ids, torch.Tensor)
        prompts = self._prompts_from(input_ids, attention_mask)
        params = [SamplingParams(temperature=temperature if do_sample else 0.0,
                                 top_k=top_k if do_sample else 0,
                                 top_p=top_p if do_sample else 1.0,
                                 seed=None if seed is None else int(seed) * 1000003 + row,   # rows draw from streams of their own
                                 max_new_tokens=max_new_tokens, eos_token_ids=tuple(eos), ignore_eos=ignore_eos)
                  for row in range(len(prompts))]
        outputs = self.generate_requests(prompts, params)
        if not as_tensor:
            return [r.output for r in outputs]
        longest = max((len(r.output) for r in outputs), default=0)
        out = torch.full((len(prompts), input_ids.shape[1] + longest), pad, dtype=torch.int64)
        out[:, :input_ids.shape[1]] = input_ids.to(torch.int64)
        for b, r in enumerate(outputs):
            out[b, input_ids.shape[1]:input_ids.shape[1] + len(r.output)] = torch.tensor(r.output, dtype=torch.int64)
        return out

    def _prompts_from(self, input_ids, attention_mask) -> List[List[int]]:
        if isinstance(input_ids, torch.Tensor):
            if input_ids.device.type != "cpu" or input_ids.dtype not in (torch.int32, torch.int64) or input_ids.ndim != 2:
                raise TypeError("input_ids must be a CPU tensor of int32 or int64 with shape [batch, width]")
            rows = input_ids.tolist()
            if attention_mask is None:
                return rows
            if attention_mask.shape != input_ids.shape:
                raise ValueError("attention_mask must have the shape of input_ids")
            mask = attention_mask.bool().tolist()
            return [[t for t, m in zip(row, mrow) if m] for row, mrow in zip(rows, mask)]
        if attention_mask is not None:
            raise ValueError("attention_mask goes with a tensor of input_ids only")
        return [list(map(int, p)) for p in input_ids]

    # ------------------------------------------------------------------ request-level interface
    def add_request(self, prompt: List[int], params: SamplingParams) -> Request:
        """Queue a prompt. It starts running with the next step() that has room for it."""
        engine = self.engine
        if not prompt:
            raise ValueError("every prompt needs at least one token")
        if min(prompt) < 0 or max(prompt) >= engine.vocab_size:
            raise ValueError(f"input_ids must contain IDs below vocabulary size {engine.vocab_size}")
        self.sampler.validate(params)
        need = -(-min(len(prompt) + params.max_new_tokens, engine.max_seq_len) // engine.cache.page_size)
        if need > engine.cache.num_pages:
            raise ValueError(f"request requires {need} KV pages; the cache has {engine.cache.num_pages}")
        if self._scheduler is None:
            self._scheduler = Scheduler(engine.cache, engine.config.max_step_tokens, engine.config.max_chunk_tokens,
                                        engine.max_seq_len, admission=engine.config.admission)
        self._next_id += 1
        return self._scheduler.add(self._next_id, prompt, params)

    def abort(self, request: Request) -> None:
        """Take a request out: its pages and slot are given back, its finish_reason becomes "aborted". A step
        that was launched ahead with it is taken back first."""
        if self._scheduler is None or request.finished:
            return
        if self._ahead is not None:
            self._take_back(self._ahead)
            self._ahead = None
        self._scheduler.abort(request.request_id)

    def has_unfinished(self) -> bool:
        return self._scheduler is not None and self._scheduler.has_work()

    def step(self) -> List[Request]:
        """One step of the engine over what the scheduler picks: token ids go to the device,
        sampled token ids come back and are appended to their requests. Returns the requests
        that finished with this step.

        While the host waits for a decode step's ids, the next decode step is already running:
        it is launched right behind, with its tokens fed from the sampler's output on the device
        (the reference's traced decode does the same, src/tt_transformers/llm_runtime/decode.py:1137-1140).
        If the next call finds that the scheduler wants exactly that step, its result is simply
        picked up; if not (somebody finished or joined), it is taken back."""
        sched = self._scheduler
        if sched is None or not sched.has_work():
            return []
        plan = sched.schedule()
        ahead, self._ahead = self._ahead, None
        if not plan:
            if ahead is not None:
                self._take_back(ahead)
            if sched.has_work() and not sched.running:
                raise RuntimeError("the scheduler can make no progress: a waiting request fits no page")
            return []
        ids = tuple(e.request.request_id for e in plan)
        all_decode = all(e.sample and e.count == 1 for e in plan)
        if ahead is not None and all_decode and ahead.ids == ids:
            flight = ahead                                   # this very step is running already
        else:
            if ahead is not None:
                self._take_back(ahead)
            flight = self._launch(plan, [StepEntry(e.request.request_id, e.tokens, [e.count - 1] if e.sample else [])
                                         for e in plan], None, 0)
        if self._may_look_ahead(plan):
            entries = [StepEntry(e.request.request_id, [0], [0]) for e in plan]     # ids come from the device
            self._ahead = self._launch(plan, entries, flight.tokens_dev, 1)
        tokens = flight.result()
        self.steps += 1
        done = sched.update(plan, tokens)
        if done and self._ahead is not None:                 # the batch changed: the step ahead is not the next one
            self._take_back(self._ahead)
            self._ahead = None
        return done

    def _launch(self, plan, entries, feedback, ahead_by: int) -> _Flight:
        cache = self.engine.cache
        lengths = {e.request_id: (cache.length(e.request_id) if cache.is_live(e.request_id) else 0) for e in entries}
        graphs = self.engine.graphs
        replays = graphs.replays if graphs is not None else 0
        logits = self.engine.step(entries, token_feedback=feedback)
        wanted = [e.request for e in plan if e.sample]
        if not wanted:
            return _Flight(tuple(e.request_id for e in entries), None, torch.empty(0, dtype=torch.int32), None, lengths)
        if (graphs is not None and graphs.replays > replays and len(wanted) == len(entries)
                and all(r.params.greedy for r in wanted)):
            # A captured step ends with the argmax of its own rows and leaves it where its next replay reads
            # its tokens: an all-greedy batch needs no sampling launch, and the step ahead no token copy.
            source, tokens_dev = graphs.greedy, OWN_ARGMAX
        else:
            source = tokens_dev = self.sampler.sample_device(logits, [r.params for r in wanted], [r.seed for r in wanted],
                                                             [len(r.output) + ahead_by for r in wanted])
        if self.engine.runtime.device.type != "cuda":
            return _Flight(tuple(e.request_id for e in entries), tokens_dev, source.cpu(), None, lengths)
        host = torch.empty(len(wanted), dtype=torch.int32, pin_memory=True)
        self.d2h_bytes += 4 * len(wanted)
        host.copy_(source, non_blocking=True)     # queued before the next replay overwrites the source
        event = torch.cuda.Event()
        event.record()
        return _Flight(tuple(e.request_id for e in entries), tokens_dev, host, event, lengths)

    def _may_look_ahead(self, plan) -> bool:
        """After this step every request of the plan decodes, nobody can join, nobody ends by
        length, and pages are plentiful: the next step is known but for its token ids."""
        engine, sched = self.engine, self._scheduler
        if not (self.look_ahead and engine.can_feed_back()) or sched.waiting:
            return False
        if len(plan) != len(sched.running) or not all(e.sample for e in plan):
            return False
        for e in plan:
            r = e.request
            if len(r.output) + 1 >= r.params.max_new_tokens or r.num_tokens + 2 >= engine.max_seq_len:
                return False
        return engine.cache.free_pages() >= 2 * len(plan)

    def _take_back(self, flight: _Flight) -> None:
        cache = self.engine.cache
        for rid in flight.ids:
            if cache.is_live(rid):
                cache.rollback(rid, flight.lengths_before[rid])

    def generate_requests(self, prompts: List[List[int]], params: List[SamplingParams]) -> List[Request]:
        """Run until every prompt is finished; the requests in input order."""
        if self._busy:
            raise RuntimeError("cannot generate: another operation on this model is active")
        self._busy = True
        try:
            requests = []
            for p, sp in zip(prompts, params):
                if sp.max_new_tokens == 0:
                    requests.append(Request(None, list(p), sp, finish_reason="length"))
                else:
                    requests.append(self.add_request(p, sp))
            first = self.steps
            while self.has_unfinished():
                self.step()
            self.engine.kernels.check_status()
            self.last_stats = {"steps": self.steps - first, "preemptions": self._scheduler.preemptions if self._scheduler else 0}
            return requests
        finally:
            if self._ahead is not None:
                self._take_back(self._ahead)
                self._ahead = None
            if self._scheduler is not None and self._scheduler.has_work():   # a failure must not leave pages taken
                for rid in self.engine.cache.live_requests():
                    self.engine.cache.release(rid)
                self._scheduler = None
            self._busy = False

    def warmup(self, **options) -> int:
        """Capture every decode and prompt step ahead of time (Engine.warmup); call it before serving."""
        if self._scheduler is not None and self._scheduler.has_work():
            raise RuntimeError("warmup() wants an idle model")
        return self.engine.warmup(**options)

    def cleanup(self) -> None:
        """Free the cache and the weights (the reference's cleanup(), hf_generation.py:416-436)."""
        self.engine.close()


def _load_tokenizer(folder: str):
    if not any(os.path.isfile(os.path.join(folder, n)) for n in ("tokenizer.json", "tokenizer.model")):
        return None
    try:
        from transformers import AutoTokenizer
        return AutoTokenizer.from_pretrained(folder, local_files_only=True)
    except Exception:            # a folder without a usable tokenizer still generates from token ids
        return None


def from_pretrained(model: Optional[str] = None, *, hf_model: Optional[str] = None, max_batch_size: int = 32,
                    max_seq_len: int = 4096, n_layers: Optional[int] = None, optimizations: Optional[str] = None,
                    dtype: str = "bfloat16", page_size: int = 16, num_pages: Optional[int] = None,
                    max_step_tokens: int = 2048, max_chunk_tokens: int = 2048, cuda_graph: bool = True,
                    gpu_memory_fraction: Optional[float] = None, graph_batch_sizes=None, admission: str = "eager",
                    device: str = "cuda:0", kernels=None) -> LLM:
    """Load the model folder `model` (config.json + safetensors; the class is chosen by
    config.json) and return an LLM ready to generate. `hf_model` is the reference's name for the same
    argument (there a hub id, here a folder); `optimizations` is its choice of precision recipe
    (src/tt_transformers/models/llama32_1b/hf_generator.py:380-394): "performance" computes in bfloat16,
    "accuracy" in float32, and either overrides `dtype`."""
    if (model is None) == (hf_model is None):
        raise TypeError("give the model folder once: from_pretrained(folder) or from_pretrained(hf_model=folder)")
    model = model if model is not None else hf_model
    if optimizations is not None:
        if optimizations not in ("performance", "accuracy"):
            raise ValueError(f"optimizations must be 'performance' or 'accuracy', got {optimizations!r}")
        dtype = "bfloat16" if optimizations == "performance" else "float32"
    dtype = {"bf16": "bfloat16", "fp32": "float32", torch.bfloat16: "bfloat16", torch.float32: "float32"}.get(dtype, dtype)
    config = EngineConfig(dtype=dtype, page_size=page_size, num_pages=num_pages, max_batch_size=max_batch_size,
                          max_seq_len=max_seq_len, max_step_tokens=max_step_tokens,
                          max_chunk_tokens=max_chunk_tokens, cuda_graph=cuda_graph, device=device,
                          gpu_memory_fraction=gpu_memory_fraction, admission=admission,
                          graph_batch_sizes=tuple(graph_batch_sizes) if graph_batch_sizes else None)
    engine = build_engine(model, config, kernels=kernels, n_layers=n_layers)
    cfg = engine.model_config
    return LLM(engine, eos_token_ids=getattr(cfg, "eos_token_ids", ()), tokenizer=_load_tokenizer(model))
