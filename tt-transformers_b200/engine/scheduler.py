"""The scheduler: which requests run in the next step, and with how many tokens.

Every step first gives each running request its next tokens (one decoded token, or the
next portion of its prompt), in the order of admission, then admits waiting requests
while a slot, pages and token budget remain. Portions may be cut anywhere; a step holds
at most `max_step_tokens` tokens and a portion at most `max_chunk_tokens`.

When pages run out: the request that was admitted last gives way. Its pages and slot are
given back, and it returns to the head of the waiting line with everything it has
produced so far as its new prompt, to be computed again later (its random stream goes on
where it was, as draws depend on the token index only). A request that runs alone and
still cannot get a page is finished with reason "out_of_pages"; no other request is
affected.

With admission "conservative" a request is admitted only when pages for its whole prompt and
all the tokens it may produce are free, and takes them all at once, as the reference's
generate() does: such a request never gives way and never runs out of pages; fewer requests
run side by side.

The reference has no scheduler of its own: generate() runs a static batch and reserves
prompt + max_new_tokens pages up front, failing before any work if they do not suffice
(src/tt_transformers/models/hf_generation.py:337-348); serving leaves scheduling to the
server in front (docs/vllm-decode.md:1-44).
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field
from typing import Deque, List, Optional

from ..cache import CacheManager, OutOfPages
from ..sampling.params import SamplingParams


@dataclass
class Request:
    request_id: object
    prompt: List[int]
    params: SamplingParams
    arrival: int = 0
    output: List[int] = field(default_factory=list)
    num_computed: int = 0                 # tokens whose keys are in the cache
    finish_reason: Optional[str] = None   # "stop" (eos), "length", "out_of_pages", "aborted"
    preemptions: int = 0

    @property
    def all_tokens(self) -> List[int]:
        return self.prompt + self.output

    @property
    def num_tokens(self) -> int:
        return len(self.prompt) + len(self.output)

    def tokens_between(self, start: int, stop: int) -> List[int]:
        """Tokens start .. stop-1 of prompt + output, without building the whole list."""
        n = len(self.prompt)
        if start >= n:
            return self.output[start - n:stop - n]
        if stop <= n:
            return self.prompt[start:stop]
        return self.prompt[start:] + self.output[:stop - n]

    @property
    def seed(self) -> int:
        return self.params.seed if self.params.seed is not None else 0x5EED + 7919 * self.arrival

    @property
    def finished(self) -> bool:
        return self.finish_reason is not None


@dataclass
class PlannedEntry:
    request: Request
    start: int            # first token (index into request.all_tokens) that this step computes
    count: int
    sample: bool          # the portion reaches the request's last token: its logits are wanted

    @property
    def tokens(self) -> List[int]:
        return self.request.tokens_between(self.start, self.start + self.count)


class Scheduler:
    def __init__(self, cache: CacheManager, max_step_tokens: int, max_chunk_tokens: int, max_seq_len: int,
                 admission: str = "eager"):
        if admission not in ("eager", "conservative"):
            raise ValueError(f"admission must be 'eager' or 'conservative', got {admission!r}")
        self.cache, self.admission = cache, admission
        self.max_step_tokens, self.max_chunk_tokens, self.max_seq_len = max_step_tokens, max_chunk_tokens, max_seq_len
        self.waiting: Deque[Request] = deque()
        self.running: List[Request] = []          # in order of admission
        self.finished: List[Request] = []
        self._arrivals = 0
        self.preemptions = 0

    # ------------------------------------------------------------------ requests in and out
    def add(self, request_id, prompt: List[int], params: SamplingParams) -> Request:
        if not prompt:
            raise ValueError("a request needs at least one prompt token")
        if len(prompt) >= self.max_seq_len:
            raise ValueError(f"the prompt of {len(prompt)} tokens leaves no room within max_seq_len {self.max_seq_len}")
        req = Request(request_id, list(prompt), params, arrival=self._arrivals)
        self._arrivals += 1
        self.waiting.append(req)
        return req

    def abort(self, request_id) -> None:
        for req in list(self.running):
            if req.request_id == request_id:
                self._finish(req, "aborted")
                return
        for req in list(self.waiting):
            if req.request_id == request_id:
                self.waiting.remove(req)
                req.finish_reason = "aborted"
                self.finished.append(req)
                return

    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    def _finish(self, req: Request, reason: str) -> None:
        req.finish_reason = reason
        if req in self.running:
            self.running.remove(req)
        if self.cache.is_live(req.request_id):
            self.cache.release(req.request_id)
        self.finished.append(req)

    def _preempt(self, req: Request) -> None:
        self.running.remove(req)
        self.cache.release(req.request_id)
        req.num_computed = 0
        req.preemptions += 1
        self.preemptions += 1
        self.waiting.appendleft(req)

    # ------------------------------------------------------------------ one step's plan
    def _fit(self, req: Request, count: int) -> int:
        """How many of the next `count` tokens of a running request the free pages allow."""
        return max(0, min(count, self.cache.room(req.request_id)))

    def schedule(self) -> List[PlannedEntry]:
        plan: List[PlannedEntry] = []
        budget = self.max_step_tokens
        preempted_before = self.preemptions
        for req in list(self.running):
            if req not in self.running or budget == 0:
                continue
            pending = req.num_tokens - req.num_computed
            count = min(pending, self.max_chunk_tokens, budget)
            while True:
                fit = self._fit(req, count)
                if fit >= 1:
                    count = fit
                    break
                victim = self.running[-1]
                if victim is req:
                    if len(self.running) == 1:
                        self._finish(req, "out_of_pages")     # alone and still no page: this request only
                    else:
                        self._preempt(req)
                    count = 0
                    break
                self._preempt(victim)
            if count == 0:
                continue
            self.cache.reserve(req.request_id, req.num_computed + count)
            plan.append(PlannedEntry(req, req.num_computed, count, sample=req.num_computed + count == req.num_tokens))
            budget -= count
        # nobody is admitted in a step in which somebody had to give way
        while (self.waiting and budget > 0 and self.cache.free_slots > 0
               and self.preemptions == preempted_before):
            req = self.waiting[0]
            pending = req.num_tokens
            count = min(pending, self.max_chunk_tokens, budget)
            fit = min(count, self.cache.room())
            if fit < 1:
                break
            if req.preemptions and self.running and self.cache.room() < pending + 1:
                break      # one that gave way comes back when all it has fits beside the others, not to give way again
            if self.admission == "conservative":
                whole = min(len(req.prompt) + req.params.max_new_tokens, self.max_seq_len)
                if self.cache.room() < whole:
                    break  # it waits until everything it may ever hold fits
                self.waiting.popleft()
                self.cache.admit(req.request_id)
                self.cache.reserve(req.request_id, whole, hold=True)
                self.running.append(req)
                plan.append(PlannedEntry(req, 0, count, sample=count == pending))
                budget -= count
                continue
            self.waiting.popleft()
            self.cache.admit(req.request_id)
            self.cache.reserve(req.request_id, fit)
            self.running.append(req)
            plan.append(PlannedEntry(req, 0, fit, sample=fit == pending))
            budget -= fit
        return plan

    # ------------------------------------------------------------------ after the step
    def update(self, plan: List[PlannedEntry], sampled: List[int]) -> List[Request]:
        """`sampled`: one token per planned entry with sample=True, in plan order. Returns
        the requests that finished with this step."""
        done, it = [], iter(sampled)
        for entry in plan:
            req = entry.request
            req.num_computed = entry.start + entry.count
            if not entry.sample:
                continue
            token = int(next(it))
            req.output.append(token)
            p = req.params
            if not p.ignore_eos and token in p.eos_token_ids:
                self._finish(req, "stop")
            elif len(req.output) >= p.max_new_tokens or req.num_tokens >= self.max_seq_len:
                self._finish(req, "length")
            if req.finished:
                done.append(req)
        return done
