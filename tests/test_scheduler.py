"""The scheduler's decisions, with the cache manager's bookkeeping but no model (no GPU)."""

import torch

from tt_transformers_b200.cache import CacheManager
from tt_transformers_b200.engine.scheduler import Scheduler
from tt_transformers_b200.parts import PagedKV
from tt_transformers_b200.sampling import SamplingParams


def make(num_pages=16, page_size=4, slots=3, step_tokens=16, chunk=8, max_seq_len=64):
    cache = CacheManager([PagedKV(1, 8)], page_size, num_pages, slots, max_seq_len, torch.device("cpu"),
                         torch.float32, allocate_storage=False)
    return cache, Scheduler(cache, step_tokens, chunk, max_seq_len)


def run_step(cache, sched, token=7):
    """What the engine does around a step, without a model: commit what was planned, sample `token`."""
    plan = sched.schedule()
    for e in plan:
        cache.commit(e.request.request_id, e.start + e.count)
    done = sched.update(plan, [token] * sum(e.sample for e in plan))
    cache.audit()
    return plan, done


def params(n=4, **kw):
    return SamplingParams(max_new_tokens=n, **kw)


def test_prompts_are_cut_under_the_budget_and_decodes_go_first():
    cache, sched = make()
    a = sched.add("a", list(range(20)), params())
    b = sched.add("b", list(range(5)), params())
    plan, _ = run_step(cache, sched)
    assert [(e.request.request_id, e.start, e.count, e.sample) for e in plan] == [("a", 0, 8, False), ("b", 0, 5, True)]
    plan, _ = run_step(cache, sched)
    # a goes on with its prompt (chunk of 8), b decodes one token
    assert [(e.request.request_id, e.start, e.count, e.sample) for e in plan] == [("a", 8, 8, False), ("b", 5, 1, True)]
    plan, _ = run_step(cache, sched)
    assert [(e.request.request_id, e.count, e.sample) for e in plan] == [("a", 4, True), ("b", 1, True)]
    assert a.output == [7] and b.output == [7, 7, 7]
    assert plan[0].tokens == list(range(16, 20))


def test_token_budget_limits_admission():
    cache, sched = make(step_tokens=10, chunk=8)
    for name in "abc":
        sched.add(name, list(range(8)), params())
    plan, _ = run_step(cache, sched)
    assert [(e.request.request_id, e.count) for e in plan] == [("a", 8), ("b", 2)]
    plan, _ = run_step(cache, sched)
    assert [(e.request.request_id, e.count) for e in plan] == [("a", 1), ("b", 6), ("c", 3)]


def test_slots_limit_admission_and_finishing_frees_them():
    cache, sched = make(slots=2)
    for name in "abc":
        sched.add(name, [1, 2, 3], params(n=2))
    plan, _ = run_step(cache, sched)
    assert [e.request.request_id for e in plan] == ["a", "b"]
    plan, done = run_step(cache, sched)
    assert [r.request_id for r in done] == ["a", "b"] and all(r.finish_reason == "length" for r in done)
    plan, _ = run_step(cache, sched)
    assert [e.request.request_id for e in plan] == ["c"]
    assert cache.free_slots == 1


def test_eos_stops_unless_ignored():
    cache, sched = make()
    a = sched.add("a", [1, 2], params(n=10, eos_token_ids=(7,)))
    b = sched.add("b", [1, 2], params(n=3, eos_token_ids=(7,), ignore_eos=True))
    run_step(cache, sched)
    assert a.finish_reason == "stop" and a.output == [7] and not b.finished
    while sched.has_work():
        run_step(cache, sched)
    assert b.finish_reason == "length" and len(b.output) == 3
    assert cache.free_pages() == 16 and cache.free_slots == 3


def test_when_pages_run_out_the_last_admitted_gives_way_and_is_computed_again():
    cache, sched = make(num_pages=6, page_size=4, step_tokens=64, chunk=64)
    a = sched.add("a", list(range(10)), params(n=12))      # 3 pages now, 6 at the end
    b = sched.add("b", list(range(9)), params(n=12))       # 3 pages now
    run_step(cache, sched)
    assert cache.free_pages() == 0
    steps = 0
    while not b.preemptions:
        plan, _ = run_step(cache, sched)
        steps += 1
        assert steps < 10
    # b gave way: its pages are back, it waits at the head of the line with what it produced
    assert sched.waiting[0] is b and b.num_computed == 0 and not cache.is_live("b")
    produced = len(b.output)
    assert produced >= 1 and sched.preemptions == 1
    while sched.has_work():
        plan, _ = run_step(cache, sched)
        for e in plan:
            if e.request is b and e.start == 0:
                assert e.tokens[:9] == list(range(9)) and len(e.tokens) <= 9 + produced + 12
    assert a.finish_reason == "length" and b.finish_reason == "length"
    assert len(a.output) == 12 and len(b.output) == 12
    assert cache.free_pages() == 6


def test_a_lone_request_that_cannot_fit_is_finished_alone():
    cache, sched = make(num_pages=2, page_size=4, step_tokens=64, chunk=64)
    a = sched.add("a", list(range(6)), params(n=20))
    b = sched.add("b", [1, 2], params(n=1))
    while not a.finished:
        run_step(cache, sched)
    assert a.finish_reason == "out_of_pages" and len(a.output) == 3      # 6 + 2 fit the two pages, the 9th does not
    while sched.has_work():
        run_step(cache, sched)
    assert b.finish_reason == "length" and cache.free_pages() == 2


def test_context_limit_and_abort():
    cache, sched = make(max_seq_len=8, num_pages=4)
    a = sched.add("a", [1, 2, 3, 4, 5], params(n=100))
    b = sched.add("b", [1], params(n=100))
    run_step(cache, sched)
    sched.abort("b")
    assert b.finish_reason == "aborted" and not cache.is_live("b")
    while sched.has_work():
        run_step(cache, sched)
    assert a.finish_reason == "length" and len(a.all_tokens) == 8
    c = sched.add("c", [1], params())
    sched.abort("c")
    assert c.finish_reason == "aborted" and not sched.has_work()


def test_seeds_follow_arrival_unless_given():
    cache, sched = make()
    a = sched.add("a", [1], params())
    b = sched.add("b", [1], params())
    c = sched.add("c", [1], params(seed=5))
    assert a.seed != b.seed and c.seed == 5


def test_conservative_admission_reserves_everything_up_front_and_never_gives_way():
    """The reference's generate() reserves prompt + max_new_tokens pages before any work
    (src/tt_transformers/models/hf_generation.py:337-343): with admission='conservative' a request starts only
    when all that fits, holds it until it ends, and so never gives way or runs out of pages."""
    cache = CacheManager([PagedKV(1, 8)], 4, 10, 3, 64, torch.device("cpu"), torch.float32, allocate_storage=False)
    sched = Scheduler(cache, 16, 8, 64, admission="conservative")
    a = sched.add("a", list(range(10)), params(n=10))       # 20 tokens: 5 pages
    b = sched.add("b", list(range(6)), params(n=10))        # 16 tokens: 4 pages
    c = sched.add("c", list(range(3)), params(n=6))         # 9 tokens: 3 pages; only one page is left beside a and b
    plan, _ = run_step(cache, sched)
    assert [(e.request.request_id, e.count) for e in plan] == [("a", 8), ("b", 6)]
    assert cache.free_pages() == 1 and [r.request_id for r in sched.waiting] == ["c"]
    steps = 0
    while sched.has_work():
        plan, _ = run_step(cache, sched)
        steps += 1
        if cache.is_live("a"):
            assert cache.free_pages() <= 1 or not cache.is_live("b")     # what is held stays held
        assert steps < 60
    assert sched.preemptions == 0
    assert [r.finish_reason for r in (a, b, c)] == ["length"] * 3 and len(c.output) == 6
    assert cache.free_pages() == 10
    # the same load admitted eagerly starts all three at once
    cache2, eager = make(num_pages=10, slots=3)
    for r in (a, b, c):
        eager.add(r.request_id, r.prompt, r.params)
    plan, _ = run_step(cache2, eager)
    assert [e.request.request_id for e in plan] == ["a", "b", "c"]


def test_held_pages_survive_a_step_taken_back():
    cache = CacheManager([PagedKV(1, 8)], 4, 10, 2, 64, torch.device("cpu"), torch.float32, allocate_storage=False)
    cache.admit("a")
    cache.reserve("a", 17, hold=True)
    assert cache.free_pages() == 5
    cache.commit("a", 6)
    cache.reserve("a", 7)
    cache.commit("a", 7)
    cache.rollback("a", 6)                      # gives back what lies beyond 6 tokens, but not what is held
    assert cache.free_pages() == 5 and cache.room("a") == 5 * 4 + 20 - 6
    cache.audit()
    cache.release("a")
    assert cache.free_pages() == 10
