"""The cache manager and the page pool: nothing is lost, held twice or freed twice (no GPU)."""

import random

import pytest
import torch

from tt_transformers_b200.cache import CacheManager, OutOfPages, OutOfSlots, PagePool
from tt_transformers_b200.cache.pages import PagePoolError
from tt_transformers_b200.parts import PagedKV, SlotState


def manager(requests, page_size=4, num_pages=10, max_slots=3, max_seq_len=64, storage=False):
    return CacheManager(requests, page_size, num_pages, max_slots, max_seq_len, torch.device("cpu"), torch.float32,
                        allocate_storage=storage)


def test_pool_hands_out_each_page_once_and_reuses_freed_pages_lowest_first():
    pool = PagePool(5)
    a = pool.allocate(3)
    assert a == [1, 2, 3] and pool.free_count == 2
    assert pool.allocate(3) is None and pool.free_count == 2         # nothing taken
    pool.free([2])
    assert pool.allocate(1) == [2]
    pool.free([3, 1])
    assert pool.allocate(2) == [1, 3] and pool.free_count == 2
    pool.free([3])
    with pytest.raises(PagePoolError):
        pool.free([4])                                               # never handed out
    pool.free([1])
    with pytest.raises(PagePoolError):
        pool.free([1])                                               # freed twice
    with pytest.raises(PagePoolError):
        pool.free([0])                                               # the scratch page is nobody's


def test_groups_by_need_and_units_by_entry():
    full, win = PagedKV(2, 16), PagedKV(2, 16, window=8)
    m = manager([full, win, full, None, 0, SlotState((3,))], storage=True)
    assert len(m.groups) == 3
    assert m.groups[0].storage["keys"].shape == (2, 11, 2, 4, 16)     # two units, pages 0..10
    assert sorted(m.groups[0].storage) == ["keys", "values"]
    assert m.groups[1].storage["values"].shape == (1, 11, 2, 4, 16)
    assert m.groups[2].storage["state"].shape == (1, 4, 3)            # three slots and the row nobody owns
    assert m._unit_of_entry[4] == m._unit_of_entry[0] and 3 not in m._unit_of_entry
    with pytest.raises(ValueError):
        manager([None, 0])


def test_reserve_commit_release():
    m = manager([PagedKV(1, 8)])
    m.admit("a")
    m.reserve("a", 9)                     # 3 pages of 4
    assert m.free_pages() == 7 and list(m.table_rows(0, [m.slot("a")])[0, :4]) == [1, 2, 3, 0]
    m.commit("a", 9)
    m.reserve("a", 12)                    # still 3 pages
    assert m.free_pages() == 7
    m.reserve("a", 13)
    assert m.free_pages() == 6
    m.trim("a")                           # the step did not run: back to what is held
    assert m.free_pages() == 7 and m.room("a") == 7 * 4 + 3
    m.audit()
    m.release("a")
    assert m.free_pages() == 10 and m.free_slots == 3
    m.audit()


def test_out_of_pages_takes_nothing_and_out_of_slots():
    m = manager([PagedKV(1, 8), PagedKV(1, 8, window=4)], num_pages=3)
    m.admit("a")
    m.reserve("a", 8)
    with pytest.raises(OutOfPages) as e:
        m.reserve("a", 17)
    assert e.value.request_id == "a"
    assert m.free_pages(0) == 1 and m.free_pages(1) == 1
    m.audit()
    m.admit("b"), m.admit("c")
    with pytest.raises(OutOfSlots):
        m.admit("d")
    with pytest.raises(ValueError):
        m.admit("a")
    with pytest.raises(ValueError):
        m.reserve("b", 65)                # beyond max_seq_len


def test_a_window_gives_pages_back_as_it_moves():
    m = manager([PagedKV(1, 8), PagedKV(1, 8, window=6)], num_pages=12)
    m.admit("a")
    length = 0
    for n in (5, 3, 1, 1, 7, 1, 1, 1):
        m.reserve("a", length + n)
        length += n
        m.commit("a", length)
        m.audit()
        # the windowed group holds only pages that positions >= length - 6 + 1 touch, and what one
        # token taken back (a step that ran ahead) would touch again
        first_needed = max(0, length - m.ROLLBACK_SLACK - 6 + 1) // 4
        row = m.table_rows(1, [m.slot("a")])[0]
        assert all(p == 0 for p in row[:first_needed]) and all(p != 0 for p in row[first_needed:-(-length // 4)])
        assert m.groups[1].pool.held_count == -(-length // 4) - first_needed
        assert m.groups[0].pool.held_count == -(-length // 4)
    m.release("a")
    assert m.free_pages(0) == 12 and m.free_pages(1) == 12


@pytest.mark.parametrize("seed", range(8))
def test_random_orders_of_requests(seed):
    rng = random.Random(seed)
    m = manager([PagedKV(2, 8), PagedKV(2, 8, window=rng.choice([3, 9, 20])), SlotState((2,))],
                page_size=rng.choice([1, 4, 8]), num_pages=rng.choice([6, 12, 30]), max_slots=4, max_seq_len=80)
    lengths, next_id = {}, 0
    for _ in range(400):
        action = rng.random()
        if action < 0.25 and m.free_slots:
            m.admit(next_id)
            lengths[next_id] = 0
            next_id += 1
        elif action < 0.8 and lengths:
            rid = rng.choice(list(lengths))
            n = rng.choice([1, 1, 1, 2, 5, 11])
            if lengths[rid] + n > 80:
                continue
            try:
                m.reserve(rid, lengths[rid] + n)
            except OutOfPages:
                m.audit()
                if rng.random() < 0.5:
                    m.trim(rid)
                continue
            if rng.random() < 0.1:
                m.trim(rid)                       # a reserved step that never ran
            else:
                lengths[rid] += n
                m.commit(rid, lengths[rid])
        elif lengths:
            rid = rng.choice(list(lengths))
            m.release(rid)
            del lengths[rid]
        m.audit()
        for rid, n in lengths.items():
            assert m.length(rid) == n
    for rid in list(lengths):
        m.release(rid)
    m.audit()
    assert all(g.pool.free_count == m.num_pages for g in m.groups if g.pool is not None)
    assert m.free_slots == 4


def test_slot_state_is_zeroed_at_admission():
    m = manager([SlotState((2, 2))], storage=True)
    slot = m.admit("a")
    m.groups[0].storage["state"][0, slot] += 5
    m.release("a")
    assert m.admit("b") == slot and float(m.groups[0].storage["state"][0, slot].abs().sum()) == 0


def test_a_request_kind_of_the_callers_own_describes_its_storage():
    """The manager asks the request what to store and how to show it: one tensor per token here, in a dtype of
    its own, beside keys and values and a per-request state."""
    from dataclasses import dataclass

    from tt_transformers_b200.parts import CacheRequest

    @dataclass(frozen=True)
    class Latent(CacheRequest):
        width: int
        paged = True

        def storage(self, page_size):
            return {"latent": ((page_size, self.width), torch.float64)}

        def view(self, tensors, *, block_table, page_size, **_):
            return ("latent view", tensors["latent"], block_table, page_size)

    m = manager([Latent(5), PagedKV(1, 8), Latent(5), SlotState((2,), dtype=torch.int32)], storage=True)
    assert [type(g.request).__name__ for g in m.groups] == ["Latent", "PagedKV", "SlotState"]
    assert m.groups[0].storage["latent"].shape == (2, 11, 4, 5) and m.groups[0].storage["latent"].dtype == torch.float64
    assert m.groups[2].storage["state"].dtype == torch.int32
    m.admit("a")
    m.reserve("a", 9)
    m.commit("a", 9)
    m.audit()

    class Batch:
        block_tables = {0: "table 0", 1: "table 1"}
        seg_slot, seg_slot_list = "slots", [0]

    kind, tensor, table, page = m.view(2, Batch)
    assert kind == "latent view" and tensor.shape == (11, 4, 5) and table == "table 0" and page == 4
    assert tensor.data_ptr() == m.groups[0].storage["latent"][1].data_ptr()
    m.release("a")
    assert m.free_pages() == 10


def test_one_token_can_be_taken_back_behind_a_window():
    m = manager([PagedKV(1, 8, window=4)], num_pages=6)
    m.admit("a")
    length = 0
    for n in (7, 1, 1, 1, 1, 1):
        m.reserve("a", length + n)
        length += n
        m.commit("a", length)
    held = m.groups[0].pool.held_count
    m.rollback("a", length - 1)                 # the step that ran ahead is not wanted after all
    m.audit()
    # every page that a query at position length - 1 reads (keys > length - 1 - 4) is still there
    row = m.table_rows(0, [m.slot("a")])[0]
    assert all(row[p // 4] != 0 for p in range(length - 1 - 4 + 1, length - 1))
    assert m.groups[0].pool.held_count <= held
    with pytest.raises(RuntimeError):
        m.rollback("a", length - 3)
