"""The library's request scheduler (nexus_scheduler_*) against the reference's
own scheduler tests (src/scheduler.rs:388-526), run on the CPU through the C
ABI, plus the cases the serving loop relies on: page reuse after release,
cancellation of pending and running requests, FIFO admission under a page
budget, empty requests refused and buffers that are too small."""
import ctypes as C

import pytest

from nexus_b200 import NexusError
from nexus_b200 import _lib as L
from nexus_b200.scheduler import ScheduledDecode, Scheduler


def test_scheduler_add_and_batch():
    # src/scheduler.rs:405-418
    s = Scheduler(4)
    s.add_request("r1", [1, 2], 3)
    s.add_request("r2", [3, 4], 3)
    batch = s.get_next_batch()
    assert batch == ["r1", "r2"]
    assert s.stats() == (0, 2, 0)


def test_scheduler_step():
    # src/scheduler.rs:420-428
    s = Scheduler(4)
    s.add_request("r1", [1, 2], 2)
    s.get_next_batch()
    assert len(s.step()) == 1


def test_scheduler_max_batch():
    # src/scheduler.rs:430-438
    s = Scheduler(2)
    for i in range(5):
        s.add_request(f"r{i}", [1], 1)
    assert len(s.get_next_batch()) <= 2


def test_scheduler_honors_request_max_tokens():
    # src/scheduler.rs:440-451
    s = Scheduler(4)
    s.add_request("r1", [1, 2], 1)
    s.get_next_batch()
    assert s.step() == ["r1"]
    assert s.stats() == (0, 0, 1)


def test_scheduler_respects_running_capacity():
    # src/scheduler.rs:453-467
    s = Scheduler(2)
    for i in range(3):
        s.add_request(f"r{i + 1}", [1], 4)
    assert len(s.get_next_batch()) == 2
    assert s.get_next_batch() == []
    assert s.stats() == (1, 2, 0)


def test_scheduler_complete_request():
    # src/scheduler.rs:469-477
    s = Scheduler(4)
    s.add_request("r1", [1], 4)
    s.get_next_batch()
    assert s.complete_request("r1")
    assert s.stats() == (0, 0, 1)


def test_decode_batch_and_append_generated():
    # src/scheduler.rs:479-506
    s = Scheduler(2)
    s.add_request("r1", [10, 11], 2)
    assert s.decode_batch() == [ScheduledDecode("r1", 11, 2, 0, 2, [0])]
    assert s.append_generated("r1", 12)
    b = s.decode_batch()
    assert (b[0].token, b[0].position, b[0].generated) == (12, 3, 1)
    assert s.append_generated("r1", 13)
    assert s.stats() == (0, 0, 1)
    assert s.tokens("r1") == [10, 11, 12, 13]


def test_scheduler_kv_page_capacity_and_release():
    # src/scheduler.rs:508-525
    s = Scheduler.with_kv_pages(4, 4, 2)
    s.add_request("r1", [1, 2, 3, 4], 4)
    s.add_request("r2", [5, 6, 7, 8], 4)
    assert len(s.get_next_batch()) == 1
    alloc = s.kv_allocation("r1")
    assert alloc.page_ids == [0, 1]
    assert alloc.capacity_tokens == 8 and alloc.page_size_tokens == 4
    assert s.kv_page_stats() == (2, 2)
    assert s.get_next_batch() == []
    assert s.complete_request("r1")
    assert s.kv_page_stats() == (0, 2)
    third = s.get_next_batch()
    assert third == ["r2"]
    # released ids are reused (they name device pool pages), smallest first
    assert s.kv_allocation("r2").page_ids == [0, 1]


def test_page_ids_stay_below_the_budget_under_churn():
    s = Scheduler.with_kv_pages(3, 16, 7)
    lens = [(5, 20), (30, 3), (1, 1), (16, 16), (40, 8), (2, 2), (17, 0)]
    for i, (p, m) in enumerate(lens):
        s.add_request(f"q{i}", list(range(p)), m)
    seen_done = set()
    for _ in range(200):
        items = s.decode_batch()
        if not items and s.stats()[0] == 0:
            break
        used = set()
        for it in items:
            assert len(it.kv_pages) == max(1, -(-(it.prompt_len + lens[int(it.id[1:])][1]) // 16))
            assert all(0 <= p < 7 for p in it.kv_pages)
            assert not used.intersection(it.kv_pages)
            used.update(it.kv_pages)
        assert s.kv_page_stats()[0] == len(used) <= 7
        for it in items:
            s.append_generated(it.id, 1000 + it.position)
        seen_done.update(s.get_completed())
    assert seen_done == {f"q{i}" for i in range(len(lens))}
    assert s.stats() == (0, 0, 0)


def test_fifo_admission_waits_for_pages():
    s = Scheduler.with_kv_pages(4, 16, 3)
    s.add_request("big", list(range(40)), 8)     # 3 pages
    s.add_request("small", [1], 1)               # 1 page: must wait behind "big"
    assert s.get_next_batch() == ["big"]
    assert s.get_next_batch() == []
    assert s.complete_request("big")
    assert s.get_next_batch() == ["small"]


def test_cancel_pending_and_unknown():
    s = Scheduler(1)
    s.add_request("a", [1], 3)
    s.add_request("b", [2], 3)
    s.get_next_batch()
    assert s.complete_request("b")          # pending
    assert not s.complete_request("zzz")
    assert not s.append_generated("b", 5)   # no longer running
    assert s.stats() == (0, 1, 1)


def test_refusals():
    s = Scheduler(2)
    with pytest.raises(NexusError, match="at least one token"):
        s.add_request("e", [], 3)            # never gives a decode item
    s.add_request("x", [1], 1)
    with pytest.raises(NexusError, match="already in use"):
        s.add_request("x", [2], 1)           # id in use
    lib = L.load()
    n = C.c_size_t()
    s.add_request("y", [2], 1)
    rc = lib.nexus_scheduler_decode_batch(s.handle, None, 1, C.byref(n))
    assert rc != 0 and n.value == 2         # too small: nothing admitted
    assert b"too small" in lib.nexus_scheduler_last_error()
    assert s.stats() == (2, 0, 0)


def test_max_tokens_zero_finishes_on_first_append():
    s = Scheduler(2)
    s.add_request("z", [7, 8], 0)
    items = s.decode_batch()
    assert items[0].token == 8
    assert s.append_generated("z", 9)       # advance() refuses: no token appended
    assert s.stats() == (0, 0, 1)
    assert s.tokens("z") == [7, 8]
