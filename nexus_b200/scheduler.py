"""Request scheduler and continuous batching over the C ABI.

``Scheduler`` mirrors the reference's ``Scheduler`` (src/scheduler.rs:126-365)
method for method -- ``add_request``, ``get_next_batch``, ``decode_batch``,
``append_generated``, ``step``, ``get_completed``, ``complete_request``,
``stats``, ``kv_page_stats``, ``kv_allocation`` -- on the library's C++
scheduler (nexus_scheduler_*).  Request ids are strings as in the reference;
they are numbered for the C ABI here.

``ContinuousBatcher`` drives a loaded model with it: every ``tick`` admits
pending requests (their KV pages become the device page tables of free
sequences, their prompts are prefilled) and runs one batched decode step over
every running request (nexus_cuda_serve_step).  The reference's server never
does this: it serializes requests behind the engine mutex and runs one
``generate_with_config`` each (src/server/mod.rs:407,416).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import _lib as L


@dataclass
class ScheduledDecode:
    """``ScheduledDecode`` (src/scheduler.rs:106-115)."""
    id: str
    token: int
    position: int
    generated: int
    prompt_len: int
    kv_pages: list


@dataclass
class KvPageAllocation:
    """``KvPageAllocation`` (src/scheduler.rs:117-124)."""
    request_id: str
    page_ids: list
    page_size_tokens: int
    capacity_tokens: int


@dataclass
class ServeEvent:
    request_id: str
    token: int
    index: int
    done: bool
    status: int


class Scheduler:
    """``Scheduler::new(max_batch_size)`` / ``Scheduler::with_kv_pages``.
    max_kv_pages None = no limit, as in ``Scheduler::new``."""

    def __init__(self, max_batch_size: int = 8, page_size_tokens: int = 16, max_kv_pages: Optional[int] = None):
        self._lib = L.load()
        h = C.c_void_p()
        L.check_scheduler(self._lib.nexus_scheduler_create(max_batch_size, page_size_tokens, max_kv_pages or 0, C.byref(h)))
        self.handle = h
        self.max_batch_size = max_batch_size
        self.page_size_tokens = max(1, page_size_tokens)
        self._num: dict[str, int] = {}
        self._name: dict[int, str] = {}

    @classmethod
    def with_kv_pages(cls, max_batch_size: int, page_size_tokens: int, max_kv_pages: int) -> "Scheduler":
        return cls(max_batch_size, page_size_tokens, max_kv_pages)

    def _id(self, name: str) -> int:
        if name not in self._num:
            n = len(self._num) + 1
            self._num[name] = n
            self._name[n] = name
        return self._num[name]

    def _ids(self, fn, cap: int) -> list[str]:
        buf = (C.c_uint64 * max(1, cap))()
        n = C.c_size_t()
        L.check_scheduler(fn(self.handle, buf, cap, C.byref(n)))
        return [self._name[buf[i]] for i in range(n.value)]

    def _room(self) -> int:
        p, r, c = self.stats()
        return p + r + c + 1

    def add_request(self, id: str, tokens: Sequence[int], max_tokens: int) -> None:
        toks = np.ascontiguousarray(np.asarray(tokens, np.uint32))
        L.check_scheduler(self._lib.nexus_scheduler_add_request(self.handle, self._id(id), toks.ctypes.data, toks.size,
                                                      max_tokens))

    def get_next_batch(self) -> list[str]:
        return self._ids(self._lib.nexus_scheduler_get_next_batch, self._room())

    def decode_batch(self) -> list[ScheduledDecode]:
        cap = self._room()
        items = (L.ScheduledDecode * cap)()
        n = C.c_size_t()
        L.check_scheduler(self._lib.nexus_scheduler_decode_batch(self.handle, items, cap, C.byref(n)))
        return [ScheduledDecode(self._name[d.id], d.token, d.position, d.generated, d.prompt_len,
                                [d.kv_pages[j] for j in range(d.n_pages)]) for d in items[:n.value]]

    def append_generated(self, id: str, token: int) -> bool:
        if id not in self._num:
            return False
        found = C.c_int()
        L.check_scheduler(self._lib.nexus_scheduler_append_generated(self.handle, self._num[id], token, C.byref(found)))
        return bool(found.value)

    def step(self) -> list[str]:
        return self._ids(self._lib.nexus_scheduler_step, self._room())

    def get_completed(self) -> list[str]:
        return self._ids(self._lib.nexus_scheduler_get_completed, self._room())

    def complete_request(self, id: str) -> bool:
        if id not in self._num:
            return False
        found = C.c_int()
        L.check_scheduler(self._lib.nexus_scheduler_complete_request(self.handle, self._num[id], C.byref(found)))
        return bool(found.value)

    def stats(self) -> tuple[int, int, int]:
        p, r, c = C.c_size_t(), C.c_size_t(), C.c_size_t()
        L.check_scheduler(self._lib.nexus_scheduler_stats(self.handle, C.byref(p), C.byref(r), C.byref(c)))
        return p.value, r.value, c.value

    def kv_page_stats(self) -> tuple[int, int]:
        used, mx = C.c_size_t(), C.c_size_t()
        L.check_scheduler(self._lib.nexus_scheduler_kv_page_stats(self.handle, C.byref(used), C.byref(mx)))
        return used.value, mx.value

    def kv_allocation(self, id: str) -> Optional[KvPageAllocation]:
        if id not in self._num:
            return None
        n, cap = C.c_size_t(), C.c_size_t()
        rc = self._lib.nexus_scheduler_kv_allocation(self.handle, self._num[id], None, 0, C.byref(n), C.byref(cap))
        if rc != 0 and n.value == 0:
            return None
        buf = (C.c_uint32 * max(1, n.value))()
        L.check_scheduler(self._lib.nexus_scheduler_kv_allocation(self.handle, self._num[id], buf, n.value, C.byref(n),
                                                        C.byref(cap)))
        return KvPageAllocation(id, list(buf[:n.value]), self.page_size_tokens, cap.value)

    def tokens(self, id: str) -> list[int]:
        """The request's tokens: its prompt, then what it generated."""
        n = C.c_size_t()
        self._lib.nexus_scheduler_tokens(self.handle, self._num[id], None, 0, C.byref(n))
        buf = (C.c_uint32 * max(1, n.value))()
        L.check_scheduler(self._lib.nexus_scheduler_tokens(self.handle, self._num[id], buf, n.value, C.byref(n)))
        return list(buf[:n.value])

    def close(self) -> None:
        if self.handle:
            self._lib.nexus_scheduler_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ContinuousBatcher:
    """Continuous batching of a loaded model (``InferenceEngine``) with a
    ``Scheduler`` whose page size is the model's and whose page budget fits its
    KV pool (by default: all of the pool, and the model's max_batch)."""

    def __init__(self, engine, max_batch_size: Optional[int] = None, max_kv_pages: Optional[int] = None):
        info = engine.info
        self.engine = engine
        self.scheduler = Scheduler(max_batch_size or info.max_batch, info.page_tokens,
                                   max_kv_pages or info.max_pages)
        self._cap = self.scheduler.max_batch_size

    def add_request(self, id: str, tokens: Sequence[int], max_tokens: int) -> None:
        self.scheduler.add_request(id, tokens, max_tokens)

    def tick(self) -> list[ServeEvent]:
        ev = (L.ServeEvent * self._cap)()
        n = C.c_size_t()
        rc = self.engine._lib.nexus_cuda_serve_step(self.engine.model, self.scheduler.handle, ev, self._cap,
                                                    C.byref(n))
        if rc != L.NEXUS_OK and rc == L.NEXUS_E_INVALID and L.load().nexus_scheduler_last_error():
            L.check_scheduler(rc)
        L.check(rc, self.engine.backend.handle)
        name = self.scheduler._name
        return [ServeEvent(name[e.request_id], e.token, e.index, bool(e.done), e.status) for e in ev[:n.value]]

    def run(self) -> dict[str, list[int]]:
        """Ticks until nothing is pending or running; returns every finished
        request's tokens (prompt + generated)."""
        out: dict[str, list[int]] = {}
        while True:
            p, r, _ = self.scheduler.stats()
            if p == 0 and r == 0:
                break
            for e in self.tick():
                if e.done:
                    out[e.request_id] = self.scheduler.tokens(e.request_id)
        self.scheduler.get_completed()
        return out
