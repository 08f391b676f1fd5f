"""Multi-sequence cache manager over a paged KV pool.

The reference engine holds one sequence and one contiguous cache
(src/engine.cpp:26-127) and never calls its paged allocator
(cuda/memory.cu:127-191).  This manager is the batched caller the paged path
needs: it admits sequences, grows their block tables a page at a time,
swaps least-recently-used sequences out to a page-locked host arena when the
pool is full (and back in, possibly into other page ids), and compacts the pool
by page copy.  Device work goes through the C ABI on two streams: swap copies on
``swap_stream`` and everything else on the caller's stream, with events keeping
page reuse ordered.

The pool is used through the methods ``alloc``, ``free``, ``pages_available``,
``swap_out``, ``swap_in``, ``compact_plan``, ``copy_pages`` and the attribute
``page_bytes``, so tests can substitute a host-only model.
"""
from __future__ import annotations

import bisect
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np

PAGE_TOKENS = 16


@dataclass
class Sequence:
    sid: int
    length: int                       # tokens cached (attended by the next decode, plus the new one)
    pages: List[int] = field(default_factory=list)
    host_slot: Optional[int] = None   # first page slot in the host arena while swapped out
    host_pages: int = 0

    @property
    def resident(self) -> bool:
        return self.host_slot is None


class HostArena:
    """First-fit allocator of runs of page slots in one page-locked buffer."""

    def __init__(self, num_slots: int):
        self.num_slots = num_slots
        self.free_runs: List[List[int]] = [[0, num_slots]] if num_slots > 0 else []  # sorted [start, length]

    def alloc(self, n: int) -> Optional[int]:
        for i, (s, ln) in enumerate(self.free_runs):
            if ln >= n:
                if ln == n:
                    self.free_runs.pop(i)
                else:
                    self.free_runs[i] = [s + n, ln - n]
                return s
        return None

    def free(self, start: int, n: int) -> None:
        starts = [r[0] for r in self.free_runs]
        i = bisect.bisect_left(starts, start)
        self.free_runs.insert(i, [start, n])
        # merge with neighbours
        merged: List[List[int]] = []
        for s, ln in self.free_runs:
            if merged and merged[-1][0] + merged[-1][1] == s:
                merged[-1][1] += ln
            else:
                merged.append([s, ln])
        self.free_runs = merged

    def free_slots(self) -> int:
        return sum(ln for _, ln in self.free_runs)


class PagedKVScheduler:
    def __init__(self, pool, host_buffer=None, host_slots: int = 0, swap_stream=None, stream=None,
                 on_swap=None):
        """``host_buffer``: page-locked uint8 tensor of ``host_slots * pool.page_bytes``
        bytes (or None for no swapping).  ``on_swap(kind, pages, fn)`` may wrap the
        swap calls (used by benchmarks to time them)."""
        self.pool = pool
        self.host = host_buffer
        self.arena = HostArena(host_slots)
        self.seqs: Dict[int, Sequence] = {}
        self.lru: "OrderedDict[int, None]" = OrderedDict()  # resident sequences, least recent first
        self.swapped: "OrderedDict[int, None]" = OrderedDict()  # swapped out, oldest first
        self.swap_stream = swap_stream
        self.stream = stream
        self.on_swap = on_swap or (lambda kind, pages, fn: fn())
        self.stats = dict(swap_out_pages=0, swap_in_pages=0, copied_pages=0, evictions=0, restores=0)

    # ------------------------------------------------------------------ helpers
    @staticmethod
    def pages_for(tokens: int) -> int:
        return (tokens + PAGE_TOKENS - 1) // PAGE_TOKENS

    def _touch(self, sid: int) -> None:
        self.lru.pop(sid, None)
        self.lru[sid] = None

    def _host_view(self, slot: int, n: int):
        pb = self.pool.page_bytes
        return self.host[slot * pb:(slot + n) * pb]

    def _make_room(self, need: int, protect=()) -> bool:
        """Swaps out least-recently-used sequences until ``need`` pages are free."""
        while self.pool.pages_available() < need:
            victim = next((s for s in self.lru if s not in protect), None)
            if victim is None or not self.evict(victim):
                return False
        return True

    # ------------------------------------------------------------------ lifecycle
    def admit(self, sid: int, length: int) -> bool:
        """New sequence with ``length`` cached tokens (pages allocated, contents
        supplied by the caller's prefill).  Evicts LRU sequences if needed."""
        need = self.pages_for(length)
        if not self._make_room(need):
            return False
        s = Sequence(sid, length, self.pool.alloc(need) if need else [])
        self.seqs[sid] = s
        self._touch(sid)
        return True

    def grow(self, sid: int, protect=()) -> bool:
        """Makes room for one more token of a resident sequence."""
        s = self.seqs[sid]
        if self.pages_for(s.length + 1) > len(s.pages):
            if not self._make_room(1, protect=set(protect) | {sid}):
                return False
            s.pages += self.pool.alloc(1)
        s.length += 1
        self._touch(sid)
        return True

    def evict(self, sid: int) -> bool:
        s = self.seqs[sid]
        if not s.resident or self.host is None:
            return False
        n = len(s.pages)
        slot = self.arena.alloc(n) if n else 0
        if slot is None:
            return False
        if n:
            self.on_swap("out", n, lambda: self.pool.swap_out(s.pages, self._host_view(slot, n),
                                                              stream=self.swap_stream))
        s.host_slot, s.host_pages, s.pages = slot, n, []
        self.lru.pop(sid, None)
        self.swapped[sid] = None
        self.stats["swap_out_pages"] += n
        self.stats["evictions"] += 1
        return True

    def restore(self, sid: int, protect=()) -> bool:
        """Swaps a sequence back in (new page ids, lowest free first)."""
        s = self.seqs[sid]
        if s.resident:
            return True
        n = s.host_pages
        if not self._make_room(n, protect=protect):
            return False
        ids: List[int] = []
        if n:
            ids = self.on_swap("in", n, lambda: self.pool.swap_in(self._host_view(s.host_slot, n), n,
                                                                 stream=self.swap_stream))
            self.arena.free(s.host_slot, n)
        s.pages, s.host_slot, s.host_pages = list(ids), None, 0
        self.swapped.pop(sid, None)
        self._touch(sid)
        self.stats["swap_in_pages"] += n
        self.stats["restores"] += 1
        return True

    def release(self, sid: int) -> None:
        s = self.seqs.pop(sid)
        if s.resident:
            self.pool.free(s.pages)
            self.lru.pop(sid, None)
        else:
            self.arena.free(s.host_slot, s.host_pages)
            self.swapped.pop(sid, None)

    def compact(self, copy_fn=None):
        """Moves in-use pages to the lowest ids and rewrites the page lists.
        ``copy_fn(src_ids, dst_ids)`` performs the device copy (vk_copy_pages)."""
        src, dst = self.pool.compact_plan()
        if not src:
            return 0
        remap = dict(zip(src, dst))
        for s in self.seqs.values():
            if s.resident:
                s.pages = [remap.get(p, p) for p in s.pages]
        if copy_fn is not None:
            copy_fn(src, dst)
        self.stats["copied_pages"] += len(src)
        return len(src)

    # ------------------------------------------------------------------ batches
    def resident_ids(self) -> List[int]:
        return [sid for sid, s in self.seqs.items() if s.resident]

    def block_table(self, sids: List[int], width: Optional[int] = None) -> np.ndarray:
        width = width or max([len(self.seqs[s].pages) for s in sids] + [1])
        bt = np.full((len(sids), width), -1, np.int32)
        for i, sid in enumerate(sids):
            pg = self.seqs[sid].pages
            bt[i, :len(pg)] = pg
        return bt

    def lengths(self, sids: List[int]) -> np.ndarray:
        return np.array([self.seqs[s].length for s in sids], np.int32)
