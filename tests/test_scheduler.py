"""CPU tests of the multi-sequence cache manager (vulcan_b200.scheduler) with a
host-only pool built on the allocator model: page ownership stays exclusive,
LRU eviction and swap-in keep every sequence's bytes, compaction packs ids."""
import numpy as np

from oracle.allocator_model import AllocatorModel
from vulcan_b200.scheduler import HostArena, PagedKVScheduler


class FakePool:
    """Host model of the pool: lowest-free-id allocation, page contents as ints."""

    def __init__(self, num_pages, page_bytes=4):
        self.m = AllocatorModel(page_bytes, num_pages)
        self.page_bytes = page_bytes
        self.data = np.zeros(num_pages, np.int64)  # one tag per page

    def alloc(self, n):
        ids = self.m.allocate_n(n)
        if ids is None:
            raise MemoryError
        return ids

    def free(self, ids):
        for i in ids:
            self.m.free_block(i)

    def pages_available(self):
        return self.m.blocks_available()

    def swap_out(self, ids, host, stream=None):
        host[:] = self.data[ids].repeat(self.page_bytes)[:len(host)]
        for i in ids:
            self.m.in_use[i] = False

    def swap_in(self, host, n, stream=None):
        ids = self.alloc(n)
        self.data[ids] = host[::self.page_bytes][:n]
        return ids

    def compact_plan(self):
        pairs = self.m.compact_plan()
        return [s for s, _ in pairs], [d for _, d in pairs]

    def copy(self, src, dst):
        self.data[dst] = self.data[src]


def _tag_pages(pool, sched, sid):
    s = sched.seqs[sid]
    for k, p in enumerate(s.pages):
        pool.data[p] = sid * 1000 + k


def _check(pool, sched):
    owned = []
    for sid, s in sched.seqs.items():
        if s.resident:
            owned += s.pages
            assert len(s.pages) == sched.pages_for(s.length)
            for k, p in enumerate(s.pages):
                assert pool.m.in_use[p]
                assert pool.data[p] == sid * 1000 + k, (sid, k, p)
    assert len(owned) == len(set(owned))
    assert sum(pool.m.in_use) == len(owned)


def test_arena_first_fit_and_merge():
    a = HostArena(10)
    assert a.alloc(4) == 0 and a.alloc(3) == 4
    a.free(0, 4)
    assert a.alloc(5) is None and a.alloc(2) == 0
    a.free(0, 2)
    a.free(4, 3)
    assert a.free_runs == [[0, 10]]


def test_admit_grow_evict_restore_compact():
    rng = np.random.default_rng(0)
    pool = FakePool(40)
    host = np.zeros(200 * pool.page_bytes, np.int64)
    sched = PagedKVScheduler(pool, host_buffer=host, host_slots=200)
    for sid in range(6):
        assert sched.admit(sid, int(rng.integers(20, 200)))
        _tag_pages(pool, sched, sid)
    _check(pool, sched)
    for step in range(60):
        for sid in list(sched.resident_ids()):
            if sid in sched.seqs and sched.seqs[sid].resident:
                before = len(sched.seqs[sid].pages)
                assert sched.grow(sid)
                if len(sched.seqs[sid].pages) > before:
                    pool.data[sched.seqs[sid].pages[-1]] = sid * 1000 + before
        if sched.swapped and step % 3 == 0:
            sid = next(iter(sched.swapped))
            assert sched.restore(sid)
        if step % 10 == 9:
            sched.compact(copy_fn=pool.copy)
            used = [i for i, u in enumerate(pool.m.in_use) if u]
            assert used == list(range(len(used)))
        _check(pool, sched)
    assert sched.stats["evictions"] > 0 and sched.stats["restores"] > 0
    bt = sched.block_table(sched.resident_ids())
    assert bt.shape[0] == len(sched.resident_ids())


def test_admit_fails_cleanly_without_swap_space():
    pool = FakePool(8)
    sched = PagedKVScheduler(pool)  # no host arena: nothing can be evicted
    assert sched.admit(0, 16 * 6)
    assert not sched.admit(1, 16 * 3)
    assert list(sched.seqs) == [0] and pool.pages_available() == 2
