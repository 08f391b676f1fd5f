"""Host-side model of the reference's paged allocator and swap semantics.

TEST INFRASTRUCTURE ONLY: the tests compare the CUDA library's allocator
against this model; the product never imports it.

Restated from VULCAN's ``MemoryManager`` (cuda/memory.cu):

* ``allocate_block`` — first free block in id order, ``-1`` when none is free
  (cuda/memory.cu:127-135).
* ``free_block`` — ids outside the pool are ignored; clears ``in_use`` and drops
  any swap copy (cuda/memory.cu:137-143).
* ``get_block_ptr`` — ``base + id * page_size``; ``None`` for a bad id
  (cuda/memory.cu:145-150).
* ``swap_to_cpu`` — bad id or a free block → ``False``; otherwise the page's
  bytes go to host storage keyed by id and the block becomes free
  (cuda/memory.cu:152-169).
* ``swap_to_gpu`` — bad id or nothing stored → ``False``; otherwise the block is
  marked in use, the bytes are restored into the SAME id and the host copy is
  dropped (cuda/memory.cu:171-191).  The reference does not check whether the
  id was reallocated meanwhile; the model keeps a ``strict`` switch that
  refuses that case, which is the library's documented behaviour.
* ``blocks_in_use`` / ``blocks_available`` / ``total_allocated_bytes``
  (cuda/memory.cu:193-207).
"""
from __future__ import annotations


class AllocatorModel:
    def __init__(self, page_size: int, max_pages: int, strict: bool = True):
        self.page_size = page_size
        self.max_pages = max_pages
        self.in_use = [False] * max_pages
        self.data = {}          # id -> bytes currently "on the GPU" (model only)
        self.cpu_swap = {}      # id -> bytes swapped out
        self.strict = strict

    def allocate_block(self) -> int:
        for i, used in enumerate(self.in_use):
            if not used:
                self.in_use[i] = True
                return i
        return -1

    def allocate_n(self, n: int):
        """All-or-nothing batch of the lowest free ids (library extension)."""
        free = [i for i, u in enumerate(self.in_use) if not u]
        if len(free) < n:
            return None
        for i in free[:n]:
            self.in_use[i] = True
        return free[:n]

    def free_block(self, block_id: int) -> None:
        if 0 <= block_id < self.max_pages:
            self.in_use[block_id] = False
            self.cpu_swap.pop(block_id, None)

    def get_block_offset(self, block_id: int):
        if 0 <= block_id < self.max_pages:
            return block_id * self.page_size
        return None

    def swap_to_cpu(self, block_id: int, page_bytes: bytes = b"") -> bool:
        if not (0 <= block_id < self.max_pages):
            return False
        if not self.in_use[block_id]:
            return False
        self.cpu_swap[block_id] = page_bytes
        self.in_use[block_id] = False
        return True

    def swap_to_gpu(self, block_id: int):
        """Returns (ok, restored_bytes)."""
        if not (0 <= block_id < self.max_pages):
            return False, None
        if block_id not in self.cpu_swap:
            return False, None
        if self.strict and self.in_use[block_id]:
            return False, None
        self.in_use[block_id] = True
        return True, self.cpu_swap.pop(block_id)

    def blocks_in_use(self) -> int:
        return sum(self.in_use)

    def blocks_available(self) -> int:
        return self.max_pages - self.blocks_in_use()

    def total_allocated_bytes(self) -> int:
        return self.blocks_in_use() * self.page_size

    def compact_plan(self):
        """Highest in-use ids move into the lowest free ids (library extension):
        returns (src, dst) pairs and updates the model."""
        pairs = []
        lo, hi = 0, self.max_pages - 1
        while True:
            while lo < self.max_pages and self.in_use[lo]:
                lo += 1
            while hi >= 0 and not self.in_use[hi]:
                hi -= 1
            if lo >= hi:
                break
            pairs.append((hi, lo))
            self.in_use[lo] = True
            self.in_use[hi] = False
        return pairs
