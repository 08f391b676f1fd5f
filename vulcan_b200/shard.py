"""Host-side partitioning of the decode path across the GPUs of one node.

Two modes, one process per GPU:

* KV-head sharding (GQA models such as Llama-2-70B, 8 KV heads): rank ``r`` of
  ``N`` owns KV heads ``[r*Hkv/N, (r+1)*Hkv/N)`` and their query heads; its pool
  holds only those heads of every page.  Block tables and lengths are the same
  on every rank (allocation runs once on the host and is replicated).  After a
  layer's decode each rank holds ``[B, Hq/N, D]``; one all-gather gives every
  rank ``[N, B, Hq/N, D]``, which ``gathered_to_heads`` views as ``[B, Hq, D]``.
* Sequence sharding (MHA models such as Llama-2-7B): sequences are dealt to
  ranks longest first onto the least-loaded rank (by tokens); no collective.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Sequence

import numpy as np


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    kv_lo: int
    kv_hi: int
    q_lo: int
    q_hi: int

    @property
    def num_kv_heads(self) -> int:
        return self.kv_hi - self.kv_lo

    @property
    def num_q_heads(self) -> int:
        return self.q_hi - self.q_lo


def head_shard(num_kv_heads: int, num_q_heads: int, world: int, rank: int) -> HeadShard:
    """KV heads (and their query heads) owned by ``rank``."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    if num_kv_heads % world:
        raise ValueError("%d KV heads do not split over %d GPUs" % (num_kv_heads, world))
    if num_q_heads % num_kv_heads:
        raise ValueError("query heads must be a multiple of KV heads")
    g = num_q_heads // num_kv_heads
    per = num_kv_heads // world
    return HeadShard(rank, world, rank * per, (rank + 1) * per, rank * per * g, (rank + 1) * per * g)


def shard_heads_of(kv: np.ndarray, shard: HeadShard, axis: int) -> np.ndarray:
    """This rank's slice of an array with a KV-head axis."""
    return np.take(kv, range(shard.kv_lo, shard.kv_hi), axis=axis)


def gathered_to_heads(gathered):
    """``[N, B, Hq/N, D]`` (rank-major all-gather) -> ``[B, Hq, D]``; works on
    numpy arrays and torch tensors (a permuted view, copied by reshape)."""
    n, b, hl, d = gathered.shape
    if hasattr(gathered, "permute"):
        return gathered.permute(1, 0, 2, 3).reshape(b, n * hl, d)
    return np.transpose(gathered, (1, 0, 2, 3)).reshape(b, n * hl, d)


def seq_shard(lengths: Sequence[int], world: int) -> List[np.ndarray]:
    """Sequence indices per rank, balanced by token count (longest first onto the
    least-loaded rank; ties go to the lower rank)."""
    lengths = np.asarray(lengths, np.int64)
    order = np.argsort(-lengths, kind="stable")
    loads = [0] * world
    owner = np.zeros(len(lengths), np.int64)
    for i in order:
        r = int(np.argmin(loads))
        owner[i] = r
        loads[r] += int(lengths[i])
    return [np.nonzero(owner == r)[0] for r in range(world)]


class GatherSchedule:
    """Host side of the step protocol of the fused output gather (vk_gather_*
    bound to a decode plan): which receive slot each layer's run writes, which
    slot each run raises this rank's flags for, what the end-of-step wait
    covers, and the flag value (the step epoch) of a step.  The decode library
    applies the same rules on the device; callers use this to pick each
    step's ``slot_base`` and to know when a slot may be read or rewritten.

    * Step ``s`` (1-based epoch ``s``) with ``L`` layers: run ``l`` writes slot
      ``(slot_base + l) % slots``; run ``l > 0`` raises this rank's flag of run
      ``l - 1``'s slot to the epoch (its stores are complete: the previous grid
      on the stream has finished); the end-of-step wait raises the last slot's
      flag and waits until every rank's flag of that slot carries the epoch.
      Since every rank raises its flags in layer order, that wait covers the
      whole step.
    * With ``2 * L`` slots, alternate steps use alternate halves
      (``slot_base`` 0, L, 0, ...), so a slot written in step ``s`` is rewritten
      in step ``s + 2``, which no rank begins before every rank has raised its
      end-of-step flag of step ``s + 1``: a rank's readers of step ``s``'s slots
      have until it ends step ``s + 1`` (its end-of-step wait) to finish.
    """

    def __init__(self, layers: int, slots: int = 0):
        if layers < 1:
            raise ValueError("layers must be >= 1")
        self.layers = layers
        self.slots = slots or 2 * layers
        if self.slots < layers:
            raise ValueError("fewer slots than layers")
        self.epoch = 0  # steps begun

    def begin_step(self) -> int:
        """Starts the next step; returns its slot_base."""
        self.epoch += 1
        return self.slot_base(self.epoch)

    def slot_base(self, epoch: int) -> int:
        if self.slots >= 2 * self.layers:
            return ((epoch - 1) % 2) * self.layers
        return 0

    def slot(self, slot_base: int, layer: int) -> int:
        return (slot_base + layer) % self.slots

    def raised_by_run(self, slot_base: int, layer: int):
        """Slot whose flag run ``layer`` raises, or None (layer 0)."""
        return self.slot(slot_base, layer - 1) if layer > 0 else None

    def slots_of_step(self, slot_base: int) -> List[int]:
        return [self.slot(slot_base, l) for l in range(self.layers)]
