"""Multi-process (gloo, world_size 2, CPU) tests of the sharding logic of the
decode path: KV-head sharding with the per-layer all-gather, sequence sharding,
and a rank that fails before the collective (the survivor must get an error
from a short process-group timeout, not hang).  Compute is the oracle."""
import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _case():
    import oracle
    from tests.helpers import random_layout
    rng = np.random.default_rng(123)
    lens = np.array([5, 300, 17, 1000], np.int32)
    Hq, Hkv, D = 16, 4, 64
    g = oracle.Geom(2, Hkv, D, 16, 0)
    bt, g.num_pages = random_layout(rng, lens)
    pool = (rng.standard_normal(g.pool_shape()) * 0.5).astype(np.float16)
    q = (rng.standard_normal((len(lens), Hq, D)) * 0.5).astype(np.float16)
    return g, bt, lens, pool, q, Hq


def _worker(rank, world, port, mode, results):
    import sys
    sys.path.insert(0, ROOT)
    try:
        import torch
        import torch.distributed as dist

        import oracle
        from vulcan_b200.shard import gathered_to_heads, head_shard, seq_shard
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        g, bt, lens, pool, q, Hq = _case()
        if mode == "heads":
            sh = head_shard(g.Hkv, Hq, world, rank)
            local_pool = np.ascontiguousarray(pool[:, :, sh.kv_lo:sh.kv_hi])
            lg = oracle.Geom(g.L, sh.num_kv_heads, g.D, g.P, g.num_pages)
            local_q = np.ascontiguousarray(q[:, sh.q_lo:sh.q_hi])
            out = oracle.decode_paged(local_pool.view(np.uint16), lg, 1, local_q.view(np.uint16), bt, lens)
            parts = [torch.zeros_like(torch.from_numpy(out)) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(out))
            full = gathered_to_heads(torch.stack(parts)).numpy()
            ref = oracle.decode_paged(pool.view(np.uint16), g, 1, q.view(np.uint16), bt, lens)
            results[rank] = bool(np.array_equal(full, ref))
        elif mode == "seqs":
            mine = seq_shard(lens, world)[rank]
            out = oracle.decode_paged(pool.view(np.uint16), g, 0, np.ascontiguousarray(q[mine]).view(np.uint16),
                                      bt[mine], lens[mine])
            buf = np.zeros((len(lens), Hq, g.D), np.float32)
            buf[mine] = out
            t = torch.from_numpy(buf)
            dist.all_reduce(t)  # each sequence is owned by exactly one rank
            ref = oracle.decode_paged(pool.view(np.uint16), g, 0, q.view(np.uint16), bt, lens)
            results[rank] = bool(np.array_equal(t.numpy(), ref))
        elif mode == "drop":
            if rank == 1:
                raise RuntimeError("injected failure on rank 1 before the collective")
            t = torch.ones(4)
            try:
                dist.all_reduce(t)
                results[rank] = "no error"
            except Exception as e:  # the survivor sees a timeout / closed-connection error
                results[rank] = "error:" + type(e).__name__
        dist.destroy_process_group()
    except Exception:
        results[rank] = "exception:" + traceback.format_exc(limit=1).splitlines()[-1]


def _spawn(mode):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        if p.is_alive():
            p.kill()
            p.join()
    return dict(results)


def test_head_sharded_decode_allgather_matches_single_rank():
    res = _spawn("heads")
    assert res == {0: True, 1: True}, res


def test_sequence_sharded_decode_matches_single_rank():
    res = _spawn("seqs")
    assert res == {0: True, 1: True}, res


def test_dropped_rank_surfaces_an_error():
    res = _spawn("drop")
    assert str(res.get(1, "")).startswith("exception:"), res
    assert str(res.get(0, "")).startswith("error:") or str(res.get(0, "")).startswith("exception:"), res


def test_shard_arithmetic():
    from vulcan_b200.shard import head_shard, seq_shard
    s = head_shard(8, 64, 8, 3)
    assert (s.kv_lo, s.kv_hi, s.q_lo, s.q_hi) == (3, 4, 24, 32)
    s = head_shard(8, 64, 2, 1)
    assert (s.kv_lo, s.kv_hi, s.q_lo, s.q_hi) == (4, 8, 32, 64)
    with pytest.raises(ValueError):
        head_shard(8, 64, 3, 0)
    parts = seq_shard([100, 90, 80, 10, 5], 2)
    assert sorted(np.concatenate(parts).tolist()) == [0, 1, 2, 3, 4]
    loads = [sum([100, 90, 80, 10, 5][i] for i in p) for p in parts]
    assert max(loads) - min(loads) <= 100


# ----------------------------------------------------------------- gather step protocol

def _protocol_worker(rank, world, port, skip_step, results):
    """The fused gather's step protocol (vulcan_b200.shard.GatherSchedule) run
    by gloo ranks with the c10d store standing in for the receive buffers and
    the flags: each layer's run writes its slot on every rank, run l > 0
    raises this rank's flag of run l-1's slot, the end-of-step wait raises the
    last slot's flag and waits (bounded) for every rank's.  Rank 1 does not
    raise its end-of-step flag in step ``skip_step``."""
    import sys
    sys.path.insert(0, ROOT)
    try:
        import time

        import torch.distributed as dist

        from vulcan_b200.shard import GatherSchedule
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
        store = dist.distributed_c10d._get_default_store()
        L, steps = 3, 6
        sched = GatherSchedule(L)
        raised = {}  # (dst, slot) -> value this rank last raised there

        def raise_flag(slot, epoch):
            for dst in range(world):
                key = "flag/%d/%d/%d" % (dst, slot, rank)
                store.add(key, epoch - raised.get((dst, slot), 0))  # flags only grow
                raised[(dst, slot)] = epoch

        def wait_slot(slot, epoch, limit=2.0):
            t0 = time.monotonic()
            for src in range(world):
                while store.add("flag/%d/%d/%d" % (rank, slot, src), 0) < epoch:
                    if time.monotonic() - t0 > limit:
                        raise TimeoutError("slot %d: rank %d's flag did not reach epoch %d" % (slot, src, epoch))
                    time.sleep(0.005)

        log = []
        for _ in range(steps):
            base = sched.begin_step()
            epoch = sched.epoch
            for l in range(L):
                slot = sched.slot(base, l)
                for dst in range(world):  # the run's peer stores
                    store.set("data/%d/%d/%d" % (dst, slot, rank), "%d:%d" % (epoch, l))
                prev = sched.raised_by_run(base, l)
                if prev is not None:
                    raise_flag(prev, epoch)
            # the previous step's slots (the other half) are still intact up to
            # this rank's end-of-step signal: no rank can begin the step that
            # rewrites them before it
            prev_ok = True
            if epoch > 1:
                pbase = sched.slot_base(epoch - 1)
                assert set(sched.slots_of_step(pbase)).isdisjoint(sched.slots_of_step(base))
                prev_ok = all(store.get("data/%d/%d/%d" % (rank, s, src)).decode() == "%d:%d" % (epoch - 1, l)
                              for l, s in enumerate(sched.slots_of_step(pbase)) for src in range(world))
            last = sched.slot(base, L - 1)
            if not (rank == 1 and epoch == skip_step):
                raise_flag(last, epoch)
            try:
                wait_slot(last, epoch)
            except TimeoutError as e:
                log.append(("timeout", epoch, str(e)))
                break
            # after the wait every rank's slice of every slot of this step is in place
            ok = all(store.get("data/%d/%d/%d" % (rank, s, src)).decode() == "%d:%d" % (epoch, l)
                     for l, s in enumerate(sched.slots_of_step(base)) for src in range(world))
            log.append(("ok", epoch, ok and prev_ok, base))
        results[rank] = log
    except Exception:
        results[rank] = "exception:" + traceback.format_exc(limit=2)


def _spawn_protocol(skip_step):
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_protocol_worker, args=(r, 2, port, skip_step, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        if p.is_alive():
            p.kill()
            p.join()
    return dict(results)


def test_gather_protocol_epochs_and_slot_alternation():
    """Six steps of three layers on two ranks: after every end-of-step wait all
    slices of the step are present, alternate steps use alternate halves of the
    2L slots (slot_base 0, 3, 0, ...), and the previous step's slots stay
    intact until this rank's end-of-step signal."""
    res = _spawn_protocol(skip_step=0)
    for r in range(2):
        log = res.get(r)
        assert isinstance(log, list) and len(log) == 6, res
        assert all(e[0] == "ok" and e[2] for e in log), log
        assert [e[3] for e in log] == [0, 3, 0, 3, 0, 3], log


def test_gather_protocol_missing_flag_times_out():
    """Rank 1 never raises its end-of-step flag in step 4: rank 0's bounded wait
    gives up with a timeout after completing steps 1-3 (no hang)."""
    res = _spawn_protocol(skip_step=4)
    log0 = res.get(0)
    assert isinstance(log0, list), res
    assert [e[0] for e in log0] == ["ok", "ok", "ok", "timeout"], log0
    assert log0[3][1] == 4 and "rank 1" in log0[3][2], log0


def test_gather_schedule_rules():
    from vulcan_b200.shard import GatherSchedule
    s = GatherSchedule(4)
    assert s.slots == 8
    assert [s.begin_step() for _ in range(4)] == [0, 4, 0, 4]
    assert s.slots_of_step(4) == [4, 5, 6, 7]
    assert s.raised_by_run(4, 0) is None and s.raised_by_run(4, 2) == 5
    one = GatherSchedule(4, slots=4)  # one slot per layer: every step reuses the same slots
    assert [one.begin_step() for _ in range(3)] == [0, 0, 0]
    with pytest.raises(ValueError):
        GatherSchedule(4, slots=3)
