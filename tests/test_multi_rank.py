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
