"""Two-GPU tests of KV-head-sharded decode: each rank holds half of the KV
heads of a 70B-shaped pool and decodes its query heads with the planned kernel
(fused append).  The output all-gathered by NCCL, and the output gathered by
the decode's own peer stores (vk_gather, two layers back to back with the
previous-slot wait), both match a single-GPU decode of the full pool within the
attention tolerance, and the two gathers agree bit for bit.  Skipped when fewer
than two GPUs are visible.  Child processes, NVLS off, short process-group
timeout."""
import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _data():
    from tests.helpers import random_layout
    import oracle
    rng = np.random.default_rng(2)
    B, Hq, Hkv, D, L = 16, 64, 8, 128, 2
    lens = np.clip(np.round(np.exp(rng.normal(np.log(2048), 0.6, B))), 256, 8192).astype(np.int32) + 1
    g = oracle.Geom(L, Hkv, D, 16, 0)
    bt, g.num_pages = random_layout(rng, lens)
    pool = (rng.standard_normal(g.pool_shape(), dtype=np.float32) * 0.5).astype(np.float16)
    q = (rng.standard_normal((B, Hq, D)) * 0.5).astype(np.float16)
    kn = (rng.standard_normal((B, Hkv, D)) * 0.5).astype(np.float16)
    vn = (rng.standard_normal((B, Hkv, D)) * 0.5).astype(np.float16)
    return g, bt, lens, pool, q, kn, vn, Hq


def _worker(rank, world, port, results):
    import sys
    sys.path.insert(0, ROOT)
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import torch.distributed as dist
        import vulcan_b200 as vk
        from vulcan_b200.shard import gathered_to_heads, head_shard
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        g, bt, lens, pool, q, kn, vn, Hq = _data()
        sh = head_shard(g.Hkv, Hq, world, rank)
        lp = vk.PagedKVPool(g.L, sh.num_kv_heads, g.D, g.num_pages)
        lp.kv_view().copy_(torch.from_numpy(np.ascontiguousarray(pool[:, :, sh.kv_lo:sh.kv_hi])).view(torch.float16))
        bt_d = torch.from_numpy(bt).to(dev)
        plan = lp.plan(lens.tolist(), sh.num_q_heads)
        out = plan.run(1, torch.from_numpy(np.ascontiguousarray(q[:, sh.q_lo:sh.q_hi])).to(dev), bt_d,
                       k_new=torch.from_numpy(np.ascontiguousarray(kn[:, sh.kv_lo:sh.kv_hi])).to(dev),
                       v_new=torch.from_numpy(np.ascontiguousarray(vn[:, sh.kv_lo:sh.kv_hi])).to(dev))
        gathered = torch.empty(world, *out.shape, dtype=out.dtype, device=dev)
        dist.all_gather_into_tensor(gathered.view(-1), out.contiguous().view(-1))
        full = gathered_to_heads(gathered).float().cpu()
        # the same layer through the fused peer-store gather: layer 0 then
        # layer 1 (which waits for layer 0's slot), append only in layer 1 of
        # a fresh copy of the shard
        lp2 = vk.PagedKVPool(g.L, sh.num_kv_heads, g.D, g.num_pages)
        lp2.kv_view().copy_(torch.from_numpy(np.ascontiguousarray(pool[:, :, sh.kv_lo:sh.kv_hi])).view(torch.float16))
        B = len(lens)
        gat = vk.Gather(rank, world, B * sh.num_q_heads * g.D * 2, slots=2)
        gat.exchange()
        gplan = lp2.plan(lens.tolist(), sh.num_q_heads)
        gplan.set_gather(gat, wait_prev=True)
        qd = torch.from_numpy(np.ascontiguousarray(q[:, sh.q_lo:sh.q_hi])).to(dev)
        gplan.run(0, qd, bt_d)
        gplan.run(1, qd, bt_d, k_new=torch.from_numpy(np.ascontiguousarray(kn[:, sh.kv_lo:sh.kv_hi])).to(dev),
                  v_new=torch.from_numpy(np.ascontiguousarray(vn[:, sh.kv_lo:sh.kv_hi])).to(dev))
        gplan.gather_wait(1)
        fused = gat.view(1, B, sh.num_q_heads, g.D)
        torch.cuda.synchronize()
        gat.check()
        lp2.check()
        same = bool(torch.equal(fused, gathered))
        lp.check()
        ok = same
        if rank == 0:  # single-GPU reference on the whole pool
            fp = vk.PagedKVPool(g.L, g.Hkv, g.D, g.num_pages)
            fp.kv_view().copy_(torch.from_numpy(pool).view(torch.float16))
            ref = fp.plan(lens.tolist(), Hq).run(1, torch.from_numpy(q).to(dev), bt_d,
                                                 k_new=torch.from_numpy(kn).to(dev),
                                                 v_new=torch.from_numpy(vn).to(dev)).float().cpu()
            err = (full - ref).abs()
            ok = same and bool((err <= 2e-3 + 1e-2 * ref.abs()).all())
        gplan.set_gather(None)
        gat.close()  # releases the peer mappings, barrier, frees
        results[rank] = ok
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        results[rank] = "exception: " + traceback.format_exc(limit=3)


def test_head_sharded_decode_two_gpus(cuda_ok):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        if p.is_alive():
            p.kill()
            p.join()
    assert dict(results) == {0: True, 1: True}, dict(results)


def _oproj_worker(rank, world, port, results):
    """Head-sharded output projection: rank r holds the attention output of its
    heads and its rows of wo; one vk_oproj run per step leaves on rank r its
    features of x @ wo (a reduce-scatter inside the GEMM launch)."""
    import sys
    sys.path.insert(0, ROOT)
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import torch.distributed as dist
        import vulcan_b200 as vk
        import oracle
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        rng = np.random.default_rng(12)
        tokens, K, N = 48, 2048, 2048
        x = (rng.standard_normal((tokens, K)) * 0.5).astype(np.float16)
        w = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)   # wo [K, N]
        kl, nl = K // world, N // world
        xr = torch.from_numpy(np.ascontiguousarray(x[:, rank * kl:(rank + 1) * kl])).to(dev)
        op = vk.OutputProjection(rank, world, 64, kl, N, device=dev)
        # this rank's rows of wo, in the reference's fp32 layout, packed
        wtr = op.pack_weight(torch.from_numpy(np.ascontiguousarray(w[rank * kl:(rank + 1) * kl]).astype(np.float32)).to(dev))
        op.exchange()
        outs = [op.run(xr, wtr).clone() for _ in range(3)]
        torch.cuda.synchronize()
        op.check()
        same = all(torch.equal(o, outs[0]) for o in outs[1:])
        ref = oracle.matmul(x.astype(np.float32), np.ascontiguousarray(w[:, rank * nl:(rank + 1) * nl]).astype(np.float32))
        got = outs[0].float().cpu().numpy()
        err = np.abs(got - ref)
        ok = same and bool((err <= 2e-3 + 1e-2 * np.abs(ref)).all())
        results[rank] = ok if ok else "same %s max err %g" % (same, err.max())
        op.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        results[rank] = "exception: " + traceback.format_exc(limit=3)


def test_output_projection_reduce_scatter_multi_gpu(cuda_ok):
    """On every visible GPU (2 to 8): each rank's features of the projection
    match the oracle's fp32 GEMM of the full x and wo, three runs in a row
    give the same bits (alternating receive slots)."""
    n = min(torch.cuda.device_count(), 8)
    if n < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _port()
    procs = [ctx.Process(target=_oproj_worker, args=(r, n, port, results)) for r in range(n)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        if p.is_alive():
            p.kill()
            p.join()
    assert dict(results) == {r: True for r in range(n)}, dict(results)
