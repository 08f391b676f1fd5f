"""GPU parity tests of the planned decode (vk_decode_plan_* / vk_decode_run):
balanced worker ranges across (sequence, head) units, fused append, fused
split merge.  Same tolerance as the other decode tests; the fused append is
bit-exact against the oracle's append."""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_close_attn, dev_f16, dev_i32, make_pool, random_layout, random_pool

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def vk(cuda_ok):
    import vulcan_b200
    vulcan_b200.load()
    return vulcan_b200


def _case(rng, lens, Hq, Hkv, D, L=2):
    g = oracle.Geom(L, Hkv, D, 16, 0)
    bt, g.num_pages = random_layout(rng, np.maximum(lens, 1))
    host = random_pool(rng, g)
    q = (rng.standard_normal((len(lens), Hq, D)) * 0.5).astype(np.float16)
    return g, bt, host, q


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("Hq,Hkv", [(8, 1), (8, 2), (4, 4), (16, 1), (12, 4), (64, 8)])
def test_planned_matches_oracle(vk, D, Hq, Hkv):
    rng = np.random.default_rng(D + Hq * 7 + Hkv)
    lens = np.array([1, 15, 16, 17, 100, 513, 1200, 3000], np.int32)
    g, bt, host, q = _case(rng, lens, Hq, Hkv, D)
    pool = make_pool(vk, g, host)
    plan = pool.plan(lens.tolist(), Hq)
    out = plan.run(1, dev_f16(q), dev_i32(bt)).float().cpu().numpy()
    assert pool.check() == 0
    ref = oracle.decode_paged(host.view(np.uint16), g, 1, q.view(np.uint16), bt, lens)
    assert_close_attn(out, ref, "planned D%d Hq%d Hkv%d (W=%d)" % (D, Hq, Hkv, plan.workers))


def test_planned_fused_append(vk):
    """k_new/v_new land at position len-1 (bit-exact vs the oracle's append) and
    are attended in the same launch."""
    rng = np.random.default_rng(5)
    lens = np.array([1, 16, 17, 250, 2049], np.int32)
    Hq, Hkv, D = 16, 2, 128
    g, bt, host, q = _case(rng, lens, Hq, Hkv, D, L=3)
    pool = make_pool(vk, g, host)
    k = (rng.standard_normal((len(lens), Hkv, D)) * 0.5).astype(np.float16)
    v = (rng.standard_normal((len(lens), Hkv, D)) * 0.5).astype(np.float16)
    plan = pool.plan(lens.tolist(), Hq)
    out = plan.run(2, dev_f16(q), dev_i32(bt), k_new=dev_f16(k), v_new=dev_f16(v)).float().cpu().numpy()
    assert pool.check() == 0
    expect = host.copy()
    assert oracle.append_paged(expect.view(np.uint16), g, 2, k[:, None].view(np.uint16), v[:, None].view(np.uint16),
                               bt, lens - 1) == 0
    assert np.array_equal(pool.kv_view().cpu().numpy().view(np.uint16), expect.view(np.uint16))
    ref = oracle.decode_paged(expect.view(np.uint16), g, 2, q.view(np.uint16), bt, lens)
    assert_close_attn(out, ref, "fused append")


def test_planned_repeated_runs_and_layers(vk):
    """Merge counters reset themselves: many launches on one uploaded plan give
    the same answers as fresh plans."""
    rng = np.random.default_rng(6)
    lens = np.array([3000, 900, 40, 2500], np.int32)
    Hq, Hkv, D = 8, 4, 128
    g, bt, host, q = _case(rng, lens, Hq, Hkv, D, L=4)
    pool = make_pool(vk, g, host)
    plan = pool.plan(lens.tolist(), Hq)
    assert plan.info(2) > 0  # some units are split across workers
    qd, btd = dev_f16(q), dev_i32(bt)
    first = [plan.run(l, qd, btd).clone() for l in range(4)]
    for rep in range(3):
        for l in range(4):
            assert torch.equal(plan.run(l, qd, btd), first[l]), (rep, l)
    for l in range(4):
        ref = oracle.decode_paged(host.view(np.uint16), g, l, q.view(np.uint16), bt, lens)
        assert_close_attn(first[l].float().cpu().numpy(), ref, "layer %d" % l)
    assert pool.check() == 0


def test_planned_zero_lengths_and_single_worker(vk):
    rng = np.random.default_rng(7)
    lens = np.array([0, 5, 0, 33], np.int32)
    Hq, Hkv, D = 8, 2, 128
    g, bt, host, q = _case(rng, lens, Hq, Hkv, D)
    pool = make_pool(vk, g, host)
    plan = pool.plan(lens.tolist(), Hq)
    out = plan.run(0, dev_f16(q), dev_i32(bt)).float().cpu().numpy()
    assert np.all(out[0] == 0) and np.all(out[2] == 0)
    ref = oracle.decode_paged(host.view(np.uint16), g, 0, q.view(np.uint16), bt, lens)
    assert_close_attn(out, ref, "zero lengths")
    plan0 = pool.plan([0, 0], Hq)  # nothing to attend at all
    out0 = plan0.run(0, dev_f16(q[:2]), dev_i32(bt[:2]))
    assert torch.count_nonzero(out0).item() == 0


def test_planned_equals_split_decode(vk):
    """The planned and the split-grid decode agree within the attention tolerance
    on a 70B-shaped layer sample."""
    rng = np.random.default_rng(8)
    B, Hq, Hkv, D = 16, 64, 8, 128
    lens = np.clip(np.round(np.exp(rng.normal(np.log(2048), 0.6, B))), 256, 8192).astype(np.int32) + 1
    g, bt, host, q = _case(rng, lens, Hq, Hkv, D, L=1)
    pool = make_pool(vk, g, host)
    a = pool.decode(0, dev_f16(q), dev_i32(bt), dev_i32(lens), int(lens.max())).float().cpu().numpy()
    b = pool.plan(lens.tolist(), Hq).run(0, dev_f16(q), dev_i32(bt)).float().cpu().numpy()
    assert_close_attn(b, a, "planned vs split")
    ref = oracle.decode_paged(host.view(np.uint16), g, 0, q[:4].view(np.uint16), bt[:4], lens[:4], nthreads=8)
    assert_close_attn(b[:4], ref, "planned vs oracle")


def test_planned_rejects_narrow_table(vk):
    g = oracle.Geom(1, 1, 128, 16, 8)
    pool = make_pool(vk, g)
    plan = pool.plan([100], 8)
    q = torch.zeros(1, 8, 128, dtype=torch.float16, device="cuda")
    with pytest.raises(vk.VKError):
        plan.run(0, q, torch.zeros(1, 3, dtype=torch.int32, device="cuda"))  # 100 tokens need 7 pages


def test_planned_fused_gather_one_rank(vk):
    """A gather of one rank: every layer's output lands in slot slot_base +
    layer of the receive buffer, bit-identical to the plain run, with and
    without an explicit `out`, with and without the previous-slot wait;
    vk_decode_plan_gather_wait passes and no timeout is recorded."""
    rng = np.random.default_rng(31)
    lens = np.array([0, 1, 17, 300, 2049], np.int32)
    Hq, Hkv, D, L = 16, 2, 128, 3
    g, bt, host, q = _case(rng, lens, Hq, Hkv, D, L=L)
    pool = make_pool(vk, g, host)
    bt_d = dev_i32(bt)
    plan = pool.plan(lens.tolist(), Hq)
    plain = [plan.run(l, dev_f16(q), bt_d).clone() for l in range(L)]
    B = len(lens)
    gat = vk.Gather(0, 1, B * Hq * D * 2, slots=2 * L)
    for step in range(4):
        base = (step % 2) * L
        gplan = pool.plan(lens.tolist(), Hq)
        gplan.set_gather(gat, slot_base=base, wait_prev=step < 2)
        for l in range(L):
            explicit = torch.empty_like(plain[0]) if l == 1 else None
            r = gplan.run(l, dev_f16(q), bt_d, out=explicit)
            if explicit is not None:
                assert torch.equal(r, plain[l])
        gplan.gather_wait(L - 1)
        for l in range(L):
            assert torch.equal(gat.view(base + l, B, Hq, D)[0], plain[l]), "step %d layer %d" % (step, l)
        gplan.set_gather(None)
    torch.cuda.synchronize()
    gat.check()
    assert pool.check() == 0
    gat.close()


# Lengths (tokens) whose units, with 16 workers per KV head, give ~120 pages
# per worker: a 1000-page unit of more than 8 pieces (merged by dealt tasks)
# next to units of 2..4 pieces (merged by their last piece), single-piece
# units, a one-token unit and an empty one.
_LMM_LENS = np.array([16000, 4000, 1600, 2600, 300, 17, 1, 6000, 0], np.int32)


def _lmm_plan(pool, lens, Hq, Hkv):
    pool.set_plan_workers(16 * Hkv)
    plan = pool.plan(lens.tolist(), Hq)
    pool.set_plan_workers(0)
    assert plan.info(3) // plan.workers >= 64, "the case must have long worker ranges"
    assert plan.info(5) == 8, "units of up to 8 pieces must merge in their last piece"
    assert plan.info(6) >= 3, "several units merged by their last piece"
    assert plan.info(7) >= 1 and plan.info(8) > 8, "one unit of more than 8 pieces merged by tasks"
    return plan


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("Hq,Hkv", [(8, 1), (16, 1), (16, 2), (64, 8)])
def test_planned_last_piece_merge(vk, D, Hq, Hkv):
    """Long worker ranges (>= 64 pages each, the one-GPU 70B regime): units of
    2..8 pieces are merged by whichever piece finishes last (acq_rel counter,
    merge in head groups of 1024/D, counter reset by the merger), a unit of
    more than 8 pieces by dealt tasks, in one plan.  Two rounds over two layers
    on one uploaded plan are bit-identical (the counters reset themselves),
    and the fused append lands bit-exact."""
    if Hkv == 8 and D != 128:
        pytest.skip("70B heads at D=128 only (pool size)")
    rng = np.random.default_rng(400 + D + Hq + Hkv)
    lens = _LMM_LENS
    g, bt, host, q = _case(rng, lens, Hq, Hkv, D, L=2)
    pool = make_pool(vk, g, host)
    plan = _lmm_plan(pool, lens, Hq, Hkv)
    qd, btd = dev_f16(q), dev_i32(bt)
    first = [plan.run(l, qd, btd).clone() for l in range(2)]
    for rep in range(2):
        for l in range(2):
            assert torch.equal(plan.run(l, qd, btd), first[l]), (rep, l)
    assert pool.check() == 0
    for l in range(2):
        ref = oracle.decode_paged(host.view(np.uint16), g, l, q.view(np.uint16), bt, lens, nthreads=8)
        assert_close_attn(first[l].float().cpu().numpy(), ref, "last-piece merge D%d Hq%d Hkv%d layer %d" % (D, Hq, Hkv, l))
    # fused append on the same branch
    B = len(lens)
    k = (rng.standard_normal((B, Hkv, D)) * 0.5).astype(np.float16)
    v = (rng.standard_normal((B, Hkv, D)) * 0.5).astype(np.float16)
    out = plan.run(1, qd, btd, k_new=dev_f16(k), v_new=dev_f16(v)).float().cpu().numpy()
    assert pool.check() == 0
    has = lens > 0  # an empty sequence has no page to append into
    expect = host.copy()
    assert oracle.append_paged(expect.view(np.uint16), g, 1, k[has][:, None].view(np.uint16),
                               v[has][:, None].view(np.uint16), bt[has], lens[has] - 1) == 0
    got = pool.kv_view().cpu().numpy()
    assert np.array_equal(got.view(np.uint16), expect.view(np.uint16)), "fused append (last-piece merge plan)"
    ref = oracle.decode_paged(expect.view(np.uint16), g, 1, q.view(np.uint16), bt, lens, nthreads=8)
    assert_close_attn(out[has], ref[has], "last-piece merge with fused append")


def _compact(pool_dev, bt, sample, lens):
    """The pages of the sampled sequences, gathered from a device pool view
    [L, num_pages, ...] into a host array, and block tables renumbered to it."""
    pages, tabs = [], np.full((len(sample), bt.shape[1]), -1, np.int32)
    for i, b in enumerate(sample):
        n = (int(lens[b]) + 15) // 16
        tabs[i, :n] = np.arange(len(pages), len(pages) + n, dtype=np.int32)
        pages.extend(int(x) for x in bt[b, :n])
    idx = torch.tensor(pages, dtype=torch.long, device=pool_dev.device)
    return pool_dev.index_select(1, idx).cpu().numpy(), tabs


def _70b_lens(rng, B=64):
    return np.clip(np.round(np.exp(rng.normal(np.log(2048), 0.6, B))), 256, 8192).astype(np.int32) + 1


def test_planned_70b_full_layer_fused_append(vk):
    """The headline configuration of one GPU: a full Llama-2-70B GQA layer (B=64,
    64/8 heads, D=128, lognormal contexts median 2048 clipped to [256, 8192]),
    default workers (one per resident warp), so ~80 pages per worker and the
    last-piece merge path; fused append of the new token.  Two layers run back
    to back with early start (programmatic dependent launch), as in the
    benchmark step.  Sampled sequences (longest, shortest and six more) are
    checked against the oracle: appended rows bit-exact, outputs within the
    attention tolerance."""
    rng = np.random.default_rng(700)
    B, Hq, Hkv, D, L = 64, 64, 8, 128, 2
    lens = _70b_lens(rng, B)
    g = oracle.Geom(L, Hkv, D, 16, 0)
    bt, g.num_pages = random_layout(rng, lens)
    pool = make_pool(vk, g)
    kv = pool.kv_view()
    kv.copy_((torch.randn(kv.shape, device="cuda", generator=torch.Generator("cuda").manual_seed(2)) * 0.5).half())
    plan = pool.plan(lens.tolist(), Hq)
    assert plan.info(5) == 8 and plan.info(6) > 0, "the 70B layer must take the last-piece merge path"
    assert plan.info(3) // plan.workers >= 64
    plan.set_early_start(True)
    sample = [int(np.argmax(lens)), int(np.argmin(lens))] + [int(x) for x in rng.choice(B, 6, replace=False)]
    before, tabs = _compact(kv, bt, sample, lens)
    q = [(rng.standard_normal((B, Hq, D)) * 0.5).astype(np.float16) for _ in range(L)]
    k = [(rng.standard_normal((B, Hkv, D)) * 0.5).astype(np.float16) for _ in range(L)]
    v = [(rng.standard_normal((B, Hkv, D)) * 0.5).astype(np.float16) for _ in range(L)]
    btd = dev_i32(bt)
    outs = [plan.run(l, dev_f16(q[l]), btd, k_new=dev_f16(k[l]), v_new=dev_f16(v[l])) for l in range(L)]
    torch.cuda.synchronize()
    assert pool.check() == 0
    after, _ = _compact(kv, bt, sample, lens)
    gs = oracle.Geom(L, Hkv, D, 16, before.shape[1])
    expect = np.ascontiguousarray(before)
    for l in range(L):
        assert oracle.append_paged(expect.view(np.uint16), gs, l, k[l][sample][:, None].view(np.uint16),
                                   v[l][sample][:, None].view(np.uint16), tabs, lens[sample] - 1) == 0
    assert np.array_equal(after.view(np.uint16), expect.view(np.uint16)), "fused append, sampled sequences"
    for l in range(L):
        ref = oracle.decode_paged(expect.view(np.uint16), gs, l, q[l][sample].view(np.uint16), tabs, lens[sample],
                                  nthreads=8)
        assert_close_attn(outs[l].float().cpu().numpy()[sample], ref, "70B full layer %d, sampled" % l)


def test_gather_wait_times_out_and_recovers(vk):
    """Two ranks of a gather driven from this process on one GPU.  Rank 0's end
    of step waits for rank 1's flag, which nothing raises: the bounded wait
    gives up after about 1 s, the host reads VK_TIMEOUT (once; the check
    clears it) and the device stays usable.  Rank 1's step then passes (its
    wait finds rank 0's flag already raised), and both receive buffers hold
    both ranks' outputs.  Only one kernel waits at a time, never on another
    running kernel."""
    import time
    rng = np.random.default_rng(32)
    lens = np.array([5, 300, 2049], np.int32)
    Hq, Hkv, D = 16, 2, 128
    g, bt, host, q0 = _case(rng, lens, Hq, Hkv, D, L=1)
    q1 = (rng.standard_normal(q0.shape) * 0.5).astype(np.float16)
    pool = make_pool(vk, g, host)
    bt_d = dev_i32(bt)
    B = len(lens)
    want0 = pool.plan(lens.tolist(), Hq).run(0, dev_f16(q0), bt_d).clone()
    want1 = pool.plan(lens.tolist(), Hq).run(0, dev_f16(q1), bt_d).clone()
    nbytes = B * Hq * D * 2
    g0, g1 = vk.Gather(0, 2, nbytes, slots=2), vk.Gather(1, 2, nbytes, slots=2)
    g0.import_local(1, g1)
    g1.import_local(0, g0)
    plan0 = pool.plan(lens.tolist(), Hq)
    plan0.set_gather(g0, slot_base=0, wait_prev=False)
    torch.cuda.synchronize()
    t0 = time.monotonic()
    plan0.run(0, dev_f16(q0), bt_d)
    plan0.gather_wait(0)
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    assert 0.9 < waited < 10.0, "the wait must give up after its 1 s bound (took %.2f s)" % waited
    with pytest.raises(vk.VKError) as e:
        g0.check()
    assert e.value.status == 4  # VK_TIMEOUT
    g0.check()  # cleared by the first check
    assert pool.check() == 0
    plan1 = pool.plan(lens.tolist(), Hq)
    plan1.set_gather(g1, slot_base=0, wait_prev=False)
    plan1.run(0, dev_f16(q1), bt_d)
    plan1.gather_wait(0)
    torch.cuda.synchronize()
    g1.check()
    assert pool.check() == 0
    for gat in (g0, g1):
        got = gat.view(0, B, Hq, D)
        assert torch.equal(got[0], want0) and torch.equal(got[1], want1)
    g0.close()
    g1.close()
