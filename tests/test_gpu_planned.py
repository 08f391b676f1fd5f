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
