"""GPU parity tests of K1 append and K2 paged decode through the C ABI, against
the CPU oracle and the golden fixtures generated from the reference's own
cpu_attention.  Tolerance (fp16 output, fp32 accumulation):
|gpu - ref| <= 2e-3 + 1e-2*|ref|; append and tables are bit-exact."""
import os

import numpy as np
import pytest
import torch

import oracle
from tests.golden import gen
from tests.helpers import (assert_close_attn, dev_f16, dev_i32, make_pool, random_layout,
                           random_pool)

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def vk(cuda_ok):
    import vulcan_b200
    vulcan_b200.load()
    return vulcan_b200


def run_decode(vk, pool, layer, q, bt, lens, max_len=None, pps=0):
    pool.set_split(pps)
    out = pool.decode(layer, dev_f16(q), dev_i32(bt), dev_i32(lens),
                      int(max_len if max_len is not None else max(1, max(lens))))
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


# ---------------------------------------------------------------- append

@pytest.mark.parametrize("T", [1, 3, 40])
def test_append_bit_exact(vk, T):
    rng = np.random.default_rng(10 + T)
    g = oracle.Geom(3, 4, 128, 16, 0)
    B = 6
    pos = rng.integers(0, 200, B).astype(np.int32)
    bt, g.num_pages = random_layout(rng, pos + T)
    host = random_pool(rng, g)
    pool = make_pool(vk, g, host)
    k = (rng.standard_normal((B, T, g.Hkv, g.D)) * 0.5).astype(np.float16)
    v = (rng.standard_normal((B, T, g.Hkv, g.D)) * 0.5).astype(np.float16)
    pool.append(1, dev_f16(k), dev_f16(v), dev_i32(bt), dev_i32(pos))
    assert pool.check() == 0
    expect = host.copy()
    assert oracle.append_paged(expect.view(np.uint16), g, 1, k.view(np.uint16), v.view(np.uint16), bt, pos) == 0
    got = pool.kv_view().cpu().numpy()
    assert np.array_equal(got.view(np.uint16), expect.view(np.uint16))


def test_append_f32_rounds_to_nearest_even(vk):
    rng = np.random.default_rng(5)
    g = oracle.Geom(1, 2, 64, 16, 4)
    pool = make_pool(vk, g)
    bt = np.array([[2, 0]], np.int32)
    x = rng.standard_normal((1, 20, 2, 64)).astype(np.float32) * 3
    x[0, 0, 0, :4] = [65504.0, 1e-8, -0.0, 2049.0]  # max, underflow, signed zero, tie
    pool.append(0, torch.from_numpy(x).cuda(), torch.from_numpy(-x).cuda(), dev_i32(bt), dev_i32([0]))
    assert pool.check() == 0
    kv = pool.kv_view().cpu().numpy()
    ref = x.astype(np.float16)
    for t in range(20):
        page, slot = bt[0][t // 16], t % 16
        assert np.array_equal(kv[0, page, :, 0, slot].view(np.uint16), ref[0, t].view(np.uint16))
        assert np.array_equal(kv[0, page, :, 1, slot].view(np.uint16), (-x[0, t]).astype(np.float16).view(np.uint16))


def test_append_rejects_bad_entries(vk):
    g = oracle.Geom(1, 1, 128, 16, 4)
    pool = make_pool(vk, g)
    k = torch.ones(2, 1, 1, 128, dtype=torch.float16, device="cuda")
    bt = dev_i32([[7, 1], [1, 2]])           # seq 0: page id 7 outside the pool
    pool.append(0, k, k, bt, dev_i32([0, 40]))  # seq 1: position 40 beyond 2 pages
    bits = pool.error_bits()
    assert bits & 0x1 and bits & 0x2
    assert pool.kv_view().abs().sum().item() == 0  # nothing written


# ---------------------------------------------------------------- decode vs fixtures

def test_decode_matches_reference_fixtures(vk):
    f = np.load(os.path.join(GOLD, "paged_decode_cases.npz"))
    for ci in range(len(gen.PAGED_CASES)):
        pre = "case%d/" % ci
        L, Hkv, D, P, NP, layer = (int(x) for x in f[pre + "geom"])
        g = oracle.Geom(L, Hkv, D, P, NP)
        pool = make_pool(vk, g, f[pre + "pool"].view(np.float16))
        for pps in (0, 1):  # auto split and one page per split (merge path)
            out = run_decode(vk, pool, layer, f[pre + "q"].view(np.float16), f[pre + "bt"], f[pre + "lens"], pps=pps)
            assert_close_attn(out, f[pre + "out"], "case %d pps %d" % (ci, pps))
        assert pool.check() == 0
        pool.close()


def test_decode_config1_append_then_attend(vk):
    """Llama-2-7B single-layer decode: append 1 token at position 512 into a
    64-page permuted table, then attend 513 keys; reference output fixture."""
    c = gen.config1_case()
    f = np.load(os.path.join(GOLD, "config1_decode.npz"))
    assert gen.digest(c) == bytes(f["sha256"]).decode()
    pool = make_pool(vk, c["geom"], c["pool_before"])
    bt = dev_i32(c["bt"])
    pool.append(0, dev_f16(c["k_new"]), dev_f16(c["v_new"]), bt, dev_i32(c["positions"]))
    got_pool = pool.kv_view().cpu().numpy()
    assert np.array_equal(got_pool.view(np.uint16), c["pool"].view(np.uint16))
    out = pool.decode(0, dev_f16(c["q"]), bt, dev_i32(c["lens"]), 513).float().cpu().numpy()
    assert_close_attn(out, f["out"], "config1")
    assert pool.check() == 0


# ---------------------------------------------------------------- decode vs oracle

@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("Hq,Hkv", [(4, 4), (8, 4), (8, 2), (8, 1), (16, 1), (12, 4)])
def test_decode_random_shapes(vk, D, Hq, Hkv):
    rng = np.random.default_rng(D * 100 + Hq * 10 + Hkv)
    lens = np.array([1, 15, 16, 17, 100, 513, 1200], np.int32)
    g = oracle.Geom(2, Hkv, D, 16, 0)
    bt, g.num_pages = random_layout(rng, lens)
    host = random_pool(rng, g)
    pool = make_pool(vk, g, host)
    q = (rng.standard_normal((len(lens), Hq, D)) * 0.5).astype(np.float16)
    ref = oracle.decode_paged(host.view(np.uint16), g, 1, q.view(np.uint16), bt, lens)
    for pps in (0, 2, 8):
        out = run_decode(vk, pool, 1, q, bt, lens, pps=pps)
        assert_close_attn(out, ref, "D%d Hq%d Hkv%d pps%d" % (D, Hq, Hkv, pps))
    assert pool.check() == 0


def test_decode_ignores_poisoned_slots(vk):
    """Every slot the sequences do not own holds NaN; outputs stay finite and match."""
    rng = np.random.default_rng(77)
    lens = np.array([3, 16, 33, 250], np.int32)
    g = oracle.Geom(1, 2, 128, 16, 0)
    bt, g.num_pages = random_layout(rng, lens)
    host = random_pool(rng, g, fill_nan=True)
    for b, n in enumerate(lens):
        for j in range(n):
            host[0, bt[b][j // 16], :, :, j % 16, :] = (rng.standard_normal((2, 2, 128)) * 0.5).astype(np.float16)
    pool = make_pool(vk, g, host)
    q = (rng.standard_normal((4, 8, 128)) * 0.5).astype(np.float16)
    ref = oracle.decode_paged(host.view(np.uint16), g, 0, q.view(np.uint16), bt, lens)
    for pps in (0, 1):
        out = run_decode(vk, pool, 0, q, bt, lens, pps=pps)
        assert_close_attn(out, ref, "poisoned pps%d" % pps)


def test_decode_single_key_returns_v0(vk):
    """CausalMask_FirstRow on the paged path: one key -> output == V[0] exactly."""
    rng = np.random.default_rng(9)
    g = oracle.Geom(1, 2, 128, 16, 3)
    host = random_pool(rng, g)
    pool = make_pool(vk, g, host)
    q = (rng.standard_normal((1, 8, 128)) * 3).astype(np.float16)
    out = run_decode(vk, pool, 0, q, np.array([[2]], np.int32), np.array([1], np.int32))
    v0 = host[0, 2, :, 1, 0].astype(np.float32)  # [Hkv, D]
    assert np.array_equal(out[0], np.repeat(v0, 4, axis=0))


def test_decode_convex_bound(vk):
    """OutputSumMatchesV: every output lies within [min V, max V] of its head."""
    rng = np.random.default_rng(11)
    lens = np.array([40, 300], np.int32)
    g = oracle.Geom(1, 1, 128, 16, 0)
    bt, g.num_pages = random_layout(rng, lens)
    host = random_pool(rng, g)
    pool = make_pool(vk, g, host)
    q = (rng.standard_normal((2, 8, 128))).astype(np.float16)
    out = run_decode(vk, pool, 0, q, bt, lens, pps=1)
    for b, n in enumerate(lens):
        vs = np.stack([host[0, bt[b][j // 16], 0, 1, j % 16] for j in range(n)]).astype(np.float32)
        assert out[b].min() >= vs.min() - 1e-3 and out[b].max() <= vs.max() + 1e-3


def test_decode_zero_and_bad_lengths(vk):
    rng = np.random.default_rng(12)
    g = oracle.Geom(1, 1, 128, 16, 4)
    pool = make_pool(vk, g, random_pool(rng, g))
    q = (rng.standard_normal((3, 2, 128))).astype(np.float16)
    bt = np.array([[0, 1], [2, 3], [1, 0]], np.int32)
    out = run_decode(vk, pool, 0, q, bt, np.array([0, 5, 33], np.int32), max_len=32)
    assert np.all(out[0] == 0)           # nothing to attend
    assert np.all(out[2] == 0)           # 33 > 2 pages: rejected
    assert pool.error_bits() & 0x4
    bt[1, 0] = 99                         # bad page id: recorded, access stays inside the pool
    run_decode(vk, pool, 0, q, bt, np.array([1, 5, 1], np.int32), max_len=32)
    assert pool.error_bits() & 0x1


def test_decode_page_permutation_invariance(vk):
    """Moving a sequence's pages to other physical ids changes nothing."""
    rng = np.random.default_rng(13)
    lens = np.array([700, 33], np.int32)
    g = oracle.Geom(1, 2, 128, 16, 0)
    bt, g.num_pages = random_layout(rng, lens, extra_pages=60)
    host = random_pool(rng, g)
    perm = rng.permutation(g.num_pages)
    host2 = np.empty_like(host)
    host2[:, perm] = host
    bt2 = np.where(bt >= 0, perm[np.maximum(bt, 0)], -1).astype(np.int32)
    q = (rng.standard_normal((2, 8, 128)) * 0.5).astype(np.float16)
    p1, p2 = make_pool(vk, g, host), make_pool(vk, g, host2)
    a = run_decode(vk, p1, 0, q, bt, lens)
    b = run_decode(vk, p2, 0, q, bt2, lens)
    assert np.array_equal(a, b)


def test_decode_70b_layer_sampled(vk):
    """One full layer of the Llama-2-70B GQA decode shape (B=64, 64/8 heads,
    lognormal contexts median 2048 clipped to [256, 8192]) checked on sampled
    sequences against the oracle."""
    rng = np.random.default_rng(70)
    B, Hq, Hkv, D = 64, 64, 8, 128
    lens = np.clip(np.round(np.exp(rng.normal(np.log(2048), 0.6, B))), 256, 8192).astype(np.int32) + 1
    g = oracle.Geom(1, Hkv, D, 16, 0)
    bt, g.num_pages = random_layout(rng, lens)
    pool = make_pool(vk, g)
    kv = pool.kv_view()
    kv.copy_((torch.randn(kv.shape, device="cuda", generator=torch.Generator("cuda").manual_seed(1)) * 0.5).half())
    q = (rng.standard_normal((B, Hq, D)) * 0.5).astype(np.float16)
    out = run_decode(vk, pool, 0, q, bt, lens, max_len=int(lens.max()))
    assert pool.check() == 0
    host = kv.cpu().numpy()
    sample = [int(np.argmax(lens)), int(np.argmin(lens)), 7, 31]
    ref = oracle.decode_paged(host.view(np.uint16), g, 0, q[sample].view(np.uint16), bt[sample], lens[sample],
                              nthreads=8)
    assert_close_attn(out[sample], ref, "70B sampled")
