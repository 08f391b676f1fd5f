"""GPU parity tests of K3 chunked prefill (vk_prefill): chunk appended with
vk_append, then causal attention over prefix + chunk, against the oracle's
restatement of cpu_attention rows (tests/test_attention.cu:66-97).  Tolerance
|gpu - ref| <= 2e-3 + 1e-2*|ref|."""
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


def _run(vk, rng, D, Hq, Hkv, T, pos, poison=False, L=2, layer=1, path=0):
    pos = np.array(pos, np.int32)
    B = len(pos)
    g = oracle.Geom(L, Hkv, D, 16, 0)
    bt, g.num_pages = random_layout(rng, pos + T, extra_pages=7)
    if poison:
        host = random_pool(rng, g, fill_nan=True)
        for b in range(B):
            for j in range(int(pos[b])):
                host[layer, bt[b][j // 16], :, :, j % 16, :] = (rng.standard_normal((Hkv, 2, D)) * 0.5).astype(np.float16)
    else:
        host = random_pool(rng, g)
    pool = make_pool(vk, g, host)
    pool.set_prefill_path(path)
    k = (rng.standard_normal((B, T, Hkv, D)) * 0.5).astype(np.float16)
    v = (rng.standard_normal((B, T, Hkv, D)) * 0.5).astype(np.float16)
    q = (rng.standard_normal((B, T, Hq, D)) * 0.5).astype(np.float16)
    bt_d = dev_i32(bt)
    pool.append(layer, dev_f16(k), dev_f16(v), bt_d, dev_i32(pos))
    out = pool.prefill(layer, dev_f16(q), bt_d, dev_i32(pos)).float().cpu().numpy()
    assert pool.check() == 0
    assert oracle.append_paged(host.view(np.uint16), g, layer, k.view(np.uint16), v.view(np.uint16), bt, pos) == 0
    ref = oracle.prefill_paged(host.view(np.uint16), g, layer, q.view(np.uint16), bt, pos, nthreads=8)
    return out, ref, pool, host, g, bt, q


# path 1 = mma.sync kernel, 2 = tcgen05/TMEM kernel (head_dim 128)
PATHS = [(64, 1), (128, 1), (128, 2)]


@pytest.mark.parametrize("D,path", PATHS)
@pytest.mark.parametrize("Hq,Hkv", [(4, 4), (8, 2), (8, 1)])
def test_prefill_matches_oracle(vk, D, path, Hq, Hkv):
    rng = np.random.default_rng(D + Hq + 10 * Hkv)
    out, ref, *_ = _run(vk, rng, D, Hq, Hkv, T=100, pos=[0, 7, 300], path=path)
    assert_close_attn(out, ref, "prefill D%d path%d Hq%d Hkv%d" % (D, path, Hq, Hkv))


@pytest.mark.parametrize("path", [1, 2])
@pytest.mark.parametrize("T", [1, 15, 64, 65, 127, 128, 129, 200, 300])
def test_prefill_chunk_lengths(vk, T, path):
    rng = np.random.default_rng(300 + T)
    out, ref, *_ = _run(vk, rng, 128, 4, 2, T=T, pos=[0, 33, 129], path=path)
    assert_close_attn(out, ref, "prefill T=%d path%d" % (T, path))


@pytest.mark.parametrize("path", [1, 2])
def test_prefill_poisoned_pool(vk, path):
    """Slots outside prefix + chunk hold NaN; outputs stay finite and match."""
    rng = np.random.default_rng(31)
    out, ref, *_ = _run(vk, rng, 128, 8, 2, T=70, pos=[3, 64, 90], poison=True, path=path)
    assert_close_attn(out, ref, "prefill poisoned path%d" % path)


def test_prefill_paths_agree(vk):
    """tcgen05 and mma.sync kernels agree within the attention tolerance."""
    rng = np.random.default_rng(34)
    a, ref, pool, host, g, bt, q = _run(vk, rng, 128, 8, 8, T=333, pos=[0, 700, 1500], path=1)
    pool.set_prefill_path(2)
    b = pool.prefill(1, dev_f16(q), dev_i32(bt), dev_i32([0, 700, 1500])).float().cpu().numpy()
    assert_close_attn(b, ref, "tcgen05 vs oracle")
    assert_close_attn(b, a, "tcgen05 vs mma.sync")


def test_prefill_last_row_equals_decode(vk):
    """The chunk's last query row is a decode of that token (same keys)."""
    rng = np.random.default_rng(32)
    out, ref, pool, host, g, bt, q = _run(vk, rng, 128, 8, 2, T=37, pos=[100, 0, 555])
    lens = np.array([100, 0, 555], np.int32) + 37
    dec = pool.decode(1, dev_f16(np.ascontiguousarray(q[:, -1])), dev_i32(bt), dev_i32(lens), int(lens.max()))
    assert_close_attn(dec.float().cpu().numpy(), ref[:, -1], "decode of last row")
    assert_close_attn(out[:, -1], ref[:, -1], "prefill last row")


def test_prefill_config4_sampled(vk):
    """Llama-2-7B chunked prefill shape (32/32 heads, D=128, 2048-token chunk,
    cached prefixes up to 4096), 2 sequences, rows checked on a sample."""
    rng = np.random.default_rng(4)
    D, H, T = 128, 32, 2048
    pos = np.array([1500, 3900], np.int32)
    g = oracle.Geom(1, H, D, 16, 0)
    bt, g.num_pages = random_layout(rng, pos + T)
    pool = make_pool(vk, g)
    kv = pool.kv_view()
    kv.copy_((torch.randn(kv.shape, device="cuda", generator=torch.Generator("cuda").manual_seed(3)) * 0.5).half())
    q = (rng.standard_normal((2, T, H, D)) * 0.5).astype(np.float16)
    out = pool.prefill(0, dev_f16(q), dev_i32(bt), dev_i32(pos)).float().cpu().numpy()
    assert pool.check() == 0
    host = kv.cpu().numpy()
    # each sampled chunk row r is a one-row prefill at position pos + r
    for r in [0, 1, 63, 64, 1000, 2047]:
        ref_r = oracle.prefill_paged(host.view(np.uint16), g, 0, np.ascontiguousarray(q[:, r:r + 1]).view(np.uint16),
                                     bt, pos + r, nthreads=8)
        assert_close_attn(out[:, r:r + 1], ref_r, "config4 row %d" % r)


def test_prefill_rejects_bad_table(vk):
    rng = np.random.default_rng(33)
    g = oracle.Geom(1, 1, 128, 16, 4)
    pool = make_pool(vk, g, random_pool(rng, g))
    q = torch.zeros(1, 40, 1, 128, dtype=torch.float16, device="cuda")
    pool.prefill(0, q, dev_i32([[0, 1]]), dev_i32([0]))  # 40 tokens need 3 pages
    assert pool.error_bits() & 0x2
