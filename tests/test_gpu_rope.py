"""GPU parity tests of the fused RoPE (vk_set_rope) against the oracle's
restatement of the reference's cpu_rope (pinned bit-exact to the reference in
test_oracle.py).

Expected values apply the oracle RoPE in fp32 to the fp16 (or fp32) inputs and
round to fp16, as the kernels do.  Appended K rows may differ from that by one
fp16 ulp, or 1e-6 near zero (CUDA's sin/cos against the host's); V rows are
bit-exact; attention
outputs are held to the usual tolerance."""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_close_attn, dev_f16, dev_i32, make_pool, random_layout, random_pool

pytestmark = pytest.mark.gpu
THETA = 10000.0


@pytest.fixture(scope="module")
def vk(cuda_ok):
    import vulcan_b200
    vulcan_b200.load()
    return vulcan_b200


def rot16(x16, positions):
    """fp16 in, RoPE in fp32 at positions (one per leading index), fp16 out."""
    return oracle.rope(x16.astype(np.float32), positions, THETA).astype(np.float16)


def assert_ulp(got16, want16, what):
    """Within one fp16 ulp, or 1e-6 absolute for values near zero (where the
    sin/cos difference of ~1e-7 * |x| spans several subnormal ulps)."""
    a = got16.view(np.int16).astype(np.int32)
    b = want16.view(np.int16).astype(np.int32)
    d = np.abs(a - b)
    near = np.abs(got16.astype(np.float32) - want16.astype(np.float32)) <= 1e-6
    bad = (d > 1) & ~near
    assert not bad.any(), "%s: %d values differ by more than 1 ulp" % (what, int(bad.sum()))


def test_append_rope_f16_and_f32(vk):
    rng = np.random.default_rng(71)
    B, T, Hkv, D, L = 3, 37, 2, 128, 2
    pos = np.array([0, 5, 4000], np.int32)
    lens = pos + T
    g = oracle.Geom(L, Hkv, D, 16, 0)
    bt, g.num_pages = random_layout(rng, lens)
    host = random_pool(rng, g)
    for f32 in (False, True):
        pool = make_pool(vk, g, host)
        pool.set_rope(THETA)
        k = (rng.standard_normal((B, T, Hkv, D)) * 0.5).astype(np.float32 if f32 else np.float16)
        v = (rng.standard_normal((B, T, Hkv, D)) * 0.5).astype(np.float32 if f32 else np.float16)
        kd = torch.from_numpy(k).cuda()
        vd = torch.from_numpy(v).cuda()
        pool.append(1, kd, vd, dev_i32(bt), dev_i32(pos))  # fp32 inputs take vk_append_f32
        torch.cuda.synchronize()
        assert pool.check() == 0
        # expected: K rotated at each token's position, V as given
        tok_pos = (pos[:, None] + np.arange(T)[None, :]).astype(np.int32)  # [B, T]
        krot = np.empty((B, T, Hkv, D), np.float16)
        for b in range(B):
            for t in range(T):
                krot[b, t] = oracle.rope(k[b, t].astype(np.float32), [tok_pos[b, t]] * Hkv, THETA).astype(np.float16)
        expect = host.copy()
        assert oracle.append_paged(expect.view(np.uint16), g, 1, krot.view(np.uint16),
                                   v.astype(np.float16).view(np.uint16), bt, pos) == 0
        got = pool.kv_view().cpu().numpy()
        assert np.array_equal(got[:, :, :, 1], expect[:, :, :, 1]), "V rows"
        assert_ulp(got[:, :, :, 0], expect[:, :, :, 0], "K rows (f32 input)" if f32 else "K rows")


@pytest.mark.parametrize("path", ["planned", "split"])
def test_decode_rope(vk, path):
    rng = np.random.default_rng(72 if path == "planned" else 73)
    Hq, Hkv, D, L = 16, 2, 128, 2
    lens = np.array([1, 17, 300, 2049, 8000], np.int32)
    g = oracle.Geom(L, Hkv, D, 16, 0)
    bt, g.num_pages = random_layout(rng, lens)
    host = random_pool(rng, g)
    pool = make_pool(vk, g, host)
    pool.set_rope(THETA)
    B = len(lens)
    q = (rng.standard_normal((B, Hq, D)) * 0.5).astype(np.float16)
    kn = (rng.standard_normal((B, Hkv, D)) * 0.5).astype(np.float16)
    vn = (rng.standard_normal((B, Hkv, D)) * 0.5).astype(np.float16)
    if path == "planned":
        out = pool.plan(lens.tolist(), Hq).run(1, dev_f16(q), dev_i32(bt), k_new=dev_f16(kn), v_new=dev_f16(vn))
    else:
        pool.append(1, dev_f16(kn[:, None]), dev_f16(vn[:, None]), dev_i32(bt), dev_i32(lens - 1))
        out = pool.decode(1, dev_f16(q), dev_i32(bt), dev_i32(lens), int(lens.max()))
    torch.cuda.synchronize()
    assert pool.check() == 0
    newpos = lens - 1
    krot = np.stack([rot16(kn[b], [newpos[b]] * Hkv) for b in range(B)])
    qrot = np.stack([rot16(q[b], [newpos[b]] * Hq) for b in range(B)])
    expect = host.copy()
    assert oracle.append_paged(expect.view(np.uint16), g, 1, krot[:, None].view(np.uint16),
                               vn[:, None].view(np.uint16), bt, newpos) == 0
    got_pool = pool.kv_view().cpu().numpy()
    assert_ulp(got_pool, expect, "pool after the fused append")
    ref = oracle.decode_paged(got_pool.view(np.uint16), g, 1, qrot.view(np.uint16), bt, lens)
    assert_close_attn(out.float().cpu().numpy(), ref, "%s decode with RoPE" % path)


@pytest.mark.parametrize("prefill_path", [1, 2])
def test_prefill_rope(vk, prefill_path):
    rng = np.random.default_rng(74 + prefill_path)
    Hq, Hkv, D, L, T = 8, 2, 128, 1, 130
    pos = np.array([0, 900], np.int32)
    lens = pos + T
    g = oracle.Geom(L, Hkv, D, 16, 0)
    bt, g.num_pages = random_layout(rng, lens)
    host = random_pool(rng, g)
    pool = make_pool(vk, g, host)
    pool.set_rope(THETA)
    pool.set_prefill_path(prefill_path)
    B = len(pos)
    q = (rng.standard_normal((B, T, Hq, D)) * 0.5).astype(np.float16)
    out = pool.prefill(0, dev_f16(q), dev_i32(bt), dev_i32(pos))
    torch.cuda.synchronize()
    assert pool.check() == 0
    qrot = np.stack([np.stack([rot16(q[b, t], [pos[b] + t] * Hq) for t in range(T)]) for b in range(B)])
    ref = oracle.prefill_paged(host.view(np.uint16), g, 0, qrot.view(np.uint16), bt, pos)
    assert_close_attn(out.float().cpu().numpy(), ref, "prefill path %d with RoPE" % prefill_path)


def test_rope_off_by_default_and_bad_base(vk):
    rng = np.random.default_rng(76)
    g = oracle.Geom(1, 1, 64, 16, 4)
    pool = make_pool(vk, g, random_pool(rng, g))
    with pytest.raises(vk.VKError):
        pool.set_rope(-1.0)
    with pytest.raises(vk.VKError):
        pool.set_rope(1.0)
    pool.set_rope(0.0)
