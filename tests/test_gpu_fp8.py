"""GPU parity tests of FP8 (e4m3 + per-row fp32 scale) KV pages against the
oracle's restatement (oracle/vk_oracle.c: or_append_fp8, or_dequant_fp8).

Append, fused append and page copy are bit-exact against the oracle on the
whole byte image of the pool (unwritten slots hold random bytes on both
sides).  Decode outputs are compared with the oracle's float64 attention over
the dequantised cache under the fp16 attention tolerance; prefill outputs
likewise (oracle.prefill_fp8)."""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import assert_close_attn, dev_f16, dev_i32, random_layout

pytestmark = pytest.mark.gpu
THETA = 10000.0


@pytest.fixture(scope="module")
def vk(cuda_ok):
    import vulcan_b200
    vulcan_b200.load()
    return vulcan_b200


def fp8_pool(vk, g, rng):
    """An FP8 pool whose bytes start random, and the same bytes on the host."""
    pool = vk.PagedKVPool(g.L, g.Hkv, g.D, g.num_pages, kv_format="fp8")
    host = rng.integers(0, 256, size=(g.L, g.num_pages, g.Hkv, pool.block_bytes), dtype=np.uint8)
    pool.block_view().copy_(torch.from_numpy(host))
    return pool, host


def rows(rng, *shape, f32=False):
    x = rng.standard_normal(shape).astype(np.float32) * 0.5
    return x if f32 else x.astype(np.float16)


def assert_bytes(pool, host, what):
    got = pool.block_view().cpu().numpy()
    bad = got != host
    assert not bad.any(), "%s: %d bytes differ (first at %s)" % (what, int(bad.sum()), np.argwhere(bad)[0])


@pytest.mark.parametrize("f32", [False, True])
def test_fp8_append_bit_exact(vk, f32):
    rng = np.random.default_rng(81 + f32)
    B, T, Hkv, D, L = 3, 37, 2, 128, 2
    pos = np.array([0, 5, 4000], np.int32)
    g = oracle.Geom(L, Hkv, D, 16, 0)
    bt, g.num_pages = random_layout(rng, pos + T)
    pool, host = fp8_pool(vk, g, rng)
    k, v = rows(rng, B, T, Hkv, D, f32=f32), rows(rng, B, T, Hkv, D, f32=f32)
    k[0, 3, 1] = 0  # an all-zero row: scale 0, codes 0
    k[1, 0, 0, 7] = 60.0  # one large element: the others quantise coarsely
    pool.append(1, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), dev_i32(bt), dev_i32(pos))
    torch.cuda.synchronize()
    assert pool.check() == 0
    assert oracle.append_fp8(host, g, 1, k, v, bt, pos) == 0
    assert_bytes(pool, host, "FP8 append (%s inputs)" % ("fp32" if f32 else "fp16"))


def fill_history(vk, pool, host, g, rng, layer, bt, lens, rope=False):
    """Appends tokens 0 .. len-2 of every sequence (GPU and oracle)."""
    for b, n in enumerate(lens):
        if n <= 1:
            continue
        k, v = rows(rng, 1, n - 1, g.Hkv, g.D), rows(rng, 1, n - 1, g.Hkv, g.D)
        pool.append(layer, dev_f16(k), dev_f16(v), dev_i32(bt[b:b + 1]), dev_i32([0]))
        kk = k.astype(np.float32)
        if rope:
            kk = np.stack([oracle.rope(kk[0, t], [t] * g.Hkv, THETA) for t in range(n - 1)])[None]
        assert oracle.append_fp8(host, g, layer, kk, v, bt[b:b + 1], np.array([0], np.int32)) == 0


@pytest.mark.parametrize("G", [8, 16])
def test_fp8_planned_decode_fused_append(vk, G):
    rng = np.random.default_rng(83 + G)
    Hkv, D, L, layer = 2, 128, 2, 1
    Hq = G * Hkv
    lens = np.array([1, 15, 16, 17, 300, 2049, 8000], np.int32)
    g = oracle.Geom(L, Hkv, D, 16, 0)
    bt, g.num_pages = random_layout(rng, lens)
    pool, host = fp8_pool(vk, g, rng)
    fill_history(vk, pool, host, g, rng, layer, bt, lens)
    torch.cuda.synchronize()
    assert pool.check() == 0
    assert_bytes(pool, host, "FP8 history append")
    B = len(lens)
    q = rows(rng, B, Hq, D)
    kn, vn = rows(rng, B, Hkv, D), rows(rng, B, Hkv, D)
    out = pool.plan(lens.tolist(), Hq).run(layer, dev_f16(q), dev_i32(bt), k_new=dev_f16(kn), v_new=dev_f16(vn))
    torch.cuda.synchronize()
    assert pool.check() == 0
    assert oracle.append_fp8(host, g, layer, kn[:, None], vn[:, None], bt, lens - 1) == 0
    assert_bytes(pool, host, "FP8 pool after the fused append")
    ref = oracle.decode_fp8(host, g, layer, q, bt, lens)
    assert_close_attn(out.float().cpu().numpy(), ref, "FP8 planned decode G=%d" % G)


def test_fp8_decode_small_v_rows(vk):
    """V rows of very different magnitudes (1e-4 .. 10) in one page: the per-page
    power-of-two normalisation of the V scales keeps fp16 P in range."""
    rng = np.random.default_rng(88)
    Hkv, D, L, layer, G = 1, 128, 1, 0, 8
    lens = np.array([16, 40, 333], np.int32)
    g = oracle.Geom(L, Hkv, D, 16, 0)
    bt, g.num_pages = random_layout(rng, lens)
    pool, host = fp8_pool(vk, g, rng)
    for b, n in enumerate(lens):
        k = rows(rng, 1, n, Hkv, D, f32=True)
        v = rows(rng, 1, n, Hkv, D, f32=True) * (10.0 ** rng.uniform(-4, 1, size=(1, n, 1, 1))).astype(np.float32)
        pool.append(layer, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), dev_i32(bt[b:b + 1]),
                    dev_i32([0]))
        assert oracle.append_fp8(host, g, layer, k, v, bt[b:b + 1], np.array([0], np.int32)) == 0
    q = rows(rng, len(lens), G * Hkv, D)
    out = pool.plan(lens.tolist(), G * Hkv).run(layer, dev_f16(q), dev_i32(bt))
    torch.cuda.synchronize()
    assert pool.check() == 0
    assert_bytes(pool, host, "FP8 append of scaled rows")
    ref = oracle.decode_fp8(host, g, layer, q, bt, lens)
    assert_close_attn(out.float().cpu().numpy(), ref, "FP8 decode, V rows over 5 decades")


def test_fp8_decode_rope(vk):
    rng = np.random.default_rng(85)
    Hkv, D, L, layer, G = 2, 128, 1, 0, 8
    Hq = G * Hkv
    lens = np.array([3, 40, 1000], np.int32)
    g = oracle.Geom(L, Hkv, D, 16, 0)
    bt, g.num_pages = random_layout(rng, lens)
    pool, host = fp8_pool(vk, g, rng)
    pool.set_rope(THETA)
    fill_history(vk, pool, host, g, rng, layer, bt, lens, rope=True)
    B = len(lens)
    q = rows(rng, B, Hq, D)
    kn, vn = rows(rng, B, Hkv, D), rows(rng, B, Hkv, D)
    out = pool.plan(lens.tolist(), Hq).run(layer, dev_f16(q), dev_i32(bt), k_new=dev_f16(kn), v_new=dev_f16(vn))
    torch.cuda.synchronize()
    assert pool.check() == 0
    newpos = lens - 1
    krot = np.stack([oracle.rope(kn[b].astype(np.float32), [newpos[b]] * Hkv, THETA) for b in range(B)])
    qrot = np.stack([oracle.rope(q[b].astype(np.float32), [newpos[b]] * Hq, THETA) for b in range(B)])
    assert oracle.append_fp8(host, g, layer, krot[:, None], vn[:, None], bt, newpos) == 0
    # K codes may differ by one step where the device's sin/cos differ from the
    # host's by an ulp; the attention output is held to the usual tolerance
    got = pool.block_view().cpu().numpy()
    ref = oracle.decode_fp8(host, g, layer, qrot.astype(np.float16), bt, lens)
    assert_close_attn(out.float().cpu().numpy(), ref, "FP8 planned decode with RoPE")
    dg = oracle.dequant_fp8(got, g)
    dh = oracle.dequant_fp8(host, g)
    for b, n in enumerate(lens):
        pages = bt[b, :(n + 15) // 16]
        a = dg[layer, pages].transpose(1, 2, 0, 3, 4).reshape(Hkv, 2, -1, D)[:, :, :n]
        h = dh[layer, pages].transpose(1, 2, 0, 3, 4).reshape(Hkv, 2, -1, D)[:, :, :n]
        assert np.array_equal(a[:, 1], h[:, 1]), "V rows"
        step = np.abs(h[:, 0]).max(axis=-1, keepdims=True) * (32.0 / 448.0)  # largest e4m3 step (416 -> 448)
        assert (np.abs(a[:, 0] - h[:, 0]) <= 1.01 * step + 1e-6).all(), "K rows with RoPE"


@pytest.mark.parametrize("pps", [0, 2])
def test_fp8_split_decode(vk, pps):
    """The split-grid decode (callers without host lengths) on FP8 pages, one
    split per sequence or two pages per split with the merge kernel."""
    rng = np.random.default_rng(93 + pps)
    Hkv, D, L, layer, G = 2, 128, 2, 0, 8
    Hq = G * Hkv
    lens = np.array([1, 16, 33, 700], np.int32)
    g = oracle.Geom(L, Hkv, D, 16, 0)
    bt, g.num_pages = random_layout(rng, lens)
    pool, host = fp8_pool(vk, g, rng)
    fill_history(vk, pool, host, g, rng, layer, bt, lens + 1)  # tokens 0 .. len-1
    pool.set_split(pps)
    q = rows(rng, len(lens), Hq, D)
    out = pool.decode(layer, dev_f16(q), dev_i32(bt), dev_i32(lens), int(lens.max()))
    torch.cuda.synchronize()
    assert pool.check() == 0
    assert_bytes(pool, host, "FP8 history append")
    ref = oracle.decode_fp8(host, g, layer, q, bt, lens)
    assert_close_attn(out.float().cpu().numpy(), ref, "FP8 split decode, pages per split %d" % pps)


@pytest.mark.parametrize("path", [1, 2])
@pytest.mark.parametrize("rope", [False, True])
def test_fp8_prefill(vk, rope, path):
    """Chunked prefill over FP8 pages, on the mma.sync kernel (path 1) and on the
    tcgen05 kernel with converter warps (path 2, the default): the chunk's rows
    are appended (quantised) first, then each chunk row attends the cached
    prefix and the chunk up to itself.  Several key tiles, a partial last page,
    two row tiles per CTA and a ragged last one."""
    rng = np.random.default_rng(89 + rope + 10 * path)
    Hq, Hkv, D, L, layer, T = 8, 2, 128, 2, 1, 300
    pos = np.array([0, 900, 37], np.int32)
    g = oracle.Geom(L, Hkv, D, 16, 0)
    bt, g.num_pages = random_layout(rng, pos + T)
    pool, host = fp8_pool(vk, g, rng)
    if rope:
        pool.set_rope(THETA)
    B = len(pos)
    fill_history(vk, pool, host, g, rng, layer, bt, pos + 1, rope=rope)  # prefix tokens 0 .. pos-1
    kc, vc = rows(rng, B, T, Hkv, D), rows(rng, B, T, Hkv, D)
    pool.append(layer, dev_f16(kc), dev_f16(vc), dev_i32(bt), dev_i32(pos))
    kk = kc.astype(np.float32)
    if rope:
        kk = np.stack([np.stack([oracle.rope(kk[b, t], [pos[b] + t] * Hkv, THETA) for t in range(T)])
                       for b in range(B)])
    assert oracle.append_fp8(host, g, layer, kk, vc, bt, pos) == 0
    q = rows(rng, B, T, Hq, D)
    pool.set_prefill_path(path)
    out = pool.prefill(layer, dev_f16(q), dev_i32(bt), dev_i32(pos))
    torch.cuda.synchronize()
    assert pool.check() == 0
    if rope:  # K codes may differ from the host's by one step (sin/cos ulps): compare against the device pool
        host = pool.block_view().cpu().numpy()
        q = np.stack([np.stack([oracle.rope(q[b, t].astype(np.float32), [pos[b] + t] * Hq, THETA)
                                for t in range(T)]) for b in range(B)]).astype(np.float16)
    else:
        assert_bytes(pool, host, "FP8 chunk append")
    ref = oracle.prefill_fp8(host, g, layer, q, bt, pos)
    assert_close_attn(out.float().cpu().numpy(), ref, "FP8 prefill path %d%s" % (path, " with RoPE" if rope else ""))


def test_fp8_prefill_paths_agree_on_stale_pages(vk):
    """The FP8 tcgen05 prefill against the mma.sync one on a pool whose unwritten
    slots hold random bytes (NaN codes included): keys past the written length
    must not reach the output on either path."""
    rng = np.random.default_rng(97)
    Hq, Hkv, D, L, layer, T = 16, 2, 128, 1, 0, 200
    pos = np.array([5, 250], np.int32)
    g = oracle.Geom(L, Hkv, D, 16, 0)
    bt, g.num_pages = random_layout(rng, pos + T + 40)
    pool, host = fp8_pool(vk, g, rng)
    fill_history(vk, pool, host, g, rng, layer, bt, pos + 1)
    pool.append(layer, dev_f16(rows(rng, 2, T, Hkv, D)), dev_f16(rows(rng, 2, T, Hkv, D)), dev_i32(bt), dev_i32(pos))
    q = dev_f16(rows(rng, 2, T, Hq, D))
    outs = []
    for path in (1, 2):
        pool.set_prefill_path(path)
        outs.append(pool.prefill(layer, q, dev_i32(bt), dev_i32(pos)).float().cpu().numpy())
    torch.cuda.synchronize()
    assert pool.check() == 0
    assert_close_attn(outs[1], outs[0], "FP8 prefill tcgen05 vs mma.sync")


def test_fp8_copy_and_swap(vk):
    rng = np.random.default_rng(86)
    g = oracle.Geom(3, 2, 128, 16, 12)
    pool, host = fp8_pool(vk, g, rng)
    src, dst = np.array([1, 4, 7], np.int32), np.array([9, 2, 11], np.int32)
    pool.copy_pages(dev_i32(src), dev_i32(dst))
    torch.cuda.synchronize()
    seg = g.Hkv * pool.block_bytes
    oracle.copy_pages(host.reshape(-1), g.L, seg, seg * g.num_pages, g.num_pages, src, dst)
    assert_bytes(pool, host, "FP8 page copy")
    ids = pool.alloc(4)
    pinned = torch.empty(4 * pool.page_bytes, dtype=torch.uint8).pin_memory()
    before = pool.block_view().cpu().numpy().copy()
    pool.swap_out(ids, pinned)
    pool.block_view().zero_()
    pool.swap_in_to(pinned, ids)
    torch.cuda.synchronize()
    after = pool.block_view().cpu().numpy()
    assert np.array_equal(after[:, ids], before[:, ids]), "FP8 swap round trip"


def test_fp8_unsupported_entry_points(vk):
    rng = np.random.default_rng(87)
    g = oracle.Geom(1, 1, 128, 16, 4)
    pool, _ = fp8_pool(vk, g, rng)
    with pytest.raises(RuntimeError):
        pool.kv_view()
    with pytest.raises(vk.VKError):
        vk.PagedKVPool(1, 1, 64, 4, kv_format="fp8")


def test_fp8_last_piece_merge(vk):
    """FP8 pages on the long-worker-range path of the planned decode (>= 64
    pages per worker): units of 2..8 pieces merged by their last piece next to
    a unit of more than 8 pieces merged by tasks; fused append bit-exact;
    repeated runs bit-identical."""
    rng = np.random.default_rng(860)
    Hkv, D, L, layer, G = 2, 128, 1, 0, 8
    Hq = G * Hkv
    lens = np.array([16000, 4000, 1600, 2600, 300, 17, 1, 6000], np.int32)
    g = oracle.Geom(L, Hkv, D, 16, 0)
    bt, g.num_pages = random_layout(rng, lens)
    pool, host = fp8_pool(vk, g, rng)
    fill_history(vk, pool, host, g, rng, layer, bt, lens)
    pool.set_plan_workers(16 * Hkv)
    plan = pool.plan(lens.tolist(), Hq)
    pool.set_plan_workers(0)
    assert plan.info(3) // plan.workers >= 64 and plan.info(5) == 8
    assert plan.info(6) >= 3 and plan.info(7) >= 1 and plan.info(8) > 8
    B = len(lens)
    q = rows(rng, B, Hq, D)
    kn, vn = rows(rng, B, Hkv, D), rows(rng, B, Hkv, D)
    qd, btd = dev_f16(q), dev_i32(bt)
    out = plan.run(layer, qd, btd, k_new=dev_f16(kn), v_new=dev_f16(vn))
    again = [plan.run(layer, qd, btd).clone() for _ in range(2)]
    torch.cuda.synchronize()
    assert pool.check() == 0
    assert torch.equal(again[0], again[1])
    assert oracle.append_fp8(host, g, layer, kn[:, None], vn[:, None], bt, lens - 1) == 0
    assert_bytes(pool, host, "FP8 fused append (last-piece merge plan)")
    ref = oracle.decode_fp8(host, g, layer, q, bt, lens)
    assert_close_attn(out.float().cpu().numpy(), ref, "FP8 last-piece merge")
    assert_close_attn(again[0].float().cpu().numpy(), ref, "FP8 last-piece merge, rerun")


def test_fp8_70b_full_layer_fused_append(vk):
    """A full Llama-2-70B GQA layer on FP8 pages (B=64, 64/8 heads, lognormal
    contexts median 2048 clipped to [256, 8192]), default workers, history
    written by the quantising append, new token by the fused append; sampled sequences (longest, shortest, six more) checked
    against the oracle: block bytes bit-exact, outputs within tolerance."""
    rng = np.random.default_rng(870)
    B, Hq, Hkv, D, L, layer = 64, 64, 8, 128, 1, 0
    lens = np.clip(np.round(np.exp(rng.normal(np.log(2048), 0.6, B))), 256, 8192).astype(np.int32) + 1
    g = oracle.Geom(L, Hkv, D, 16, 0)
    bt, g.num_pages = random_layout(rng, lens)
    pool = vk.PagedKVPool(L, Hkv, D, g.num_pages, kv_format="fp8")
    blocks = pool.block_view()
    blocks.zero_()
    gen = torch.Generator("cuda").manual_seed(3)
    btd = dev_i32(bt)
    for b, n in enumerate(lens):
        kh = (torch.randn((1, int(n) - 1, Hkv, D), device="cuda", generator=gen) * 0.5).half()
        vh = (torch.randn((1, int(n) - 1, Hkv, D), device="cuda", generator=gen) * 0.5).half()
        pool.append(layer, kh, vh, btd[b:b + 1], dev_i32([0]))
    plan = pool.plan(lens.tolist(), Hq)
    # FP8 runs more resident warps than fp16 (6 CTAs per SM), so this layer has
    # ~40 pages per worker and its split units are merged by dealt tasks
    assert plan.info(5) == (8 if plan.info(3) // plan.workers >= 64 else 1)
    assert plan.info(7) > 0 or plan.info(6) > 0
    sample = [int(np.argmax(lens)), int(np.argmin(lens))] + [int(x) for x in rng.choice(B, 6, replace=False)]
    pages, tabs = [], np.full((len(sample), bt.shape[1]), -1, np.int32)
    for i, b in enumerate(sample):
        n = (int(lens[b]) + 15) // 16
        tabs[i, :n] = np.arange(len(pages), len(pages) + n, dtype=np.int32)
        pages.extend(int(x) for x in bt[b, :n])
    idx = torch.tensor(pages, dtype=torch.long, device="cuda")
    before = blocks.index_select(1, idx).cpu().numpy()
    q = rows(rng, B, Hq, D)
    kn, vn = rows(rng, B, Hkv, D), rows(rng, B, Hkv, D)
    out = plan.run(layer, dev_f16(q), btd, k_new=dev_f16(kn), v_new=dev_f16(vn))
    torch.cuda.synchronize()
    assert pool.check() == 0
    after = blocks.index_select(1, idx).cpu().numpy()
    gs = oracle.Geom(L, Hkv, D, 16, len(pages))
    expect = np.ascontiguousarray(before)
    assert oracle.append_fp8(expect, gs, layer, kn[sample][:, None], vn[sample][:, None], tabs, lens[sample] - 1) == 0
    bad = after != expect
    assert not bad.any(), "FP8 fused append, sampled sequences: %d bytes differ" % int(bad.sum())
    ref = oracle.decode_fp8(expect, gs, layer, q[sample], tabs, lens[sample])
    assert_close_attn(out.float().cpu().numpy()[sample], ref, "FP8 70B full layer, sampled")
