"""GPU tests of K4 page copy / compaction, K5 pinned-host swap, and the
MemoryManager / KVCache mirrors of the reference's allocator tests
(tests/test_memory.cpp).  Copies and swaps are bit-exact."""
import numpy as np
import pytest
import torch

import oracle
from oracle.allocator_model import AllocatorModel
from tests.helpers import dev_f16, dev_i32, device_view, make_pool, random_layout, random_pool

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def vk(cuda_ok):
    import vulcan_b200
    vulcan_b200.load()
    return vulcan_b200


def test_copy_pages_bit_exact(vk):
    rng = np.random.default_rng(20)
    g = oracle.Geom(4, 2, 128, 16, 24)  # 128 KiB pages
    host = random_pool(rng, g)
    pool = make_pool(vk, g, host)
    src = np.array([3, 9, 17, 0], np.int32)
    dst = np.array([20, 4, 1, 23], np.int32)
    pool.copy_pages(dev_i32(src), dev_i32(dst))
    assert pool.check() == 0
    expect = host.copy()
    oracle.copy_pages(expect.view(np.uint8), g.L, g.seg_bytes, g.seg_bytes * g.num_pages, g.num_pages, src, dst)
    assert np.array_equal(pool.kv_view().cpu().numpy().view(np.uint16), expect.view(np.uint16))


def test_copy_pages_odd_page_size(vk):
    """A raw byte pool whose page is not a multiple of the 32 KiB copy chunk."""
    pool = vk.PagedKVPool(0, 0, 0, 6, page_tokens=0, page_bytes=40016)
    data = torch.randint(0, 255, (6 * 40016,), dtype=torch.uint8, device="cuda")
    pool.storage.copy_(data)
    pool.copy_pages(dev_i32([5, 1]), dev_i32([0, 3]))
    torch.cuda.synchronize()
    got = pool.storage.view(6, 40016).cpu()
    d = data.view(6, 40016).cpu()
    assert torch.equal(got[0], d[5]) and torch.equal(got[3], d[1]) and torch.equal(got[2], d[2])


def test_compaction_preserves_attention(vk):
    rng = np.random.default_rng(21)
    g = oracle.Geom(1, 2, 128, 16, 64)
    pool = make_pool(vk, g, random_pool(rng, g))
    ids = pool.alloc(64)
    assert ids == list(range(64))
    lens = np.array([100, 37, 260], np.int32)
    bt = np.full((3, 17), -1, np.int32)
    keep = rng.permutation(64)[:7 + 3 + 17]
    bt[0, :7], bt[1, :3], bt[2, :17] = keep[:7], keep[7:10], keep[10:27]
    pool.free(sorted(set(range(64)) - set(keep.tolist())))
    q = dev_f16((rng.standard_normal((3, 8, 128)) * 0.5).astype(np.float16))
    before = pool.decode(0, q, dev_i32(bt), dev_i32(lens), 260).cpu()
    model = AllocatorModel(1, 64)
    model.in_use = [bool(pool.page_in_use(i)) for i in range(64)]
    src, dst = pool.compact_plan()
    assert list(zip(src, dst)) == model.compact_plan()
    pool.copy_pages(dev_i32(src), dev_i32(dst))
    page_map = np.arange(64, dtype=np.int32)
    page_map[src] = dst
    bt_dev = dev_i32(bt)
    vk.remap_block_tables(bt_dev, dev_i32(page_map))
    assert np.array_equal(bt_dev.cpu().numpy(), oracle.remap_block_tables(bt, page_map))
    assert sorted(bt_dev.cpu().numpy()[bt_dev.cpu().numpy() >= 0].tolist()) == list(range(27))
    after = pool.decode(0, q, bt_dev, dev_i32(lens), 260).cpu()
    assert torch.equal(before, after)
    assert pool.check() == 0


def test_swap_round_trip_and_remap(vk):
    rng = np.random.default_rng(22)
    g = oracle.Geom(2, 2, 128, 16, 16)
    host = random_pool(rng, g)
    pool = make_pool(vk, g, host)
    ids = pool.alloc(16)
    victims = [3, 4, 5, 11]  # a run of three plus a single page
    pinned = torch.empty(len(victims) * pool.page_bytes, dtype=torch.uint8, pin_memory=True)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        pool.swap_out(victims, pinned)
    s.synchronize()
    assert pool.pages_in_use() == 12
    assert [pool.page_in_use(i) for i in victims] == [0, 0, 0, 0]
    # host buffer: whole pages back to back, each page's layer segments in order
    expect = np.ascontiguousarray(host.transpose(1, 0, 2, 3, 4, 5)[victims]).view(np.uint8).reshape(-1)
    assert np.array_equal(pinned.numpy(), expect)
    # scribble over the freed pages, then swap back in (lowest free ids first)
    pool.kv_view()[:, victims] = 0
    got_ids = pool.swap_in(pinned, 4)
    torch.cuda.synchronize()
    assert got_ids == victims
    assert np.array_equal(pool.kv_view().cpu().numpy().view(np.uint16), host.view(np.uint16))
    assert ids == list(range(16)) and pool.pages_in_use() == 16


def test_swap_in_to_requires_free_ids(vk):
    g = oracle.Geom(1, 1, 64, 16, 4)
    pool = make_pool(vk, g)
    pool.alloc(2)
    pinned = torch.zeros(2 * pool.page_bytes, dtype=torch.uint8, pin_memory=True)
    with pytest.raises(vk.VKError):
        pool.swap_in_to(pinned, [1, 2])  # 1 is in use
    pool.swap_in_to(pinned, [2, 3])
    assert pool.pages_in_use() == 4


# ---------------------------------------------------------------- MemoryManager mirror

def test_memory_manager_reference_tests(vk):
    """tests/test_memory.cpp:99-212 on the library's MemoryManager."""
    m = vk.MemoryManager(4096, 16)                                     # Construction
    assert (m.blocks_in_use(), m.blocks_available(), m.total_allocated_bytes()) == (0, 16, 0)
    m = vk.MemoryManager(4096, 8)                                      # AllocateAndFree
    i = m.allocate_block()
    assert i >= 0 and m.blocks_in_use() == 1 and m.blocks_available() == 7
    assert m.get_block_ptr(i)
    m.free_block(i)
    assert m.blocks_in_use() == 0 and m.blocks_available() == 8
    m = vk.MemoryManager(1024, 4)                                      # AllocateAll
    ids = [m.allocate_block() for _ in range(4)]
    assert ids == [0, 1, 2, 3] and m.blocks_available() == 0
    assert m.allocate_block() == -1
    m.free_block(ids[0])
    assert m.blocks_available() == 1 and m.allocate_block() >= 0
    m = vk.MemoryManager(4096, 8)                                      # BlockPointersPersist
    a, b = m.allocate_block(), m.allocate_block()
    assert abs(m.get_block_ptr(b) - m.get_block_ptr(a)) == 4096
    m = vk.MemoryManager(1024, 4)                                      # InvalidBlockId
    assert m.get_block_ptr(-1) is None and m.get_block_ptr(999) is None
    assert not m.swap_to_cpu(-1) and not m.swap_to_gpu(999)


def test_memory_manager_swap(vk):
    m = vk.MemoryManager(1024, 4)
    i = m.allocate_block()
    data = torch.arange(1024, dtype=torch.int32).to(torch.uint8)
    block = device_view(m.get_block_ptr(i), 1024)
    block.copy_(data.cuda())
    assert m.swap_to_cpu(i) and m.blocks_in_use() == 0
    block.zero_()
    assert m.swap_to_gpu(i) and m.blocks_in_use() == 1
    torch.cuda.synchronize()
    assert torch.equal(block.cpu(), data)
    # the reference test's sequence: the reused id is freed before swap-in,
    # which drops the swap copy (cuda/memory.cu:137-143) -> swap_to_gpu False
    assert m.swap_to_cpu(i)
    t = m.allocate_block()
    assert t == i
    m.free_block(t)
    assert not m.swap_to_gpu(i) and m.blocks_in_use() == 0


# ---------------------------------------------------------------- KVCache mirror

def test_kvcache_mirror(vk):
    c = vk.KVCache(4, 128, 64, 2)                                      # Construction
    assert c.current_length() == 0 and c.max_seq_len() == 128 and c.memory_usage() > 0
    heads, head_dim = 2, 4 * 16                                        # AppendAndGet (+ readback)
    c = vk.KVCache(heads, 32, head_dim, 1)
    k = torch.arange(heads * head_dim, dtype=torch.float32, device="cuda")[None] + 1
    v = k + 99
    c.append(0, k, v, 0, 1)
    assert c.current_length() == 1
    kp, vp = c.get(0)
    assert kp and vp and vp - kp == 16 * head_dim * 2
    page = c.block_table[0, 0].item()
    kv = c.pool.kv_view()[0, page]
    assert torch.equal(kv[:, 0, 0].float().cpu().reshape(-1), k.cpu().reshape(-1))
    assert torch.equal(kv[:, 1, 0].float().cpu().reshape(-1), v.cpu().reshape(-1))
    c.append(5, k, v, 0, 1)                                            # bad layer: ignored
    c.append(0, k, v, 32, 1)                                           # overflow: ignored
    assert c.current_length() == 1
    c.set_length(42)                                                   # Reset
    assert c.current_length() == 42
    c.reset()
    assert c.current_length() == 0
    c = vk.KVCache(8, 2048, 128, 32)                                   # MemoryUsageCalculation (fp16)
    assert c.memory_usage() == 2 * 32 * 8 * 2048 * 128 * 2


def test_kvcache_decode_matches_oracle(vk):
    rng = np.random.default_rng(30)
    Hkv, D, Hq = 2, 128, 8
    c = vk.KVCache(Hkv, 100, D, 2)
    k = torch.from_numpy((rng.standard_normal((37, Hkv * D)) * 0.5).astype(np.float32)).cuda()
    v = torch.from_numpy((rng.standard_normal((37, Hkv * D)) * 0.5).astype(np.float32)).cuda()
    c.append(1, k, v, 0, 37)
    q = (rng.standard_normal((Hq, D)) * 0.5).astype(np.float16)
    out = c.decode(1, dev_f16(q)).float().cpu().numpy()
    host = c.pool.kv_view().cpu().numpy()
    g = oracle.Geom(2, Hkv, D, 16, c.pool.num_pages)
    ref = oracle.decode_paged(host.view(np.uint16), g, 1, q[None].view(np.uint16),
                              c.block_table.cpu().numpy(), np.array([37], np.int32))
    from tests.helpers import assert_close_attn
    assert_close_attn(out[None], ref, "kvcache decode")
