"""GPU tests that run the reference's own implementation (compiled from its
sources into oracle/_ref) beside the library on identical inputs:
MemoryManager id sequences and swap results, KVCache::append row placement,
launch_attention outputs on the reference's six attention cases, and
launch_matmul against the oracle's restatement (bit for bit)."""
import ctypes
import os

import numpy as np
import pytest
import torch

import oracle
from tests.helpers import dev_i32, device_view

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
vp, ci, csz = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t


@pytest.fixture(scope="module")
def ref(cuda_ok):
    R = oracle.ref_lib()
    if R is None:
        pytest.skip("oracle/_ref not built")
    sig = {
        "ref_mm_create": (vp, [csz, ci]), "ref_mm_destroy": (None, [vp]), "ref_mm_allocate": (ci, [vp]),
        "ref_mm_free": (None, [vp, ci]), "ref_mm_ptr": (vp, [vp, ci]), "ref_mm_swap_to_cpu": (ci, [vp, ci]),
        "ref_mm_swap_to_gpu": (ci, [vp, ci]), "ref_mm_in_use": (ci, [vp]), "ref_mm_available": (ci, [vp]),
        "ref_mm_total_bytes": (csz, [vp]), "ref_kv_create": (vp, [ci, ci, ci, ci]),
        "ref_kv_destroy": (None, [vp]), "ref_kv_append": (None, [vp, ci, vp, vp, ci, ci]),
        "ref_kv_get": (None, [vp, ci, ctypes.POINTER(vp), ctypes.POINTER(vp)]), "ref_kv_len": (ci, [vp]),
        "ref_kv_memory": (csz, [vp]), "ref_launch_attention": (None, [vp, vp, vp, vp, ci, ci, ci, ci]),
        "ref_launch_matmul": (None, [vp, vp, vp, ci, ci, ci]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(R, name)
        fn.restype, fn.argtypes = res, args
    torch.cuda.init()
    return R


@pytest.fixture(scope="module")
def vk(cuda_ok):
    import vulcan_b200
    vulcan_b200.load()
    return vulcan_b200


def test_allocator_sequence_matches_reference(ref, vk):
    """A seeded mix of allocate/free/swap on the reference MemoryManager and the
    library's: identical ids, counts and return values at every step."""
    rng = np.random.default_rng(40)
    r = ref.ref_mm_create(256, 32)
    m = vk.MemoryManager(256, 32)
    try:
        live = []
        for step in range(400):
            op = rng.integers(0, 5)
            if op <= 1:
                a, b = ref.ref_mm_allocate(r), m.allocate_block()
                assert a == b, step
                if a >= 0:
                    live.append(a)
            elif op == 2 and live:
                i = live.pop(int(rng.integers(0, len(live))))
                ref.ref_mm_free(r, i)
                m.free_block(i)
            elif op == 3:
                i = int(rng.integers(-2, 34))
                assert bool(ref.ref_mm_swap_to_cpu(r, i)) == m.swap_to_cpu(i), step
                if i in live:
                    live.remove(i)
            else:
                i = int(rng.integers(-2, 34))
                a = bool(ref.ref_mm_swap_to_gpu(r, i))
                b = m.swap_to_gpu(i)
                if a or b:
                    # the reference restores into an id even if it was reallocated
                    # meanwhile; the library refuses that case (documented)
                    if a != b:
                        assert a and not b and m._pool.page_in_use(i) == 1
                        m._swap.pop(i, None)       # the reference consumed its copy
                    else:
                        live.append(i)
                    assert ref.ref_mm_in_use(r) == m.blocks_in_use(), step
                    continue
            assert ref.ref_mm_in_use(r) == m.blocks_in_use(), step
            assert ref.ref_mm_available(r) == m.blocks_available(), step
            assert ref.ref_mm_total_bytes(r) == m.total_allocated_bytes(), step
    finally:
        ref.ref_mm_destroy(r)


def test_reference_swap_test_sequence(ref):
    """The reference's SwapToCPUAndBack sequence on the reference itself: its
    free_block drops the swap copy, so swap_to_gpu returns false."""
    r = ref.ref_mm_create(1024, 4)
    try:
        i = ref.ref_mm_allocate(r)
        assert ref.ref_mm_swap_to_cpu(r, i) == 1
        t = ref.ref_mm_allocate(r)
        assert t == i
        ref.ref_mm_free(r, t)
        assert ref.ref_mm_swap_to_gpu(r, i) == 0
    finally:
        ref.ref_mm_destroy(r)


def test_kvcache_append_matches_reference(ref, vk):
    """Reference KVCache::append (fp32, contiguous) vs the library's paged append
    (fp16): every appended row lands at the same (head, position), fp16 of the
    reference row bit for bit."""
    rng = np.random.default_rng(41)
    Hkv, S, D, L = 4, 96, 128, 2
    rc = ref.ref_kv_create(Hkv, S, D, L)
    c = vk.KVCache(Hkv, S, D, L)
    try:
        pos = 0
        for T in (5, 1, 1, 30, 1, 11):
            k = torch.from_numpy((rng.standard_normal((T, Hkv * D)) * 0.5).astype(np.float32)).cuda()
            v = torch.from_numpy((rng.standard_normal((T, Hkv * D)) * 0.5).astype(np.float32)).cuda()
            ref.ref_kv_append(rc, 1, vp(k.data_ptr()), vp(v.data_ptr()), pos, T)
            c.append(1, k, v, pos, T)
            pos += T
            assert ref.ref_kv_len(rc) == c.current_length() == pos
        kp, vpp = vp(), vp()
        ref.ref_kv_get(rc, 1, ctypes.byref(kp), ctypes.byref(vpp))
        rk = device_view(kp.value, Hkv * S * D * 4).view(torch.float32).view(Hkv, S, D).cpu()
        rv = device_view(vpp.value, Hkv * S * D * 4).view(torch.float32).view(Hkv, S, D).cpu()
        kv = c.pool.kv_view()[1].cpu()  # [pages, Hkv, 2, 16, D]
        bt = c.block_table[0].cpu()
        for j in range(pos):
            page = int(bt[j // 16])
            assert torch.equal(kv[page, :, 0, j % 16], rk[:, j].half()), j
            assert torch.equal(kv[page, :, 1, j % 16], rv[:, j].half()), j
    finally:
        ref.ref_kv_destroy(rc)


def test_launch_attention_matches_reference(ref, vk):
    """The six reference attention cases: the reference GPU kernel and the
    library's launch_attention both within the reference's tolerances of its
    golden outputs, and within 1e-5 of each other."""
    f = np.load(os.path.join(GOLD, "ref_attention_cases.npz"))
    tol = {"SingleHead_SmallSeq": 1e-4}
    for n in sorted({k.split("/")[0] for k in f.files}):
        q, k, v, o = (torch.from_numpy(f[n + s]).cuda() for s in ("/q", "/k", "/v", "/o"))
        B, H, S, D = q.shape
        out_ref = torch.zeros_like(q)
        out_new = torch.zeros_like(q)
        ref.ref_launch_attention(vp(q.data_ptr()), vp(k.data_ptr()), vp(v.data_ptr()), vp(out_ref.data_ptr()),
                                 B, H, S, D)
        vk.launch_attention(q, k, v, out_new, B, H, S, D)
        torch.cuda.synchronize()
        t = tol.get(n, 1e-3)
        assert (out_ref - o).abs().max().item() < t, n
        assert (out_new - o).abs().max().item() < t, n
        assert (out_new - out_ref).abs().max().item() < 1e-5, n


def test_launch_attention_longer_vs_oracle(vk):
    rng = np.random.default_rng(42)
    q, k, v = (rng.standard_normal((2, 3, 300, 128)).astype(np.float32) * 0.5 for _ in range(3))
    ref_out = oracle.attention_causal(q, k, v)
    out = torch.zeros(2, 3, 300, 128, device="cuda")
    vk.launch_attention(*(torch.from_numpy(x).cuda() for x in (q, k, v)), out, 2, 3, 300, 128)
    assert np.abs(out.cpu().numpy() - ref_out).max() < 1e-4


def test_reference_memory_usage_formula(ref, vk):
    rc = ref.ref_kv_create(8, 2048, 128, 32)
    try:
        assert ref.ref_kv_memory(rc) == 2 * 32 * 8 * 2048 * 128 * 4  # fp32 reference
    finally:
        ref.ref_kv_destroy(rc)
    assert vk.KVCache(8, 2048, 128, 32).memory_usage() == 2 * 32 * 8 * 2048 * 128 * 2  # fp16 pages


@pytest.mark.parametrize("m,k,n", [(1, 4096, 512), (7, 300, 130), (64, 1024, 256), (33, 77, 65)])
def test_oracle_matmul_matches_reference_launch_matmul(ref, m, k, n):
    """Pins oracle.matmul: the reference's own launch_matmul (cuda/matmul.cu,
    compiled from its sources, run on the GPU) gives the same fp32 bits."""
    rng = np.random.default_rng(m + k + n)
    a = (rng.standard_normal((m, k)) * 0.5).astype(np.float32)
    b = (rng.standard_normal((k, n)) * 0.02).astype(np.float32)
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    dc = torch.empty(m, n, dtype=torch.float32, device="cuda")
    ref.ref_launch_matmul(vp(da.data_ptr()), vp(db.data_ptr()), vp(dc.data_ptr()), m, k, n)
    torch.cuda.synchronize()
    got = oracle.matmul(a, b)
    assert np.array_equal(dc.cpu().numpy().view(np.uint32), got.view(np.uint32)), \
        "max diff %g" % np.abs(dc.cpu().numpy() - got).max()
