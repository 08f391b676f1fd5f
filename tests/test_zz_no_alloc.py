"""GPU test of vk_decode_static, the decode entry point that allocates no device
memory (its split-K scratch is a fixed array inside the library), for callers
that cannot call cudaMalloc.  It must give the same output as vk_decode, call
after call, and refuse shapes whose scratch would exceed the fixed array.

This file is collected last on purpose, so that a run stopping at the first
failure has already run every other test."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from tests.helpers import ATOL, RTOL, dev_f16, dev_i32, make_pool, random_layout, random_pool

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 32 << 20  # VK_DECODE_STATIC_SCRATCH_BYTES


@pytest.fixture(scope="module")
def vk(cuda_ok):
    import vulcan_b200
    vulcan_b200.load()
    return vulcan_b200


def _static_decode(lib, pool, layer, q, bt, lens, max_len, out):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.vk_decode_static(pool.handle, layer, ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                ctypes.c_void_p(bt.data_ptr()), bt.shape[1], ctypes.c_void_p(lens.data_ptr()),
                                q.shape[0], q.shape[1], max_len, 0.0, ctypes.c_void_p(stream))


def _filled_pool(vk, rng, g, fmt, bt, lens):
    """A pool of either format holding every token the decode will read, and
    its host image for the oracle (fp16 values, or FP8 block bytes written by
    the quantising append and mirrored by the oracle's append)."""
    if fmt == "fp16":
        host = random_pool(rng, g)
        return make_pool(vk, g, host), host
    pool = vk.PagedKVPool(g.L, g.Hkv, g.D, g.num_pages, kv_format="fp8")
    host = np.zeros((g.L, g.num_pages, g.Hkv, pool.block_bytes), np.uint8)
    pool.block_view().zero_()
    for layer in range(g.L):
        for b, n in enumerate(lens):
            k = (rng.standard_normal((1, int(n), g.Hkv, g.D)) * 0.5).astype(np.float16)
            v = (rng.standard_normal((1, int(n), g.Hkv, g.D)) * 0.5).astype(np.float16)
            pool.append(layer, dev_f16(k), dev_f16(v), dev_i32(bt[b:b + 1]), dev_i32([0]))
            assert oracle.append_fp8(host, g, layer, k, v, bt[b:b + 1], np.zeros(1, np.int32)) == 0
    torch.cuda.synchronize()
    assert np.array_equal(pool.block_view().cpu().numpy(), host)
    return pool, host


def _oracle(g, fmt, host, layer, q, bt, lens):
    if fmt == "fp16":
        return oracle.decode_paged(host.view(np.uint16), g, layer, q.view(np.uint16), bt, lens, nthreads=8)
    return oracle.decode_fp8(host, g, layer, q, bt, lens)


@pytest.mark.parametrize("fmt", ["fp16", "fp8"])
def test_decode_static_matches_decode_two_calls(vk, fmt):
    """Two calls in a row with different lengths (so different split counts,
    and the second call finds the first call's partials in the array): each
    output matches vk_decode with a caller workspace and the CPU oracle within
    the attention tolerance."""
    from vulcan_b200 import _lib
    lib = _lib.load()
    rng = np.random.default_rng(2024 + (fmt == "fp8"))
    g = oracle.Geom(2, 4, 128, 16, 0)
    lens_a = np.array([3000, 17, 1, 900, 2500, 64, 333, 1024], np.int32)
    lens_b = np.array([40, 2999, 700, 5, 16, 1500, 2048, 90], np.int32)  # different split counts
    most = np.maximum(lens_a, lens_b)
    bt, g.num_pages = random_layout(rng, most)
    pool, host = _filled_pool(vk, rng, g, fmt, bt, most)
    pool.set_split(4)  # many splits per sequence, so the scratch is really used
    max_len = 3000
    assert 0 < pool.workspace_size(8, 32, max_len) <= SCRATCH_BYTES
    bt_d = dev_i32(bt)
    for call, lens in enumerate((lens_a, lens_b)):
        qh = (rng.standard_normal((8, 32, 128)) * 0.5).astype(np.float16)
        q = dev_f16(qh)
        lens_d = dev_i32(lens)
        want = pool.decode(1, q, bt_d, lens_d, max_len)
        got = torch.full_like(q, float("nan"))
        assert _static_decode(lib, pool, 1, q, bt_d, lens_d, max_len, got) == _lib.VK_OK, \
            lib.vk_last_error_string()
        torch.cuda.synchronize()
        assert torch.isfinite(got).all(), "call %d" % call
        diff = (got.float() - want.float()).abs()
        assert bool((diff <= ATOL + RTOL * want.float().abs()).all()), "call %d max diff %g" % (call, diff.max())
        ref = _oracle(g, fmt, host, 1, qh, bt, lens)
        err = np.abs(got.float().cpu().numpy() - ref)
        assert (err <= ATOL + RTOL * np.abs(ref)).all(), "call %d vs oracle: max err %g" % (call, err.max())
    assert pool.check() == 0


def test_decode_static_rejects_oversized_scratch(vk):
    from vulcan_b200 import _lib
    lib = _lib.load()
    g = oracle.Geom(1, 8, 128, 16, 8)
    pool = make_pool(vk, g)
    pool.set_split(1)
    B, Hq, max_len = 64, 64, 8192
    assert pool.workspace_size(B, Hq, max_len) > SCRATCH_BYTES
    q = torch.zeros(B, Hq, 128, dtype=torch.float16, device="cuda")
    out = torch.zeros_like(q)
    bt = torch.zeros(B, 512, dtype=torch.int32, device="cuda")
    lens = torch.ones(B, dtype=torch.int32, device="cuda")
    st = _static_decode(lib, pool, 0, q, bt, lens, max_len, out)
    assert st == _lib.VK_INVALID_ARG
    assert b"scratch" in lib.vk_last_error_string()
