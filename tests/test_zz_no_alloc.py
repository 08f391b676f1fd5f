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


def test_decode_static_matches_decode_two_calls(vk):
    from vulcan_b200 import _lib
    lib = _lib.load()
    rng = np.random.default_rng(2024)
    g = oracle.Geom(2, 4, 128, 16, 0)
    lens_a = np.array([3000, 17, 1, 900, 2500, 64, 333, 1024], np.int32)
    lens_b = np.array([40, 2999, 700, 5, 16, 1500, 2048, 90], np.int32)  # different split counts
    bt, g.num_pages = random_layout(rng, np.maximum(lens_a, lens_b))
    pool = make_pool(vk, g, random_pool(rng, g))
    pool.set_split(4)  # many splits per sequence, so the scratch is really used
    max_len = 3000
    assert 0 < pool.workspace_size(8, 32, max_len) <= SCRATCH_BYTES
    bt_d = dev_i32(bt)
    for call, lens in enumerate((lens_a, lens_b)):
        q = dev_f16((rng.standard_normal((8, 32, 128)) * 0.5).astype(np.float16))
        lens_d = dev_i32(lens)
        want = pool.decode(1, q, bt_d, lens_d, max_len)
        got = torch.full_like(q, float("nan"))
        assert _static_decode(lib, pool, 1, q, bt_d, lens_d, max_len, got) == _lib.VK_OK, \
            lib.vk_last_error_string()
        torch.cuda.synchronize()
        diff = (got.float() - want.float()).abs()
        assert torch.isfinite(got).all(), "call %d" % call
        assert bool((diff <= ATOL + RTOL * want.float().abs()).all()), "call %d max diff %g" % (call, diff.max())
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
