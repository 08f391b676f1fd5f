"""Shared helpers for the GPU parity tests (upload numpy pools, compare with the
oracle under the fp16 attention tolerance)."""
import numpy as np
import torch

import oracle

# fp16 attention outputs vs the fp32 oracle: |gpu - ref| <= ATOL + RTOL*|ref|
ATOL = 2e-3
RTOL = 1e-2


def assert_close_attn(gpu, ref, what=""):
    gpu = np.asarray(gpu, np.float32)
    ref = np.asarray(ref, np.float32)
    assert gpu.shape == ref.shape, (gpu.shape, ref.shape)
    assert np.isfinite(gpu).all(), what + ": non-finite output"
    err = np.abs(gpu - ref)
    bound = ATOL + RTOL * np.abs(ref)
    bad = err > bound
    assert not bad.any(), "%s: %d/%d outside tolerance, max err %.3g" % (what, bad.sum(), bad.size, err.max())


def make_pool(vk, g: oracle.Geom, host_pool_f16=None):
    """A torch-backed PagedKVPool with the same geometry, optionally filled."""
    pool = vk.PagedKVPool(g.L, g.Hkv, g.D, g.num_pages, page_tokens=g.P)
    if host_pool_f16 is not None:
        pool.kv_view().copy_(torch.from_numpy(np.ascontiguousarray(host_pool_f16)).view(torch.float16))
    return pool


def dev_i32(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.int32)).cuda()


def dev_f16(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float16)).cuda()


def random_layout(rng, lens, num_pages=None, P=16, extra_pages=5):
    """Random physical pages for sequences of the given lengths; returns (bt, num_pages)."""
    need = [(int(n) + P - 1) // P for n in lens]
    total = sum(need)
    num_pages = num_pages or total + extra_pages
    perm = rng.permutation(num_pages).astype(np.int32)
    width = max(1, max(need))
    bt = np.full((len(lens), width), -1, np.int32)
    off = 0
    for b, k in enumerate(need):
        bt[b, :k] = perm[off:off + k]
        off += k
    return bt, num_pages


def random_pool(rng, g: oracle.Geom, fill_nan=False):
    shape = g.pool_shape()
    if fill_nan:
        return np.full(shape, np.float16(np.nan), np.float16)
    return (rng.standard_normal(shape, dtype=np.float32) * 0.5).astype(np.float16)


class _RawDeviceBuffer:
    """Exposes raw device bytes through __cuda_array_interface__."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (int(ptr), False),
                                         "version": 3, "strides": None}


def device_view(ptr, nbytes):
    """A uint8 CUDA tensor aliasing ``nbytes`` of device memory at ``ptr``."""
    return torch.as_tensor(_RawDeviceBuffer(ptr, nbytes), device="cuda")
