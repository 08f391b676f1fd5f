"""CPU oracle for the paged KV-cache path — TEST INFRASTRUCTURE ONLY.

Loads ``liboracle.so`` (the C restatement in ``vk_oracle.c``) and, when it has
been built, ``_ref/libvulcan_ref.so`` (the reference's own golden attention and
library, compiled from its sources).  Only ``tests/``, ``__graft_entry__.smoke``
and the CPU-baseline leg of ``bench.py`` may import this package; the product
library never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None

_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_c_int = ctypes.c_int


def build(ref: bool = False) -> None:
    """Compile liboracle.so (and oracle/_ref when ``ref`` is set)."""
    subprocess.run(["make", "-s", "-C", _HERE, "all"] + (["ref"] if ref else []), check=True)


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        L.or_attention_causal.argtypes = [_f32p, _f32p, _f32p, _f32p] + [_c_int] * 4
        L.or_attention_causal.restype = None
        L.or_decode_paged.argtypes = ([_u16p] + [_c_int] * 6 + [_u16p, _f32p, _i32p, _c_int, _i32p]
                                      + [_c_int, _c_int, ctypes.c_float, _c_int])
        L.or_decode_paged.restype = _c_int
        L.or_decode_paged_f64.argtypes = ([_u16p] + [_c_int] * 6 + [_u16p, _f64p, _i32p, _c_int,
                                          _i32p, _c_int, _c_int, ctypes.c_double])
        L.or_decode_paged_f64.restype = _c_int
        L.or_prefill_paged.argtypes = ([_u16p] + [_c_int] * 6 + [_u16p, _f32p, _i32p, _c_int, _i32p]
                                       + [_c_int, _c_int, _c_int, ctypes.c_float, _c_int])
        L.or_prefill_paged.restype = _c_int
        L.or_append_paged.argtypes = ([_u16p] + [_c_int] * 6 + [_u16p, _u16p, _i32p, _c_int, _i32p]
                                      + [_c_int, _c_int])
        L.or_append_paged.restype = _c_int
        L.or_copy_pages.argtypes = [_u8p, _c_int, ctypes.c_uint64, ctypes.c_uint64, _c_int, _i32p, _i32p, _c_int]
        L.or_copy_pages.restype = _c_int
        L.or_remap_block_tables.argtypes = [_i32p, ctypes.c_int64, _i32p, _c_int]
        L.or_remap_block_tables.restype = None
        L.or_rope.argtypes = [_f32p, _f32p, _c_int, _c_int, ctypes.c_float]
        L.or_e4m3_encode_array.argtypes = [_f32p, _u8p, ctypes.c_int64]
        L.or_e4m3_decode_array.argtypes = [_u8p, _f32p, ctypes.c_int64]
        L.or_fp8_quant_row.argtypes = [_f32p, _c_int, _u8p, ctypes.POINTER(ctypes.c_float)]
        L.or_append_fp8.argtypes = ([_u8p] + [_c_int] * 6 + [_f32p, _f32p, _i32p, _c_int, _i32p, _c_int, _c_int])
        L.or_append_fp8.restype = _c_int
        L.or_dequant_fp8.argtypes = [_u8p] + [_c_int] * 5 + [_f32p]
        L.or_rope.restype = None
        L.or_matmul.argtypes = [_f32p, _f32p, _f32p] + [_c_int] * 4
        L.or_matmul.restype = None
        _LIB = L
    return _LIB


def ref_lib():
    """The reference's own code compiled from its sources, or None if not built."""
    global _REF
    if _REF is None:
        path = os.path.join(_HERE, "_ref", "libvulcan_ref.so")
        if not os.path.exists(path):
            return None
        R = ctypes.CDLL(path)
        R.ref_random_floats.argtypes = [_c_int, ctypes.c_float, ctypes.c_float, _c_int, _f32p]
        R.ref_random_floats.restype = None
        R.ref_cpu_attention.argtypes = [_f32p, _f32p, _f32p, _f32p] + [_c_int] * 4
        R.ref_cpu_attention.restype = None
        R.ref_kernels_random_floats.argtypes = [_c_int, ctypes.c_float, ctypes.c_float, _c_int, _f32p]
        R.ref_kernels_random_floats.restype = None
        R.ref_cpu_rope.argtypes = [_f32p, _c_int, _c_int, ctypes.c_float, _f32p]
        R.ref_cpu_rope.restype = None
        R.ref_launch_matmul.argtypes = [ctypes.c_void_p] * 3 + [_c_int] * 3
        R.ref_launch_matmul.restype = None
        _REF = R
    return _REF


# ---------------------------------------------------------------- wrappers

class Geom:
    """Pool geometry: layers, kv heads, head dim, page tokens, pages."""

    def __init__(self, L, Hkv, D, P, num_pages):
        self.L, self.Hkv, self.D, self.P, self.num_pages = L, Hkv, D, P, num_pages

    @property
    def page_elems(self):
        return self.L * self.Hkv * 2 * self.P * self.D

    @property
    def seg_bytes(self):
        """Bytes of one page in one layer."""
        return self.Hkv * 2 * self.P * self.D * 2

    def pool_shape(self):
        """Layer-major pool: [layer, page, kv head, K|V, slot, d]."""
        return (self.L, self.num_pages, self.Hkv, 2, self.P, self.D)


def attention_causal(Q, K, V):
    """Contiguous [B,H,S,D] fp32 causal attention (cpu_attention restated)."""
    B, H, S, D = Q.shape
    O = np.zeros_like(Q, dtype=np.float32)
    lib().or_attention_causal(np.ascontiguousarray(Q, np.float32), np.ascontiguousarray(K, np.float32),
                              np.ascontiguousarray(V, np.float32), O, B, H, S, D)
    return O


def decode_paged(pool_u16, g: Geom, layer, q_u16, block_tables, seq_lens, scale=0.0, nthreads=1):
    B, Hq, D = q_u16.shape
    out = np.zeros((B, Hq, D), np.float32)
    rc = lib().or_decode_paged(np.ascontiguousarray(pool_u16).reshape(-1), g.L, g.Hkv, g.D, g.P,
                               g.num_pages, layer, np.ascontiguousarray(q_u16).reshape(-1), out,
                               np.ascontiguousarray(block_tables, np.int32).reshape(-1),
                               block_tables.shape[1], np.ascontiguousarray(seq_lens, np.int32),
                               B, Hq, float(scale), int(nthreads))
    if rc != 0:
        raise ValueError("oracle decode: bad block table")
    return out


def decode_paged_f64(pool_u16, g: Geom, layer, q_u16, block_tables, seq_lens, scale=0.0):
    B, Hq, D = q_u16.shape
    out = np.zeros((B, Hq, D), np.float64)
    rc = lib().or_decode_paged_f64(np.ascontiguousarray(pool_u16).reshape(-1), g.L, g.Hkv, g.D, g.P,
                                   g.num_pages, layer, np.ascontiguousarray(q_u16).reshape(-1), out,
                                   np.ascontiguousarray(block_tables, np.int32).reshape(-1),
                                   block_tables.shape[1], np.ascontiguousarray(seq_lens, np.int32),
                                   B, Hq, float(scale))
    if rc != 0:
        raise ValueError("oracle decode: bad block table")
    return out


def prefill_paged(pool_u16, g: Geom, layer, q_u16, block_tables, positions, scale=0.0, nthreads=1):
    B, T, Hq, D = q_u16.shape
    out = np.zeros((B, T, Hq, D), np.float32)
    rc = lib().or_prefill_paged(np.ascontiguousarray(pool_u16).reshape(-1), g.L, g.Hkv, g.D, g.P,
                                g.num_pages, layer, np.ascontiguousarray(q_u16).reshape(-1), out,
                                np.ascontiguousarray(block_tables, np.int32).reshape(-1),
                                block_tables.shape[1], np.ascontiguousarray(positions, np.int32),
                                B, T, Hq, float(scale), int(nthreads))
    if rc != 0:
        raise ValueError("oracle prefill: bad block table")
    return out


def append_paged(pool_u16, g: Geom, layer, k_u16, v_u16, block_tables, positions):
    """In-place append into a host pool copy; returns 0 or -1 (bad entry skipped)."""
    B, T = k_u16.shape[0], k_u16.shape[1]
    flat = pool_u16.reshape(-1)
    assert flat.base is pool_u16 or flat is pool_u16 or np.shares_memory(flat, pool_u16)
    return lib().or_append_paged(flat, g.L, g.Hkv, g.D, g.P, g.num_pages, layer,
                                 np.ascontiguousarray(k_u16).reshape(-1),
                                 np.ascontiguousarray(v_u16).reshape(-1),
                                 np.ascontiguousarray(block_tables, np.int32).reshape(-1),
                                 block_tables.shape[1], np.ascontiguousarray(positions, np.int32), B, T)


def copy_pages(pool_bytes, nseg, seg_bytes, seg_stride, num_pages, src, dst):
    """In-place page copy on a host byte image of the pool (see or_copy_pages)."""
    flat = pool_bytes.reshape(-1)
    rc = lib().or_copy_pages(flat, nseg, seg_bytes, seg_stride, num_pages, np.ascontiguousarray(src, np.int32),
                             np.ascontiguousarray(dst, np.int32), len(src))
    if rc != 0:
        raise ValueError("oracle copy: bad id")


def remap_block_tables(bt, page_map):
    flat = np.ascontiguousarray(bt, np.int32).reshape(-1).copy()
    lib().or_remap_block_tables(flat, flat.size, np.ascontiguousarray(page_map, np.int32), len(page_map))
    return flat.reshape(bt.shape)


def ref_attention_causal(Q, K, V):
    """The reference's own cpu_attention (compiled from its test file)."""
    R = ref_lib()
    if R is None:
        raise RuntimeError("oracle/_ref not built")
    B, H, S, D = Q.shape
    O = np.zeros((B, H, S, D), np.float32)
    R.ref_cpu_attention(np.ascontiguousarray(Q, np.float32), np.ascontiguousarray(K, np.float32),
                        np.ascontiguousarray(V, np.float32), O, B, H, S, D)
    return O


def ref_random_floats(n, lo, hi, seed):
    R = ref_lib()
    if R is None:
        raise RuntimeError("oracle/_ref not built")
    out = np.zeros(n, np.float32)
    R.ref_random_floats(n, lo, hi, seed, out)
    return out


def rope(x, positions, theta_base=10000.0):
    """cpu_rope (tests/test_kernels.cu:697-716) over the last axis of x (fp32),
    row r of x.reshape(-1, D) at positions.reshape(-1)[r // rows_per_pos]:
    positions has one entry per leading index of x.shape[:-1] prefix it
    broadcasts against (same shape as x.shape[:k] for some k)."""
    x = np.ascontiguousarray(x, np.float32)
    D = x.shape[-1]
    pos = np.asarray(positions, np.int32)
    rows = x.reshape(-1, D)
    per = rows.shape[0] // max(1, pos.size)
    out = np.empty_like(rows)
    L = lib()
    for r in range(rows.shape[0]):
        L.or_rope(np.ascontiguousarray(rows[r]), out[r], D, int(pos.reshape(-1)[r // per]), float(theta_base))
    return out.reshape(x.shape)


def ref_rope(x, pos, theta_base=10000.0):
    """The reference's own cpu_rope on one vector (needs oracle/_ref)."""
    R = ref_lib()
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    R.ref_cpu_rope(x, x.size, int(pos), float(theta_base), out)
    return out


def ref_kernels_random_floats(n, lo, hi, seed):
    """random_floats of the reference's kernel tests (tests/test_kernels.cu:30-37)."""
    R = ref_lib()
    out = np.empty(n, np.float32)
    R.ref_kernels_random_floats(n, lo, hi, seed, out)
    return out


# ---------------------------------------------------------------- FP8 pages
# (group-wise symmetric quantisation of docs/ADRs/003-quantization-format.md:11-18
# with an OCP E4M3 element; block layout in vk_oracle.c)

FP8_QMAX = 448.0


def fp8_block_bytes(D, P=16):
    return 2 * P * D + 8 * P


def _check_fp8_pool(pool_u8, g: Geom):
    if pool_u8.dtype != np.uint8 or pool_u8.size != g.L * g.num_pages * g.Hkv * fp8_block_bytes(g.D, g.P):
        raise ValueError("FP8 pool image does not match the geometry")


def e4m3_encode(x):
    """Nearest-even E4M3 codes of fp32 values, finite overflow saturated to +-448."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint8)
    lib().or_e4m3_encode_array(x.reshape(-1), out.reshape(-1), x.size)
    return out


def e4m3_decode(c):
    c = np.ascontiguousarray(c, np.uint8)
    out = np.empty(c.shape, np.float32)
    lib().or_e4m3_decode_array(c.reshape(-1), out.reshape(-1), c.size)
    return out


def fp8_quant_row(x):
    """(codes uint8 [n], scale float32) of one group."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    codes = np.empty(x.size, np.uint8)
    sc = ctypes.c_float()
    lib().or_fp8_quant_row(x, x.size, codes, ctypes.byref(sc))
    return codes, np.float32(sc.value)


def append_fp8(pool_u8, g: Geom, layer, k, v, block_tables, positions):
    """In-place append of fp32 (or fp16, widened exactly) rows [B, T, Hkv, D] into
    a host byte image of an FP8 pool; returns 0 or -1 (bad entry skipped)."""
    _check_fp8_pool(pool_u8, g)
    k = np.ascontiguousarray(np.asarray(k).astype(np.float32))
    v = np.ascontiguousarray(np.asarray(v).astype(np.float32))
    B, T = k.shape[0], k.shape[1]
    flat = pool_u8.reshape(-1)
    assert np.shares_memory(flat, pool_u8)
    return lib().or_append_fp8(flat, g.L, g.Hkv, g.D, g.P, g.num_pages, layer, k.reshape(-1), v.reshape(-1),
                               np.ascontiguousarray(block_tables, np.int32).reshape(-1), block_tables.shape[1],
                               np.ascontiguousarray(positions, np.int32), B, T)


def dequant_fp8(pool_u8, g: Geom):
    """fp32 [L, num_pages, Hkv, 2, P, D]: code * scale of every slot."""
    _check_fp8_pool(pool_u8, g)
    out = np.empty((g.L, g.num_pages, g.Hkv, 2, g.P, g.D), np.float32)
    lib().or_dequant_fp8(np.ascontiguousarray(pool_u8).reshape(-1), g.L, g.Hkv, g.D, g.P, g.num_pages,
                         out.reshape(-1))
    return out


def decode_fp8(pool_u8, g: Geom, layer, q, block_tables, seq_lens, scale=0.0):
    """Paged GQA decode over the dequantised FP8 cache, the arithmetic of one
    cpu_attention row (tests/test_attention.cu:66-97) per (sequence, query
    head) in float64.  q: [B, Hq, D] (fp16 or fp32).  Returns float64 [B, Hq, D]."""
    deq = dequant_fp8(pool_u8, g)[layer].astype(np.float64)  # [NP, Hkv, 2, P, D]
    q = np.asarray(q).astype(np.float64)
    B, Hq, D = q.shape
    G = Hq // g.Hkv
    sc = scale if scale > 0 else 1.0 / np.sqrt(D)
    out = np.zeros((B, Hq, D))
    for b in range(B):
        n = int(seq_lens[b])
        if n <= 0:
            continue
        pages = np.asarray(block_tables[b][: (n + g.P - 1) // g.P])
        kv = deq[pages]  # [np, Hkv, 2, P, D]
        K = kv[:, :, 0].transpose(1, 0, 2, 3).reshape(g.Hkv, -1, D)[:, :n]
        V = kv[:, :, 1].transpose(1, 0, 2, 3).reshape(g.Hkv, -1, D)[:, :n]
        for h in range(Hq):
            s = K[h // G] @ q[b, h] * sc
            p = np.exp(s - s.max())
            out[b, h] = (p / p.sum()) @ V[h // G]
    return out


def prefill_fp8(pool_u8, g: Geom, layer, q, block_tables, positions, scale=0.0):
    """Chunked prefill over the dequantised FP8 cache: query token t of sequence
    b at position positions[b] + t attends keys 0..positions[b] + t, the causal
    row rule of cpu_attention (tests/test_attention.cu:66-97) in float64.
    q: [B, T, Hq, D].  Returns float64 [B, T, Hq, D]."""
    deq = dequant_fp8(pool_u8, g)[layer].astype(np.float64)  # [NP, Hkv, 2, P, D]
    q = np.asarray(q).astype(np.float64)
    B, T, Hq, D = q.shape
    G = Hq // g.Hkv
    sc = scale if scale > 0 else 1.0 / np.sqrt(D)
    out = np.zeros((B, T, Hq, D))
    for b in range(B):
        n = int(positions[b]) + T
        pages = np.asarray(block_tables[b][: (n + g.P - 1) // g.P])
        kv = deq[pages]
        K = kv[:, :, 0].transpose(1, 0, 2, 3).reshape(g.Hkv, -1, D)[:, :n]
        V = kv[:, :, 1].transpose(1, 0, 2, 3).reshape(g.Hkv, -1, D)[:, :n]
        rows = int(positions[b]) + np.arange(T)
        hide = np.arange(n)[None, :] > rows[:, None]  # [T, n]
        for h in range(Hq):
            s = q[b, :, h] @ K[h // G].T * sc
            s[hide] = -np.inf
            p = np.exp(s - s.max(axis=1, keepdims=True))
            out[b, :, h] = (p / p.sum(axis=1, keepdims=True)) @ V[h // G]
    return out


# ---------------------------------------------------------------- wo projection

def matmul(A, B, nthreads=8):
    """launch_matmul's contract (cuda/matmul.cu:42-103): fp32 C = A @ B with one
    in-order fused multiply-add chain per element, as the reference kernel runs."""
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    M, K = A.shape
    K2, N = B.shape
    if K != K2:
        raise ValueError("inner dimensions differ")
    C = np.empty((M, N), np.float32)
    lib().or_matmul(A.reshape(-1), B.reshape(-1), C.reshape(-1), M, K, N, nthreads)
    return C
