"""Seeded synthetic inputs shared by the fixture generator and the tests.

Values are fp16 draws of N(0, 0.5^2) from numpy's PCG64 generator; block
tables are seeded permutations of the physical page ids.  Pools are layer-major
[layer, page, kv head, K|V, slot, d], the library's device layout.  Only the slots that a
case uses are filled (the rest stay zero), as a freshly created pool is
zero-filled.
"""
import hashlib

import numpy as np

import oracle

PAGE_TOKENS = 16

# (num_q_heads, num_kv_heads, sequence lengths) — GQA groups 8, 4, 2, 1 and the
# page-boundary lengths 1, 15, 16, 17, 31, 33.
PAGED_CASES = [
    (8, 1, [1, 15, 16, 17]),
    (4, 1, [33, 100, 257]),
    (4, 2, [2, 31, 64]),
    (2, 2, [5, 48]),
]
PAGED_SEED = 7100
CONFIG1_SEED = 7000


def normal_f16(rng, shape, std=0.5):
    return (rng.standard_normal(shape, dtype=np.float32) * std).astype(np.float16)


def fill_sequences(rng, pool, g, layer, bt, lens):
    """Writes random K/V for tokens 0..lens[b]-1 of every sequence."""
    for b, n in enumerate(lens):
        for j in range(int(n)):
            page = bt[b][j // g.P]
            pool[layer, page, :, :, j % g.P, :] = normal_f16(rng, (g.Hkv, 2, g.D))


def paged_case(index):
    Hq, Hkv, lens = PAGED_CASES[index]
    rng = np.random.Generator(np.random.PCG64(PAGED_SEED + index))
    L, D, P, layer = 2, 128, PAGE_TOKENS, 1
    lens = np.array(lens, np.int32)
    pages_per_seq = [(int(n) + P - 1) // P for n in lens]
    width = max(pages_per_seq)
    num_pages = sum(pages_per_seq) + 3
    g = oracle.Geom(L, Hkv, D, P, num_pages)
    perm = rng.permutation(num_pages).astype(np.int32)
    bt = np.full((len(lens), width), -1, np.int32)
    off = 0
    for b, npg in enumerate(pages_per_seq):
        bt[b, :npg] = perm[off:off + npg]
        off += npg
    pool = np.zeros(g.pool_shape(), np.float16)
    fill_sequences(rng, pool, g, layer, bt, lens)
    q = normal_f16(rng, (len(lens), Hq, D))
    return dict(geom=g, layer=layer, pool=pool, bt=bt, lens=lens, q=q)


def config1_case():
    """Llama-2-7B single-layer decode: 32/32 heads, D=128, batch 1, 512 cached
    tokens, 1 appended token, 64 physical pages in a seeded permutation."""
    rng = np.random.Generator(np.random.PCG64(CONFIG1_SEED))
    H = Hkv = 32
    D, P, num_pages, ctx = 128, PAGE_TOKENS, 64, 512
    g = oracle.Geom(1, Hkv, D, P, num_pages)
    bt = rng.permutation(num_pages).astype(np.int32)[None, :]
    pool_before = np.zeros(g.pool_shape(), np.float16)
    fill_sequences(rng, pool_before, g, 0, bt, [ctx])
    k_new = normal_f16(rng, (1, 1, Hkv, D))
    v_new = normal_f16(rng, (1, 1, Hkv, D))
    q = normal_f16(rng, (1, H, D))
    positions = np.array([ctx], np.int32)
    pool = pool_before.copy()
    rc = oracle.append_paged(pool.view(np.uint16), g, 0, k_new.view(np.uint16), v_new.view(np.uint16),
                             bt, positions)
    assert rc == 0
    return dict(geom=g, pool_before=pool_before, pool=pool, bt=bt, k_new=k_new, v_new=v_new, q=q,
                positions=positions, lens=positions + 1)


def digest(c):
    h = hashlib.sha256()
    for key in ("pool_before", "bt", "k_new", "v_new", "q"):
        h.update(np.ascontiguousarray(c[key]).tobytes())
    return h.hexdigest()
