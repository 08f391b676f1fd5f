"""CPU tests of the oracle: pinned against the reference's golden vectors and
known-answer properties, plus the allocator model against the reference's
allocator tests.  No GPU needed."""
import os

import numpy as np
import pytest

import oracle
from oracle.allocator_model import AllocatorModel
from tests.golden import gen

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLD, name))


# ---------------------------------------------------------------- attention

def test_oracle_matches_reference_attention_fixtures():
    """cpu_attention restated == the reference's own output, bit for bit, on the
    six attention tests of tests/test_attention.cu:107-264."""
    f = load("ref_attention_cases.npz")
    names = sorted({k.split("/")[0] for k in f.files})
    assert len(names) == 6
    for n in names:
        out = oracle.attention_causal(f[n + "/q"], f[n + "/k"], f[n + "/v"])
        assert np.array_equal(out, f[n + "/o"]), n


def test_reference_known_answers_on_fixtures():
    f = load("ref_attention_cases.npz")
    # CausalMask_FirstRow (tests/test_attention.cu:156-182): row 0 == V[0]
    o, v = f["CausalMask_FirstRow/o"], f["CausalMask_FirstRow/v"]
    assert np.allclose(o[0, 0, 0], v[0, 0, 0], atol=1e-5)
    # OutputSumMatchesV (:232-264): outputs inside [min V, max V]
    o, v = f["OutputSumMatchesV/o"], f["OutputSumMatchesV/v"]
    assert o.min() >= v.min() - 1e-4 and o.max() <= v.max() + 1e-4


def test_oracle_paged_decode_matches_fixtures():
    f = load("paged_decode_cases.npz")
    for ci in range(len(gen.PAGED_CASES)):
        pre = "case%d/" % ci
        L, Hkv, D, P, NP, layer = (int(x) for x in f[pre + "geom"])
        g = oracle.Geom(L, Hkv, D, P, NP)
        out = oracle.decode_paged(f[pre + "pool"], g, layer, f[pre + "q"], f[pre + "bt"], f[pre + "lens"])
        assert np.array_equal(out, f[pre + "out"]), ci
        # multithreaded oracle is the same arithmetic per (b, h)
        out4 = oracle.decode_paged(f[pre + "pool"], g, layer, f[pre + "q"], f[pre + "bt"], f[pre + "lens"],
                                   nthreads=4)
        assert np.array_equal(out4, out)


def test_fixture_inputs_regenerate():
    """The seeded generator still produces the fixture inputs."""
    f = load("paged_decode_cases.npz")
    for ci in range(len(gen.PAGED_CASES)):
        c = gen.paged_case(ci)
        assert np.array_equal(c["pool"].view(np.uint16), f["case%d/pool" % ci])
        assert np.array_equal(c["q"].view(np.uint16), f["case%d/q" % ci])
    c1 = load("config1_decode.npz")
    assert gen.digest(gen.config1_case()) == bytes(c1["sha256"]).decode()


def test_oracle_config1_matches_fixture():
    c = gen.config1_case()
    f = load("config1_decode.npz")
    out = oracle.decode_paged(c["pool"].view(np.uint16), c["geom"], 0, c["q"].view(np.uint16), c["bt"],
                              c["lens"])
    assert np.array_equal(out, f["out"])


def test_oracle_fp32_error_small_vs_f64():
    """The fp32 oracle is within 1e-5 of a double-precision evaluation."""
    c = gen.paged_case(1)
    g = c["geom"]
    o32 = oracle.decode_paged(c["pool"].view(np.uint16), g, c["layer"], c["q"].view(np.uint16), c["bt"], c["lens"])
    o64 = oracle.decode_paged_f64(c["pool"].view(np.uint16), g, c["layer"], c["q"].view(np.uint16), c["bt"],
                                  c["lens"])
    assert np.abs(o32 - o64).max() < 1e-5


def test_oracle_decode_equals_last_row_of_prefill():
    c = gen.paged_case(2)
    g = c["geom"]
    pool = c["pool"].view(np.uint16)
    B = len(c["lens"])
    # prefill a 1-token chunk at position len-1 == decode
    q4 = c["q"].view(np.uint16)[:, None]
    pre = oracle.prefill_paged(pool, g, c["layer"], q4, c["bt"], c["lens"] - 1)
    dec = oracle.decode_paged(pool, g, c["layer"], c["q"].view(np.uint16), c["bt"], c["lens"])
    assert np.array_equal(pre[:, 0], dec)
    assert B == 3


def test_oracle_bad_table_detected():
    c = gen.paged_case(0)
    bt = c["bt"].copy()
    bt[1, 0] = c["geom"].num_pages + 5
    with pytest.raises(ValueError):
        oracle.decode_paged(c["pool"].view(np.uint16), c["geom"], c["layer"], c["q"].view(np.uint16), bt,
                            c["lens"])


# ---------------------------------------------------------------- append / copy

def test_oracle_append_scatter_rule():
    """Token t of sequence b lands at page bt[b][pos//16], slot pos%16, every head
    (src/kv_cache.cpp:94-121 with page indirection)."""
    rng = np.random.default_rng(3)
    g = oracle.Geom(3, 2, 64, 16, 12)
    pool = np.zeros(g.pool_shape(), np.uint16)
    B, T = 2, 5
    bt = np.array([[4, 7, 1], [9, 0, 11]], np.int32)
    pos = np.array([14, 30], np.int32)
    k = rng.integers(0, 65535, (B, T, 2, 64), dtype=np.uint16)
    v = rng.integers(0, 65535, (B, T, 2, 64), dtype=np.uint16)
    assert oracle.append_paged(pool, g, 2, k, v, bt, pos) == 0
    for b in range(B):
        for t in range(T):
            p = pos[b] + t
            for h in range(2):
                assert np.array_equal(pool[2, bt[b][p // 16], h, 0, p % 16], k[b, t, h])
                assert np.array_equal(pool[2, bt[b][p // 16], h, 1, p % 16], v[b, t, h])
    assert np.count_nonzero(pool[:2]) == 0  # other layers untouched
    # overflow past the table: reported, nothing written for that token
    pool2 = np.zeros_like(pool)
    assert oracle.append_paged(pool2, g, 0, k, v, bt, np.array([44, 0], np.int32)) == -1


def test_oracle_copy_and_remap():
    page = 64
    pool = np.arange(10 * page, dtype=np.uint32).astype(np.uint8).reshape(10, page)
    before = pool.copy()
    oracle.copy_pages(pool, 1, page, 0, 10, np.array([7, 8], np.int32), np.array([1, 2], np.int32))
    assert np.array_equal(pool[1], before[7]) and np.array_equal(pool[2], before[8])
    assert np.array_equal(pool[7], before[7])
    # three layer segments of 16 bytes per page (layer-major)
    seg = np.arange(3 * 10 * 16, dtype=np.uint32).astype(np.uint8).reshape(3, 10, 16)
    before = seg.copy()
    oracle.copy_pages(seg, 3, 16, 160, 10, np.array([9], np.int32), np.array([0], np.int32))
    assert np.array_equal(seg[:, 0], before[:, 9]) and np.array_equal(seg[:, 1:], before[:, 1:])
    bt = np.array([[7, 3, -1], [8, 9, 0]], np.int32)
    pm = np.arange(10, dtype=np.int32)
    pm[7], pm[8] = 1, 2
    assert np.array_equal(oracle.remap_block_tables(bt, pm), [[1, 3, -1], [2, 9, 0]])


# ---------------------------------------------------------------- allocator model

def test_model_allocate_all():
    """MemoryManagerTest.AllocateAll (tests/test_memory.cpp:122-146)."""
    m = AllocatorModel(1024, 4)
    ids = [m.allocate_block() for _ in range(4)]
    assert ids == [0, 1, 2, 3]
    assert m.blocks_in_use() == 4 and m.blocks_available() == 0
    assert m.allocate_block() == -1
    m.free_block(ids[0])
    assert m.blocks_available() == 1
    assert m.allocate_block() == 0


def test_model_swap_round_trip():
    """Swap out then in restores the bytes into the same id (cuda/memory.cu:152-191)."""
    m = AllocatorModel(1024, 4)
    i = m.allocate_block()
    data = bytes(range(256)) * 4
    assert m.swap_to_cpu(i, data)
    assert m.blocks_in_use() == 0
    ok, restored = m.swap_to_gpu(i)
    assert ok and restored == data and m.blocks_in_use() == 1


def test_model_swap_sequence_of_reference_test():
    """The call sequence of MemoryManagerTest.SwapToCPUAndBack
    (tests/test_memory.cpp:169-203) under the reference's implementation: the
    reused id is freed before swap-in, and free_block erases the swap copy of
    that id (cuda/memory.cu:137-143), so swap_to_gpu returns False although the
    test expects True.  The implementation, not the test's expectation, is what
    the library reproduces."""
    m = AllocatorModel(1024, 4)
    i = m.allocate_block()
    assert m.swap_to_cpu(i, b"x" * 1024)
    t = m.allocate_block()
    assert t == i
    m.free_block(t)
    ok, _ = m.swap_to_gpu(i)
    assert not ok and m.blocks_in_use() == 0


def test_model_invalid_ids():
    """MemoryManagerTest.InvalidBlockId (tests/test_memory.cpp:205-212)."""
    m = AllocatorModel(1024, 4)
    assert m.get_block_offset(-1) is None and m.get_block_offset(999) is None
    assert not m.swap_to_cpu(-1)
    assert not m.swap_to_gpu(999)[0]
    m.free_block(-3)  # ignored
    assert m.blocks_in_use() == 0


def test_model_compaction():
    m = AllocatorModel(1, 10)
    for _ in range(10):
        m.allocate_block()
    for i in (0, 2, 3, 6):
        m.free_block(i)
    pairs = m.compact_plan()
    assert pairs == [(9, 0), (8, 2), (7, 3)]
    assert [i for i, u in enumerate(m.in_use) if u] == list(range(6))


def test_oracle_rope_matches_reference_golden():
    """The oracle's RoPE restatement is bit-identical to the reference's own
    cpu_rope (tests/test_kernels.cu:697-716) on its three tests' inputs and on
    further head dims, positions and bases (tests/golden/rope_cases.npz)."""
    z = np.load(os.path.join(GOLD, "rope_cases.npz"))
    names = sorted({k.split("/")[0] for k in z.files})
    assert len(names) >= 9
    for name in names:
        d, pos = (int(v) for v in z[name + "/meta"])
        got = oracle.rope(z[name + "/x"][None], [pos], float(z[name + "/theta"]))[0]
        assert np.array_equal(got.view(np.uint32), z[name + "/y"].view(np.uint32)), name


def test_oracle_rope_properties():
    """Position 0 is the identity and every rotated pair keeps its norm (the
    reference's Position0_Identity and PreservesNorm tests)."""
    z = np.load(os.path.join(GOLD, "rope_cases.npz"))
    x0 = z["Position0_Identity/x"]
    assert np.array_equal(oracle.rope(x0[None], [0])[0], x0)
    x = z["PreservesNorm/x"]
    y = oracle.rope(x[None], [42])[0]
    n_in = np.hypot(x[0::2], x[1::2])
    n_out = np.hypot(y[0::2], y[1::2])
    assert np.abs(n_in - n_out).max() < 1e-4
