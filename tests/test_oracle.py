"""CPU tests of the oracle: pinned against the reference's golden vectors and
known-answer properties, plus the allocator model against the reference's
allocator tests.  No GPU needed."""
import os

import numpy as np
import torch
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


# ---------------------------------------------------------------- FP8 pages

def test_e4m3_encoder_matches_torch():
    """The oracle's E4M3 encoder (nearest even) and decoder agree with torch's
    float8_e4m3fn on every code and on in-range values including ties."""
    rng = np.random.default_rng(90)
    steps = oracle.e4m3_decode(np.arange(256, dtype=np.uint8))
    fin = np.isfinite(steps)
    vals = np.unique(steps[fin]).astype(np.float32)
    mids = ((vals[:-1] + vals[1:]) / 2).astype(np.float32)  # ties between neighbouring codes
    x = np.concatenate([vals, mids,
                        (rng.standard_normal(50000) * 40).astype(np.float32),
                        np.float32(2.0) ** rng.integers(-12, 9, 5000).astype(np.float32),
                        np.array([0.0, -0.0, 2 ** -10, 3 * 2 ** -11, 1e-30], np.float32)])
    x = x[np.abs(x) <= 448]
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(oracle.e4m3_encode(x), want)
    td = torch.from_numpy(np.arange(256, dtype=np.uint8)).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(steps), np.isnan(td))
    assert np.array_equal(steps[fin], td[fin])
    # saturation: finite values past 448 clamp to +-448 (code 0x7E / 0xFE)
    assert list(oracle.e4m3_encode(np.array([449, 464, 470, 1e9, -500], np.float32))) == [0x7E] * 4 + [0xFE]


def test_fp8_group_rule():
    """ADR-003's symmetric group rule with qmax 448: the largest element maps to
    +-448, every element is within half a step of code * scale, zero rows give
    scale 0."""
    rng = np.random.default_rng(91)
    for _ in range(50):
        x = (rng.standard_normal(128) * rng.uniform(0.01, 10)).astype(np.float32)
        codes, scale = oracle.fp8_quant_row(x)
        assert scale == np.float32(np.abs(x).max()) / np.float32(448.0)
        deq = oracle.e4m3_decode(codes).astype(np.float64) * scale
        i = np.argmax(np.abs(x))
        assert abs(oracle.e4m3_decode(codes[i:i + 1])[0]) == 448.0
        y = np.abs(x.astype(np.float64)) / scale
        half = np.where(y < 2 ** -6, 2.0 ** -10, 2.0 ** (np.floor(np.log2(np.maximum(y, 2 ** -6))) - 4))
        assert (np.abs(deq - x) <= half * scale * 1.0001 + 1e-12).all()
    codes, scale = oracle.fp8_quant_row(np.zeros(128, np.float32))
    assert scale == 0 and not codes.any()


def test_fp8_append_dequant_round_trip():
    """Append then dequantise returns code * scale at each token's slot for K and V
    (the block layout functions are mutually consistent) and leaves other slots."""
    rng = np.random.default_rng(92)
    g = oracle.Geom(2, 2, 128, 16, 6)
    bb = oracle.fp8_block_bytes(128)
    pool = rng.integers(0, 256, size=(g.L, g.num_pages, g.Hkv, bb), dtype=np.uint8)
    before = pool.copy()
    bt = np.array([[3, 1, 4]], np.int32)
    T = 20
    k = (rng.standard_normal((1, T, 2, 128)) * 0.5).astype(np.float32)
    v = (rng.standard_normal((1, T, 2, 128)) * 0.5).astype(np.float32)
    assert oracle.append_fp8(pool, g, 1, k, v, bt, np.array([9], np.int32)) == 0
    deq = oracle.dequant_fp8(pool, g)
    for t in range(T):
        pos = 9 + t
        page, slot = bt[0, pos // 16], pos % 16
        for h in range(2):
            for kv, x in ((0, k), (1, v)):
                codes, scale = oracle.fp8_quant_row(x[0, t, h])
                want = oracle.e4m3_decode(codes) * scale
                assert np.array_equal(deq[1, page, h, kv, slot], want)
    untouched = [p for p in range(g.num_pages) if p not in (3, 1)]
    assert np.array_equal(pool[:, untouched], before[:, untouched])
    assert np.array_equal(pool[0], before[0])


def test_fp8_oracle_prefill_last_row_is_decode():
    """The FP8 oracle's prefill and decode agree: the last row of a chunk that
    ends a sequence is that sequence's decode row (same keys, same query)."""
    rng = np.random.default_rng(94)
    Hq, Hkv, D, T = 4, 2, 128, 21
    pos = np.array([0, 37, 250], np.int32)
    lens = pos + T
    g = oracle.Geom(1, Hkv, D, 16, int(((lens + 15) // 16).sum()) + 2)
    perm = rng.permutation(g.num_pages).astype(np.int32)
    width = int(((lens + 15) // 16).max())
    bt = np.full((len(lens), width), -1, np.int32)
    off = 0
    for b, n in enumerate(lens):
        k = (n + 15) // 16
        bt[b, :k] = perm[off:off + k]
        off += k
    pool = np.zeros((1, g.num_pages, Hkv, oracle.fp8_block_bytes(D)), np.uint8)
    for b, n in enumerate(lens):
        kv = (rng.standard_normal((2, 1, n, Hkv, D)) * 0.5).astype(np.float32)
        assert oracle.append_fp8(pool, g, 0, kv[0], kv[1], bt[b:b + 1], np.zeros(1, np.int32)) == 0
    q = (rng.standard_normal((len(lens), T, Hq, D)) * 0.5).astype(np.float32)
    pre = oracle.prefill_fp8(pool, g, 0, q, bt, pos)
    dec = oracle.decode_fp8(pool, g, 0, q[:, -1], bt, lens)
    assert np.allclose(pre[:, -1], dec, rtol=1e-12, atol=1e-12)


def test_oracle_matmul_contract():
    """oracle.matmul restates launch_matmul (cuda/matmul.cu:42-103): C = A @ B,
    fp32, one in-order fused multiply-add chain per element (checked against an
    explicit fmaf-order loop on a small case and float64 on a larger one)."""
    from fractions import Fraction

    def fma32(x, y, z):  # x*y + z rounded once to the nearest float32 (ties to even)
        exact = Fraction(float(x)) * Fraction(float(y)) + Fraction(float(z))
        c = np.float32(float(exact))
        best = min((c, np.nextafter(c, np.float32(np.inf)), np.nextafter(c, np.float32(-np.inf))),
                   key=lambda v: (abs(Fraction(float(v)) - exact), int(v.view(np.uint32)) & 1))
        return np.float32(best)

    rng = np.random.default_rng(11)
    a = rng.standard_normal((3, 5)).astype(np.float32)
    b = rng.standard_normal((5, 4)).astype(np.float32)
    c = oracle.matmul(a, b)
    for i in range(3):
        for j in range(4):
            s = np.float32(0)
            for k in range(5):
                s = fma32(a[i, k], b[k, j], s)
            assert c[i, j] == s
    a = (rng.standard_normal((17, 700)) * 0.5).astype(np.float32)
    b = (rng.standard_normal((700, 33)) * 0.02).astype(np.float32)
    c = oracle.matmul(a, b)
    assert np.abs(c - a.astype(np.float64) @ b.astype(np.float64)).max() < 1e-5
