"""Generates the golden fixtures in this directory from the reference's own code.

Run from the repository root after ``make -C oracle all ref`` (which compiles
the reference's golden attention from its sources into oracle/_ref):

    python tests/golden/make_golden.py

Outputs:
  ref_attention_cases.npz  The six attention tests of the reference
      (tests/test_attention.cu:107-264): inputs drawn with the reference's own
      ``random_floats`` (std::mt19937 + uniform_real_distribution, same seeds
      and ranges) and outputs of its ``cpu_attention``.
  paged_decode_cases.npz   Paged fp16 GQA decode cases (edge lengths 1, 15,
      16, 17, 33, 100, 257; G = 1, 2, 4, 8): pool, block tables, lengths and
      the reference ``cpu_attention`` last row over the gathered keys.
  config1_decode.npz       The Llama-2-7B single-layer decode workload (32/32
      heads, D=128, context 512 + 1 appended token, 64-page permuted table):
      seed, SHA-256 of the regenerated inputs and the reference output.
  rope_cases.npz           The reference's three RoPE tests
      (tests/test_kernels.cu:718-780: inputs from its ``random_floats`` with
      the same seeds, ranges, head dims and positions) and further positions
      and head dims (64, 128, 256; positions up to 8191), each with the output
      of its ``cpu_rope``.
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402
from tests.golden import gen  # noqa: E402

# name, head_dim, lo, hi, seed, position, theta -- tests/test_kernels.cu:718-780 first
ROPE_CASES = [
    ("Position0_Identity", 64, -1.0, 1.0, 1100, 0, 10000.0),
    ("PreservesNorm", 128, -2.0, 2.0, 1200, 42, 10000.0),
    ("AgainstCPUReference", 128, -1.0, 1.0, 1300, 100, 10000.0),
    ("d64_pos1", 64, -1.0, 1.0, 1400, 1, 10000.0),
    ("d128_pos511", 128, -1.0, 1.0, 1401, 511, 10000.0),
    ("d128_pos4095", 128, -0.5, 0.5, 1402, 4095, 10000.0),
    ("d128_pos8191", 128, -1.0, 1.0, 1403, 8191, 10000.0),
    ("d256_pos2048", 256, -1.0, 1.0, 1404, 2048, 10000.0),
    ("d128_pos777_theta500k", 128, -1.0, 1.0, 1405, 777, 500000.0),
]

REF_CASES = [
    # name, B, H, S, D, lo, hi, seeds (q, k, v)  -- tests/test_attention.cu
    ("SingleHead_SmallSeq", 1, 1, 4, 8, -1.0, 1.0, (2000, 2001, 2002)),
    ("MultiHead_4Heads", 1, 4, 8, 16, -0.5, 0.5, (2010, 2011, 2012)),
    ("CausalMask_FirstRow", 1, 1, 4, 4, -1.0, 1.0, (2020, 2021, 2022)),
    ("LongerSequence_32", 1, 2, 32, 32, -0.3, 0.3, (2030, 2031, 2032)),
    ("Batched_2x4Heads", 2, 4, 8, 16, -0.5, 0.5, (2040, 2041, 2042)),
    ("OutputSumMatchesV", 1, 1, 8, 8, -1.0, 1.0, (2050, 2051, 2052)),
]


def ref_decode_rows(pool, g, layer, q, bt, lens):
    """Reference cpu_attention run on each (sequence, head)'s gathered keys; the
    last row is the decode output."""
    B, Hq, D = q.shape
    G = Hq // g.Hkv
    out = np.zeros((B, Hq, D), np.float32)
    for b in range(B):
        n = int(lens[b])
        if n == 0:
            continue
        idx = np.arange(n)
        pages = bt[b][idx // g.P]
        for h in range(Hq):
            kv = h // G
            K = pool[layer, pages, kv, 0, idx % g.P].astype(np.float32)
            V = pool[layer, pages, kv, 1, idx % g.P].astype(np.float32)
            Q = np.zeros((n, D), np.float32)
            Q[n - 1] = q[b, h].astype(np.float32)
            out[b, h] = oracle.ref_attention_causal(Q[None, None], K[None, None], V[None, None])[0, 0, n - 1]
    return out


def main():
    if oracle.ref_lib() is None:
        raise SystemExit("build oracle/_ref first: make -C oracle all ref")
    arrays = {}
    for name, B, H, S, D, lo, hi, seeds in REF_CASES:
        n = B * H * S * D
        q, k, v = (oracle.ref_random_floats(n, lo, hi, s).reshape(B, H, S, D) for s in seeds)
        arrays[name + "/q"], arrays[name + "/k"], arrays[name + "/v"] = q, k, v
        arrays[name + "/o"] = oracle.ref_attention_causal(q, k, v)
    np.savez_compressed(os.path.join(HERE, "ref_attention_cases.npz"), **arrays)

    arrays = {}
    for ci, (Hq, Hkv, lens) in enumerate(gen.PAGED_CASES):
        c = gen.paged_case(ci)
        g = c["geom"]
        out = ref_decode_rows(c["pool"], g, c["layer"], c["q"], c["bt"], c["lens"])
        pre = "case%d/" % ci
        arrays[pre + "pool"] = c["pool"].view(np.uint16)
        arrays[pre + "q"] = c["q"].view(np.uint16)
        arrays[pre + "bt"] = c["bt"]
        arrays[pre + "lens"] = c["lens"]
        arrays[pre + "geom"] = np.array([g.L, g.Hkv, g.D, g.P, g.num_pages, c["layer"]], np.int32)
        arrays[pre + "out"] = out
    np.savez_compressed(os.path.join(HERE, "paged_decode_cases.npz"), **arrays)

    c = gen.config1_case()
    g = c["geom"]
    out = ref_decode_rows(c["pool"], g, 0, c["q"], c["bt"], c["lens"])
    np.savez_compressed(os.path.join(HERE, "config1_decode.npz"), seed=np.int64(gen.CONFIG1_SEED),
                        sha256=np.frombuffer(gen.digest(c).encode(), np.uint8), out=out)
    arrays = {}
    for name, d, lo, hi, seed, pos, theta in ROPE_CASES:
        x = oracle.ref_kernels_random_floats(d, lo, hi, seed)
        arrays[name + "/x"] = x
        arrays[name + "/meta"] = np.array([d, pos], np.int32)
        arrays[name + "/theta"] = np.float32(theta)
        arrays[name + "/y"] = oracle.ref_rope(x, pos, theta)
    np.savez_compressed(os.path.join(HERE, "rope_cases.npz"), **arrays)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
