"""Builds and runs the C++ facade tests (tests/cpp/test_facade.cpp): the
VULCAN-compatible vulcan::KVCache, vulcan::cuda::MemoryManager / GPUBuffer and
launch_attention, linked against libvulcan_kv.so, checked like the reference's
own gtests."""
import os
import subprocess

import pytest

from vulcan_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def build_facade_test(out_path):
    lib_dir = os.path.dirname(_lib.LIB_PATH)
    cmd = ["nvcc", "-std=c++17", "-O2", "-I" + os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "cpp", "test_facade.cpp"), "-o", out_path,
           "-L" + lib_dir, "-lvulcan_kv", "-Xlinker", "-rpath=" + lib_dir]
    subprocess.run(cmd, check=True, capture_output=True, text=True)


def test_facade_test_program_builds(tmp_path):
    """Compiles and links without a GPU."""
    _lib.load()
    build_facade_test(str(tmp_path / "test_facade"))
    assert os.path.exists(tmp_path / "test_facade")


@pytest.mark.gpu
def test_facade_cpp(tmp_path, cuda_ok):
    _lib.load()
    exe = str(tmp_path / "test_facade")
    build_facade_test(exe)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    print(r.stdout, r.stderr)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failures" in r.stdout


# ----------------------------------------------------------------- batched caller

def build_batch_test(out_path):
    lib_dir = os.path.dirname(_lib.LIB_PATH)
    cmd = ["nvcc", "-std=c++17", "-O2", "-I" + os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "cpp", "test_batch.cpp"), "-o", out_path,
           "-L" + lib_dir, "-lvulcan_kv", "-Xlinker", "-rpath=" + lib_dir]
    subprocess.run(cmd, check=True, capture_output=True, text=True)


def read_dump(path):
    """Records written by tests/cpp/test_batch.cpp: name -> numpy array."""
    import struct

    import numpy as np
    data = open(path, "rb").read()
    recs, off = {}, 0
    while off < len(data):
        (n,) = struct.unpack_from("<I", data, off)
        off += 4
        name = data[off:off + n].decode()
        off += n
        dt, nd = struct.unpack_from("<II", data, off)
        off += 8
        dims = struct.unpack_from("<%dq" % nd, data, off)
        off += 8 * nd
        dtype = np.dtype({0: np.float16, 1: np.int32, 2: np.uint8}[dt])
        cnt = int(np.prod(dims))
        recs[name] = np.frombuffer(data, dtype, cnt, off).reshape(dims)
        off += cnt * dtype.itemsize
    return recs


def test_batch_test_program_builds(tmp_path):
    """Compiles and links without a GPU."""
    _lib.load()
    build_batch_test(str(tmp_path / "test_batch"))
    assert os.path.exists(tmp_path / "test_batch")


@pytest.mark.gpu
@pytest.mark.parametrize("fmt,theta", [("fp16", 0.0), ("fp16", 10000.0), ("fp8", 0.0)])
def test_batched_caller_cpp(tmp_path, cuda_ok, fmt, theta):
    """vulcan::PagedAttention driven by an engine-shaped C++ program (prompt
    chunks, decode steps, a sequence released and another admitted into its
    pages, over 3 layers).  Every step is replayed through the CPU oracle from
    an empty pool: appended rows land where the oracle puts them (the final pool
    image byte-exact without RoPE) and every output is within the attention
    tolerance."""
    import numpy as np

    import oracle
    from tests.helpers import assert_close_attn
    _lib.load()
    exe, dump = str(tmp_path / "test_batch"), str(tmp_path / "batch.dump")
    build_batch_test(exe)
    r = subprocess.run([exe, dump, fmt, repr(theta)], capture_output=True, text=True, timeout=300)
    print(r.stdout, r.stderr)
    assert r.returncode == 0, r.stdout + r.stderr
    d = read_dump(dump)
    L, Hkv, D, NP, W, is8 = (int(x) for x in d["geom"])
    assert bool(is8) == (fmt == "fp8")
    g = oracle.Geom(L, Hkv, D, 16, NP)
    if fmt == "fp8":
        host = np.zeros((L, NP, Hkv, oracle.fp8_block_bytes(D)), np.uint8)
    else:
        host = np.zeros(g.pool_shape(), np.float16)
    steps = int(d["steps"][0])
    assert steps == 8
    for s in range(steps):
        pre = "s%d." % s
        pos, bt = d[pre + "pos"], np.ascontiguousarray(d[pre + "bt"])
        for l in range(L):
            lp = pre + "l%d." % l
            q, k, v, out = (np.ascontiguousarray(d[lp + x]) for x in ("q", "k", "v", "out"))
            B, T = q.shape[:2]
            qpos = pos[:, None] + np.arange(T, dtype=np.int32)[None, :]
            if theta:
                k = oracle.rope(k.astype(np.float32), qpos, theta).astype(np.float16)
                q = oracle.rope(q.astype(np.float32), qpos, theta).astype(np.float16)
            if fmt == "fp8":
                assert oracle.append_fp8(host, g, l, k, v, bt, pos) == 0
                ref = (oracle.decode_fp8(host, g, l, q[:, 0], bt, pos + 1)[:, None] if T == 1 else
                       oracle.prefill_fp8(host, g, l, q, bt, pos))
            else:
                u16 = host.view(np.uint16)
                assert oracle.append_paged(u16, g, l, k.view(np.uint16), v.view(np.uint16), bt, pos) == 0
                ref = (oracle.decode_paged(u16, g, l, np.ascontiguousarray(q[:, 0]).view(np.uint16), bt,
                                           pos + 1)[:, None] if T == 1 else
                       oracle.prefill_paged(u16, g, l, q.view(np.uint16), bt, pos, nthreads=8))
            assert_close_attn(out.astype(np.float32), ref, "%s theta %g step %d layer %d (T=%d)" % (fmt, theta, s, l, T))
    if not theta:
        got = d["pool"]
        assert np.array_equal(got, host.reshape(-1).view(np.uint8)), "final pool image"
