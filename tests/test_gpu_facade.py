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
