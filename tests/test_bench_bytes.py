"""CPU checks of the byte and FLOP accounting that bench.py's roofline
fractions are computed from (the algorithmic bytes of one decode layer)."""
import importlib.util
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_module", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_decode_bytes_fp16_and_fp8():
    b = _bench()
    ctx = np.array([0, 15, 2047], np.int64)  # lens 1, 16, 2048
    Hq, Hkv, D = 64, 8, 128
    f16 = b.algorithmic_bytes(ctx, Hq, Hkv, D, "fp16")
    f8 = b.algorithmic_bytes(ctx, Hq, Hkv, D, "fp8")
    tokens = int((ctx + 1).sum())
    table = 4 * (1 + 1 + 128)
    qo = 3 * 2 * Hq * D * 2
    # K+V per token and KV head: 512 B of fp16, 2*128 codes + 2 fp32 scales for FP8
    assert f16["decode"] == tokens * Hkv * 512 + qo + table
    assert f8["decode"] == tokens * Hkv * 264 + qo + table
    # the new token: fp16 K/V read, written in the page format
    assert f16["append"] == 3 * Hkv * (512 + 512)
    assert f8["append"] == 3 * Hkv * (512 + 264)
    assert f16["total"] == f16["decode"] + f16["append"]


def test_workload_70b_shape():
    b = _bench()
    wl = b.workload("70b")
    assert (wl["B"], wl["Hq"], wl["Hkv"], wl["D"], wl["L"]) == (64, 64, 8, 128, 80)
    assert wl["ctx"].min() + 1 >= 256 and wl["ctx"].max() + 1 <= 8192
