"""CPU tests of the C-ABI library: it loads, exports every symbol the header
declares, and rejects bad arguments on the host without touching a GPU."""
import ctypes
import os
import subprocess

import pytest

from vulcan_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_library_exports_every_header_symbol():
    lib = _lib.load()
    declared = _lib.header_symbols()
    assert len(declared) >= 30
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing
    # the ctypes table binds exactly the declared functions
    assert sorted(_lib.SIGNATURES) == declared


def test_exported_symbols_are_c_linkage():
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    for s in _lib.header_symbols():
        assert s in exported, s


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.vk_version() >= 100
    for code, name in _lib.STATUS.items():
        assert lib.vk_status_string(code).decode() == name


def test_host_side_argument_checks():
    lib = _lib.load()
    handle = ctypes.c_void_p()
    assert lib.vk_pool_create(None, ctypes.byref(handle)) == _lib.VK_INVALID_ARG
    assert b"cfg" in lib.vk_last_error_string()
    cfg = _lib.VkPoolCfg(1, 1, 128, 16, 0, 0, 0)  # zero pages
    assert lib.vk_pool_create(ctypes.byref(cfg), ctypes.byref(handle)) == _lib.VK_INVALID_ARG
    cfg = _lib.VkPoolCfg(1, 1, 100, 16, 4, 0, 0)  # head_dim not a multiple of 8
    assert lib.vk_pool_create(ctypes.byref(cfg), ctypes.byref(handle)) == _lib.VK_INVALID_ARG
    cfg = _lib.VkPoolCfg(1, 1, 128, 16, 4, 0, 0)
    assert lib.vk_pool_create_in(ctypes.byref(cfg), ctypes.c_void_p(0x1001), 1 << 30,
                                 ctypes.byref(handle)) == _lib.VK_INVALID_ARG  # misaligned
    assert lib.vk_pool_create_in(ctypes.byref(cfg), ctypes.c_void_p(0x100000), 10,
                                 ctypes.byref(handle)) == _lib.VK_INVALID_ARG  # too small
    # NULL pools
    ids = (ctypes.c_int32 * 2)()
    assert lib.vk_alloc_pages(None, 1, ids) == _lib.VK_INVALID_ARG
    assert lib.vk_page_ptr(None, 0) is None
    assert lib.vk_pages_in_use(None) == 0
    assert lib.vk_decode(None, 0, None, None, None, 1, None, 1, 1, 16, 0.0, None, 0, None) == _lib.VK_INVALID_ARG
    assert lib.vk_set_decode_workers(None, 4) == _lib.VK_INVALID_ARG
    assert lib.vk_attention_f32(None, None, None, None, 1, 1, 4, 512, None) == _lib.VK_UNSUPPORTED
    assert lib.vk_attention_f32(None, None, None, None, 1, 1, 4, 8, None) == _lib.VK_INVALID_ARG
    assert lib.vk_attention_f32(None, None, None, None, 0, 1, 4, 8, None) == _lib.VK_OK  # empty
    assert lib.vk_remap_block_tables(None, 0, None, 0, None) == _lib.VK_OK
    assert lib.vk_remap_block_tables(None, 5, None, 3, None) == _lib.VK_INVALID_ARG


def test_product_does_not_reference_oracle():
    """The product library and package never load the oracle."""
    for root, _, files in os.walk(os.path.join(ROOT, "vulcan_b200")):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".cpp")):
                text = open(os.path.join(root, f)).read()
                assert "import oracle" not in text and "liboracle" not in text, f
    out = subprocess.run(["nm", "-D", "--undefined-only", _lib.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    assert "or_" not in " ".join(l.split()[-1] for l in out.splitlines() if l.strip() and l.split()[-1].startswith("or_"))


def test_build_flags_target_sm100a():
    from vulcan_b200 import build
    assert "arch=compute_100a,code=sm_100a" in build.NVCC_FLAGS


def test_fp8_pool_argument_checks():
    """vk_pool_create_fmt rejects bad formats and shapes on the host, before any
    device call: an unknown format, FP8 with head_dim other than 128 or pages of
    other than 16 tokens, and a byte-page pool with a format."""
    lib = _lib.load()
    handle = ctypes.c_void_p()
    cfg = _lib.VkPoolCfg(1, 1, 128, 16, 4, 0, 0)
    assert lib.vk_pool_create_fmt(ctypes.byref(cfg), 7, None, 0, ctypes.byref(handle)) == _lib.VK_INVALID_ARG
    assert b"kv_format" in lib.vk_last_error_string()
    cfg64 = _lib.VkPoolCfg(1, 1, 64, 16, 4, 0, 0)
    assert lib.vk_pool_create_fmt(ctypes.byref(cfg64), 1, None, 0, ctypes.byref(handle)) == _lib.VK_UNSUPPORTED
    cfg8 = _lib.VkPoolCfg(1, 1, 128, 8, 4, 0, 0)
    assert lib.vk_pool_create_fmt(ctypes.byref(cfg8), 1, None, 0, ctypes.byref(handle)) == _lib.VK_UNSUPPORTED
    raw = _lib.VkPoolCfg(0, 0, 0, 0, 4, 0, 4096)
    assert lib.vk_pool_create_fmt(ctypes.byref(raw), 1, None, 0, ctypes.byref(handle)) == _lib.VK_INVALID_ARG
    assert lib.vk_pool_create_fmt(ctypes.byref(cfg), 1, ctypes.c_void_p(0x1001), 1 << 30,
                                  ctypes.byref(handle)) == _lib.VK_INVALID_ARG  # misaligned caller memory
    assert lib.vk_pool_kv_format(None) == -1
