"""ctypes binding of libvulcan_kv.so (the C ABI declared in include/vk_paged_kv.h).

The library is the product: there is no Python or CPU fallback.  Loading fails
loudly when the shared library is missing and cannot be built.
"""
from __future__ import annotations

import ctypes
import os
import re

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libvulcan_kv.so")
HEADER = os.path.join(os.path.dirname(_PKG), "include", "vk_paged_kv.h")

c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_u32 = ctypes.c_uint32
c_u64 = ctypes.c_uint64
c_sz = ctypes.c_size_t
c_f32 = ctypes.c_float
vp = ctypes.c_void_p
i32p = ctypes.POINTER(ctypes.c_int32)
u32p = ctypes.POINTER(ctypes.c_uint32)


class VkPoolCfg(ctypes.Structure):
    _fields_ = [("num_layers", c_i32), ("num_kv_heads", c_i32), ("head_dim", c_i32),
                ("page_tokens", c_i32), ("num_pages", c_i32), ("device", c_i32),
                ("page_bytes", c_u64)]


# name -> (restype, argtypes)
SIGNATURES = {
    "vk_pool_create": (c_i32, [ctypes.POINTER(VkPoolCfg), ctypes.POINTER(vp)]),
    "vk_pool_create_in": (c_i32, [ctypes.POINTER(VkPoolCfg), vp, c_sz, ctypes.POINTER(vp)]),
    "vk_pool_destroy": (c_i32, [vp]),
    "vk_pool_base": (vp, [vp]),
    "vk_pool_page_bytes": (c_u64, [vp]),
    "vk_pool_create_fmt": (c_i32, [ctypes.POINTER(VkPoolCfg), c_i32, vp, c_sz, ctypes.POINTER(vp)]),
    "vk_pool_kv_format": (c_i32, [vp]),
    "vk_pool_num_pages": (c_i32, [vp]),
    "vk_pool_check": (c_i32, [vp, u32p]),
    "vk_alloc_pages": (c_i32, [vp, c_i32, i32p]),
    "vk_free_pages": (c_i32, [vp, i32p, c_i32]),
    "vk_page_ptr": (vp, [vp, c_i32]),
    "vk_pages_in_use": (c_i32, [vp]),
    "vk_pages_available": (c_i32, [vp]),
    "vk_allocated_bytes": (c_u64, [vp]),
    "vk_page_in_use": (c_i32, [vp, c_i32]),
    "vk_append": (c_i32, [vp, c_i32, vp, vp, vp, c_i32, vp, c_i32, c_i32, vp]),
    "vk_append_f32": (c_i32, [vp, c_i32, vp, vp, vp, c_i32, vp, c_i32, c_i32, vp]),
    "vk_decode_workspace_size": (c_sz, [vp, c_i32, c_i32, c_i32]),
    "vk_decode": (c_i32, [vp, c_i32, vp, vp, vp, c_i32, vp, c_i32, c_i32, c_i32, c_f32, vp, c_sz,
                          vp]),
    "vk_decode_static": (c_i32, [vp, c_i32, vp, vp, vp, c_i32, vp, c_i32, c_i32, c_i32, c_f32, vp]),
    "vk_decode_pages_per_split": (c_i32, [vp, c_i32, c_i32]),
    "vk_decode_plan_create": (c_i32, [vp, i32p, c_i32, c_i32, ctypes.POINTER(vp)]),
    "vk_decode_plan_destroy": (c_i32, [vp]),
    "vk_decode_plan_workspace_size": (c_sz, [vp]),
    "vk_decode_plan_upload": (c_i32, [vp, vp, c_sz, vp]),
    "vk_decode_plan_info": (c_i32, [vp, c_i32]),
    "vk_decode_plan_set_early_start": (c_i32, [vp, c_i32]),
    "vk_decode_run": (c_i32, [vp, vp, c_i32, vp, vp, vp, c_i32, vp, vp, c_f32, vp, vp]),
    "vk_set_decode_split": (c_i32, [vp, c_i32]),
    "vk_set_decode_workers": (c_i32, [vp, c_i32]),
    "vk_gather_create": (c_i32, [c_i32, c_i32, c_i32, c_u64, c_i32, ctypes.POINTER(vp)]),
    "vk_gather_destroy": (c_i32, [vp]),
    "vk_gather_release_peers": (c_i32, [vp]),
    "vk_gather_export": (c_i32, [vp, vp]),
    "vk_gather_import": (c_i32, [vp, c_i32, vp]),
    "vk_gather_import_local": (c_i32, [vp, c_i32, vp]),
    "vk_oproj_create": (c_i32, [c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, vp]),
    "vk_oproj_export": (c_i32, [vp, vp]),
    "vk_oproj_import": (c_i32, [vp, c_i32, vp]),
    "vk_oproj_import_local": (c_i32, [vp, c_i32, vp]),
    "vk_oproj_release_peers": (c_i32, [vp]),
    "vk_oproj_destroy": (c_i32, [vp]),
    "vk_oproj_splits": (c_i32, [vp]),
    "vk_oproj_run": (c_i32, [vp, vp, c_i32, vp, vp, c_i32, c_i32, vp]),
    "vk_oproj_check": (c_i32, [vp]),
    "vk_oproj_packed_bytes": (c_sz, [c_i32, c_i32]),
    "vk_oproj_pack_weight": (c_i32, [vp, c_i32, c_i32, c_i32, vp, vp]),
    "vk_oproj_pack_weight_t16": (c_i32, [vp, c_i32, c_i32, c_i32, vp, vp]),
    "vk_gather_buffer": (vp, [vp, c_i32]),
    "vk_decode_plan_gather_wait": (c_i32, [vp, vp, c_i32, vp]),
    "vk_gather_check": (c_i32, [vp]),
    "vk_decode_plan_set_gather": (c_i32, [vp, vp, c_i32, c_i32]),
    "vk_prefill": (c_i32, [vp, c_i32, vp, vp, vp, c_i32, vp, c_i32, c_i32, c_i32, c_f32, vp]),
    "vk_set_prefill_path": (c_i32, [vp, c_i32]),
    "vk_set_rope": (c_i32, [vp, c_f32]),
    "vk_copy_pages": (c_i32, [vp, vp, vp, c_i32, vp]),
    "vk_remap_block_tables": (c_i32, [vp, c_i64, vp, c_i32, vp]),
    "vk_compact_plan": (c_i32, [vp, i32p, i32p, c_i32, i32p]),
    "vk_swap_out": (c_i32, [vp, i32p, c_i32, vp, vp]),
    "vk_swap_in": (c_i32, [vp, vp, c_i32, i32p, vp]),
    "vk_swap_in_to": (c_i32, [vp, vp, i32p, c_i32, vp]),
    "vk_attention_f32": (c_i32, [vp, vp, vp, vp, c_i32, c_i32, c_i32, c_i32, vp]),
    "vk_last_error_string": (ctypes.c_char_p, []),
    "vk_status_string": (ctypes.c_char_p, [c_i32]),
    "vk_version": (c_i32, []),
}

STATUS = {0: "VK_OK", 1: "VK_INVALID_ARG", 2: "VK_OUT_OF_PAGES", 3: "VK_CUDA_ERROR",
          4: "VK_TIMEOUT", 5: "VK_BAD_BLOCK_TABLE", 6: "VK_NOT_FOUND", 7: "VK_UNSUPPORTED"}
VK_OK, VK_INVALID_ARG, VK_OUT_OF_PAGES, VK_CUDA_ERROR = 0, 1, 2, 3
VK_TIMEOUT, VK_BAD_BLOCK_TABLE, VK_NOT_FOUND, VK_UNSUPPORTED = 4, 5, 6, 7

_LIB = None


def header_symbols(path: str = HEADER):
    """Names of the functions declared in the C header."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(vk_[a-z0-9_]+)\s*\(", text)))


def load(build_if_missing: bool = True):
    """Loads (building first if needed) libvulcan_kv.so and declares signatures."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(LIB_PATH):
        if not build_if_missing:
            raise RuntimeError("libvulcan_kv.so is missing: run python -m vulcan_b200.build")
        from . import build as _build
        _build.build()
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


class VKError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        msg = load().vk_last_error_string().decode(errors="replace")
        super().__init__("%s%s: %s" % (what + ": " if what else "", STATUS.get(status, status), msg))


def check(status: int, what: str = "") -> None:
    if status != VK_OK:
        raise VKError(status, what)
