"""vulcan_b200 — B200-native paged KV-cache subsystem for VULCAN.

The product is libvulcan_kv.so (C ABI in include/vk_paged_kv.h): hand-written
sm_100a kernels for KV append, paged GQA decode with split-K, chunked prefill,
page copy and pinned-host swap.  This package binds it with ctypes and mirrors
the reference's KVCache / MemoryManager / launch_attention interfaces.
"""
from ._lib import VKError, load  # noqa: F401
from .paged_kv import (DecodePlan, Gather, KVCache, MemoryManager, PagedKVPool, default_scale,  # noqa: F401
                       launch_attention, remap_block_tables)

__all__ = ["VKError", "load", "DecodePlan", "Gather", "KVCache", "MemoryManager", "PagedKVPool", "default_scale",
           "launch_attention", "remap_block_tables"]
