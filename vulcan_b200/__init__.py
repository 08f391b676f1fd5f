"""vulcan_b200 — B200-native paged KV-cache subsystem for VULCAN.

The product is libvulcan_kv.so (C ABI in include/vk_paged_kv.h): hand-written
sm_100a kernels for KV append, paged GQA decode with split-K, chunked prefill,
page copy, pinned-host swap and the output projection fused with its
reduce-scatter.  This package binds it with ctypes and mirrors
the reference's KVCache / MemoryManager / launch_attention interfaces.
"""
from ._lib import VKError, load  # noqa: F401
from .paged_kv import (DecodePlan, Gather, KVCache, MemoryManager, OutputProjection, PagedKVPool,  # noqa: F401
                       default_scale, launch_attention, remap_block_tables)

__all__ = ["VKError", "load", "DecodePlan", "Gather", "KVCache", "MemoryManager", "OutputProjection", "PagedKVPool",
           "default_scale", "launch_attention", "remap_block_tables"]
