"""Python mirror of VULCAN's KV-cache interfaces over the B200 C ABI.

Three layers, all calling libvulcan_kv.so (no CPU path):

* ``PagedKVPool`` — the batched paged API: page allocator, append (K1),
  paged GQA decode with split-K (K2), chunked prefill (K3), page copy (K4) and
  pinned-host swap (K5).  Tensors are torch tensors; work is enqueued on the
  current CUDA stream.
* ``MemoryManager`` — the reference's ``vulcan::cuda::MemoryManager``
  (include/cuda/memory.h:87-128): byte pages, ``allocate_block`` returning -1
  when full, ``get_block_ptr`` returning None for a bad id, ``swap_to_cpu`` /
  ``swap_to_gpu`` returning False on failure.
* ``KVCache`` — the reference's ``vulcan::KVCache`` (include/vulcan/kv_cache.h:
  34-92) for one sequence: ``append(layer, k_new, v_new, start_pos,
  num_tokens)`` with fp32 inputs, length bookkeeping, ``memory_usage``.  Pages
  are fp16 and taken on demand.

``launch_attention`` mirrors ``vulcan::cuda::launch_attention``
(include/cuda/kernels.h:99-101) on contiguous fp32 tensors.
"""
from __future__ import annotations

import ctypes
import math
import sys
from typing import List, Optional, Sequence

import torch

from . import _lib
from ._lib import VKError, check

PAGE_TOKENS = 16
KV_FORMATS = {"fp16": 0, "fp8": 1}  # page formats (VK_KV_FP16, VK_KV_FP8)


def _stream(stream=None) -> int:
    if stream is None:
        stream = torch.cuda.current_stream()
    return int(stream.cuda_stream) if hasattr(stream, "cuda_stream") else int(stream)


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _i32_array(ids: Sequence[int]):
    arr = (ctypes.c_int32 * max(1, len(ids)))(*ids)
    return arr


def _need(t: torch.Tensor, dtype, name: str, device=True):
    if t.dtype != dtype:
        raise TypeError("%s must be %s, got %s" % (name, dtype, t.dtype))
    if device and not t.is_cuda:
        raise TypeError("%s must be a CUDA tensor" % name)
    if not t.is_contiguous():
        raise ValueError("%s must be contiguous" % name)


class PagedKVPool:
    """A paged fp16 KV pool for ``num_layers`` layers and ``num_kv_heads`` heads.

    Layer-major fp16 layout (see include/vk_paged_kv.h):
    ``[num_layers, num_pages, num_kv_heads, 2 (K,V), page_tokens, head_dim]``,
    so one layer's pages form one contiguous region.  The pool storage is a
    torch allocation handed to the library (``vk_pool_create_in``) unless
    ``own_memory`` is set.
    """

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, num_pages: int,
                 page_tokens: int = PAGE_TOKENS, device=None, own_memory: bool = False,
                 page_bytes: int = 0, zero: bool = True, kv_format: str = "fp16"):
        self._lib = _lib.load()
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                           (device.index if isinstance(device, torch.device) else int(device)))
        self.device = dev
        self.num_layers, self.num_kv_heads, self.head_dim = num_layers, num_kv_heads, head_dim
        self.page_tokens, self.num_pages = page_tokens, num_pages
        if kv_format not in KV_FORMATS:
            raise ValueError("kv_format must be one of %s" % sorted(KV_FORMATS))
        self.kv_format = kv_format
        fmt = KV_FORMATS[kv_format]
        cfg = _lib.VkPoolCfg(num_layers, num_kv_heads, head_dim, page_tokens, num_pages, dev.index,
                             page_bytes)
        self.kv = page_bytes == 0
        # bytes of one (layer, page, head) block: fp16 K and V rows, or FP8 codes + 32 fp32 scales
        self.block_bytes = (2 * page_tokens * head_dim + 8 * page_tokens if kv_format == "fp8"
                            else 2 * page_tokens * head_dim * 2)
        self.page_bytes = page_bytes if page_bytes else num_layers * num_kv_heads * self.block_bytes
        handle = ctypes.c_void_p()
        self.storage = None
        with torch.cuda.device(dev):
            if own_memory:
                check(self._lib.vk_pool_create_fmt(ctypes.byref(cfg), fmt, None, 0, ctypes.byref(handle))
                      if fmt else self._lib.vk_pool_create(ctypes.byref(cfg), ctypes.byref(handle)), "vk_pool_create")
            else:
                nbytes = self.page_bytes * num_pages
                self.storage = (torch.zeros if zero else torch.empty)(nbytes, dtype=torch.uint8, device=dev)
                check(self._lib.vk_pool_create_fmt(ctypes.byref(cfg), fmt, _ptr(self.storage), nbytes,
                                                   ctypes.byref(handle))
                      if fmt else self._lib.vk_pool_create_in(ctypes.byref(cfg), _ptr(self.storage), nbytes,
                                                              ctypes.byref(handle)), "vk_pool_create_in")
        if self.kv and self._lib.vk_pool_kv_format(handle) != fmt:
            raise RuntimeError("library reports another page format than requested")
        if self._lib.vk_pool_page_bytes(handle) != self.page_bytes:
            raise RuntimeError("library reports %d bytes per page, expected %d"
                               % (self._lib.vk_pool_page_bytes(handle), self.page_bytes))
        self.handle = handle
        self._ws = None

    # ------------------------------------------------------------------ views
    def kv_view(self) -> torch.Tensor:
        """fp16 view [L, num_pages, Hkv, 2, page_tokens, head_dim] of the pool."""
        if self.storage is None or not self.kv or self.kv_format != "fp16":
            raise RuntimeError("kv_view needs a torch-backed fp16 KV pool")
        return self.storage.view(torch.float16).view(self.num_layers, self.num_pages, self.num_kv_heads,
                                                     2, self.page_tokens, self.head_dim)

    def block_view(self) -> torch.Tensor:
        """uint8 view [L, num_pages, Hkv, block_bytes] of the pool (either format)."""
        if self.storage is None or not self.kv:
            raise RuntimeError("block_view needs a torch-backed KV pool")
        return self.storage.view(self.num_layers, self.num_pages, self.num_kv_heads, self.block_bytes)

    @property
    def base_ptr(self) -> int:
        return self._lib.vk_pool_base(self.handle) or 0

    # -------------------------------------------------------------- allocator
    def alloc(self, n: int) -> List[int]:
        ids = (ctypes.c_int32 * max(1, n))()
        check(self._lib.vk_alloc_pages(self.handle, n, ids), "vk_alloc_pages")
        return list(ids[:n])

    def free(self, ids: Sequence[int]) -> None:
        check(self._lib.vk_free_pages(self.handle, _i32_array(ids), len(ids)), "vk_free_pages")

    def page_ptr(self, page_id: int) -> Optional[int]:
        return self._lib.vk_page_ptr(self.handle, page_id)

    def pages_in_use(self) -> int:
        return self._lib.vk_pages_in_use(self.handle)

    def pages_available(self) -> int:
        return self._lib.vk_pages_available(self.handle)

    def allocated_bytes(self) -> int:
        return self._lib.vk_allocated_bytes(self.handle)

    def page_in_use(self, page_id: int) -> int:
        return self._lib.vk_page_in_use(self.handle, page_id)

    def check(self) -> int:
        """Synchronises, reads and clears the device error word; raises on error."""
        bits = ctypes.c_uint32(0)
        st = self._lib.vk_pool_check(self.handle, ctypes.byref(bits))
        if st != _lib.VK_OK:
            raise VKError(st, "device error bits 0x%x" % bits.value)
        return bits.value

    def error_bits(self) -> int:
        """Like check() but returns the bits instead of raising."""
        bits = ctypes.c_uint32(0)
        self._lib.vk_pool_check(self.handle, ctypes.byref(bits))
        return bits.value

    # ----------------------------------------------------------------- kernels
    def append(self, layer: int, k_new: torch.Tensor, v_new: torch.Tensor, block_tables: torch.Tensor,
               positions: torch.Tensor, stream=None) -> None:
        """k_new/v_new: [B, T, Hkv, D] fp16 (or fp32); block_tables [B, W] int32; positions [B] int32."""
        B, T = k_new.shape[0], k_new.shape[1]
        _need(block_tables, torch.int32, "block_tables")
        _need(positions, torch.int32, "positions")
        if k_new.dtype == torch.float32:
            fn = self._lib.vk_append_f32
        else:
            _need(k_new, torch.float16, "k_new")
            fn = self._lib.vk_append
        _need(v_new, k_new.dtype, "v_new")
        check(fn(self.handle, layer, _ptr(k_new), _ptr(v_new), _ptr(block_tables), block_tables.shape[1],
                 _ptr(positions), B, T, _stream(stream)), "vk_append")

    def workspace_size(self, batch: int, num_q_heads: int, max_seq_len: int) -> int:
        return self._lib.vk_decode_workspace_size(self.handle, batch, num_q_heads, max_seq_len)

    def pages_per_split(self, batch: int, max_seq_len: int) -> int:
        return self._lib.vk_decode_pages_per_split(self.handle, batch, max_seq_len)

    def set_split(self, pages_per_split: int) -> None:
        check(self._lib.vk_set_decode_split(self.handle, pages_per_split), "vk_set_decode_split")

    def set_rope(self, theta_base: float) -> None:
        """Fused RoPE in append, decode and prefill (see vk_set_rope); 0 = off."""
        check(self._lib.vk_set_rope(self.handle, float(theta_base)), "vk_set_rope")

    def set_plan_workers(self, max_workers: int) -> None:
        """Caps the workers of plans made afterwards (0 = one per resident warp)."""
        check(self._lib.vk_set_decode_workers(self.handle, max_workers), "vk_set_decode_workers")

    def workspace(self, batch: int, num_q_heads: int, max_seq_len: int) -> Optional[torch.Tensor]:
        need = self.workspace_size(batch, num_q_heads, max_seq_len)
        if need == 0:
            return None
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._ws

    def decode(self, layer: int, q: torch.Tensor, block_tables: torch.Tensor, seq_lens: torch.Tensor,
               max_seq_len: int, out: Optional[torch.Tensor] = None, scale: float = 0.0,
               workspace: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
        """q: [B, Hq, D] fp16; seq_lens [B] int32 (tokens to attend); returns [B, Hq, D] fp16."""
        _need(q, torch.float16, "q")
        _need(block_tables, torch.int32, "block_tables")
        _need(seq_lens, torch.int32, "seq_lens")
        B, Hq, _ = q.shape
        if out is None:
            out = torch.empty_like(q)
        if workspace is None:
            workspace = self.workspace(B, Hq, max_seq_len)
        ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
        check(self._lib.vk_decode(self.handle, layer, _ptr(q), _ptr(out), _ptr(block_tables),
                                  block_tables.shape[1], _ptr(seq_lens), B, Hq, max_seq_len, float(scale),
                                  _ptr(workspace), ws_bytes, _stream(stream)), "vk_decode")
        return out

    def plan(self, seq_lens: Sequence[int], num_q_heads: int,
             workspace: Optional[torch.Tensor] = None) -> "DecodePlan":
        """Host-side balanced schedule for one decode step (lengths include the new token)."""
        return DecodePlan(self, seq_lens, num_q_heads, workspace)

    def prefill(self, layer: int, q: torch.Tensor, block_tables: torch.Tensor, positions: torch.Tensor,
                out: Optional[torch.Tensor] = None, scale: float = 0.0, stream=None) -> torch.Tensor:
        """q: [B, T, Hq, D] fp16; positions [B] int32 (chunk start); returns [B, T, Hq, D] fp16."""
        _need(q, torch.float16, "q")
        _need(block_tables, torch.int32, "block_tables")
        _need(positions, torch.int32, "positions")
        B, T, Hq, _ = q.shape
        if out is None:
            out = torch.empty_like(q)
        check(self._lib.vk_prefill(self.handle, layer, _ptr(q), _ptr(out), _ptr(block_tables),
                                   block_tables.shape[1], _ptr(positions), B, T, Hq, float(scale),
                                   _stream(stream)), "vk_prefill")
        return out

    def set_prefill_path(self, path: int) -> None:
        """0 automatic, 1 mma.sync kernel, 2 tcgen05/TMEM kernel."""
        check(self._lib.vk_set_prefill_path(self.handle, path), "vk_set_prefill_path")

    def copy_pages(self, src_ids: torch.Tensor, dst_ids: torch.Tensor, stream=None) -> None:
        _need(src_ids, torch.int32, "src_ids")
        _need(dst_ids, torch.int32, "dst_ids")
        check(self._lib.vk_copy_pages(self.handle, _ptr(src_ids), _ptr(dst_ids), src_ids.numel(),
                                      _stream(stream)), "vk_copy_pages")

    def compact_plan(self, cap: Optional[int] = None):
        cap = self.num_pages if cap is None else cap
        src = (ctypes.c_int32 * max(1, cap))()
        dst = (ctypes.c_int32 * max(1, cap))()
        n = ctypes.c_int32(0)
        check(self._lib.vk_compact_plan(self.handle, src, dst, cap, ctypes.byref(n)), "vk_compact_plan")
        return list(src[:n.value]), list(dst[:n.value])

    def swap_out(self, ids: Sequence[int], host: torch.Tensor, stream=None) -> None:
        """Copies pages ``ids`` into pinned ``host`` (uint8, >= len(ids)*page_bytes) and frees them."""
        check(self._lib.vk_swap_out(self.handle, _i32_array(ids), len(ids), _ptr(host), _stream(stream)),
              "vk_swap_out")

    def swap_in(self, host: torch.Tensor, n: int, stream=None) -> List[int]:
        ids = (ctypes.c_int32 * max(1, n))()
        check(self._lib.vk_swap_in(self.handle, _ptr(host), n, ids, _stream(stream)), "vk_swap_in")
        return list(ids[:n])

    def swap_in_to(self, host: torch.Tensor, ids: Sequence[int], stream=None) -> None:
        check(self._lib.vk_swap_in_to(self.handle, _ptr(host), _i32_array(ids), len(ids), _stream(stream)),
              "vk_swap_in_to")

    def close(self) -> None:
        if getattr(self, "handle", None) is not None and self.handle.value:
            self._lib.vk_pool_destroy(self.handle)
            self.handle = ctypes.c_void_p()
        self.storage = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DecodePlan:
    """vk_decode_plan: built on the host from the step's lengths, uploaded once
    into a device workspace, then run once per layer (vk_decode_run)."""

    def __init__(self, pool: PagedKVPool, seq_lens: Sequence[int], num_q_heads: int,
                 workspace: Optional[torch.Tensor] = None):
        self.pool = pool
        self._lib = pool._lib
        lens = [int(x) for x in seq_lens]
        self.batch, self.num_q_heads = len(lens), num_q_heads
        h = ctypes.c_void_p()
        check(self._lib.vk_decode_plan_create(pool.handle, _i32_array(lens), len(lens), num_q_heads,
                                              ctypes.byref(h)), "vk_decode_plan_create")
        self.handle = h
        nbytes = max(256, self._lib.vk_decode_plan_workspace_size(h))
        if workspace is not None and workspace.numel() >= nbytes and workspace.data_ptr() % 256 == 0:
            self.workspace = workspace
        else:
            self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=pool.device)
        self.uploaded = False

    def info(self, what: int) -> int:
        return self._lib.vk_decode_plan_info(self.handle, what)

    def set_early_start(self, enable: bool = True) -> None:
        """Programmatic dependent launch for back-to-back runs (see the C header)."""
        check(self._lib.vk_decode_plan_set_early_start(self.handle, int(bool(enable))),
              "vk_decode_plan_set_early_start")

    def set_gather(self, gather: Optional["Gather"], slot_base: int = 0, wait_prev: bool = True) -> None:
        """Binds a fused output gather (see Gather); a run of layer l then writes
        every rank's receive slice of slot ``(slot_base + l) % slots`` and may
        leave ``out`` as None.  ``wait_prev``: wait for the previous slot first."""
        check(self._lib.vk_decode_plan_set_gather(self.handle, gather.handle if gather else None,
                                                  int(slot_base), int(bool(wait_prev))),
              "vk_decode_plan_set_gather")
        self.gather = gather

    def gather_wait(self, layer: int, stream=None) -> None:
        """Raises this rank's flags for layer's slot (its run precedes on the
        stream) and makes the stream wait for every rank's slice of it."""
        check(self._lib.vk_decode_plan_gather_wait(self.handle, _ptr(self.workspace), layer, _stream(stream)),
              "vk_decode_plan_gather_wait")

    @property
    def workers(self) -> int:
        return self.info(0)

    @property
    def ctas(self) -> int:
        return self.info(1)

    def upload(self, stream=None) -> None:
        check(self._lib.vk_decode_plan_upload(self.handle, _ptr(self.workspace), self.workspace.numel(),
                                              _stream(stream)), "vk_decode_plan_upload")
        self.uploaded = True

    def run(self, layer: int, q: torch.Tensor, block_tables: torch.Tensor, out: Optional[torch.Tensor] = None,
            k_new: Optional[torch.Tensor] = None, v_new: Optional[torch.Tensor] = None, scale: float = 0.0,
            stream=None) -> torch.Tensor:
        """q [B, Hq, D] fp16; optional k_new/v_new [B, Hkv, D] fp16 appended at position len-1."""
        if not self.uploaded:
            self.upload(stream)
        _need(q, torch.float16, "q")
        _need(block_tables, torch.int32, "block_tables")
        if k_new is not None:
            _need(k_new, torch.float16, "k_new")
            _need(v_new, torch.float16, "v_new")
        if out is None and getattr(self, "gather", None) is None:
            out = torch.empty_like(q)
        check(self._lib.vk_decode_run(self.pool.handle, self.handle, layer, _ptr(q), _ptr(out), _ptr(block_tables),
                                      block_tables.shape[1], _ptr(k_new), _ptr(v_new), float(scale),
                                      _ptr(self.workspace), _stream(stream)), "vk_decode_run")
        return out

    def close(self) -> None:
        if getattr(self, "handle", None) is not None and self.handle.value:
            self._lib.vk_decode_plan_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class _DeviceArray:
    """__cuda_array_interface__ over library-owned device memory."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape), "typestr": typestr,
                                         "version": 3, "strides": None}


class Gather:
    """vk_gather: head-sharded output all-gather fused into the planned decode.

    Each rank creates one with the same ``slice_bytes`` (its [B, Hq/world, D]
    fp16 output) and ``slots``; the ranks then swap ``export()`` handles over
    any host transport (``exchange`` does it with torch.distributed) and
    ``import_peer`` every other rank's.  ``view(slot, B, Hq_local, D)`` is the
    rank's receive buffer of a slot as [world, B, Hq_local, D] fp16.  A step
    binds it to a plan (``DecodePlan.set_gather``), runs the layers in order and
    ends with ``DecodePlan.gather_wait(L - 1)``."""

    HANDLE_BYTES = 64

    def __init__(self, rank: int, world: int, slice_bytes: int, slots: int, device=None):
        self._lib = _lib.load()
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                           (device.index if isinstance(device, torch.device) else int(device)))
        self.device, self.rank, self.world, self.slots, self.slice_bytes = dev, rank, world, slots, slice_bytes
        h = ctypes.c_void_p()
        check(self._lib.vk_gather_create(dev.index, rank, world, slice_bytes, slots, ctypes.byref(h)),
              "vk_gather_create")
        self.handle = h

    def export(self) -> bytes:
        buf = ctypes.create_string_buffer(self.HANDLE_BYTES)
        check(self._lib.vk_gather_export(self.handle, buf), "vk_gather_export")
        return buf.raw

    def import_peer(self, peer: int, handle: bytes) -> None:
        buf = ctypes.create_string_buffer(bytes(handle), self.HANDLE_BYTES)
        check(self._lib.vk_gather_import(self.handle, peer, buf), "vk_gather_import")
        self._ipc_peers = True

    def import_local(self, peer: int, other: "Gather") -> None:
        """Rank ``peer`` is ``other``, a gather of this process (one host
        process driving several ranks; see vk_gather_import_local)."""
        check(self._lib.vk_gather_import_local(self.handle, peer, other.handle), "vk_gather_import_local")

    def exchange(self, group=None) -> None:
        """Swaps handles with every rank through torch.distributed (host side)."""
        import torch.distributed as dist
        handles = [None] * self.world
        dist.all_gather_object(handles, self.export(), group=group)
        for r, hd in enumerate(handles):
            if r != self.rank:
                self.import_peer(r, hd)

    def buffer_ptr(self, slot: int) -> int:
        p = self._lib.vk_gather_buffer(self.handle, slot)
        if not p:
            raise VKError(1, "vk_gather_buffer")
        return p

    def view(self, slot: int, batch: int, heads_local: int, head_dim: int) -> torch.Tensor:
        n = self.world * batch * heads_local * head_dim
        if n * 2 > self.world * self.slice_bytes:
            raise ValueError("view larger than the slot")
        arr = _DeviceArray(self.buffer_ptr(slot), (self.world, batch, heads_local, head_dim), "<f2")
        return torch.as_tensor(arr, device=self.device)

    def check(self) -> None:
        check(self._lib.vk_gather_check(self.handle), "vk_gather_check")

    def release_peers(self) -> None:
        check(self._lib.vk_gather_release_peers(self.handle), "vk_gather_release_peers")

    def close(self, group=None) -> None:
        """Two-phase teardown: release the peer mappings, meet every rank at a
        torch.distributed barrier (when peers were imported from other
        processes), then free the buffer."""
        if getattr(self, "handle", None) is not None and self.handle.value:
            if self.world > 1:
                self.release_peers()
                if getattr(self, "_ipc_peers", False):
                    import torch.distributed as dist
                    dist.barrier(group=group)
            self._lib.vk_gather_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            if getattr(self, "handle", None) is not None and self.handle.value:
                self._lib.vk_gather_destroy(self.handle)
                self.handle = ctypes.c_void_p()
        except Exception:
            pass


class OutputProjection:
    """vk_oproj: the `wo` projection after head-sharded attention fused with its
    reduce-scatter over output features (see include/vk_paged_kv.h).

    Every rank creates one with the same world, max_tokens, k_local (its heads
    x head_dim) and n_out; peers are joined like a Gather (``exchange`` over
    torch.distributed, or ``import_local`` for ranks of this process).  ``run``
    takes this rank's attention output x [tokens, k_local] fp16 and its rows of
    wo packed by ``pack_weight`` (fp32 [k_local, n_out] rows, the reference's
    layout) or ``pack_weight_t16`` (fp16 [n_out, k_local] rows of wo
    transposed), and returns y [tokens, n_out/world] fp16: this rank's features
    of the sum over ranks."""

    HANDLE_BYTES = 64

    def __init__(self, rank: int, world: int, max_tokens: int, k_local: int, n_out: int, device=None):
        self._lib = _lib.load()
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                           (device.index if isinstance(device, torch.device) else int(device)))
        self.device, self.rank, self.world = dev, rank, world
        self.max_tokens, self.k_local, self.n_out = max_tokens, k_local, n_out
        h = ctypes.c_void_p()
        check(self._lib.vk_oproj_create(dev.index, rank, world, max_tokens, k_local, n_out, ctypes.byref(h)),
              "vk_oproj_create")
        self.handle = h
        self._ipc_peers = False

    @property
    def splits(self) -> int:
        return self._lib.vk_oproj_splits(self.handle)

    def export(self) -> bytes:
        buf = ctypes.create_string_buffer(self.HANDLE_BYTES)
        check(self._lib.vk_oproj_export(self.handle, buf), "vk_oproj_export")
        return buf.raw

    def import_peer(self, peer: int, handle: bytes) -> None:
        buf = ctypes.create_string_buffer(bytes(handle), self.HANDLE_BYTES)
        check(self._lib.vk_oproj_import(self.handle, peer, buf), "vk_oproj_import")
        self._ipc_peers = True

    def import_local(self, peer: int, other: "OutputProjection") -> None:
        check(self._lib.vk_oproj_import_local(self.handle, peer, other.handle), "vk_oproj_import_local")

    def exchange(self, group=None) -> None:
        import torch.distributed as dist
        handles = [None] * self.world
        dist.all_gather_object(handles, self.export(), group=group)
        for r, hd in enumerate(handles):
            if r != self.rank:
                self.import_peer(r, hd)

    def run(self, x: torch.Tensor, w_packed: torch.Tensor, y: Optional[torch.Tensor] = None,
            stream=None) -> torch.Tensor:
        """x and y may be row-strided views (unit stride along a row)."""
        for t, name in ((x, "x"),) + (((y, "y"),) if y is not None else ()):
            if t.dtype != torch.float16 or not t.is_cuda or t.dim() != 2 or t.stride(1) != 1:
                raise ValueError("%s must be a 2-D fp16 CUDA tensor with unit stride along its rows" % name)
        nbytes = self._lib.vk_oproj_packed_bytes(self.k_local, self.n_out)
        if not w_packed.is_cuda or w_packed.numel() * w_packed.element_size() != nbytes:
            raise ValueError("w_packed must be a packed weight of %d bytes (pack_weight / pack_weight_t16)" % nbytes)
        tokens = x.shape[0]
        if y is None:
            y = torch.empty(tokens, self.n_out // self.world, dtype=torch.float16, device=x.device)
        check(self._lib.vk_oproj_run(self.handle, _ptr(x), x.stride(0), _ptr(w_packed), _ptr(y), y.stride(0),
                                     tokens, _stream(stream)), "vk_oproj_run")
        return y

    @staticmethod
    def pack_weight(w: torch.Tensor, stream=None) -> torch.Tensor:
        """fp32 wo rows [k_rows, n] (the reference's layout, row-strided view
        allowed) -> packed fp16 weight (uint8 tensor)."""
        if w.dtype != torch.float32 or not w.is_cuda or w.dim() != 2 or w.stride(1) != 1:
            raise ValueError("w must be a 2-D fp32 CUDA tensor with unit stride along its rows")
        k_rows, n = w.shape
        lib = _lib.load()
        wp = torch.empty(max(1, lib.vk_oproj_packed_bytes(k_rows, n)), dtype=torch.uint8, device=w.device)
        check(lib.vk_oproj_pack_weight(_ptr(w), w.stride(0), k_rows, n, _ptr(wp), _stream(stream)),
              "vk_oproj_pack_weight")
        return wp

    @staticmethod
    def pack_weight_t16(w_t: torch.Tensor, stream=None) -> torch.Tensor:
        """fp16 rows of wo transposed [n, k_rows] (an nn.Linear [out, in] weight
        or its column slice) -> packed fp16 weight (uint8 tensor)."""
        if w_t.dtype != torch.float16 or not w_t.is_cuda or w_t.dim() != 2 or w_t.stride(1) != 1:
            raise ValueError("w_t must be a 2-D fp16 CUDA tensor with unit stride along its rows")
        n, k_rows = w_t.shape
        lib = _lib.load()
        wp = torch.empty(max(1, lib.vk_oproj_packed_bytes(k_rows, n)), dtype=torch.uint8, device=w_t.device)
        check(lib.vk_oproj_pack_weight_t16(_ptr(w_t), w_t.stride(0), n, k_rows, _ptr(wp), _stream(stream)),
              "vk_oproj_pack_weight_t16")
        return wp

    def check(self) -> None:
        check(self._lib.vk_oproj_check(self.handle), "vk_oproj_check")

    def close(self, group=None) -> None:
        if getattr(self, "handle", None) is not None and self.handle.value:
            if self.world > 1:
                check(self._lib.vk_oproj_release_peers(self.handle), "vk_oproj_release_peers")
                if self._ipc_peers:
                    import torch.distributed as dist
                    dist.barrier(group=group)
            self._lib.vk_oproj_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            if getattr(self, "handle", None) is not None and self.handle.value:
                self._lib.vk_oproj_destroy(self.handle)
                self.handle = ctypes.c_void_p()
        except Exception:
            pass


def remap_block_tables(block_tables: torch.Tensor, page_map: torch.Tensor, stream=None) -> None:
    _need(block_tables, torch.int32, "block_tables")
    _need(page_map, torch.int32, "page_map")
    check(_lib.load().vk_remap_block_tables(_ptr(block_tables), block_tables.numel(), _ptr(page_map),
                                            page_map.numel(), _stream(stream)), "vk_remap_block_tables")


def launch_attention(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, O: torch.Tensor, batch: int,
                     heads: int, seq_len: int, head_dim: int, stream=None) -> None:
    """vulcan::cuda::launch_attention on contiguous fp32 [B, H, S, D] tensors."""
    for t, n in ((Q, "Q"), (K, "K"), (V, "V"), (O, "O")):
        _need(t, torch.float32, n)
    check(_lib.load().vk_attention_f32(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), batch, heads, seq_len, head_dim,
                                       _stream(stream)), "vk_attention_f32")


class MemoryManager:
    """vulcan::cuda::MemoryManager(page_size, max_pages) over a raw byte-page pool."""

    DEFAULT_PAGE_SIZE = 16 * 1024

    def __init__(self, page_size: int = DEFAULT_PAGE_SIZE, max_pages: int = 1024, device=None):
        self.page_size = page_size
        self.max_pages = max_pages
        self._pool = PagedKVPool(0, 0, 0, max_pages, page_tokens=0, device=device, own_memory=True,
                                 page_bytes=page_size)
        self._swap = {}  # id -> pinned host tensor

    def allocate_block(self) -> int:
        try:
            return self._pool.alloc(1)[0]
        except VKError as e:
            if e.status == _lib.VK_OUT_OF_PAGES:
                return -1
            raise

    def free_block(self, block_id: int) -> None:
        self._pool.free([block_id])
        self._swap.pop(block_id, None)

    def get_block_ptr(self, block_id: int) -> Optional[int]:
        return self._pool.page_ptr(block_id)

    def swap_to_cpu(self, block_id: int) -> bool:
        if not (0 <= block_id < self.max_pages) or self._pool.page_in_use(block_id) != 1:
            return False
        host = torch.empty(self.page_size, dtype=torch.uint8, pin_memory=True)
        st = torch.cuda.current_stream(self._pool.device)
        if self._pool._lib.vk_swap_out(self._pool.handle, _i32_array([block_id]), 1, _ptr(host),
                                       _stream(st)) != _lib.VK_OK:
            return False
        st.synchronize()
        self._swap[block_id] = host
        return True

    def swap_to_gpu(self, block_id: int) -> bool:
        if not (0 <= block_id < self.max_pages) or block_id not in self._swap:
            return False
        st = torch.cuda.current_stream(self._pool.device)
        if self._pool._lib.vk_swap_in_to(self._pool.handle, _ptr(self._swap[block_id]),
                                         _i32_array([block_id]), 1, _stream(st)) != _lib.VK_OK:
            return False
        st.synchronize()
        del self._swap[block_id]
        return True

    def blocks_in_use(self) -> int:
        return self._pool.pages_in_use()

    def blocks_available(self) -> int:
        return self._pool.pages_available()

    def total_allocated_bytes(self) -> int:
        return self._pool.allocated_bytes()


class KVCache:
    """vulcan::KVCache(num_kv_heads, max_seq_len, head_dim, num_layers) for one
    sequence on a paged fp16 pool; pages are taken on demand by ``append``."""

    def __init__(self, num_kv_heads: int, max_seq_len: int, head_dim: int, num_layers: int, device=None):
        self._num_kv_heads, self._max_seq_len = num_kv_heads, max_seq_len
        self._head_dim, self._num_layers = head_dim, num_layers
        pages = (max_seq_len + PAGE_TOKENS - 1) // PAGE_TOKENS
        self.pool = PagedKVPool(num_layers, num_kv_heads, head_dim, pages, device=device)
        self.block_table = torch.full((1, pages), -1, dtype=torch.int32, device=self.pool.device)
        self._pages: List[int] = []
        self._current_len = 0

    def _ensure_pages(self, end: int) -> None:
        need = (end + PAGE_TOKENS - 1) // PAGE_TOKENS
        if need > len(self._pages):
            new = self.pool.alloc(need - len(self._pages))
            self.block_table[0, len(self._pages):need] = torch.tensor(new, dtype=torch.int32)
            self._pages += new

    def append(self, layer: int, k_new: torch.Tensor, v_new: torch.Tensor, start_pos: int,
               num_tokens: int) -> None:
        """k_new/v_new: [num_tokens, num_kv_heads*head_dim] (fp32 or fp16) CUDA tensors."""
        if layer < 0 or layer >= self._num_layers:
            return  # the reference returns silently (src/kv_cache.cpp:86)
        if start_pos + num_tokens > self._max_seq_len:
            print("[VULCAN] KV Cache overflow: pos=%d + tokens=%d > max_seq=%d"
                  % (start_pos, num_tokens, self._max_seq_len), file=sys.stderr)
            return
        self._ensure_pages(start_pos + num_tokens)
        k = k_new.reshape(1, num_tokens, self._num_kv_heads, self._head_dim)
        v = v_new.reshape(1, num_tokens, self._num_kv_heads, self._head_dim)
        pos = torch.tensor([start_pos], dtype=torch.int32, device=self.pool.device)
        self.pool.append(layer, k, v, self.block_table, pos)
        self._current_len = max(self._current_len, start_pos + num_tokens)

    def get(self, layer: int):
        """Device addresses of this layer's K and V blocks of physical page 0;
        the element (page, kv head, slot, d) of the layer is at
        ``k + (page*Hkv + head)*2*P*D*2 + (slot*D + d)*2`` (V: same from ``v``)."""
        if layer < 0 or layer >= self._num_layers:
            return None, None
        seg = self._num_kv_heads * 2 * PAGE_TOKENS * self._head_dim * 2
        k = self.pool.base_ptr + layer * seg * self.pool.num_pages
        return k, k + PAGE_TOKENS * self._head_dim * 2

    def decode(self, layer: int, q: torch.Tensor, num_q_heads: Optional[int] = None) -> torch.Tensor:
        """Attention of one query token ([num_q_heads, head_dim] fp16) over the cached tokens."""
        hq = num_q_heads or q.shape[0]
        lens = torch.tensor([self._current_len], dtype=torch.int32, device=self.pool.device)
        return self.pool.decode(layer, q.reshape(1, hq, self._head_dim).contiguous(), self.block_table, lens,
                                self._max_seq_len)[0]

    def current_length(self) -> int:
        return self._current_len

    def set_length(self, length: int) -> None:
        self._current_len = length

    def reset(self) -> None:
        self._current_len = 0

    def max_seq_len(self) -> int:
        return self._max_seq_len

    def memory_usage(self) -> int:
        """Bytes of fp16 storage for max_seq_len tokens: 2*L*Hkv*ceil(S/16)*16*D*2."""
        pages = (self._max_seq_len + PAGE_TOKENS - 1) // PAGE_TOKENS
        return 2 * self._num_layers * self._num_kv_heads * pages * PAGE_TOKENS * self._head_dim * 2


def default_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
