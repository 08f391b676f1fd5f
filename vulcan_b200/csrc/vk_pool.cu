// Pool lifetime, the host-side page allocator, swap and compaction, and the
// C-ABI diagnostics of libvulcan_kv.so.
//
// Reference behaviour followed (VULCAN, cuda/memory.cu):
//   - one device allocation carved into equal pages (:73-116); the reference
//     halves max_pages on OOM, this library reports VK_CUDA_ERROR instead so
//     the caller sizes the pool explicitly;
//   - allocate_block: lowest free id, -1 when full (:127-135);
//   - free_block: bad ids ignored, swap copy dropped (:137-143);
//   - get_block_ptr: base + id*page, nullptr on a bad id (:145-150);
//   - swap_to_cpu / swap_to_gpu (:152-191), here batched and asynchronous.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "vk_internal.h"
#include "vk_fp8.cuh"

namespace vk {

static thread_local std::string g_last_error;

vk_status fail(vk_status s, const std::string& msg) {
    g_last_error = msg;
    return s;
}

vk_status cuda_fail(cudaError_t e, const char* what) {
    g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return VK_CUDA_ERROR;
}

// ---------------------------------------------------------------- allocator

void Allocator::reset(int32_t n) {
    num_pages = n;
    used = 0;
    hint = 0;
    free_bits.assign((static_cast<size_t>(n) + 63) / 64, ~0ull);
    if (n % 64) free_bits.back() = (1ull << (n % 64)) - 1;
}

int32_t Allocator::take_lowest() {
    for (size_t w = hint; w < free_bits.size(); ++w) {
        if (free_bits[w]) {
            const int bit = __builtin_ctzll(free_bits[w]);
            free_bits[w] &= ~(1ull << bit);
            hint = w;
            ++used;
            return static_cast<int32_t>(w * 64 + bit);
        }
    }
    hint = free_bits.size();
    return -1;
}

bool Allocator::is_used(int32_t id) const {
    return !((free_bits[static_cast<size_t>(id) >> 6] >> (id & 63)) & 1ull);
}

void Allocator::set_used(int32_t id) {
    if (!is_used(id)) {
        free_bits[static_cast<size_t>(id) >> 6] &= ~(1ull << (id & 63));
        ++used;
    }
}

void Allocator::set_free(int32_t id) {
    if (is_used(id)) {
        free_bits[static_cast<size_t>(id) >> 6] |= (1ull << (id & 63));
        --used;
        hint = std::min(hint, static_cast<size_t>(id) >> 6);
    }
}

// ---------------------------------------------------------------- tensor map

PFN_cuTensorMapEncodeTiled_v12000 tmap_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// Rows of head_dim fp16 elements over the whole pool; a TMA box is 64 elements
// (128 bytes, 128-byte swizzle) by 2*page_tokens rows: the K and V rows of one
// (layer, page, head) for one 64-wide slice of the head dimension.  The rows of
// (layer, page, head) start at ((layer*num_pages + page)*Hkv + head)*2*page_tokens.
static vk_status make_tmap(vk_pool* p) {
    const uint64_t rows =
        static_cast<uint64_t>(p->num_pages) * p->cfg.num_layers * p->cfg.num_kv_heads * 2 *
        p->cfg.page_tokens;
    if (rows >= (1ull << 31)) return VK_OK;  // TMA coordinates are int32: kernels refuse
    auto encode = tmap_encode_fn();
    if (!encode) return fail(VK_CUDA_ERROR, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(p->cfg.head_dim), rows};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(p->cfg.head_dim) * 2};
    cuuint32_t box[2] = {64, static_cast<cuuint32_t>(2 * p->cfg.page_tokens)};
    cuuint32_t box16[2] = {64, static_cast<cuuint32_t>(p->cfg.page_tokens)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(&p->tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p->base, dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r == CUDA_SUCCESS)
        r = encode(&p->tmap16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p->base, dims, strides, box16, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char buf[96];
        std::snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
        return fail(VK_CUDA_ERROR, buf);
    }
    p->tmap_ok = true;
    return VK_OK;
}

// bytes of the K and V rows of one (layer, page, head)
static uint64_t kv_head_bytes(const vk_pool_cfg* c, int fmt) {
    if (fmt == VK_KV_FP8) return static_cast<uint64_t>(fp8_head_bytes(c->head_dim));
    return 2ull * c->page_tokens * c->head_dim * 2;
}

static vk_status check_cfg(const vk_pool_cfg* c, int fmt, bool* kv, uint64_t* page_bytes) {
    if (!c) return fail(VK_INVALID_ARG, "cfg is NULL");
    if (c->num_pages <= 0) return fail(VK_INVALID_ARG, "num_pages must be > 0");
    if (fmt != VK_KV_FP16 && fmt != VK_KV_FP8) return fail(VK_INVALID_ARG, "unknown kv_format");
    if (c->page_bytes) {
        if (fmt != VK_KV_FP16) return fail(VK_INVALID_ARG, "a byte-page pool (page_bytes != 0) has no KV format");
        *kv = false;
        *page_bytes = c->page_bytes;
        return VK_OK;
    }
    if (c->num_layers <= 0 || c->num_kv_heads <= 0 || c->head_dim <= 0 || c->page_tokens <= 0)
        return fail(VK_INVALID_ARG, "num_layers, num_kv_heads, head_dim, page_tokens must be > 0");
    if (c->head_dim % 8)
        return fail(VK_INVALID_ARG, "head_dim must be a multiple of 8 (16-byte rows)");
    if (fmt == VK_KV_FP8 && (c->head_dim != kFp8Dim || c->page_tokens != kPageTokens))
        return fail(VK_UNSUPPORTED, "FP8 pages need head_dim 128 and page_tokens 16");
    *kv = true;
    *page_bytes = static_cast<uint64_t>(c->num_layers) * c->num_kv_heads * kv_head_bytes(c, fmt);
    return VK_OK;
}

// Layer-major layout: segment `layer` of page `id` starts at
// base + layer*seg_stride + id*seg_bytes, so one layer's pages form one
// contiguous region of num_pages*seg_bytes.
static void set_geometry(vk_pool* p) {
    if (p->kv) {
        p->head_bytes = kv_head_bytes(&p->cfg, p->kv_format);
        p->seg_bytes = p->head_bytes * p->cfg.num_kv_heads;
        p->nseg = p->cfg.num_layers;
        p->seg_stride = p->seg_bytes * static_cast<uint64_t>(p->num_pages);
    } else {
        p->seg_bytes = p->page_bytes;
        p->nseg = 1;
        p->seg_stride = 0;
    }
}

static vk_status finish_create(vk_pool* p, vk_pool** out) {
    cudaError_t e = cudaMalloc(&p->d_err, sizeof(uint32_t));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(error word)");
    e = cudaMemset(p->d_err, 0, sizeof(uint32_t));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(error word)");
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, p->device) == cudaSuccess &&
        sms > 0)
        p->num_sms = sms;
    if (p->kv && p->kv_format == VK_KV_FP16) {  // FP8 blocks are fetched with untiled bulk copies
        vk_status s = make_tmap(p);
        if (s != VK_OK) return s;
    }
    p->alloc.reset(p->num_pages);
    *out = p;
    return VK_OK;
}

}  // namespace vk

using namespace vk;

extern "C" {

static vk_status pool_create_owned(const vk_pool_cfg* cfg, int fmt, vk_pool** out_pool) {
    if (!out_pool) return fail(VK_INVALID_ARG, "out_pool is NULL");
    *out_pool = nullptr;
    bool kv = false;
    uint64_t pb = 0;
    vk_status s = check_cfg(cfg, fmt, &kv, &pb);
    if (s != VK_OK) return s;
    DeviceGuard g(cfg->device);
    auto* p = new vk_pool();
    p->cfg = *cfg;
    p->kv = kv;
    p->kv_format = fmt;
    p->device = cfg->device;
    p->page_bytes = pb;
    p->num_pages = cfg->num_pages;
    set_geometry(p);
    const uint64_t bytes = pb * static_cast<uint64_t>(cfg->num_pages);
    cudaError_t e = cudaMalloc(&p->base, bytes);
    if (e != cudaSuccess) {
        delete p;
        return cuda_fail(e, "cudaMalloc(pool)");
    }
    p->owns_mem = true;
    // Zero-filled like the reference's cache (src/kv_cache.cpp:33-35).
    e = cudaMemset(p->base, 0, bytes);
    if (e != cudaSuccess) {
        cudaFree(p->base);
        delete p;
        return cuda_fail(e, "cudaMemset(pool)");
    }
    s = finish_create(p, out_pool);
    if (s != VK_OK) {
        if (p->d_err) cudaFree(p->d_err);
        cudaFree(p->base);
        delete p;
        *out_pool = nullptr;
    }
    return s;
}

static vk_status pool_create_in(const vk_pool_cfg* cfg, int fmt, void* device_mem, size_t bytes,
                                vk_pool** out_pool) {
    if (!out_pool) return fail(VK_INVALID_ARG, "out_pool is NULL");
    *out_pool = nullptr;
    bool kv = false;
    uint64_t pb = 0;
    vk_status s = check_cfg(cfg, fmt, &kv, &pb);
    if (s != VK_OK) return s;
    if (!device_mem || (reinterpret_cast<uintptr_t>(device_mem) & 255))
        return fail(VK_INVALID_ARG, "device_mem must be non-NULL and 256-byte aligned");
    if (bytes < pb * static_cast<uint64_t>(cfg->num_pages))
        return fail(VK_INVALID_ARG, "device_mem smaller than num_pages * page_bytes");
    DeviceGuard g(cfg->device);
    auto* p = new vk_pool();
    p->cfg = *cfg;
    p->kv = kv;
    p->kv_format = fmt;
    p->device = cfg->device;
    p->page_bytes = pb;
    p->num_pages = cfg->num_pages;
    set_geometry(p);
    p->base = static_cast<char*>(device_mem);
    p->owns_mem = false;
    s = finish_create(p, out_pool);
    if (s != VK_OK) {
        if (p->d_err) cudaFree(p->d_err);
        delete p;
        *out_pool = nullptr;
    }
    return s;
}

vk_status vk_pool_create(const vk_pool_cfg* cfg, vk_pool** out_pool) {
    return pool_create_owned(cfg, VK_KV_FP16, out_pool);
}

vk_status vk_pool_create_in(const vk_pool_cfg* cfg, void* device_mem, size_t bytes, vk_pool** out_pool) {
    return pool_create_in(cfg, VK_KV_FP16, device_mem, bytes, out_pool);
}

vk_status vk_pool_create_fmt(const vk_pool_cfg* cfg, int32_t kv_format, void* device_mem, size_t bytes,
                             vk_pool** out_pool) {
    if (cfg && cfg->page_bytes) {
        if (out_pool) *out_pool = nullptr;
        return fail(VK_INVALID_ARG, "vk_pool_create_fmt makes KV pools: page_bytes must be 0");
    }
    return device_mem ? pool_create_in(cfg, kv_format, device_mem, bytes, out_pool)
                      : pool_create_owned(cfg, kv_format, out_pool);
}

int32_t vk_pool_kv_format(const vk_pool* pool) { return pool && pool->kv ? pool->kv_format : -1; }

vk_status vk_pool_destroy(vk_pool* pool) {
    if (!pool) return VK_OK;
    DeviceGuard g(pool->device);
    if (pool->owns_mem && pool->base) cudaFree(pool->base);
    if (pool->d_err) cudaFree(pool->d_err);
    if (pool->rope_freq) cudaFree(pool->rope_freq);
    delete pool;
    return VK_OK;
}

void* vk_pool_base(const vk_pool* pool) { return pool ? pool->base : nullptr; }
uint64_t vk_pool_page_bytes(const vk_pool* pool) { return pool ? pool->page_bytes : 0; }
int32_t vk_pool_num_pages(const vk_pool* pool) { return pool ? pool->num_pages : 0; }

vk_status vk_pool_check(vk_pool* pool, uint32_t* out_bits) {
    if (!pool) return fail(VK_INVALID_ARG, "pool is NULL");
    DeviceGuard g(pool->device);
    uint32_t bits = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
    e = cudaMemcpy(&bits, pool->d_err, sizeof bits, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(error word)");
    e = cudaMemset(pool->d_err, 0, sizeof bits);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(error word)");
    if (out_bits) *out_bits = bits;
    if (bits & VK_ERR_TIMEOUT) return fail(VK_TIMEOUT, "a device-side wait timed out");
    if (bits) {
        char buf[96];
        std::snprintf(buf, sizeof buf, "kernel rejected block-table/position/length (bits 0x%x)",
                      bits);
        return fail(VK_BAD_BLOCK_TABLE, buf);
    }
    return VK_OK;
}

// ---------------------------------------------------------------- allocator

vk_status vk_alloc_pages(vk_pool* pool, int32_t n, int32_t* out_ids) {
    if (!pool || (n > 0 && !out_ids) || n < 0) return fail(VK_INVALID_ARG, "bad alloc arguments");
    if (pool->num_pages - pool->alloc.used < n) {
        for (int32_t i = 0; i < n; ++i) out_ids[i] = -1;
        return fail(VK_OUT_OF_PAGES, "not enough free pages");
    }
    for (int32_t i = 0; i < n; ++i) out_ids[i] = pool->alloc.take_lowest();
    return VK_OK;
}

vk_status vk_free_pages(vk_pool* pool, const int32_t* ids, int32_t n) {
    if (!pool || (n > 0 && !ids) || n < 0) return fail(VK_INVALID_ARG, "bad free arguments");
    for (int32_t i = 0; i < n; ++i) {
        const int32_t id = ids[i];
        if (id < 0 || id >= pool->num_pages) continue;  // ignored, as the reference does
        pool->alloc.set_free(id);
    }
    return VK_OK;
}

void* vk_page_ptr(const vk_pool* pool, int32_t id) {
    if (!pool || id < 0 || id >= pool->num_pages) return nullptr;
    return pool->base + static_cast<uint64_t>(id) * pool->seg_bytes;
}

int32_t vk_pages_in_use(const vk_pool* pool) { return pool ? pool->alloc.used : 0; }
int32_t vk_pages_available(const vk_pool* pool) {
    return pool ? pool->num_pages - pool->alloc.used : 0;
}
uint64_t vk_allocated_bytes(const vk_pool* pool) {
    return pool ? static_cast<uint64_t>(pool->alloc.used) * pool->page_bytes : 0;
}
int32_t vk_page_in_use(const vk_pool* pool, int32_t id) {
    if (!pool || id < 0 || id >= pool->num_pages) return -1;
    return pool->alloc.is_used(id) ? 1 : 0;
}

// ---------------------------------------------------------------- swap

// Host buffers hold whole pages back to back (page i of the call at
// host + i*page_bytes, its layer segments consecutive).  Byte pools copy runs of
// consecutive ids with one cudaMemcpyAsync each; KV pools copy each page's
// layer segments with one strided 2-D copy.
static vk_status copy_runs(vk_pool* pool, const int32_t* ids, int32_t n, char* host, bool to_host,
                           cudaStream_t st) {
    if (pool->nseg > 1) {
        for (int32_t i = 0; i < n; ++i) {
            char* dev = pool->base + static_cast<uint64_t>(ids[i]) * pool->seg_bytes;
            char* h = host + static_cast<uint64_t>(i) * pool->page_bytes;
            cudaError_t e =
                to_host ? cudaMemcpy2DAsync(h, pool->seg_bytes, dev, pool->seg_stride, pool->seg_bytes, pool->nseg,
                                            cudaMemcpyDeviceToHost, st)
                        : cudaMemcpy2DAsync(dev, pool->seg_stride, h, pool->seg_bytes, pool->seg_bytes, pool->nseg,
                                            cudaMemcpyHostToDevice, st);
            if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy2DAsync(swap)");
        }
        return VK_OK;
    }
    int32_t i = 0;
    while (i < n) {
        int32_t j = i + 1;
        while (j < n && ids[j] == ids[j - 1] + 1) ++j;
        const uint64_t bytes = static_cast<uint64_t>(j - i) * pool->page_bytes;
        char* dev = pool->base + static_cast<uint64_t>(ids[i]) * pool->page_bytes;
        char* h = host + static_cast<uint64_t>(i) * pool->page_bytes;
        cudaError_t e = to_host ? cudaMemcpyAsync(h, dev, bytes, cudaMemcpyDeviceToHost, st)
                                : cudaMemcpyAsync(dev, h, bytes, cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(swap)");
        i = j;
    }
    return VK_OK;
}

vk_status vk_swap_out(vk_pool* pool, const int32_t* ids, int32_t n, void* host_buf, void* stream) {
    if (!pool || n < 0 || (n > 0 && (!ids || !host_buf)))
        return fail(VK_INVALID_ARG, "bad swap_out arguments");
    for (int32_t i = 0; i < n; ++i) {
        if (ids[i] < 0 || ids[i] >= pool->num_pages)
            return fail(VK_INVALID_ARG, "swap_out: id outside the pool");
        if (!pool->alloc.is_used(ids[i]))
            return fail(VK_INVALID_ARG, "swap_out: id is not allocated");  // reference returns false
    }
    DeviceGuard g(pool->device);
    vk_status s = copy_runs(pool, ids, n, static_cast<char*>(host_buf), true, as_stream(stream));
    if (s != VK_OK) return s;
    for (int32_t i = 0; i < n; ++i) pool->alloc.set_free(ids[i]);
    return VK_OK;
}

vk_status vk_swap_in(vk_pool* pool, const void* host_buf, int32_t n, int32_t* out_ids,
                     void* stream) {
    if (!pool || n < 0 || (n > 0 && (!out_ids || !host_buf)))
        return fail(VK_INVALID_ARG, "bad swap_in arguments");
    vk_status s = vk_alloc_pages(pool, n, out_ids);
    if (s != VK_OK) return s;
    DeviceGuard g(pool->device);
    s = copy_runs(pool, out_ids, n, static_cast<char*>(const_cast<void*>(host_buf)), false,
                  as_stream(stream));
    if (s != VK_OK) vk_free_pages(pool, out_ids, n);
    return s;
}

vk_status vk_swap_in_to(vk_pool* pool, const void* host_buf, const int32_t* ids, int32_t n,
                        void* stream) {
    if (!pool || n < 0 || (n > 0 && (!ids || !host_buf)))
        return fail(VK_INVALID_ARG, "bad swap_in_to arguments");
    for (int32_t i = 0; i < n; ++i) {
        if (ids[i] < 0 || ids[i] >= pool->num_pages)
            return fail(VK_INVALID_ARG, "swap_in_to: id outside the pool");
        if (pool->alloc.is_used(ids[i]))
            return fail(VK_INVALID_ARG, "swap_in_to: id is in use");
        for (int32_t j = 0; j < i; ++j)
            if (ids[j] == ids[i]) return fail(VK_INVALID_ARG, "swap_in_to: duplicate id");
    }
    DeviceGuard g(pool->device);
    vk_status s = copy_runs(pool, ids, n, static_cast<char*>(const_cast<void*>(host_buf)), false,
                            as_stream(stream));
    if (s != VK_OK) return s;
    for (int32_t i = 0; i < n; ++i) pool->alloc.set_used(ids[i]);
    return VK_OK;
}

// ---------------------------------------------------------------- compaction

vk_status vk_compact_plan(vk_pool* pool, int32_t* src_ids, int32_t* dst_ids, int32_t cap,
                          int32_t* out_n) {
    if (!pool || !out_n || cap < 0 || (cap > 0 && (!src_ids || !dst_ids)))
        return fail(VK_INVALID_ARG, "bad compact_plan arguments");
    int32_t n = 0, lo = 0, hi = pool->num_pages - 1;
    while (true) {
        while (lo < pool->num_pages && pool->alloc.is_used(lo)) ++lo;
        while (hi >= 0 && !pool->alloc.is_used(hi)) --hi;
        if (lo >= hi || n == cap) break;
        src_ids[n] = hi;
        dst_ids[n] = lo;
        pool->alloc.set_used(lo);
        pool->alloc.set_free(hi);
        ++n;
    }
    *out_n = n;
    return VK_OK;
}

vk_status vk_copy_pages(vk_pool* pool, const int32_t* src_ids, const int32_t* dst_ids, int32_t n,
                        void* stream) {
    if (!pool || n < 0 || (n > 0 && (!src_ids || !dst_ids)))
        return fail(VK_INVALID_ARG, "bad copy_pages arguments");
    if (n == 0) return VK_OK;
    DeviceGuard g(pool->device);
    return launch_copy_pages(pool, src_ids, dst_ids, n, as_stream(stream));
}

vk_status vk_remap_block_tables(int32_t* block_tables, int64_t entries, const int32_t* page_map,
                                int32_t map_len, void* stream) {
    if (entries < 0 || map_len < 0 || (entries > 0 && (!block_tables || !page_map)))
        return fail(VK_INVALID_ARG, "bad remap arguments");
    if (entries == 0) return VK_OK;
    return launch_remap(block_tables, entries, page_map, map_len, as_stream(stream));
}

// ---------------------------------------------------------------- append

static vk_status append_common(vk_pool* pool, int32_t layer, const void* k, const void* v, bool f32,
                               const int32_t* bt, int32_t bt_stride, const int32_t* pos,
                               int32_t batch, int32_t tokens, void* stream) {
    if (!pool) return fail(VK_INVALID_ARG, "pool is NULL");
    if (!pool->kv) return fail(VK_UNSUPPORTED, "append needs a KV pool (page_bytes == 0)");
    if (layer < 0 || layer >= pool->cfg.num_layers) return fail(VK_INVALID_ARG, "layer out of range");
    if (batch < 0 || tokens < 0 || bt_stride <= 0) return fail(VK_INVALID_ARG, "bad batch/tokens/bt_stride");
    if (batch == 0 || tokens == 0) return VK_OK;
    if (!k || !v || !bt || !pos) return fail(VK_INVALID_ARG, "NULL array");
    DeviceGuard g(pool->device);
    if (pool->kv_format == VK_KV_FP8)
        return launch_append_fp8(pool, layer, k, v, f32, bt, bt_stride, pos, batch, tokens, as_stream(stream));
    return launch_append(pool, layer, k, v, f32, bt, bt_stride, pos, batch, tokens, as_stream(stream));
}

vk_status vk_append(vk_pool* pool, int32_t layer, const void* k_new, const void* v_new,
                    const int32_t* block_tables, int32_t bt_stride, const int32_t* positions,
                    int32_t batch, int32_t tokens, void* stream) {
    return append_common(pool, layer, k_new, v_new, false, block_tables, bt_stride, positions,
                         batch, tokens, stream);
}

vk_status vk_append_f32(vk_pool* pool, int32_t layer, const float* k_new, const float* v_new,
                        const int32_t* block_tables, int32_t bt_stride, const int32_t* positions,
                        int32_t batch, int32_t tokens, void* stream) {
    return append_common(pool, layer, k_new, v_new, true, block_tables, bt_stride, positions, batch,
                         tokens, stream);
}

// ---------------------------------------------------------------- diagnostics

const char* vk_last_error_string(void) { return g_last_error.c_str(); }

const char* vk_status_string(vk_status s) {
    switch (s) {
        case VK_OK: return "VK_OK";
        case VK_INVALID_ARG: return "VK_INVALID_ARG";
        case VK_OUT_OF_PAGES: return "VK_OUT_OF_PAGES";
        case VK_CUDA_ERROR: return "VK_CUDA_ERROR";
        case VK_TIMEOUT: return "VK_TIMEOUT";
        case VK_BAD_BLOCK_TABLE: return "VK_BAD_BLOCK_TABLE";
        case VK_NOT_FOUND: return "VK_NOT_FOUND";
        case VK_UNSUPPORTED: return "VK_UNSUPPORTED";
    }
    return "VK_UNKNOWN";
}

int32_t vk_version(void) { return 100; }

}  // extern "C"
