// K1 append (block-table scatter of new K/V rows), K4 page copy and the
// block-table remap kernel.
//
// Append restates the row scatter of VULCAN's KVCache::append
// (src/kv_cache.cpp:94-121) with page indirection: token t of sequence b at
// pos = positions[b]+t goes to page block_tables[b][pos/16], slot pos%16, for
// every KV head.  The reference issues 2*Hkv*T blocking cudaMemcpy calls; here
// one launch moves every row with 16-byte vector loads and stores, one warp per
// (token, group of 4 KV heads) covering their K rows and V rows.
#include "vk_internal.h"
#include "vk_fp8.cuh"
#include "vk_ptx.cuh"
#include "vk_rope.cuh"

namespace vk {

struct AppendParams {
    char* base;
    const void* k;
    const void* v;
    const int32_t* bt;
    const int32_t* pos;
    uint32_t* err;
    uint64_t seg_bytes, layer_off, head_bytes;
    int bt_stride, B, T, Hkv, D, P, num_pages;
    const float* rope_freq;  // non-null: K rows are rotated (RoPE) at their positions
};

constexpr int kAppendHeads = 4;  // KV heads per warp: their rows' loads are in flight together

// One warp per (token, group of 4 KV heads): the position checks and the page
// lookup once, then the K and V rows of the group's heads, every load of a
// pass issued before its first store (2 KiB per warp in flight at D=128).
template <bool F32>
__global__ void __launch_bounds__(256) append_kernel(const AppendParams p) {
    const int64_t wid = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int groups = (p.Hkv + kAppendHeads - 1) / kAppendHeads;
    if (wid >= static_cast<int64_t>(p.B) * p.T * groups) return;
    const int h0 = static_cast<int>(wid % groups) * kAppendHeads;
    const int64_t tok = wid / groups;  // b*T + t
    const int t = static_cast<int>(tok % p.T);
    const int b = static_cast<int>(tok / p.T);
    const int pos = p.pos[b] + t;
    if (pos < 0 || pos / p.P >= p.bt_stride) {
        if (lane == 0) atomicOr(p.err, VK_ERR_TABLE_INDEX);
        return;
    }
    const int32_t page = p.bt[static_cast<int64_t>(b) * p.bt_stride + pos / p.P];
    if (page < 0 || page >= p.num_pages) {
        if (lane == 0) atomicOr(p.err, VK_ERR_PAGE_ID);
        return;
    }
    char* dst0 = p.base + p.layer_off + static_cast<uint64_t>(page) * p.seg_bytes +
                 static_cast<uint64_t>(pos % p.P) * p.D * 2;
    const int vpr = p.D / 8;  // 16-byte vectors per row (8 fp16)
    // vectors [i0, i0 + 64) of each head's K|V rows per pass (one pass for D <= 256)
    for (int i0 = 0; i0 < 2 * vpr; i0 += 64) {
    uint4 val[kAppendHeads][2];
#pragma unroll
    for (int j = 0; j < kAppendHeads; ++j) {
        const int h = h0 + j;
        const int64_t src_elem = (tok * p.Hkv + h) * p.D;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int i = i0 + lane + 32 * k;
            if (h >= p.Hkv || i >= 2 * vpr) continue;
            const bool is_v = i >= vpr;
            const int vi = is_v ? i - vpr : i;
            if constexpr (F32) {
                const float4* src =
                    reinterpret_cast<const float4*>(static_cast<const float*>(is_v ? p.v : p.k) + src_elem) + 2 * vi;
                float4 a = __ldg(src), c = __ldg(src + 1);
                if (!is_v && p.rope_freq != nullptr) {  // rotate in fp32, then round
                    const int i0 = vi * 4;
                    float2 r;
                    r = rope_pair(a.x, a.y, i0, pos, p.rope_freq); a.x = r.x; a.y = r.y;
                    r = rope_pair(a.z, a.w, i0 + 1, pos, p.rope_freq); a.z = r.x; a.w = r.y;
                    r = rope_pair(c.x, c.y, i0 + 2, pos, p.rope_freq); c.x = r.x; c.y = r.y;
                    r = rope_pair(c.z, c.w, i0 + 3, pos, p.rope_freq); c.z = r.x; c.w = r.y;
                }
                val[j][k].x = pack_half2(a.x, a.y);
                val[j][k].y = pack_half2(a.z, a.w);
                val[j][k].z = pack_half2(c.x, c.y);
                val[j][k].w = pack_half2(c.z, c.w);
            } else {
                const uint4* src =
                    reinterpret_cast<const uint4*>(static_cast<const __half*>(is_v ? p.v : p.k) + src_elem) + vi;
                val[j][k] = __ldg(src);
                if (!is_v && p.rope_freq != nullptr) val[j][k] = rope_uint4(val[j][k], vi * 8, pos, p.rope_freq);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < kAppendHeads; ++j) {
        const int h = h0 + j;
        char* dst_k = dst0 + static_cast<uint64_t>(h) * p.head_bytes;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int i = i0 + lane + 32 * k;
            if (h >= p.Hkv || i >= 2 * vpr) continue;
            const bool is_v = i >= vpr;
            const int vi = is_v ? i - vpr : i;
            reinterpret_cast<uint4*>(dst_k + (is_v ? static_cast<uint64_t>(p.P) * p.D * 2 : 0))[vi] = val[j][k];
        }
    }
    }
}

vk_status launch_append(vk_pool* pool, int layer, const void* k, const void* v, bool f32,
                        const int32_t* bt, int bt_stride, const int32_t* pos, int B, int T,
                        cudaStream_t st) {
    const int D = pool->cfg.head_dim;
    const uintptr_t align = f32 ? 32 : 16;
    if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) % align)
        return fail(VK_INVALID_ARG, "k_new/v_new must be 16-byte aligned (32 for fp32)");
    AppendParams p;
    p.base = pool->base;
    p.k = k;
    p.v = v;
    p.bt = bt;
    p.pos = pos;
    p.err = pool->d_err;
    p.seg_bytes = pool->seg_bytes;
    p.layer_off = static_cast<uint64_t>(layer) * pool->seg_stride;
    p.head_bytes = pool->head_bytes;
    p.bt_stride = bt_stride;
    p.B = B;
    p.T = T;
    p.Hkv = pool->cfg.num_kv_heads;
    p.D = D;
    p.P = pool->cfg.page_tokens;
    p.num_pages = pool->num_pages;
    p.rope_freq = pool->kv ? pool->rope_freq : nullptr;
    const int64_t groups = (p.Hkv + kAppendHeads - 1) / kAppendHeads;
    const int64_t threads = static_cast<int64_t>(B) * T * groups * 32;
    const int64_t blocks = (threads + 255) / 256;
    if (blocks > 0x7fffffff) return fail(VK_INVALID_ARG, "append too large for one launch");
    if (f32)
        append_kernel<true><<<static_cast<unsigned>(blocks), 256, 0, st>>>(p);
    else
        append_kernel<false><<<static_cast<unsigned>(blocks), 256, 0, st>>>(p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? VK_OK : cuda_fail(e, "append_kernel launch");
}

// ---------------------------------------------------------------- K1 on FP8 pools

// One warp per (token, kv head): the K row (rotated first when RoPE is on) and
// the V row are quantised in fp32 (vk_fp8.cuh) from the fp16 or fp32 inputs and
// written as codes and scales into the token's slot of its page block.
template <bool F32>
__global__ void __launch_bounds__(256) append_fp8_kernel(const AppendParams p) {
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t rows = static_cast<int64_t>(p.B) * p.T * p.Hkv;
    if (row >= rows) return;
    const int h = static_cast<int>(row % p.Hkv);
    const int64_t bt_idx = row / p.Hkv;
    const int t = static_cast<int>(bt_idx % p.T);
    const int b = static_cast<int>(bt_idx / p.T);
    const int pos = p.pos[b] + t;
    if (pos < 0 || pos / p.P >= p.bt_stride) {
        if (lane == 0) atomicOr(p.err, VK_ERR_TABLE_INDEX);
        return;
    }
    const int32_t page = p.bt[static_cast<int64_t>(b) * p.bt_stride + pos / p.P];
    if (page < 0 || page >= p.num_pages) {
        if (lane == 0) atomicOr(p.err, VK_ERR_PAGE_ID);
        return;
    }
    const int64_t src = row * kFp8Dim + 4 * lane;
    float xk[4], xv[4];
    if constexpr (F32) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p.k) + src));
        const float4 c = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p.v) + src));
        xk[0] = a.x; xk[1] = a.y; xk[2] = a.z; xk[3] = a.w;
        xv[0] = c.x; xv[1] = c.y; xv[2] = c.z; xv[3] = c.w;
    } else {
        const uint2 kw = __ldg(reinterpret_cast<const uint2*>(static_cast<const __half*>(p.k) + src));
        const uint2 vw = __ldg(reinterpret_cast<const uint2*>(static_cast<const __half*>(p.v) + src));
        float2 f;
        f = __half22float2(*reinterpret_cast<const __half2*>(&kw.x)); xk[0] = f.x; xk[1] = f.y;
        f = __half22float2(*reinterpret_cast<const __half2*>(&kw.y)); xk[2] = f.x; xk[3] = f.y;
        f = __half22float2(*reinterpret_cast<const __half2*>(&vw.x)); xv[0] = f.x; xv[1] = f.y;
        f = __half22float2(*reinterpret_cast<const __half2*>(&vw.y)); xv[2] = f.x; xv[3] = f.y;
    }
    if (p.rope_freq != nullptr) {
        float2 f;
        f = rope_pair(xk[0], xk[1], 2 * lane, pos, p.rope_freq); xk[0] = f.x; xk[1] = f.y;
        f = rope_pair(xk[2], xk[3], 2 * lane + 1, pos, p.rope_freq); xk[2] = f.x; xk[3] = f.y;
    }
    float ks, vs;
    const uint32_t kc = fp8_quant_row(xk, ks);
    const uint32_t vc = fp8_quant_row(xv, vs);
    char* blk = p.base + p.layer_off + static_cast<uint64_t>(page) * p.seg_bytes + static_cast<uint64_t>(h) * p.head_bytes;
    fp8_store_token(blk, pos % p.P, lane, kc, vc, ks, vs);
}

vk_status launch_append_fp8(vk_pool* pool, int layer, const void* k, const void* v, bool f32,
                            const int32_t* bt, int bt_stride, const int32_t* pos, int B, int T,
                            cudaStream_t st) {
    if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) % 16)
        return fail(VK_INVALID_ARG, "k_new/v_new must be 16-byte aligned");
    AppendParams p;
    p.base = pool->base;
    p.k = k;
    p.v = v;
    p.bt = bt;
    p.pos = pos;
    p.err = pool->d_err;
    p.seg_bytes = pool->seg_bytes;
    p.layer_off = static_cast<uint64_t>(layer) * pool->seg_stride;
    p.head_bytes = pool->head_bytes;
    p.bt_stride = bt_stride;
    p.B = B;
    p.T = T;
    p.Hkv = pool->cfg.num_kv_heads;
    p.D = pool->cfg.head_dim;
    p.P = pool->cfg.page_tokens;
    p.num_pages = pool->num_pages;
    p.rope_freq = pool->rope_freq;
    const int64_t threads = static_cast<int64_t>(B) * T * p.Hkv * 32;
    const int64_t blocks = (threads + 255) / 256;
    if (blocks > 0x7fffffff) return fail(VK_INVALID_ARG, "append too large for one launch");
    if (f32)
        append_fp8_kernel<true><<<static_cast<unsigned>(blocks), 256, 0, st>>>(p);
    else
        append_fp8_kernel<false><<<static_cast<unsigned>(blocks), 256, 0, st>>>(p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? VK_OK : cuda_fail(e, "append_fp8_kernel launch");
}

// ---------------------------------------------------------------- K4 copy

constexpr int kCopyThreads = 512;
constexpr int kCopyUnroll = 4;
constexpr uint64_t kCopyChunk = static_cast<uint64_t>(kCopyThreads) * kCopyUnroll * 16;  // 32 KiB

// grid.x = (32 KiB chunks of a segment) x segments, grid.y = page pairs.  Each
// CTA moves one chunk of one layer segment of one page with 16-byte loads
// issued ahead of the stores.
__global__ void __launch_bounds__(kCopyThreads) copy_pages_kernel(char* base, uint64_t seg_bytes,
                                                                  uint64_t seg_stride, int chunks_per_seg,
                                                                  const int32_t* src, const int32_t* dst,
                                                                  int num_pages, uint32_t* err) {
    const int pair = blockIdx.y;
    const int32_t s = src[pair], d = dst[pair];
    if (s < 0 || s >= num_pages || d < 0 || d >= num_pages) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(err, VK_ERR_PAGE_ID);
        return;
    }
    const int seg = blockIdx.x / chunks_per_seg;
    const uint64_t off = static_cast<uint64_t>(blockIdx.x % chunks_per_seg) * kCopyChunk;
    const uint64_t seg_off = static_cast<uint64_t>(seg) * seg_stride;
    const uint4* sp = reinterpret_cast<const uint4*>(base + seg_off + static_cast<uint64_t>(s) * seg_bytes + off);
    uint4* dp = reinterpret_cast<uint4*>(base + seg_off + static_cast<uint64_t>(d) * seg_bytes + off);
    const uint64_t left = seg_bytes - off;
    const int nvec = static_cast<int>((left < kCopyChunk ? left : kCopyChunk) / 16);
    uint4 r[kCopyUnroll];
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) {
        const int i = threadIdx.x + u * kCopyThreads;
        if (i < nvec) r[u] = __ldcs(sp + i);
    }
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) {
        const int i = threadIdx.x + u * kCopyThreads;
        if (i < nvec) __stcs(dp + i, r[u]);
    }
}

vk_status launch_copy_pages(vk_pool* pool, const int32_t* src, const int32_t* dst, int n,
                            cudaStream_t st) {
    if (pool->seg_bytes % 16) return fail(VK_UNSUPPORTED, "copy needs page segments of a multiple of 16 bytes");
    if (n > 65535) return fail(VK_INVALID_ARG, "copy_pages: at most 65535 pages per call");
    const uint64_t chunks = (pool->seg_bytes + kCopyChunk - 1) / kCopyChunk;
    const uint64_t blocks = chunks * static_cast<uint64_t>(pool->nseg);
    if (blocks > 0x7fffffff) return fail(VK_INVALID_ARG, "page too large");
    dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(n));
    copy_pages_kernel<<<grid, kCopyThreads, 0, st>>>(pool->base, pool->seg_bytes, pool->seg_stride,
                                                     static_cast<int>(chunks), src, dst, pool->num_pages,
                                                     pool->d_err);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? VK_OK : cuda_fail(e, "copy_pages_kernel launch");
}

// ---------------------------------------------------------------- remap

__global__ void remap_kernel(int32_t* bt, int64_t entries, const int32_t* map, int map_len) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < entries;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int32_t e = bt[i];
        if (e >= 0 && e < map_len) bt[i] = map[e];
    }
}

vk_status launch_remap(int32_t* bt, int64_t entries, const int32_t* map, int map_len,
                       cudaStream_t st) {
    int64_t blocks = (entries + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    remap_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(bt, entries, map, map_len);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? VK_OK : cuda_fail(e, "remap_kernel launch");
}

}  // namespace vk
