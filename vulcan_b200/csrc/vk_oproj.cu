// Output projection after head-sharded attention, fused with its
// reduce-scatter (row 8f.3: the `wo` matmul of the reference's self_attention,
// src/transformer.cpp:191-194, launch_matmul's contract C = A * B,
// cuda/matmul.cu:42-103).
//
// With KV heads sharded over `world` GPUs, rank r holds the attention output of
// its heads, x_r = x[:, K_r] ([tokens, k_local] fp16, k_local = its heads x
// head_dim), and the matching rows of wo, W_r = wo[K_r, :].  The projection is
// y = sum_r x_r W_r; rank r keeps the output features
// [r*n_out/world, (r+1)*n_out/world) of y (a reduce-scatter over features), so
// no rank needs another rank's attention output.
//
// One launch per layer computes and communicates tile by tile:
//
//  * CTA (tile, split): 128 output features x all tokens, over one of `splits`
//    ranges of k_local.  out^T tile = W_r^T x_r^T on tcgen05 (kind::f16,
//    M = 128 features, N = tokens rounded to 16, fp32 accumulator in TMEM):
//    warp 4 streams the weights and x into a ring of up to 8 stages (~192 KiB,
//    one CTA per SM), warp 5 issues the
//    MMAs (one thread) and owns the TMEM.  The weights are packed once
//    (vk_oproj_pack_weight*) into 16 KiB blocks of 128 features x 64 k, each
//    already in the 128-byte-swizzled shared-memory layout the MMA reads, so
//    a stage's weights are one contiguous bulk copy (strided 128-byte row reads
//    ran at a third of HBM bandwidth); x, re-read by every tile from L2, comes
//    by 2-D TMA.
//  * Epilogue (warps 0-3, one thread per feature = TMEM lane): the fp32 partial
//    goes straight to the receive buffer of the rank that owns the tile, over
//    NVLink for a peer (plain stores, coalesced: a warp writes 32 consecutive
//    features of one token), then one system-scope release raises the tile's
//    flag for (this rank, this split) on the owner.
//  * Then every CTA sums a token slice of one tile of its own rank: it waits
//    (bounded, 1 s) until the flags of all world*splits contributions to that
//    tile carry this run's sequence number, then adds them in rank-then-split
//    order (so the result does not depend on arrival order) and writes y in
//    fp16.  Spreading the sum over the grid keeps it to a few round trips.
//
// The grid is launched cooperatively (every CTA resident at once), so a CTA
// that waits for the other splits of its tile on this GPU cannot block them.
// Every rank makes the same runs in the same order on one stream each; run n
// uses receive slot n % 2 and flag value n.  A rank can reuse a slot only after
// finishing the next run, which needs every rank's contributions to it, and
// those start after the rank's earlier run has completed: two slots suffice.
// The run number lives in device memory (read by every CTA at its start, moved
// on by the last CTA to finish), so a captured launch can be replayed.
#include <algorithm>
#include <cstdio>
#include <cstring>

#include "vk_gather.cuh"
#include "vk_internal.h"
#include "vk_ptx.cuh"
#include "vk_tc.cuh"

namespace vk {

constexpr int kOpFeat = 128;       // output features per tile (MMA M, TMEM lanes)
constexpr int kOpK = 64;           // k per stage (one 128-byte swizzled row)
constexpr int kOpMaxStages = 8;    // ring depth: as many stages as fit in ~192 KiB
constexpr int kOpRingBytes = 192 * 1024;
constexpr int kOpSmemLimit = 232448;  // dynamic shared memory of one CTA on sm_100
constexpr int kOpThreads = 192;    // warps 0-3 epilogue, 4 TMA, 5 MMA
constexpr int kOpMaxTokens = 256;
constexpr int kOpSlots = 2;

struct OprojParams {
    const char* w;           // packed weights [n_out/128][k_local/64][16 KiB]
    __half* y;
    int ldy;                 // row stride of y (elements)
    int tokens, ntok;        // tokens, tokens rounded up to 16 (MMA N)
    int kblocks;             // k_local / 64
    int kb_per_split, splits;
    int stages;              // ring depth (<= kOpMaxStages)
    int tiles_local;         // tiles each rank owns: n_out / world / 128
    int rank, world;
    char* base[kMaxGatherRanks];
    uint64_t slot_bytes, slice_bytes, flags_off, err_off;
    int feat_local;          // n_out / world (row stride of a receive slice)
};

__host__ __device__ constexpr int op_stage_bytes(int ntok) { return kOpFeat * 128 + ntok * 128; }
__host__ __device__ constexpr int op_stages(int ntok) {
    return kOpRingBytes / op_stage_bytes(ntok) < kOpMaxStages ? kOpRingBytes / op_stage_bytes(ntok) : kOpMaxStages;
}
__host__ __device__ constexpr int op_smem_bytes(int ntok, int stages) { return stages * op_stage_bytes(ntok) + 1024 + 256; }

__device__ __forceinline__ uint32_t* op_flag(const OprojParams& p, int slot, int on_rank, int tloc, int contrib) {
    return reinterpret_cast<uint32_t*>(p.base[on_rank] + p.flags_off) +
           (static_cast<int64_t>(slot) * p.tiles_local + tloc) * (p.world * p.splits) + contrib;
}

// Sum of the contributions to one tile for tokens [tok_lo, tok_hi): warp w
// takes a quarter of the tokens, lane l the 4 features 4l..4l+3 (float4 loads,
// 8-byte fp16 stores); y = sum over c = 0 .. ncontrib-1 in that order, fp32.
// CC contributions x TB tokens are loaded before any is added, so the loads of
// a batch are in flight together.
template <int CC, int TB>
__device__ __forceinline__ void op_sum_slice(const OprojParams& p, const float* tile_src, __half* tile_y, int ncontrib,
                                             int tok_lo, int tok_hi, int warp, int lane) {
    const int64_t slice4 = static_cast<int64_t>(p.slice_bytes / 16);  // float4 per contribution slice
    const int64_t row4 = p.feat_local / 4;                            // float4 per token row
    const float4* base = reinterpret_cast<const float4*>(tile_src) + lane;
    const int per_w = (tok_hi - tok_lo + 3) / 4;
    const int a = tok_lo + warp * per_w, b = min(tok_hi, a + per_w);
    for (int t0 = a; t0 < b; t0 += TB) {
        float4 acc[TB];
#pragma unroll
        for (int j = 0; j < TB; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int c0 = 0; c0 < ncontrib; c0 += CC) {
            float4 v[CC][TB];
#pragma unroll
            for (int cc = 0; cc < CC; ++cc)
#pragma unroll
                for (int j = 0; j < TB; ++j) {
                    const int c = c0 + cc, tok = t0 + j;
                    v[cc][j] = (c < ncontrib && tok < b) ? __ldcg(base + c * slice4 + tok * row4)
                                                         : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
            for (int cc = 0; cc < CC; ++cc)
#pragma unroll
                for (int j = 0; j < TB; ++j)
                    if (c0 + cc < ncontrib) {
                        acc[j].x += v[cc][j].x;
                        acc[j].y += v[cc][j].y;
                        acc[j].z += v[cc][j].z;
                        acc[j].w += v[cc][j].w;
                    }
        }
#pragma unroll
        for (int j = 0; j < TB; ++j)
            if (t0 + j < b) {
                const __half2 lo = __floats2half2_rn(acc[j].x, acc[j].y), hi = __floats2half2_rn(acc[j].z, acc[j].w);
                uint2 w2;
                w2.x = *reinterpret_cast<const uint32_t*>(&lo);
                w2.y = *reinterpret_cast<const uint32_t*>(&hi);
                *reinterpret_cast<uint2*>(tile_y + static_cast<int64_t>(t0 + j) * p.ldy + 4 * lane) = w2;
            }
    }
}

__device__ __forceinline__ uint32_t ld_acquire_gpu32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void named_bar(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__global__ void __launch_bounds__(kOpThreads, 1)
oproj_kernel(const __grid_constant__ CUtensorMap tmap_x, const OprojParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const int stage_bytes = op_stage_bytes(p.ntok);
    const int NS = p.stages;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NS * stage_bytes);
    uint64_t* full = bars;                  // [stages]
    uint64_t* empty = bars + NS;            // [stages]
    uint64_t* acc_full = bars + 2 * NS;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * NS + 1);
    uint32_t* err = reinterpret_cast<uint32_t*>(p.base[p.rank] + p.err_off);
    uint32_t* runs = err + 1;       // runs completed on this rank
    uint32_t* exits = err + 2;      // CTAs of this run that have finished
    const uint32_t seq = *reinterpret_cast<volatile uint32_t*>(runs) + 1u;
    const int slot = static_cast<int>(seq % kOpSlots);

    const int tile = blockIdx.x, split = blockIdx.y;
    const int owner = tile / p.tiles_local, tloc = tile % p.tiles_local;
    const int kb0 = split * p.kb_per_split;
    const int nkb = max(0, min(p.kblocks, kb0 + p.kb_per_split) - kb0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t tmem_cols = p.ntok <= 32 ? 32u : p.ntok <= 64 ? 64u : p.ntok <= 128 ? 128u : 256u;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2 * NS + 1; ++i) mbar_init(smem_u32(&bars[i]), 1);
        mbar_fence_init();
    }
    if (warp == 5) {
        tmem_alloc(smem_u32(tmem_slot), tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        // -------------------------------------------------------- TMA producer
        if (lane == 0) {
            prefetch_tmap(&tmap_x);
            const uint64_t pol = l2_evict_first_policy();   // weights: read once
            const uint64_t pol_x = l2_evict_last_policy();  // x: read by every tile
            for (int i = 0; i < nkb; ++i) {
                const int st = i % NS;
                if (i >= NS && !mbar_wait(smem_u32(&empty[st]), ((i / NS) - 1) & 1, err)) break;
                const uint32_t bar = smem_u32(&full[st]);
                mbar_expect_tx(bar, stage_bytes);
                const uint32_t dst = sbase + st * stage_bytes;
                const int k0 = (kb0 + i) * kOpK;
                bulk_load(dst, p.w + (static_cast<int64_t>(tile) * p.kblocks + kb0 + i) * (kOpFeat * 128),
                          kOpFeat * 128, bar, pol);                                  // 128 features x 64 k
                tma_load_2d(dst + kOpFeat * 128, &tmap_x, k0, 0, bar, pol_x);     // ntok tokens x 64 k
            }
        }
    } else if (warp == 5) {
        // -------------------------------------------------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_f16(kOpFeat, static_cast<uint32_t>(p.ntok));
            bool ok = true;
            for (int i = 0; i < nkb && ok; ++i) {
                const int st = i % NS;
                ok = mbar_wait(smem_u32(&full[st]), (i / NS) & 1, err);
                if (!ok) break;
                tc_fence_after();
                const uint32_t a = sbase + st * stage_bytes;
                const uint64_t da = umma_desc_sw128(a, 16, 1024);
                const uint64_t db = umma_desc_sw128(a + kOpFeat * 128, 16, 1024);
#pragma unroll
                for (int ks = 0; ks < kOpK / 16; ++ks)
                    umma_ss(tmem, da + static_cast<uint64_t>((ks * 32) >> 4), db + static_cast<uint64_t>((ks * 32) >> 4),
                            idesc, (i > 0 || ks > 0) ? 1u : 0u);
                umma_commit(smem_u32(&empty[st]));
            }
            umma_commit(smem_u32(&acc_full[0]));  // after every MMA issued above
        }
    } else {
        // -------------------------------------------------------- epilogue: partial -> owner
        const int t = threadIdx.x;                 // feature row of the tile = TMEM lane
        const bool ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(acc_full), 0, err));
        tc_fence_after();
        float* dst = reinterpret_cast<float*>(p.base[owner] + static_cast<uint64_t>(slot) * p.slot_bytes +
                                              static_cast<uint64_t>(p.rank * p.splits + split) * p.slice_bytes) +
                     tloc * kOpFeat + t;
        const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
        for (int c = 0; c < p.ntok; c += 32) {
            float v[32];
            tmem_ld32(lane_addr + c, v);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int tok = c + j;
                if (tok < p.tokens) dst[static_cast<int64_t>(tok) * p.feat_local] = (ok && nkb > 0) ? v[j] : 0.f;
            }
        }
        named_bar(1, 128);  // every epilogue thread's stores precede the flag
        if (t == 0) {
            // one rank: everything stays on this GPU, so GPU scope suffices
            // (a system-scope fence after the partial's stores measured ~7 us)
            if (p.world == 1) {
                asm volatile("fence.acq_rel.gpu;" ::: "memory");
                asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(op_flag(p, slot, owner, tloc, p.rank * p.splits + split)),
                             "r"(seq)
                             : "memory");
            } else {
                asm volatile("fence.acq_rel.sys;" ::: "memory");
                st_release_sys(op_flag(p, slot, owner, tloc, p.rank * p.splits + split), seq);
            }
        }
        // ---------------------------------------------------- sum a slice of a tile this rank owns
        // Every CTA, once its own partial is out, sums the contributions to a
        // token slice of one of this rank's tiles (CTA c: tile c % tiles_local,
        // slice c / tiles_local), so the reduction is spread over the grid.
        const int cta = tile * p.splits + split;
        const int per_tile = static_cast<int>(gridDim.x * gridDim.y) / p.tiles_local;
        const int jt = cta % p.tiles_local, slice = cta / p.tiles_local;
        if (slice < per_tile) {
            const int tok_lo = slice * p.tokens / per_tile, tok_hi = (slice + 1) * p.tokens / per_tile;
            const int ncontrib = p.world * p.splits;
            if (t == 0) {
                const uint64_t t0 = global_ns();
                for (int c = 0; c < ncontrib; ++c) {
                    const uint32_t* f = op_flag(p, slot, p.rank, jt, c);
                    bool timed_out = false;
                    while (static_cast<int32_t>((p.world == 1 ? ld_acquire_gpu32(f) : ld_acquire_sys(f)) - seq) < 0) {
                        if ((*reinterpret_cast<volatile uint32_t*>(err) & VK_ERR_TIMEOUT) ||
                            global_ns() - t0 > kGatherWaitNs) {
                            atomicOr(err, VK_ERR_TIMEOUT);
                            timed_out = true;
                            break;
                        }
                        __nanosleep(64);
                    }
                    if (timed_out) break;
                }
            }
            named_bar(1, 128);
            const float* src = reinterpret_cast<const float*>(p.base[p.rank] + static_cast<uint64_t>(slot) * p.slot_bytes) +
                               jt * kOpFeat;
            __half* yo = p.y + jt * kOpFeat;
            if (ncontrib <= 2) op_sum_slice<2, 8>(p, src, yo, ncontrib, tok_lo, tok_hi, warp, lane);
            else if (ncontrib <= 4) op_sum_slice<4, 4>(p, src, yo, ncontrib, tok_lo, tok_hi, warp, lane);
            else op_sum_slice<8, 2>(p, src, yo, ncontrib, tok_lo, tok_hi, warp, lane);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, tmem_cols);
    }
    // the last CTA to finish moves the run number on (every CTA has read it)
    if (threadIdx.x == 0 && atomicAdd(exits, 1u) == gridDim.x * gridDim.y - 1) {
        *exits = 0u;
        *runs = seq;
    }
}

// Byte offset of weight element (feature f, k) in the packed layout: 16 KiB
// blocks [n/128][k_rows/64], each 128 rows (features) of 64 k; the 16-byte
// chunk c of row r sits at chunk c ^ (r & 7) (the 128-byte swizzle of a TMA
// box, which the UMMA descriptor expects).
__device__ __forceinline__ int64_t op_packed_off(int f, int k, int kblocks) {
    const int r = f & 127, c = (k & 63) >> 3;
    return ((static_cast<int64_t>(f >> 7) * kblocks + (k >> 6)) * 128 + r) * 128 + ((c ^ (r & 7)) << 4) + ((k & 7) << 1);
}

// fp32 [k_rows, n] (row stride ldw, the reference's wo rows) -> packed fp16
__global__ void oproj_pack_kernel(const float* __restrict__ w, int ldw, int k_rows, int n, char* __restrict__ wp) {
    __shared__ float tile[32][33];
    const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int k = k0 + r, c = n0 + threadIdx.x;
        tile[r][threadIdx.x] = (k < k_rows && c < n) ? w[static_cast<int64_t>(k) * ldw + c] : 0.f;
    }
    __syncthreads();
    const int kblocks = k_rows >> 6;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int f = n0 + r, k = k0 + threadIdx.x;
        if (f < n && k < k_rows)
            *reinterpret_cast<__half*>(wp + op_packed_off(f, k, kblocks)) = __float2half(tile[threadIdx.x][r]);
    }
}

// fp16 [n, k_rows] rows (row stride ldw: an nn.Linear [out, in] weight or a
// column slice of it) -> packed; one thread per 16-byte chunk
__global__ void oproj_pack_t16_kernel(const __half* __restrict__ wt, int ldw, int n, int k_rows, char* __restrict__ wp) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int chunks = k_rows >> 3;
    if (i >= static_cast<int64_t>(n) * chunks) return;
    const int f = static_cast<int>(i / chunks), k = static_cast<int>(i % chunks) * 8;
    const uint4 v = *reinterpret_cast<const uint4*>(wt + static_cast<int64_t>(f) * ldw + k);
    *reinterpret_cast<uint4*>(wp + op_packed_off(f, k, k_rows >> 6)) = v;
}

static int op_occupancy(int device, int ntok) {
    static bool attr_set[64] = {};
    if (device < 0 || device >= 64) return 0;
    if (!attr_set[device]) {
        if (cudaFuncSetAttribute(oproj_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kOpSmemLimit) != cudaSuccess)
            return 0;
        attr_set[device] = true;
    }
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, oproj_kernel, kOpThreads, op_smem_bytes(ntok, op_stages(ntok))) !=
        cudaSuccess)
        return 0;
    return occ;
}

}  // namespace vk

struct vk_oproj {
    int device = 0, rank = 0, world = 0, max_tokens = 0, k_local = 0, n_out = 0;
    int splits = 1, stages = 4, tiles_local = 0, num_sms = 148;
    uint64_t slice_bytes = 0, slot_bytes = 0, flags_off = 0, err_off = 0, total = 0;
    char* own = nullptr;
    char* peer[vk::kMaxGatherRanks] = {};
    bool imported[vk::kMaxGatherRanks] = {};
    bool local[vk::kMaxGatherRanks] = {};
};

using namespace vk;

extern "C" {

vk_status vk_oproj_create(int32_t device, int32_t rank, int32_t world, int32_t max_tokens, int32_t k_local,
                          int32_t n_out, vk_oproj** out) {
    if (!out) return fail(VK_INVALID_ARG, "out is NULL");
    *out = nullptr;
    if (world < 1 || world > kMaxGatherRanks) return fail(VK_UNSUPPORTED, "output projection supports 1..8 ranks");
    if (rank < 0 || rank >= world) return fail(VK_INVALID_ARG, "rank outside [0, world)");
    if (max_tokens < 1 || max_tokens > kOpMaxTokens) return fail(VK_UNSUPPORTED, "max_tokens must be in 1..256");
    if (k_local <= 0 || k_local % kOpK) return fail(VK_UNSUPPORTED, "k_local must be a positive multiple of 64");
    if (n_out <= 0 || n_out % (kOpFeat * world)) return fail(VK_UNSUPPORTED, "n_out must be a multiple of 128 * world");
    DeviceGuard dg(device);
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms <= 0)
        return fail(VK_CUDA_ERROR, "cannot query the device");
    const int ntok = (max_tokens + 15) / 16 * 16;
    const int occ = op_occupancy(device, ntok);
    if (occ <= 0) return fail(VK_CUDA_ERROR, "occupancy query for the output projection kernel failed");
    const int tiles = n_out / kOpFeat;
    const int kblocks = k_local / kOpK;
    if (tiles > sms * occ) return fail(VK_UNSUPPORTED, "n_out too large: every tile's CTA must be resident at once");
    // splits of k so that the grid fills the GPU (each split keeps >= 2 k-blocks)
    // k splits: enough CTAs to cover the SMs (each keeps >= 2 k-blocks), but
    // the fp32 partials they add (splits * max_tokens * 4 bytes per feature)
    // stay within ~1/8 of the weight bytes (k_local * 2 per feature)
    int splits = std::max(1, std::min(sms * occ / tiles, kblocks / 2));
    splits = std::min(splits, std::max(1, (k_local * 2) / (8 * max_tokens * 4)));
    const int kb_per_split = (kblocks + splits - 1) / splits;
    splits = (kblocks + kb_per_split - 1) / kb_per_split;  // no empty split
    auto* h = new vk_oproj();
    h->device = device;
    h->rank = rank;
    h->world = world;
    h->max_tokens = max_tokens;
    h->k_local = k_local;
    h->n_out = n_out;
    h->splits = splits;
    h->stages = op_stages(ntok);
    h->tiles_local = tiles / world;
    h->num_sms = sms;
    const uint64_t feat_local = static_cast<uint64_t>(n_out / world);
    h->slice_bytes = (static_cast<uint64_t>(max_tokens) * feat_local * 4 + 255) & ~uint64_t(255);
    h->slot_bytes = h->slice_bytes * static_cast<uint64_t>(world) * splits;
    h->flags_off = h->slot_bytes * kOpSlots;
    const uint64_t nflags = static_cast<uint64_t>(kOpSlots) * h->tiles_local * world * splits;
    h->err_off = h->flags_off + ((nflags * 4 + 255) & ~uint64_t(255));
    h->total = h->err_off + 256;
    cudaError_t e = cudaMalloc(&h->own, h->total);
    if (e == cudaSuccess) e = cudaMemset(h->own, 0, h->total);
    if (e != cudaSuccess) {
        if (h->own) cudaFree(h->own);
        delete h;
        return cuda_fail(e, "output projection buffers");
    }
    *out = h;
    return VK_OK;
}

int32_t vk_oproj_splits(const vk_oproj* h) { return h ? h->splits : -1; }

vk_status vk_oproj_export(const vk_oproj* h, void* handle_out) {
    if (!h || !handle_out) return fail(VK_INVALID_ARG, "projection or handle is NULL");
    DeviceGuard dg(h->device);
    cudaIpcMemHandle_t ipc;
    cudaError_t e = cudaIpcGetMemHandle(&ipc, h->own);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
    std::memcpy(handle_out, &ipc, sizeof(ipc));
    return VK_OK;
}

vk_status vk_oproj_import(vk_oproj* h, int32_t peer, const void* handle) {
    if (!h || !handle) return fail(VK_INVALID_ARG, "projection or handle is NULL");
    if (peer < 0 || peer >= h->world || peer == h->rank) return fail(VK_INVALID_ARG, "peer outside [0, world) or own rank");
    if (h->imported[peer]) return fail(VK_INVALID_ARG, "peer already imported");
    DeviceGuard dg(h->device);
    cudaIpcMemHandle_t ipc;
    std::memcpy(&ipc, handle, sizeof(ipc));
    void* ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&ptr, ipc, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    h->peer[peer] = static_cast<char*>(ptr);
    h->imported[peer] = true;
    return VK_OK;
}

vk_status vk_oproj_import_local(vk_oproj* h, int32_t peer, const vk_oproj* ph) {
    if (!h || !ph) return fail(VK_INVALID_ARG, "projection or peer projection is NULL");
    if (peer < 0 || peer >= h->world || peer == h->rank) return fail(VK_INVALID_ARG, "peer outside [0, world) or own rank");
    if (h->imported[peer]) return fail(VK_INVALID_ARG, "peer already imported");
    if (ph->rank != peer || ph->world != h->world || ph->total != h->total || ph->splits != h->splits)
        return fail(VK_INVALID_ARG, "peer projection has another rank or shape");
    if (ph->device != h->device) {
        DeviceGuard dg(h->device);
        int ok = 0;
        cudaError_t e = cudaDeviceCanAccessPeer(&ok, h->device, ph->device);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceCanAccessPeer");
        if (!ok) return fail(VK_UNSUPPORTED, "no peer access between the two devices");
        e = cudaDeviceEnablePeerAccess(ph->device, 0);
        if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
        else if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceEnablePeerAccess");
    }
    h->peer[peer] = ph->own;
    h->imported[peer] = true;
    h->local[peer] = true;
    return VK_OK;
}

vk_status vk_oproj_release_peers(vk_oproj* h) {
    if (!h) return fail(VK_INVALID_ARG, "projection is NULL");
    DeviceGuard dg(h->device);
    cudaError_t e = cudaDeviceSynchronize();
    for (int r = 0; r < h->world; ++r)
        if (h->imported[r]) {
            if (!h->local[r]) {
                cudaError_t c = cudaIpcCloseMemHandle(h->peer[r]);
                if (e == cudaSuccess) e = c;
            }
            h->imported[r] = h->local[r] = false;
            h->peer[r] = nullptr;
        }
    return e == cudaSuccess ? VK_OK : cuda_fail(e, "closing peer mappings");
}

vk_status vk_oproj_destroy(vk_oproj* h) {
    if (!h) return VK_OK;
    vk_status s = vk_oproj_release_peers(h);
    DeviceGuard dg(h->device);
    cudaError_t e = cudaFree(h->own);
    delete h;
    if (s != VK_OK) return s;
    return e == cudaSuccess ? VK_OK : cuda_fail(e, "cudaFree(output projection buffers)");
}

vk_status vk_oproj_check(vk_oproj* h) {
    if (!h) return fail(VK_INVALID_ARG, "projection is NULL");
    DeviceGuard dg(h->device);
    uint32_t bits = 0;
    cudaError_t e = cudaMemcpy(&bits, h->own + h->err_off, sizeof(bits), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(projection error word)");
    if (bits == 0) return VK_OK;
    e = cudaMemset(h->own + h->err_off, 0, sizeof(bits));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(projection error word)");
    return fail(VK_TIMEOUT, "an output-projection wait gave up: a contribution did not arrive within 1 s");
}

size_t vk_oproj_packed_bytes(int32_t k_rows, int32_t n) {
    if (k_rows <= 0 || n <= 0 || k_rows % kOpK || n % kOpFeat) return 0;
    return static_cast<size_t>(k_rows) * n * 2;
}

vk_status vk_oproj_pack_weight(const float* w, int32_t ldw, int32_t k_rows, int32_t n, void* w_packed, void* stream) {
    if (!w || !w_packed || vk_oproj_packed_bytes(k_rows, n) == 0 || ldw < n)
        return fail(VK_INVALID_ARG, "bad weight pack arguments (k_rows a multiple of 64, n of 128)");
    if (reinterpret_cast<uintptr_t>(w_packed) & 15) return fail(VK_INVALID_ARG, "w_packed must be 16-byte aligned");
    const dim3 grid((n + 31) / 32, (k_rows + 31) / 32), block(32, 8);
    oproj_pack_kernel<<<grid, block, 0, as_stream(stream)>>>(w, ldw, k_rows, n, static_cast<char*>(w_packed));
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? VK_OK : cuda_fail(e, "oproj_pack_kernel launch");
}

vk_status vk_oproj_pack_weight_t16(const void* w_t, int32_t ldw, int32_t n, int32_t k_rows, void* w_packed,
                                   void* stream) {
    if (!w_t || !w_packed || vk_oproj_packed_bytes(k_rows, n) == 0 || ldw < k_rows || (ldw % 8))
        return fail(VK_INVALID_ARG, "bad weight pack arguments (k_rows a multiple of 64, n of 128, ldw of 8)");
    if ((reinterpret_cast<uintptr_t>(w_t) | reinterpret_cast<uintptr_t>(w_packed)) & 15)
        return fail(VK_INVALID_ARG, "w_t and w_packed must be 16-byte aligned");
    const int64_t chunks = static_cast<int64_t>(n) * (k_rows / 8);
    oproj_pack_t16_kernel<<<static_cast<unsigned>((chunks + 255) / 256), 256, 0, as_stream(stream)>>>(
        static_cast<const __half*>(w_t), ldw, n, k_rows, static_cast<char*>(w_packed));
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? VK_OK : cuda_fail(e, "oproj_pack_t16_kernel launch");
}

vk_status vk_oproj_run(vk_oproj* h, const void* x, int32_t ldx, const void* w_packed, void* y, int32_t ldy,
                       int32_t tokens, void* stream) {
    if (!h) return fail(VK_INVALID_ARG, "projection is NULL");
    for (int r = 0; r < h->world; ++r)
        if (r != h->rank && !h->imported[r]) return fail(VK_INVALID_ARG, "projection has peers not imported");
    if (!x || !w_packed || !y) return fail(VK_INVALID_ARG, "NULL array");
    if (tokens < 1 || tokens > h->max_tokens) return fail(VK_INVALID_ARG, "tokens outside 1..max_tokens");
    if (ldx < h->k_local || (ldx % 8)) return fail(VK_INVALID_ARG, "ldx must be >= k_local and a multiple of 8");
    if (ldy < h->n_out / h->world) return fail(VK_INVALID_ARG, "ldy smaller than n_out / world");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w_packed)) & 15)
        return fail(VK_INVALID_ARG, "x and w_packed must be 16-byte aligned");
    if ((reinterpret_cast<uintptr_t>(y) & 7) || (ldy % 4)) return fail(VK_INVALID_ARG, "y must be 8-byte aligned with ldy a multiple of 4");
    auto encode = tmap_encode_fn();
    if (!encode) return fail(VK_CUDA_ERROR, "cuTensorMapEncodeTiled unavailable");
    const int ntok = (tokens + 15) / 16 * 16;
    alignas(64) CUtensorMap tx;
    {
        // rows past `tokens` read as zeros (out-of-bounds fill)
        cuuint64_t dims[2] = {static_cast<cuuint64_t>(h->k_local), static_cast<cuuint64_t>(tokens)};
        cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldx) * 2};
        cuuint32_t box[2] = {kOpK, static_cast<cuuint32_t>(ntok)};
        cuuint32_t estr[2] = {1, 1};
        CUresult r = encode(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(VK_CUDA_ERROR, "cuTensorMapEncodeTiled(x) failed");
    }
    OprojParams p{};
    p.w = static_cast<const char*>(w_packed);
    p.y = static_cast<__half*>(y);
    p.ldy = ldy;
    p.tokens = tokens;
    p.ntok = ntok;
    p.kblocks = h->k_local / kOpK;
    p.splits = h->splits;
    p.kb_per_split = (p.kblocks + h->splits - 1) / h->splits;
    p.stages = h->stages;
    p.tiles_local = h->tiles_local;
    p.rank = h->rank;
    p.world = h->world;
    for (int r = 0; r < kMaxGatherRanks; ++r) p.base[r] = r < h->world ? (r == h->rank ? h->own : h->peer[r]) : nullptr;
    p.slot_bytes = h->slot_bytes;
    p.slice_bytes = h->slice_bytes;
    p.flags_off = h->flags_off;
    p.err_off = h->err_off;
    p.feat_local = h->n_out / h->world;
    DeviceGuard dg(h->device);
    const int smem = op_smem_bytes(ntok, h->stages);  // at most the max_tokens configuration sized at create
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(h->n_out / kOpFeat, h->splits);
    cfg.blockDim = dim3(kOpThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = as_stream(stream);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, oproj_kernel, tx, p);
    if (e != cudaSuccess) return cuda_fail(e, "oproj_kernel launch");
    return VK_OK;
}

}  // extern "C"
