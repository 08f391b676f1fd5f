// K3 chunked prefill on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Same contract and arithmetic as the mma.sync prefill in vk_prefill.cu (the
// causal j <= row rule of cpu_attention, tests/test_attention.cu:66-97, over a
// cached prefix), head_dim 128.  One CTA per (256 query rows, query head,
// sequence), one CTA per SM, 10 warps.  The 256 rows are two 128-row tiles A
// and B whose softmax steps alternate, so the tensor core always has the other
// tile's MMAs to run while one tile's softmax is on the CUDA cores:
//
//  * TMEM (512 columns): S_A at 0, S_B at 128, O_A at 256, O_B at 384.  P of a
//    tile is written as fp16 pairs over the first 64 columns of its S (after
//    the softmax has read them) and is the A operand of O += P V straight from
//    TMEM (tcgen05.mma with A in tensor memory), so P never touches shared
//    memory.
//  * warp 9 allocates TMEM and one of its threads issues every tcgen05.mma, in
//    the order S_A0, S_B0, PV_A0, S_A1, PV_B0, S_B1, PV_A1, S_A2, ... (a tile's
//    next S is issued after its PV, so P is read before S is rewritten; the
//    MMAs of one thread execute in issue order).  Completions are
//    tcgen05.commit arrivals on mbarriers; a K or V stage is released by the
//    commit after the last MMA that reads it.
//  * warp 8 lane 0 streams K and V pages with 2-D TMA boxes of 16 rows x 128 B
//    (128-byte swizzle) into separate 2-stage rings; a key tile's K and V land
//    on one barrier, so the issuer takes one data wait per key tile (its waits
//    cost ~200 cycles each even when the phase has long completed).
//  * Q: both 128-row tiles arrive by TMA (a 3-D map over [tokens][heads][d]
//    made per call) issued by thread 0 as soon as the barriers exist, so Q
//    lands together with the first K/V tile; with RoPE the softmax threads
//    rotate their rows in shared memory before Q is released to the MMAs.
//    (q not 16-byte aligned: the softmax threads load their rows instead.)
//  * warps 0-3 (tile A) and 4-7 (tile B): one thread per query row (its TMEM
//    lane).  Per key tile: the S row read from TMEM once into registers, its
//    max (masked on the causal diagonal), P = 2^(s*scale - m) packed to fp16
//    into TMEM, and O
//    rescaled in TMEM only when the row max grows by more than 2^8 (P stays
//    <= 2^8; exact after the final divide).  The scale is folded into one FMA
//    per element, the max (3-input) and sum run as four independent chains,
//    and only tiles on the causal diagonal pay for the mask.
//  * V stages start zeroed, and V rows of keys at or beyond the written length
//    in the last key tile are zeroed before that tile's PV, so stale bytes
//    cannot reach O.  All waits are bounded.
//  * FP8 pages (FMT 1, vk_fp8.cuh): warp 8 bulk-copies each key tile's e4m3
//    codes and fp32 row scales into a staging buffer, K and V apart (the next
//    tile's K loads while this tile's V is converted), and warps 10-11
//    dequantise them (code x scale as fp16 pairs; for K the
//    scale is split into two fp16 parts so it adds no rounding of its own)
//    into the same swizzled K ring and into a V^T ring (rows of head
//    dimension, keys contiguous: the FP8 block stores V element-major, so the
//    conversion writes 16-byte chunks, and PV reads V as a K-major operand).
//    Keys at or beyond the written length are written as zeros.
#include "vk_fp8.cuh"
#include "vk_internal.h"
#include "vk_ptx.cuh"
#include "vk_rope.cuh"
#include "vk_tc.cuh"

namespace vk {

constexpr int kTcRows = 128;                  // rows of one tile; a CTA has two
constexpr int kTcKeys = 128;
constexpr int kTcThreads = 320;               // fp16 pages
constexpr int kTcThreads8 = 384;              // FP8 pages: two more warps convert
constexpr int kTcD = 128;
// shared memory map (bytes from a 1024-aligned base)
constexpr int kTcQ = 0;                       // [2 tiles][2 halves][128 rows][128 B]
constexpr int kTcK = 65536;                   // 2 stages x 32 KiB
constexpr int kTcV = kTcK + 2 * 32768;        // 2 stages x 32 KiB
constexpr int kTcBar = kTcV + 2 * 32768;      // mbarriers + TMEM address
constexpr int kTcSmem = kTcBar + 256 + 1024;
// FP8 pages: staging for one key tile after the V ring, K and V apart: each
// half holds 8 pages' codes (2 KiB each) then their 16 row scales (64 bytes)
constexpr int kTcStage8 = kTcBar;
constexpr int kStgCodes = kPageTokens * kTcD;                      // 2,048
constexpr int kStgScales = (kTcKeys / kPageTokens) * kStgCodes;    // 16,384
constexpr int kStgHalf = kStgScales + (kTcKeys / kPageTokens) * 64;
constexpr int kStgPageBytes = kStgCodes + 64;                      // bytes per page and half
constexpr int kTcBar8 = kTcStage8 + 2 * kStgHalf;
static_assert(2 * kStgHalf == (kTcKeys / kPageTokens) * 4224, "FP8 staging holds one tile of page blocks");
constexpr int kTcSmem8 = kTcBar8 + 256 + 1024;
static_assert(kTcSmem8 <= 232448, "FP8 prefill shared memory");
constexpr uint32_t kTcCols = 512;

struct TcParams {
    const __half* q;
    __half* out;
    const int32_t* bt;
    const int32_t* pos;
    uint32_t* err;
    int bt_stride, T, Hq, Hkv, G, layer, num_pages, q_tiles;
    float scale_log2;
    const float* rope_freq;  // non-null: q rotated (RoPE) at its position
    // FP8 pages: block of (layer, page, head) at pool_base + layer_off + page * seg_bytes + head * head_bytes
    const char* pool_base;
    uint64_t layer_off, seg_bytes, head_bytes;
    int q_tma;  // 1: Q tiles arrive by TMA (q 16-byte aligned); 0: loaded by the softmax warps
};

// 3-input max (one instruction on sm_100)
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// Causal mask of a row's scores: key 32c + i is hidden when 32c + i > lim.
template <int NC>
__device__ __forceinline__ void mask_row(float (&v)[NC][32], int lim) {
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (c * 32 + i > lim) v[c][i] = -INFINITY;
}

__device__ __forceinline__ bool wait_warp(uint32_t bar, uint32_t parity, uint32_t* err) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, err));
}

template <int FMT>
__global__ void __launch_bounds__(FMT ? kTcThreads8 : kTcThreads, 1) prefill_tc_kernel(const __grid_constant__ CUtensorMap tmap16,
                                                                  const __grid_constant__ CUtensorMap tmapq,
                                                                  const TcParams p) {
    constexpr int P = kPageTokens;
    constexpr int NTHR = FMT ? kTcThreads8 : kTcThreads;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (FMT ? kTcBar8 : kTcBar));
    // barrier slots
    uint64_t* k_full = bars + 0;   // [2]  fp16 pages: K and V of the stage landed; FP8: K converted
    uint64_t* k_empty = bars + 2;  // [2]
    uint64_t* v_full = bars + 4;   // [2]  FP8 pages: V converted
    uint64_t* v_empty = bars + 6;  // [2]
    uint64_t* s_full = bars + 8;   // [tile]   S of the tile written
    uint64_t* p_full = bars + 10;  // [tile]   P written, O rescaled (one arrival per softmax warp of the tile)
    uint64_t* o_full = bars + 12;  // [tile]   PV of the tile done
    uint64_t* q_full = bars + 14;  // Q of both tiles in shared memory (by TMA without RoPE, else one arrival per softmax warp)
    uint64_t* q_land = bars + 15;  // Q tiles landed by TMA, before RoPE is applied in shared memory
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
    uint64_t* stg_full = bars + 17;   // FP8 [K, V]: the tile's K (V) codes and scales are staged
    uint64_t* stg_empty = bars + 19;  // FP8 [K, V]: the converters are done with them

    // FP8 pages: heavy tiles first across the whole grid (CTAs start in linear
    // order, x fastest: x runs over (head, sequence), y over the 256-row tiles
    // from the last, most keys, to the first), measured 453 -> 495 TFLOP/s.
    // fp16 pages keep heavy-first within each (head, sequence): the global
    // order drew the power cap there (1.73-1.82 GHz) and ran 4% slower.
    const int qt = p.q_tiles - 1 - static_cast<int>(FMT ? blockIdx.y : blockIdx.x);
    const int h = FMT ? static_cast<int>(blockIdx.x) % p.Hq : static_cast<int>(blockIdx.y);
    const int b = FMT ? static_cast<int>(blockIdx.x) / p.Hq : static_cast<int>(blockIdx.z);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos0 = p.pos[b];
    const int q0 = qt * 2 * kTcRows;
    if (pos0 < 0 || (pos0 + p.T + P - 1) / P > p.bt_stride) {
        if (threadIdx.x == 0 && qt == 0 && h == 0) atomicOr(p.err, VK_ERR_TABLE_INDEX);
        return;
    }
    // key tiles of each row tile (B may be empty at the end of the chunk)
    const int rowsA = min(kTcRows, p.T - q0);
    const int rowsB = max(0, min(kTcRows, p.T - q0 - kTcRows));
    const int lenA = pos0 + q0 + rowsA;                      // keys tile A attends
    const int lenB = rowsB > 0 ? pos0 + q0 + kTcRows + rowsB : 0;
    const int ntA = (lenA + kTcKeys - 1) / kTcKeys;
    const int ntB = (lenB + kTcKeys - 1) / kTcKeys;
    const int kv_len = max(lenA, lenB);
    const int ntiles = max(ntA, ntB);
    const int hkv = h / p.G;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 8; ++i) mbar_init(smem_u32(&bars[i]), 1);
        for (int t = 0; t < 2; ++t) {
            mbar_init(smem_u32(&s_full[t]), 1);
            mbar_init(smem_u32(&p_full[t]), 4);
            mbar_init(smem_u32(&o_full[t]), 1);
        }
        mbar_init(smem_u32(q_full), (p.q_tma && p.rope_freq == nullptr) ? 1 : 8);
        mbar_init(smem_u32(q_land), 1);
        if (FMT) {
            for (int hf = 0; hf < 2; ++hf) {
                mbar_init(smem_u32(&stg_full[hf]), 1);
                mbar_init(smem_u32(&stg_empty[hf]), 1);
            }
        }
        mbar_fence_init();
        if (p.q_tma) {
            // both 128-row Q tiles, two 64-column halves each (128-byte swizzle:
            // the layout the MMA descriptors read); rows past the chunk read the
            // next rows of q or zeros, and are never stored
            const uint32_t bar = smem_u32(p.rope_freq == nullptr ? q_full : q_land);
            prefetch_tmap(&tmapq);
            mbar_expect_tx(bar, 2 * 2 * kTcRows * 128);
            const uint64_t pol = l2_evict_first_policy();
            for (int t = 0; t < 2; ++t)
                for (int hb = 0; hb < 2; ++hb)
                    tma_load_3d(sbase + kTcQ + t * 32768 + hb * 16384, &tmapq, hb * 64, h, b * p.T + q0 + t * kTcRows,
                                bar, pol);
        }
    }
    // zero both V stages: rows a last tile does not load keep finite values
    for (int i = threadIdx.x; i < 2 * 32768 / 16; i += NTHR)
        asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(sbase + kTcV + i * 16), "r"(0u) : "memory");
    fence_async_smem();
    if (warp == 9) {
        tmem_alloc(smem_u32(tmem_slot), kTcCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (FMT && warp == 8) {
        // ------------------------------------------------------------ FP8 page blocks -> staging
        // K and V are staged apart (each page's codes and its scales are two
        // bulk copies): the next tile's K loads while this tile's V is being
        // converted, and its V while its K is.
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            const int32_t* btrow = p.bt + static_cast<int64_t>(b) * p.bt_stride;
            bool ok = true;
            for (int j = 0; j < ntiles && ok; ++j) {
                const int npg = min(kTcKeys / P, (kv_len - j * kTcKeys + P - 1) / P);
                int pages[kTcKeys / P];
                for (int i = 0; i < npg; ++i) {
                    int pg = btrow[j * (kTcKeys / P) + i];
                    if (pg < 0 || pg >= p.num_pages) {
                        atomicOr(p.err, VK_ERR_PAGE_ID);
                        pg = 0;
                    }
                    pages[i] = pg;
                }
                for (int kv = 0; kv < 2; ++kv) {
                    if (j >= 1 && !mbar_wait(smem_u32(&stg_empty[kv]), (j - 1) & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    const uint32_t bar = smem_u32(&stg_full[kv]);
                    mbar_expect_tx(bar, npg * kStgPageBytes);
                    const uint32_t dst = sbase + kTcStage8 + kv * kStgHalf;
                    for (int i = 0; i < npg; ++i) {
                        const char* blk = p.pool_base + p.layer_off + static_cast<uint64_t>(pages[i]) * p.seg_bytes +
                                          static_cast<uint64_t>(hkv) * p.head_bytes;
                        bulk_load(dst + i * kStgCodes, blk + kv * kStgCodes, kStgCodes, bar, pol);
                        bulk_load(dst + kStgScales + i * 64, blk + fp8_scale_off(kv, 0, kTcD), 64, bar, pol);
                    }
                }
            }
        }
    } else if (FMT && warp >= 10) {
        // ------------------------------------------------------------ FP8 -> fp16 converters (64 threads)
        const int ct = threadIdx.x - 320;
        volatile int* okp = reinterpret_cast<volatile int*>(tmem_slot) + 1;  // broadcast slot
        const uint32_t kstg = sbase + kTcStage8, vstg = sbase + kTcStage8 + kStgHalf;
        // K: chunk (page, token, 16 elements) -> key row, two 16-byte fp16
        // chunks; code x scale as fp16 pairs with the scale split into s_hi +
        // s_lo (both fp16): t = code * s_hi, then t + code * s_lo, so the row
        // scale carries no fp16 rounding of its own.  Four chunks per round,
        // their loads issued first.
        auto convert_k = [&](int st, int key_end) {
#pragma unroll 1
            for (int i0 = 0; i0 < kTcKeys * 8 / 64; i0 += 4) {
                uint4 codes[4];
                float s1[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int q = ct + 64 * (i0 + u);
                    const int pg = q >> 7, t = (q >> 3) & 15, c = q & 7;
                    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                                 : "=r"(codes[u].x), "=r"(codes[u].y), "=r"(codes[u].z), "=r"(codes[u].w)
                                 : "r"(kstg + pg * kStgCodes + fp8_k_off(t, 16 * c, kTcD)));
                    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(s1[u]) : "r"(kstg + kStgScales + pg * 64 + t * 4));
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int q = ct + 64 * (i0 + u);
                    const int pg = q >> 7, t = (q >> 3) & 15, c = q & 7, key = pg * P + t;
                    const __half shi = __float2half_rn(s1[u]);
                    const __half slo = __float2half_rn(s1[u] - __half2float(shi));
                    const __half2 hi2 = __half2half2(shi), lo2 = __half2half2(slo);
                    const uint32_t w[4] = {codes[u].x, codes[u].y, codes[u].z, codes[u].w};
                    uint32_t o[8];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        uint32_t a, b2;
                        e4m3x4_to_h2x2(w[k], a, b2);
                        const __half2 ca = *reinterpret_cast<const __half2*>(&a);
                        const __half2 cb = *reinterpret_cast<const __half2*>(&b2);
                        const __half2 ra = __hfma2(ca, lo2, __hmul2(ca, hi2));
                        const __half2 rb = __hfma2(cb, lo2, __hmul2(cb, hi2));
                        o[2 * k] = *reinterpret_cast<const uint32_t*>(&ra);
                        o[2 * k + 1] = *reinterpret_cast<const uint32_t*>(&rb);
                    }
                    if (key >= key_end) {  // past the written length: zeros (the bytes may be anything)
#pragma unroll
                        for (int k = 0; k < 8; ++k) o[k] = 0u;
                    }
                    const int hb = c >> 2, cc = (c & 3) * 2;
                    const uint32_t row = sbase + kTcK + st * 32768 + hb * 16384 + key * 128;
                    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(row + ((cc ^ (key & 7)) << 4)),
                                 "r"(o[0]), "r"(o[1]), "r"(o[2]), "r"(o[3])
                                 : "memory");
                    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(row + (((cc + 1) ^ (key & 7)) << 4)),
                                 "r"(o[4]), "r"(o[5]), "r"(o[6]), "r"(o[7])
                                 : "memory");
                }
            }
        };
        // V: per page, this thread's rows d = ct and ct + 64 of V^T (keys
        // pg*16 .. pg*16+15).  The block holds token t at position fp8_v_pos(t):
        // byte permutes put the tokens in order, then codes -> fp16 (exact)
        // times the tokens' scales as fp16 pairs.
        auto convert_v = [&](int st, int key_end) {
#pragma unroll 1
            for (int pg = 0; pg < kTcKeys / P; ++pg) {
                const int valid = key_end - pg * P;
                uint32_t o[2][8];
                if (valid > 0) {
                    uint4 raw[2];
#pragma unroll
                    for (int dd = 0; dd < 2; ++dd)
                        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                                     : "=r"(raw[dd].x), "=r"(raw[dd].y), "=r"(raw[dd].z), "=r"(raw[dd].w)
                                     : "r"(vstg + pg * kStgCodes + (ct + 64 * dd) * P));
                    float sv[16];
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                                     : "=f"(sv[4 * k]), "=f"(sv[4 * k + 1]), "=f"(sv[4 * k + 2]), "=f"(sv[4 * k + 3])
                                     : "r"(vstg + kStgScales + pg * 64 + 16 * k));
                    __half2 sp[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k)  // keys past the written length: scale 0 (and cleared below)
                        sp[k] = __floats2half2_rn(2 * k < valid ? sv[2 * k] : 0.f, 2 * k + 1 < valid ? sv[2 * k + 1] : 0.f);
#pragma unroll
                    for (int dd = 0; dd < 2; ++dd) {
                        // positions 0..15 hold tokens 0,1,8,9,2,3,10,11,4,5,12,13,6,7,14,15
                        uint32_t nat[4];
                        asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(nat[0]) : "r"(raw[dd].x), "r"(raw[dd].y));  // 0..3
                        asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(nat[1]) : "r"(raw[dd].z), "r"(raw[dd].w));  // 4..7
                        asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(nat[2]) : "r"(raw[dd].x), "r"(raw[dd].y));  // 8..11
                        asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(nat[3]) : "r"(raw[dd].z), "r"(raw[dd].w));  // 12..15
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            uint32_t a, b2;
                            e4m3x4_to_h2x2(nat[k], a, b2);
                            const __half2 ra = __hmul2(*reinterpret_cast<const __half2*>(&a), sp[2 * k]);
                            const __half2 rb = __hmul2(*reinterpret_cast<const __half2*>(&b2), sp[2 * k + 1]);
                            o[dd][2 * k] = *reinterpret_cast<const uint32_t*>(&ra);
                            o[dd][2 * k + 1] = *reinterpret_cast<const uint32_t*>(&rb);
                        }
                        if (valid < P) {  // a NaN code times scale 0 stays NaN: clear those keys
#pragma unroll
                            for (int k = 0; k < 8; ++k) {
                                if (2 * k >= valid) o[dd][k] &= 0xffff0000u;
                                if (2 * k + 1 >= valid) o[dd][k] &= 0x0000ffffu;
                            }
                        }
                    }
                } else {
#pragma unroll
                    for (int dd = 0; dd < 2; ++dd)
#pragma unroll
                        for (int k = 0; k < 8; ++k) o[dd][k] = 0u;
                }
                const int hb = pg >> 2, cc = (pg & 3) * 2;
#pragma unroll
                for (int dd = 0; dd < 2; ++dd) {
                    const int d = ct + 64 * dd;
                    const uint32_t row = sbase + kTcV + st * 32768 + hb * 16384 + d * 128;
                    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(row + ((cc ^ (d & 7)) << 4)),
                                 "r"(o[dd][0]), "r"(o[dd][1]), "r"(o[dd][2]), "r"(o[dd][3])
                                 : "memory");
                    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(row + (((cc + 1) ^ (d & 7)) << 4)),
                                 "r"(o[dd][4]), "r"(o[dd][5]), "r"(o[dd][6]), "r"(o[dd][7])
                                 : "memory");
                }
            }
        };
        // one converter thread waits (bounded), the 64 meet at named barrier 2
        auto sync_on = [&](uint32_t bar1, uint32_t par1, uint32_t bar2, uint32_t par2, bool second) -> bool {
            if (ct == 0) {
                bool ok = mbar_wait(bar1, par1, p.err);
                if (ok && second) ok = mbar_wait(bar2, par2, p.err);
                *okp = ok ? 1 : 0;
            }
            asm volatile("bar.sync 2, 64;" ::: "memory");
            return *okp != 0;
        };
        // per key tile: K (k_full; the next tile's K starts loading), then V
        // (v_full; the next tile's V starts loading): S can start on a tile
        // whose V is still being converted
        for (int j = 0; j < ntiles; ++j) {
            const int st = j & 1;
            const int key_end = kv_len - j * kTcKeys;  // keys of this tile below the written length
            const uint32_t ph = j & 1, pe = ((j >> 1) - 1) & 1;
            if (!sync_on(smem_u32(&stg_full[0]), ph, smem_u32(&k_empty[st]), pe, j >= 2)) break;
            convert_k(st, key_end);
            fence_async_smem();  // the generic-proxy stores precede the tensor core's reads
            asm volatile("bar.sync 2, 64;" ::: "memory");
            if (ct == 0) {
                mbar_arrive(smem_u32(&stg_empty[0]));
                mbar_arrive(smem_u32(&k_full[st]));
            }
            if (!sync_on(smem_u32(&stg_full[1]), ph, smem_u32(&v_empty[st]), pe, j >= 2)) break;
            convert_v(st, key_end);
            fence_async_smem();
            asm volatile("bar.sync 2, 64;" ::: "memory");
            if (ct == 0) {
                mbar_arrive(smem_u32(&stg_empty[1]));
                mbar_arrive(smem_u32(&v_full[st]));
            }
        }
    } else if (warp == 8) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            prefetch_tmap(&tmap16);
            const uint64_t pol = l2_evict_first_policy();
            const int32_t* btrow = p.bt + static_cast<int64_t>(b) * p.bt_stride;
            bool ok = true;
            for (int j = 0; j < ntiles && ok; ++j) {
                const int st = j & 1;
                const int npg = min(kTcKeys / P, (kv_len - j * kTcKeys + P - 1) / P);
                int pages[kTcKeys / P];
                for (int i = 0; i < npg; ++i) {
                    int pg = btrow[j * (kTcKeys / P) + i];
                    if (pg < 0 || pg >= p.num_pages) {
                        atomicOr(p.err, VK_ERR_PAGE_ID);
                        pg = 0;
                    }
                    pages[i] = pg;
                }
                for (int kv = 0; kv < 2 && ok; ++kv) {  // K ring, then V ring; both land on k_full
                    uint64_t* empty = kv ? v_empty : k_empty;
                    if (j >= 2 && !mbar_wait(smem_u32(&empty[st]), ((j >> 1) - 1) & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    const uint32_t bar = smem_u32(&k_full[st]);
                    if (kv == 0) mbar_expect_tx(bar, 2 * npg * 2 * (P * 128));
                    const uint32_t dst0 = sbase + (kv ? kTcV : kTcK) + st * 32768;
                    for (int i = 0; i < npg; ++i) {
                        const int row = ((p.layer * p.num_pages + pages[i]) * p.Hkv + hkv) * (2 * P) + kv * P;
#pragma unroll
                        for (int hb = 0; hb < 2; ++hb)
                            tma_load_2d(dst0 + hb * 16384 + i * (P * 128), &tmap16, hb * 64, row, bar, pol);
                    }
                }
            }
        }
    } else if (warp == 9) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            // fp16 pages: V stage [key][d] (B MN-major); FP8 pages: V^T [d][key] (B K-major)
            const uint32_t id_s = idesc_f16_128x128(0), id_pv = idesc_f16_128x128(FMT ? 0u : 1u);
            bool ok = mbar_wait(smem_u32(q_full), 0, p.err);
            tc_fence_after();
            const int nt[2] = {ntA, ntB};
            int k_waited = -1;  // highest key tile whose K stage has been waited for
            // Descriptors are formed once; within a tile only the start-address
            // field moves (by constants), so each MMA costs one add at issue:
            // the issuing warp shares its SM sub-partition with two softmax
            // warps, and every issue slot it spends delays the tensor pipe.
            const uint64_t dq0 = umma_desc_sw128(sbase + kTcQ, 16, 1024);
            const uint64_t dk0 = umma_desc_sw128(sbase + kTcK, 16, 1024);
            const uint64_t dv0 = FMT ? umma_desc_sw128(sbase + kTcV, 16, 1024) : umma_desc_sw128(sbase + kTcV, 16384, 1024);
            auto issue_s = [&](int t, int j) {
                const int st = j & 1;
                if (j > k_waited) {
                    ok = ok && mbar_wait(smem_u32(&k_full[st]), (j >> 1) & 1, p.err);
                    k_waited = j;
                }
                if (!ok) return;
                tc_fence_after();
                const uint64_t dq = dq0 + static_cast<uint64_t>(t * (32768 >> 4));
                const uint64_t dk = dk0 + static_cast<uint64_t>(st * (32768 >> 4));
                const uint32_t dt = tmem + t * 128;
#pragma unroll
                for (int ks = 0; ks < kTcD / 16; ++ks) {
                    const uint64_t off = ((ks >> 2) * 16384 + (ks & 3) * 32) >> 4;
                    umma_ss(dt, dq + off, dk + off, id_s, ks > 0);
                }
                umma_commit(smem_u32(&s_full[t]));
                // the last S that reads this K stage releases it
                if (t == 1 || j >= ntB) umma_commit(smem_u32(&k_empty[st]));
            };
            auto issue_pv = [&](int t, int j) {
                const int st = j & 1;
                // P first: waiting on the data barriers earlier (they complete long
                // before the softmax ends) measured 3% slower, the spinning issuer
                // taking issue slots from the softmax warps of its sub-partition.
                ok = ok && mbar_wait(smem_u32(&p_full[t]), j & 1, p.err);
                if (FMT && (t == 0 || j >= ntA)) ok = ok && mbar_wait(smem_u32(&v_full[st]), (j >> 1) & 1, p.err);
                if (!ok) return;
                tc_fence_after();
                const uint64_t dv = dv0 + static_cast<uint64_t>(st * (32768 >> 4));
                const uint32_t dpo = tmem + 256 + t * 128, dpa = tmem + t * 128;
#pragma unroll
                for (int ks = 0; ks < kTcKeys / 16; ++ks) {
                    // next 16 keys: fp16 V advances 16 rows (2 KiB); FP8's V^T 32 bytes
                    // along its 128-byte rows, then to the second 64-key half
                    const uint64_t adv = FMT ? static_cast<uint64_t>(((ks >> 2) * 16384 + (ks & 3) * 32) >> 4)
                                             : static_cast<uint64_t>(ks * (2048 >> 4));
                    umma_ts(dpo, dpa + ks * 8, dv + adv, id_pv, (j > 0 || ks > 0) ? 1u : 0u);
                }
                umma_commit(smem_u32(&o_full[t]));
                if (t == 1 || j >= ntB) umma_commit(smem_u32(&v_empty[st]));
            };
            if (ntA > 0) issue_s(0, 0);
            if (ntB > 0) issue_s(1, 0);
            for (int j = 0; j < ntiles && ok; ++j) {
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                    if (j < nt[t]) {
                        issue_pv(t, j);
                        if (j + 1 < nt[t]) issue_s(t, j + 1);
                    }
                }
            }
        }
    } else {
        // ------------------------------------------------------------ softmax (one query row per thread)
        const int t = warp >> 2;              // row tile
        const int r = threadIdx.x & 127;      // row in the tile = TMEM lane
        const int qrow = q0 + t * kTcRows + r;
        const bool valid_row = qrow < p.T;
        const int qpos = pos0 + qrow;
        const int ntt = t ? ntB : ntA;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
        const uint32_t s_col = t * 128, o_col = 256 + t * 128;
        bool alive0 = true;
        // Q row -> shared memory (K-major, 128-byte swizzle)
        if (p.q_tma && p.rope_freq != nullptr) {
            // landed by TMA: rotate this thread's row in place
            if (!wait_warp(smem_u32(q_land), 0, p.err)) alive0 = false;
            if (alive0) {
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    const uint32_t addr =
                        sbase + kTcQ + t * 32768 + (c >> 3) * 16384 + r * 128 + (((c & 7) ^ (r & 7)) << 4);
                    uint4 v;
                    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                                 : "r"(addr));
                    v = rope_uint4(v, c * 8, qpos, p.rope_freq);
                    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
                                 "r"(v.w)
                                 : "memory");
                }
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(q_full));
        } else if (!p.q_tma) {
            const uint4* src = reinterpret_cast<const uint4*>(
                p.q + ((static_cast<int64_t>(b) * p.T + (valid_row ? qrow : 0)) * p.Hq + h) * kTcD);
            // all 16 loads first: a shared store (asm with a memory clobber)
            // between them would serialise 16 round trips to HBM (~13k cycles
            // of the CTA's start, measured)
            uint4 qv[16];
#pragma unroll
            for (int c = 0; c < 16; ++c) qv[c] = valid_row ? __ldg(src + c) : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                uint4 v = qv[c];
                if (p.rope_freq != nullptr) v = rope_uint4(v, c * 8, qpos, p.rope_freq);
                const uint32_t addr =
                    sbase + kTcQ + t * 32768 + (c >> 3) * 16384 + r * 128 + (((c & 7) ^ (r & 7)) << 4);
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
                             "r"(v.w)
                             : "memory");
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(q_full));
        }
        const float sc = p.scale_log2;
        float m_ref = -INFINITY, l = 0.f;  // m_ref in the scaled (log2) domain
        bool alive = alive0;
        for (int j = 0; j < ntt && alive; ++j) {
            if (!wait_warp(smem_u32(&s_full[t]), j & 1, p.err)) { alive = false; break; }
            tc_fence_after();
            const int key0 = j * kTcKeys;
            // keys past the tile's first row need the causal mask
            const bool need_mask = key0 + kTcKeys - 1 > pos0 + q0 + t * kTcRows;
            const int lim = qpos - key0;  // key c is visible iff c <= lim
            // the whole S row in registers (one TMEM pass); row max of the raw
            // scores (scale > 0 commutes with max); masked keys read as -inf,
            // so their P below is 2^-inf = 0
            float v[kTcKeys / 32][32];
#pragma unroll
            for (int c = 0; c < kTcKeys / 32; ++c) tmem_ld32(lane_base + s_col + c * 32, v[c]);
            tmem_wait_ld();
            if (need_mask) mask_row(v, lim);
            float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int c = 0; c < kTcKeys / 32; ++c)
#pragma unroll
                for (int i = 0; i < 32; i += 8) {
                    mx4[0] = max3f(mx4[0], v[c][i], v[c][i + 1]);
                    mx4[1] = max3f(mx4[1], v[c][i + 2], v[c][i + 3]);
                    mx4[2] = max3f(mx4[2], v[c][i + 4], v[c][i + 5]);
                    mx4[3] = max3f(mx4[3], v[c][i + 6], v[c][i + 7]);
                }
            const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * sc;
            float alpha = 1.f;
            if (mx > m_ref + 8.f || m_ref == -INFINITY) {  // lazy rescale
                const float m_new = fmaxf(m_ref, mx);
                alpha = ex2(m_ref - m_new);
                m_ref = m_new;
            }
            if (!FMT && j == ntiles - 1 && key0 + kTcKeys > kv_len) {
                // the CTA's last key tile: zero V rows of keys at or beyond the
                // written length before any PV of it (both tiles may do it; same
                // zeros)
                if (!wait_warp(smem_u32(&k_full[j & 1]), (j >> 1) & 1, p.err)) { alive = false; break; }
                if (key0 + r >= kv_len) {
#pragma unroll
                    for (int hb = 0; hb < 2; ++hb)
#pragma unroll
                        for (int c = 0; c < 8; ++c) {
                            const uint32_t addr = sbase + kTcV + (j & 1) * 32768 + hb * 16384 + r * 128 + (c << 4);
                            asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0u) : "memory");
                        }
                }
                fence_async_smem();
            }
            // P = 2^(s*sc - m_ref), packed to fp16 over the first 64 columns of
            // S (column 16c+i holds keys 32c+2i, 32c+2i+1)
            const float mneg = m_ref == -INFINITY ? 0.f : -m_ref;
            float sum4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < kTcKeys / 32; ++c) {
                uint32_t pk[16];
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    const float a0 = ex2(fmaf(v[c][i], sc, mneg));
                    const float a1 = ex2(fmaf(v[c][i + 1], sc, mneg));
                    sum4[(i >> 1) & 3] += a0 + a1;
                    pk[i >> 1] = pack_half2(a0, a1);
                }
                tmem_st16(lane_base + s_col + c * 16, pk);
            }
            l = l * alpha + ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
            // tcgen05.ld/st are warp-collective: rescale O if any row of the warp
            // needs it (PV of the previous tile completed before this S was written), before the
            // PV of this tile starts.  Done after P is stored, when the S row's
            // 128 registers are dead: the kernel's 10 warps get 168 registers a
            // thread, and rescaling with the row still live spilled ~280 bytes
            // into the max pass (677 -> 765 TFLOP/s on the 7B chunked prefill).
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
                for (int c = 0; c < kTcD / 32; ++c) {
                    float v[32];
                    tmem_ld32(lane_base + o_col + c * 32, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] *= alpha;
                    tmem_st32(lane_base + o_col + c * 32, v);
                }
            }
            tmem_wait_st();
            // tcgen05.wait::st above is warp-collective: the warp's P and O
            // stores are complete when lane 0 signals for the warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&p_full[t]));
        }
        if (alive && ntt > 0 && wait_warp(smem_u32(&o_full[t]), (ntt - 1) & 1, p.err)) {
            tc_fence_after();
            const float inv = 1.f / l;
            __half* dst = p.out + ((static_cast<int64_t>(b) * p.T + (valid_row ? qrow : 0)) * p.Hq + h) * kTcD;
#pragma unroll
            for (int c = 0; c < kTcD / 32; ++c) {
                float v[32];
                tmem_ld32(lane_base + o_col + c * 32, v);
                tmem_wait_ld();
                if (valid_row) {
#pragma unroll
                    for (int i = 0; i < 32; i += 8) {
                        uint4 w;
                        w.x = pack_half2(v[i] * inv, v[i + 1] * inv);
                        w.y = pack_half2(v[i + 2] * inv, v[i + 3] * inv);
                        w.z = pack_half2(v[i + 4] * inv, v[i + 5] * inv);
                        w.w = pack_half2(v[i + 6] * inv, v[i + 7] * inv);
                        *reinterpret_cast<uint4*>(dst + c * 32 + i) = w;
                    }
                }
            }
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc(tmem, kTcCols);
    }
}

vk_status launch_prefill_tc(vk_pool* pool, const TcParams& p, const CUtensorMap& tq, int B, cudaStream_t st) {
    static uint64_t attr_set[2] = {0, 0};
    const int fmt = pool->kv_format == VK_KV_FP8 ? 1 : 0;
    const uint64_t bit = 1ull << (pool->device & 63);
    if (!(attr_set[fmt] & bit)) {
        cudaError_t e = fmt ? cudaFuncSetAttribute(prefill_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem8)
                            : cudaFuncSetAttribute(prefill_tc_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(prefill_tc)");
        attr_set[fmt] |= bit;
    }
    if (fmt) prefill_tc_kernel<1><<<dim3(p.Hq * B, p.q_tiles), kTcThreads8, kTcSmem8, st>>>(pool->tmap16, tq, p);
    else prefill_tc_kernel<0><<<dim3(p.q_tiles, p.Hq, B), kTcThreads, kTcSmem, st>>>(pool->tmap16, tq, p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? VK_OK : cuda_fail(e, "prefill_tc_kernel launch");
}

vk_status prefill_tc(vk_pool* pool, int layer, const void* q, void* out, const int32_t* bt, int bt_stride,
                     const int32_t* positions, int B, int T, int Hq, float scale, cudaStream_t st) {
    TcParams p;
    p.q = static_cast<const __half*>(q);
    p.out = static_cast<__half*>(out);
    p.bt = bt;
    p.pos = positions;
    p.err = pool->d_err;
    p.bt_stride = bt_stride;
    p.T = T;
    p.Hq = Hq;
    p.Hkv = pool->cfg.num_kv_heads;
    p.G = Hq / p.Hkv;
    p.layer = layer;
    p.num_pages = pool->num_pages;
    p.q_tiles = (T + 2 * kTcRows - 1) / (2 * kTcRows);
    const float sc = scale > 0.f ? scale : 1.0f / sqrtf(static_cast<float>(kTcD));
    p.scale_log2 = sc * 1.4426950408889634f;
    p.rope_freq = pool->rope_freq;
    p.pool_base = pool->base;
    p.layer_off = static_cast<uint64_t>(layer) * pool->seg_stride;
    p.seg_bytes = pool->seg_bytes;
    p.head_bytes = pool->head_bytes;
    // Q by TMA: a 3-D view [B*T tokens][Hq heads][128 d] of q, boxes of 64 d x
    // 1 head x 128 tokens; needs q 16-byte aligned (else the softmax warps load it)
    alignas(64) CUtensorMap tq = pool->tmap16;  // placeholder when unused
    p.q_tma = 0;
    auto encode = tmap_encode_fn();
    const uint64_t ntok = static_cast<uint64_t>(B) * T;
    if (encode && !(reinterpret_cast<uintptr_t>(q) & 15) && ntok + 2 * kTcRows < (1ull << 31)) {
        cuuint64_t dims[3] = {static_cast<cuuint64_t>(kTcD), static_cast<cuuint64_t>(Hq), ntok};
        cuuint64_t strides[2] = {static_cast<cuuint64_t>(kTcD) * 2, static_cast<cuuint64_t>(Hq) * kTcD * 2};
        cuuint32_t box[3] = {64, 1, static_cast<cuuint32_t>(kTcRows)};
        cuuint32_t estr[3] = {1, 1, 1};
        if (encode(&tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(q), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
            p.q_tma = 1;
        else
            tq = pool->tmap16;
    }
    return launch_prefill_tc(pool, p, tq, B, st);
}

}  // namespace vk
