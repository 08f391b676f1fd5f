// K3: chunked-prefill attention over the paged cache.
//
// The prefill use of VULCAN's attention (src/transformer.cpp:136-189 with
// num_tokens = chunk, src/engine.cpp:70-101): query token t of sequence b sits at
// position pos_b + t and attends cached keys 0..pos_b+t -- the causal
// j <= row rule of cpu_attention (tests/test_attention.cu:69) with a cached
// prefix.  The chunk's own K/V are appended first (vk_append).
//
// Design (B200, tensor cores through mma.sync):
//  * One CTA per (64-query tile, query head, sequence); heavy tiles (later in
//    the chunk, more keys) are scheduled first.
//  * Warp 4 lane 0 streams 64-key tiles (four 16-token pages) with 2-D TMA
//    loads (128-byte swizzle) into a 2-stage ring; warps 0-3 each own 16 query
//    rows.
//  * S = Q K^T and O += P V with mma.m16n8k16 (fp16 in, fp32 accumulate); the
//    S accumulator is re-used as the A operand of P V in registers; online
//    softmax per row with quad shuffles; causal masking only on tiles that cross
//    the diagonal; V of slots beyond the written tokens is zeroed in registers.
//  * FP8 pools (FMT = 1, D = 128; block format in vk_fp8.cuh): a page block
//    arrives in one bulk copy; K codes become the B operand of S through
//    ldmatrix and a conversion, with Q's fragments loaded in the permuted
//    contraction order of the decode (elements 4c..4c+3 per lane and 16-step);
//    V codes become the B operand of P V without a transpose (element-major
//    rows); K scales multiply the scores, V scales the probabilities (relative
//    to a power of two per key tile, carried in the rescale of O).
#include <cmath>
#include <vector>

#include "vk_internal.h"
#include "vk_fp8.cuh"
#include "vk_ptx.cuh"
#include "vk_rope.cuh"

namespace vk {

constexpr int kPreWarps = 4;                 // consumer warps (16 query rows each)
constexpr int kPreThreads = (kPreWarps + 1) * 32;
constexpr int kPreRows = 16 * kPreWarps;     // query rows per CTA
constexpr int kPreKeys = 64;                 // keys per KV tile (4 pages)
constexpr int kPreStages = 2;

struct PrefillParams {
    const __half* q;      // [B, T, Hq, D]
    __half* out;          // [B, T, Hq, D]
    const int32_t* bt;
    const int32_t* pos;
    uint32_t* err;
    int bt_stride, T, Hq, Hkv, G, L, layer, num_pages, q_tiles;
    float scale_log2;
    const float* rope_freq;  // non-null: q rotated (RoPE) at its position
    // FP8 pools: block addressing for the bulk copies
    const char* pool_base;
    uint64_t seg_bytes, layer_off, head_bytes;
};

template <int D, int FMT>
__host__ __device__ constexpr int prefill_page_bytes() {
    return FMT ? fp8_head_bytes(D) : 2 * kPageTokens * D * 2;
}

template <int D, int FMT>
__host__ __device__ constexpr int prefill_smem_bytes() {
    return kPreStages * 4 * prefill_page_bytes<D, FMT>() + 2 * kPreStages * 8 + 1024;
}

template <int D, int FMT>
__global__ void __launch_bounds__(kPreThreads) prefill_kernel(const __grid_constant__ CUtensorMap tmap,
                                                              const PrefillParams p) {
    static_assert(FMT == 0 || D == kFp8Dim, "FP8 blocks are defined for head_dim 128");
    constexpr int P = kPageTokens;
    constexpr int PB = prefill_page_bytes<D, FMT>();  // one page (K + V rows) in shared memory
    constexpr int SB = 4 * PB;                   // one 64-key stage
    constexpr int NB = D / 64;
    constexpr int KS = D / 16;                   // k-steps over the head dimension
    constexpr int DT = D / 8;                    // 8-wide output column tiles

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPreStages * SB);
    uint64_t* empty = full + kPreStages;

    const int qt = p.q_tiles - 1 - static_cast<int>(blockIdx.x);  // heavy tiles first
    const int h = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos0 = p.pos[b];
    const int row0 = qt * kPreRows;
    if (pos0 < 0 || (pos0 + p.T + P - 1) / P > p.bt_stride) {
        if (threadIdx.x == 0 && qt == 0 && h == 0) atomicOr(p.err, VK_ERR_TABLE_INDEX);
        return;
    }
    const int kv_len = pos0 + min(p.T, row0 + kPreRows);  // keys seen by the tile's last row
    const int ntiles = (kv_len + kPreKeys - 1) / kPreKeys;
    const int hkv = h / p.G;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPreStages; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), kPreWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kPreWarps) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            if (FMT == 0) prefetch_tmap(&tmap);
            const uint64_t pol = l2_evict_first_policy();
            const int32_t* btrow = p.bt + static_cast<int64_t>(b) * p.bt_stride;
            for (int j = 0; j < ntiles; ++j) {
                const int st = j % kPreStages;
                if (j >= kPreStages && !mbar_wait(smem_u32(&empty[st]), ((j / kPreStages) - 1) & 1, p.err)) break;
                const int npg = min(4, (kv_len - j * kPreKeys + P - 1) / P);
                const uint32_t bar = smem_u32(&full[st]);
                mbar_expect_tx(bar, npg * PB);
                for (int i = 0; i < npg; ++i) {
                    int page = btrow[j * 4 + i];
                    if (page < 0 || page >= p.num_pages) {
                        atomicOr(p.err, VK_ERR_PAGE_ID);
                        page = 0;
                    }
                    const uint32_t dst = smem_u32(smem + st * SB + i * PB);
                    if constexpr (FMT == 1) {
                        bulk_load(dst, p.pool_base + p.layer_off + static_cast<uint64_t>(page) * p.seg_bytes +
                                           static_cast<uint64_t>(hkv) * p.head_bytes,
                                  PB, bar, pol);
                    } else {
                        const int row = ((p.layer * p.num_pages + page) * p.Hkv + hkv) * (2 * P);
#pragma unroll
                        for (int hb = 0; hb < NB; ++hb)
                            tma_load_2d(dst + hb * (2 * P * 128), &tmap, hb * 64, row, bar, pol);
                    }
                }
            }
        }
    } else {
        // ---------------------------------------------------------------- consumers
        const int g = lane >> 2, c = lane & 3;
        const int mi = lane >> 3, rr = lane & 7;
        const int wrow0 = row0 + warp * 16;           // first chunk row of this warp
        const int r_lo = wrow0 + g, r_hi = wrow0 + g + 8;
        const int qpos_lo = pos0 + r_lo, qpos_hi = pos0 + r_hi;

        // Q rows as A fragments (rows beyond the chunk are zero)
        uint32_t qa[KS][4];
        {
            const __half* qlo = p.q + ((static_cast<int64_t>(b) * p.T + min(r_lo, p.T - 1)) * p.Hq + h) * D;
            const __half* qhi = p.q + ((static_cast<int64_t>(b) * p.T + min(r_hi, p.T - 1)) * p.Hq + h) * D;
            const bool vlo = r_lo < p.T, vhi = r_hi < p.T;
            // the second pair of a lane's k-slots: elements d+8 (fp16 pages) or
            // d+2 (FP8: the lane holds elements 4c..4c+3 of each 16-step)
            constexpr int D2 = FMT ? 2 : 8;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                const int d = ks * 16 + (FMT ? 4 : 2) * c;
                qa[ks][0] = vlo ? __ldg(reinterpret_cast<const unsigned int*>(qlo + d)) : 0u;
                qa[ks][1] = vhi ? __ldg(reinterpret_cast<const unsigned int*>(qhi + d)) : 0u;
                qa[ks][2] = vlo ? __ldg(reinterpret_cast<const unsigned int*>(qlo + d + D2)) : 0u;
                qa[ks][3] = vhi ? __ldg(reinterpret_cast<const unsigned int*>(qhi + d + D2)) : 0u;
                if (p.rope_freq != nullptr) {
                    qa[ks][0] = rope_word(qa[ks][0], d, qpos_lo, p.rope_freq);
                    qa[ks][1] = rope_word(qa[ks][1], d, qpos_hi, p.rope_freq);
                    qa[ks][2] = rope_word(qa[ks][2], d + D2, qpos_lo, p.rope_freq);
                    qa[ks][3] = rope_word(qa[ks][3], d + D2, qpos_hi, p.rope_freq);
                }
            }
        }
        float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
        float vf = 1.f;  // FP8: acc holds the true sums divided by vf (a power of two)
        float acc[DT][4];
#pragma unroll
        for (int n = 0; n < DT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;

        for (int j = 0; j < ntiles; ++j) {
            const int st = j % kPreStages;
            if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&full[st]), (j / kPreStages) & 1, p.err))) break;
            const uint32_t sb = smem_u32(smem + st * SB);
            const int key0 = j * kPreKeys;

            // S[16 x 64] = Q K^T
            float s[8][4];
#pragma unroll
            for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
            if constexpr (FMT == 1) {
#pragma unroll
                for (int np = 0; np < 4; ++np) {  // keys [16*np, 16*np+16): page np
#pragma unroll
                    for (int kp = 0; kp < KS / 2; ++kp) {
                        // matrices: keys 0-7 / 8-15 of 16-byte chunk 2kp, then of 2kp+1
                        const int kr = rr + (mi & 1) * 8;
                        const int ch = 2 * kp + (mi >> 1);
                        uint32_t r[4], b0, b1;
                        ldsm_x4(r, sb + np * PB + kr * D + ((ch ^ (kr & 7)) << 4));
                        e4m3x4_to_h2x2(r[0], b0, b1);
                        mma16816(s[2 * np], qa[2 * kp], b0, b1);
                        e4m3x4_to_h2x2(r[1], b0, b1);
                        mma16816(s[2 * np + 1], qa[2 * kp], b0, b1);
                        e4m3x4_to_h2x2(r[2], b0, b1);
                        mma16816(s[2 * np], qa[2 * kp + 1], b0, b1);
                        e4m3x4_to_h2x2(r[3], b0, b1);
                        mma16816(s[2 * np + 1], qa[2 * kp + 1], b0, b1);
                    }
                }
            } else {
#pragma unroll
                for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
                    for (int np = 0; np < 4; ++np) {  // keys [16*np, 16*np+16): page np
                        const int kr = rr + (mi >> 1) * 8;
                        const int d = ks * 16 + (mi & 1) * 8;
                        uint32_t bk[4];
                        ldsm_x4(bk, sb + np * PB + (d >> 6) * (2 * P * 128) + swz128(kr, (d & 63) >> 3));
                        mma16816(s[2 * np], qa[ks], bk[0], bk[1]);
                        mma16816(s[2 * np + 1], qa[ks], bk[2], bk[3]);
                    }
                }
            }

            // FP8: per-key scales of the lane's keys (8-key group n, column
            // 2c + e); keys at or beyond kv_len are unwritten (any bits)
            float ksc[8][2], vsc[8][2];
            float ratio = 1.f;
            if constexpr (FMT == 1) {
                float vmax = 0.f;
#pragma unroll
                for (int n = 0; n < 8; ++n)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int t = (n & 1) * 8 + 2 * c + e;  // token in page n/2
                        const uint32_t blk = sb + (n >> 1) * PB;
                        const bool ok = key0 + n * 8 + 2 * c + e < kv_len;
                        ksc[n][e] = p.scale_log2 * lds_f32(blk + fp8_scale_off(0, t, D));
                        vsc[n][e] = ok ? lds_f32(blk + fp8_scale_off(1, t, D)) : 0.f;
                        vmax = fmaxf(vmax, vsc[n][e]);
                    }
                vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 1));
                vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 2));
                const int ex = min(60, max(-60, static_cast<int>((__float_as_uint(vmax) >> 23) & 0xffu) - 127));
                const float inv_f = __uint_as_float(static_cast<uint32_t>(127 - ex) << 23);  // 2^-ex
                ratio = vf * inv_f;                                                           // exact
                vf = __uint_as_float(static_cast<uint32_t>(127 + ex) << 23);
#pragma unroll
                for (int n = 0; n < 8; ++n) vsc[n][0] *= inv_f, vsc[n][1] *= inv_f;
            }

            // causal mask on tiles crossing this warp's diagonal
            const bool need_mask = key0 + kPreKeys - 1 > pos0 + wrow0;
            float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
            for (int n = 0; n < 8; ++n) {
                const int k0 = key0 + n * 8 + 2 * c;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int key = k0 + (e & 1);
                    const int qp = e < 2 ? qpos_lo : qpos_hi;
                    float v = s[n][e] * (FMT ? ksc[n][e & 1] : p.scale_log2);
                    if (need_mask && key > qp) v = -INFINITY;
                    s[n][e] = v;
                }
                mx_lo = fmaxf(mx_lo, fmaxf(s[n][0], s[n][1]));
                mx_hi = fmaxf(mx_hi, fmaxf(s[n][2], s[n][3]));
            }
#pragma unroll
            for (int o = 1; o < 4; o <<= 1) {
                mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, o));
                mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, o));
            }
            const float n_lo = fmaxf(m_lo, mx_lo), n_hi = fmaxf(m_hi, mx_hi);
            const float a_lo = ex2(m_lo - n_lo), a_hi = ex2(m_hi - n_hi);
            m_lo = n_lo;
            m_hi = n_hi;
            float ps_lo = 0.f, ps_hi = 0.f;
            uint32_t pa[4][4];  // P as A fragments, one per 16-key step
#pragma unroll
            for (int n = 0; n < 8; ++n) {
                const float p0 = ex2(s[n][0] - n_lo), p1 = ex2(s[n][1] - n_lo);
                const float p2 = ex2(s[n][2] - n_hi), p3 = ex2(s[n][3] - n_hi);
                ps_lo += p0 + p1;
                ps_hi += p2 + p3;
                if constexpr (FMT == 1) {  // times each key's V scale (relative to vf)
                    pa[n >> 1][(n & 1) * 2 + 0] = pack_half2(p0 * vsc[n][0], p1 * vsc[n][1]);
                    pa[n >> 1][(n & 1) * 2 + 1] = pack_half2(p2 * vsc[n][0], p3 * vsc[n][1]);
                } else {
                    pa[n >> 1][(n & 1) * 2 + 0] = pack_half2(p0, p1);
                    pa[n >> 1][(n & 1) * 2 + 1] = pack_half2(p2, p3);
                }
            }
            l_lo = l_lo * a_lo + ps_lo;
            l_hi = l_hi * a_hi + ps_hi;
            const float c_lo = FMT ? a_lo * ratio : a_lo, c_hi = FMT ? a_hi * ratio : a_hi;
#pragma unroll
            for (int n = 0; n < DT; ++n) {
                acc[n][0] *= c_lo;
                acc[n][1] *= c_lo;
                acc[n][2] *= c_hi;
                acc[n][3] *= c_hi;
            }

            // O[16 x D] += P[16 x 64] V[64 x D]
            const bool tail = key0 + kPreKeys > kv_len;
            if constexpr (FMT == 1) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    uint32_t keep0 = 0xffffffffu, keep1 = 0xffffffffu;  // keys 2c, 2c+1 / 2c+8, 2c+9
                    if (tail) {
                        const int t0 = key0 + kk * 16 + 2 * c;
                        keep0 = (t0 < kv_len ? 0x0000ffffu : 0u) | (t0 + 1 < kv_len ? 0xffff0000u : 0u);
                        keep1 = (t0 + 8 < kv_len ? 0x0000ffffu : 0u) | (t0 + 9 < kv_len ? 0xffff0000u : 0u);
                    }
#pragma unroll
                    for (int dq = 0; dq < D / 32; ++dq) {
                        // matrices: element rows 32dq + 8i + 0..7 (16 bytes each), output tiles 4dq + i
                        uint32_t r[4];
                        ldsm_x4(r, sb + kk * PB + P * D + (32 * dq + 8 * mi + rr) * P);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            uint32_t b0, b1;
                            e4m3x4_to_h2x2(r[i], b0, b1);
                            mma16816(acc[4 * dq + i], pa[kk], b0 & keep0, b1 & keep1);
                        }
                    }
                }
            } else {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
                for (int dp = 0; dp < DT / 2; ++dp) {
                    const int kr = rr + (mi & 1) * 8;
                    const int d = dp * 16 + (mi >> 1) * 8;
                    uint32_t bv[4];
                    ldsm_x4_t(bv, sb + kk * PB + (d >> 6) * (2 * P * 128) + swz128(P + kr, (d & 63) >> 3));
                    if (tail) {  // zero V of slots at or beyond the written length
                        const int t0 = key0 + kk * 16 + 2 * c;
#pragma unroll
                        for (int r = 0; r < 4; ++r) {
                            const int t = t0 + ((r & 1) ? 8 : 0);
                            const uint32_t keep = (t < kv_len ? 0x0000ffffu : 0u) | (t + 1 < kv_len ? 0xffff0000u : 0u);
                            bv[r] &= keep;
                        }
                    }
                    mma16816(acc[2 * dp], pa[kk], bv[0], bv[1]);
                    mma16816(acc[2 * dp + 1], pa[kk], bv[2], bv[3]);
                }
            }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&empty[st]));
        }

#pragma unroll
        for (int o = 1; o < 4; o <<= 1) {
            l_lo += __shfl_xor_sync(0xffffffffu, l_lo, o);
            l_hi += __shfl_xor_sync(0xffffffffu, l_hi, o);
        }
        const float i_lo = (FMT ? vf : 1.f) / l_lo, i_hi = (FMT ? vf : 1.f) / l_hi;
        __half* olo = p.out + ((static_cast<int64_t>(b) * p.T + r_lo) * p.Hq + h) * D;
        __half* ohi = p.out + ((static_cast<int64_t>(b) * p.T + r_hi) * p.Hq + h) * D;
#pragma unroll
        for (int n = 0; n < DT; ++n) {
            const int d = n * 8 + 2 * c;
            if (r_lo < p.T) *reinterpret_cast<__half2*>(olo + d) = __floats2half2_rn(acc[n][0] * i_lo, acc[n][1] * i_lo);
            if (r_hi < p.T) *reinterpret_cast<__half2*>(ohi + d) = __floats2half2_rn(acc[n][2] * i_hi, acc[n][3] * i_hi);
        }
    }
}

template <int D, int FMT>
static vk_status launch_prefill_t(vk_pool* pool, const PrefillParams& p, int B, cudaStream_t st) {
    constexpr int smem = prefill_smem_bytes<D, FMT>();
    static uint64_t attr_set = 0;
    const uint64_t bit = 1ull << (pool->device & 63);
    if (!(attr_set & bit)) {
        cudaError_t e = cudaFuncSetAttribute(prefill_kernel<D, FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(prefill)");
        attr_set |= bit;
    }
    dim3 grid(p.q_tiles, p.Hq, B);
    prefill_kernel<D, FMT><<<grid, kPreThreads, smem, st>>>(pool->tmap, p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? VK_OK : cuda_fail(e, "prefill_kernel launch");
}

}  // namespace vk

using namespace vk;

extern "C" vk_status vk_prefill(vk_pool* pool, int32_t layer, const void* q, void* out,
                                const int32_t* block_tables, int32_t bt_stride,
                                const int32_t* positions, int32_t batch, int32_t tokens,
                                int32_t num_q_heads, float scale, void* stream) {
    if (!pool) return fail(VK_INVALID_ARG, "pool is NULL");
    const bool fp8 = pool->kv && pool->kv_format == VK_KV_FP8;
    if (!pool->kv || (!fp8 && !pool->tmap_ok)) return fail(VK_UNSUPPORTED, "prefill needs a KV pool addressable by TMA");
    if (pool->cfg.page_tokens != kPageTokens) return fail(VK_UNSUPPORTED, "prefill supports page_tokens == 16");
    const int D = pool->cfg.head_dim, Hkv = pool->cfg.num_kv_heads;
    if (D != 64 && D != 128) return fail(VK_UNSUPPORTED, "prefill supports head_dim 64 and 128");
    if (layer < 0 || layer >= pool->cfg.num_layers) return fail(VK_INVALID_ARG, "layer out of range");
    if (batch < 0 || tokens < 0 || bt_stride <= 0) return fail(VK_INVALID_ARG, "bad batch/tokens/bt_stride");
    if (num_q_heads <= 0 || num_q_heads % Hkv) return fail(VK_INVALID_ARG, "num_q_heads must be a positive multiple of num_kv_heads");
    if (batch == 0 || tokens == 0) return VK_OK;
    if (!q || !out || !block_tables || !positions) return fail(VK_INVALID_ARG, "NULL array");
    if ((reinterpret_cast<uintptr_t>(q) & 3) || (reinterpret_cast<uintptr_t>(out) & 3))
        return fail(VK_INVALID_ARG, "q and out must be 4-byte aligned");
    if (batch > 65535 || num_q_heads > 65535) return fail(VK_INVALID_ARG, "batch and num_q_heads must be <= 65535");
    PrefillParams p;
    p.q = static_cast<const __half*>(q);
    p.out = static_cast<__half*>(out);
    p.bt = block_tables;
    p.pos = positions;
    p.err = pool->d_err;
    p.bt_stride = bt_stride;
    p.T = tokens;
    p.Hq = num_q_heads;
    p.Hkv = Hkv;
    p.G = num_q_heads / Hkv;
    p.L = pool->cfg.num_layers;
    p.layer = layer;
    p.num_pages = pool->num_pages;
    p.q_tiles = (tokens + kPreRows - 1) / kPreRows;
    p.rope_freq = pool->rope_freq;
    p.pool_base = pool->base;
    p.seg_bytes = pool->seg_bytes;
    p.layer_off = static_cast<uint64_t>(layer) * pool->seg_stride;
    p.head_bytes = pool->head_bytes;
    const float sc = scale > 0.f ? scale : 1.0f / sqrtf(static_cast<float>(D));
    p.scale_log2 = sc * 1.4426950408889634f;
    DeviceGuard g(pool->device);
    cudaStream_t st = as_stream(stream);
    if (fp8) {  // FP8 pages (head_dim 128): the tcgen05 kernel with converter warps; path 1: mma.sync
        if (pool->prefill_path == 1) return launch_prefill_t<128, 1>(pool, p, batch, st);
        return prefill_tc(pool, layer, q, out, block_tables, bt_stride, positions, batch, tokens, num_q_heads, scale,
                          st);
    }
    const bool tc = D == 128 && pool->prefill_path != 1;
    if (pool->prefill_path == 2 && !tc) return fail(VK_UNSUPPORTED, "the tcgen05 prefill supports head_dim 128");
    if (tc)
        return prefill_tc(pool, layer, q, out, block_tables, bt_stride, positions, batch, tokens, num_q_heads, scale,
                          st);
    return D == 128 ? launch_prefill_t<128, 0>(pool, p, batch, st) : launch_prefill_t<64, 0>(pool, p, batch, st);
}

extern "C" vk_status vk_set_rope(vk_pool* pool, float theta_base) {
    if (!pool) return fail(VK_INVALID_ARG, "pool is NULL");
    if (!(theta_base >= 0.f) || theta_base == 1.0f) return fail(VK_INVALID_ARG, "RoPE base must be 0 (off) or > 0 and != 1");
    if (theta_base == 0.f) {
        pool->rope_theta = 0.f;
        if (pool->rope_freq) {
            DeviceGuard g(pool->device);
            cudaFree(pool->rope_freq);
            pool->rope_freq = nullptr;
        }
        return VK_OK;
    }
    if (!pool->kv || (pool->cfg.head_dim & 1)) return fail(VK_UNSUPPORTED, "RoPE needs a KV pool with an even head_dim");
    // frequencies with cpu_rope's float steps (tests/test_kernels.cu:703-705)
    const int D = pool->cfg.head_dim, half = D / 2;
    std::vector<float> freq(half);
    for (int i = 0; i < half; ++i)
        freq[i] = 1.0f / std::pow(theta_base, 2.0f * static_cast<float>(i) / static_cast<float>(D));
    DeviceGuard g(pool->device);
    if (!pool->rope_freq) {
        cudaError_t e = cudaMalloc(&pool->rope_freq, sizeof(float) * half);
        if (e != cudaSuccess) {
            pool->rope_freq = nullptr;
            return cuda_fail(e, "cudaMalloc(RoPE table)");
        }
    }
    cudaError_t e = cudaMemcpy(pool->rope_freq, freq.data(), sizeof(float) * half, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(RoPE table)");
    pool->rope_theta = theta_base;
    return VK_OK;
}

extern "C" vk_status vk_set_prefill_path(vk_pool* pool, int32_t path) {
    if (!pool || path < 0 || path > 2) return fail(VK_INVALID_ARG, "path must be 0 (auto), 1 (mma.sync) or 2 (tcgen05)");
    pool->prefill_path = path;
    return VK_OK;
}
