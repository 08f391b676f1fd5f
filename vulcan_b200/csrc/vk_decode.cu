// K2: paged GQA decode attention with split-K and a merge kernel.
//
// Replaces the decode use of VULCAN's attention_kernel / launch_attention
// (cuda/attention.cu:38-131), which the engine launches once per query head
// with the contiguous cache (src/transformer.cpp:157-189).  The arithmetic
// being reproduced is one causal row of cpu_attention
// (tests/test_attention.cu:66-97): s_j = (q . k_j) / sqrt(D) over all cached
// keys, softmax, weighted sum of V.  The GQA mapping is
// kv_head = q_head / (Hq / Hkv) (src/transformer.cpp:173-179).
//
// Design (B200):
//  * One CTA per (split, kv head, sequence).  A split is a run of at most
//    `pps` pages of the sequence; all G = Hq/Hkv query heads of the KV head are
//    served from the same page loads, so every K/V byte is read once.
//  * Warp 4 is the producer: one thread walks the block table and issues 2-D
//    TMA loads (128-byte swizzle, L2 evict-first) of each page's K and V rows
//    for this (layer, kv head) into an 8-stage shared-memory ring, completing
//    on mbarriers.  Warps 0-3 consume pages round-robin.
//  * Per page a consumer warp computes S^T = K Q^T on the tensor cores
//    (mma.m16n8k16, tokens as M=16, query heads as N=8), runs an online
//    softmax per head in registers (shuffles across the 8 token lanes), turns
//    P^T into the B operand with movmatrix.trans and accumulates
//    O^T += V^T P^T (ldmatrix.trans of V).  fp16 operands, fp32 accumulation.
//  * The four warps' (m, l, O) are combined in shared memory.  A sequence with
//    one split writes fp16 output directly; otherwise the split writes its
//    normalised partial and log-sum-exp and the merge kernel combines them.
//  * Every wait is bounded; bad block-table entries are recorded in the pool's
//    error word and replaced by page 0 so no access leaves the pool.
//  * FP8 pools (FMT = 1, D = 128): a page block arrives in one bulk copy and
//    the consumers fold it in with page_update_fp8 (vk_fp8.cuh).
#include <algorithm>

#include "vk_fp8.cuh"
#include "vk_internal.h"
#include "vk_ptx.cuh"
#include "vk_rope.cuh"

namespace vk {

constexpr int kDecodeConsumers = 4;
constexpr int kDecodeThreads = (kDecodeConsumers + 1) * 32;
constexpr int kDecodeStages = 8;

struct DecodeParams {
    const __half* q;
    __half* out;
    float* ws_o;    // [B, Hq, max_splits, D]
    float* ws_lse;  // [B, Hq, max_splits]
    const int32_t* bt;
    const int32_t* seq_lens;
    uint32_t* err;
    int bt_stride, Hq, Hkv, G, L, layer, num_pages, pps, max_splits;
    float scale_log2;
    const float* rope_freq;  // non-null: q rotated (RoPE) at position seq_len - 1
    // FP8 pools: block addressing for the bulk copies
    const char* pool_base;
    uint64_t seg_bytes, layer_off, head_bytes;
};

template <int D, int FMT>
__host__ __device__ constexpr int stage_bytes() {
    return FMT ? fp8_head_bytes(D) : 2 * kPageTokens * D * 2;
}

template <int D, int FMT>
__host__ __device__ constexpr int decode_smem_bytes() {
    return kDecodeStages * stage_bytes<D, FMT>() + 2 * kDecodeStages * 8 + 1024;
}

// Length of sequence b clamped to the table capacity, recording bad lengths.
__device__ __forceinline__ int checked_len(const DecodeParams& p, int b, bool report) {
    int n = p.seq_lens[b];
    if (n < 0 || n > p.bt_stride * kPageTokens) {
        if (report) atomicOr(p.err, VK_ERR_SEQ_LEN);
        n = 0;
    }
    return n;
}

template <int D, int NT, int FMT>
__global__ void __launch_bounds__(kDecodeThreads) decode_kernel(const __grid_constant__ CUtensorMap tmap,
                                                                const DecodeParams p) {
    static_assert(FMT == 0 || D == kFp8Dim, "FP8 blocks are defined for head_dim 128");
    // the combine after the ring reuses its shared memory
    static_assert(kDecodeStages * stage_bytes<D, FMT>() >= 4 * (2 + D) * NT * 8 * 4, "combine does not fit");
    constexpr int P = kPageTokens;
    constexpr int SB = stage_bytes<D, FMT>();
    constexpr int NB = D / 64;   // 128-byte TMA boxes per row
    constexpr int KS = D / 16;   // k-steps of S^T, m-tiles of O^T
    constexpr int NH = NT * 8;   // query heads per CTA tile (>= G)

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kDecodeStages * SB);
    uint64_t* empty = full + kDecodeStages;

    const int split = blockIdx.x, hkv = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int seq_len = checked_len(p, b, threadIdx.x == 0 && split == 0 && hkv == 0);
    const int npages = (seq_len + P - 1) / P;
    const int nsplit = (npages + p.pps - 1) / p.pps;

    if (npages == 0) {  // nothing to attend: zeros, like an empty weighted sum
        if (split == 0)
            for (int i = threadIdx.x; i < p.G * D; i += blockDim.x)
                p.out[(static_cast<int64_t>(b) * p.Hq + hkv * p.G + i / D) * D + i % D] = __float2half(0.f);
        return;
    }
    if (split >= nsplit) return;
    const int pbeg = split * p.pps;
    const int n = min(npages, pbeg + p.pps) - pbeg;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kDecodeStages; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        mbar_fence_init();
    }
    __syncthreads();

    // Per-warp softmax state (valid in consumer warps).
    float m_run[NT][2], l_run[NT][2], acc[NT][KS][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        m_run[nt][0] = m_run[nt][1] = -INFINITY;
        l_run[nt][0] = l_run[nt][1] = 0.f;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) acc[nt][mt][0] = acc[nt][mt][1] = acc[nt][mt][2] = acc[nt][mt][3] = 0.f;
    }

    if (warp == kDecodeConsumers) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            if (FMT == 0) prefetch_tmap(&tmap);
            const uint64_t pol = l2_evict_first_policy();
            const int32_t* btrow = p.bt + static_cast<int64_t>(b) * p.bt_stride + pbeg;
            for (int i = 0; i < n; ++i) {
                const int st = i % kDecodeStages;
                if (i >= kDecodeStages &&
                    !mbar_wait(smem_u32(&empty[st]), ((i / kDecodeStages) - 1) & 1, p.err))
                    break;
                int page = btrow[i];
                if (page < 0 || page >= p.num_pages) {
                    atomicOr(p.err, VK_ERR_PAGE_ID);
                    page = 0;
                }
                const uint32_t bar = smem_u32(&full[st]);
                mbar_expect_tx(bar, SB);
                const uint32_t dst = smem_u32(smem + st * SB);
                if constexpr (FMT == 1) {
                    bulk_load(dst, p.pool_base + p.layer_off + static_cast<uint64_t>(page) * p.seg_bytes +
                                       static_cast<uint64_t>(hkv) * p.head_bytes,
                              SB, bar, pol);
                } else {
                    const int row = ((p.layer * p.num_pages + page) * p.Hkv + hkv) * (2 * P);
#pragma unroll
                    for (int hb = 0; hb < NB; ++hb)
                        tma_load_2d(dst + hb * (2 * P * 128), &tmap, hb * 64, row, bar, pol);
                }
            }
        }
    } else {
        // ------------------------------------------------------------ consumers
        // Q as the B operand (k = head dim, n = query head): 2 regs per k-step.
        // (FP8: the permuted contraction order of page_update_fp8, elements
        // 4c..4c+3 of each 16-step, so the second pair is at d+2)
        constexpr int D2 = FMT ? 2 : 8;
        uint32_t qf[NT][KS][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int hl = nt * 8 + (lane >> 2);
            const bool ok = hl < p.G;
            const __half* qrow = p.q + (static_cast<int64_t>(b) * p.Hq + hkv * p.G + (ok ? hl : 0)) * D;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                const int d = ks * 16 + (lane & 3) * (FMT ? 4 : 2);
                qf[nt][ks][0] = ok ? *reinterpret_cast<const uint32_t*>(qrow + d) : 0u;
                qf[nt][ks][1] = ok ? *reinterpret_cast<const uint32_t*>(qrow + d + D2) : 0u;
            }
        }
        if (p.rope_freq != nullptr) {  // fused RoPE at the new token's position
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int ks = 0; ks < KS; ++ks) {
                    const int d = ks * 16 + (lane & 3) * (FMT ? 4 : 2);
                    qf[nt][ks][0] = rope_word(qf[nt][ks][0], d, seq_len - 1, p.rope_freq);
                    qf[nt][ks][1] = rope_word(qf[nt][ks][1], d + D2, seq_len - 1, p.rope_freq);
                }
        }
        WarpSoftmaxState<D, NT> st8;  // FP8 pages: page_update_fp8's state
        if constexpr (FMT == 1) st8.reset();
        const int g8 = lane >> 2;           // token row of this lane in S^T (and +8)
        const int mi = lane >> 3, rr = lane & 7;  // ldmatrix: matrix index, row in matrix
        bool alive = true;
        for (int i = warp; i < n && alive; i += kDecodeConsumers) {
            const int st = i % kDecodeStages;
            // warp-uniform outcome, so a timed-out wait never splits the warp
            if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&full[st]), (i / kDecodeStages) & 1, p.err))) {
                alive = false;
                break;
            }
            const uint32_t sb = smem_u32(smem + st * SB);
            const int valid = min(P, seq_len - (pbeg + i) * P);
            if constexpr (FMT == 1) {
                page_update_fp8<D, NT>(sb, valid, qf, st8, p.scale_log2, lane);
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&empty[st]));
                continue;
            }

            // S^T[16 tokens x 8 heads] = K Q^T
            float s[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                const int tok = rr + (mi & 1) * 8;
                const int d = ks * 16 + (mi >> 1) * 8;
                uint32_t a[4];
                ldsm_x4(a, sb + (d >> 6) * (2 * P * 128) + swz128(tok, (d & 63) >> 3));
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma16816(s[nt], a, qf[nt][ks][0], qf[nt][ks][1]);
            }

            // Online softmax per head; P^T to B fragments.
            uint32_t pb[NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const bool v0 = g8 < valid, v1 = g8 + 8 < valid;
                const float x0 = v0 ? s[nt][0] * p.scale_log2 : -INFINITY;
                const float x1 = v0 ? s[nt][1] * p.scale_log2 : -INFINITY;
                const float x2 = v1 ? s[nt][2] * p.scale_log2 : -INFINITY;
                const float x3 = v1 ? s[nt][3] * p.scale_log2 : -INFINITY;
                float mA = fmaxf(x0, x2), mB = fmaxf(x1, x3);
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) {
                    mA = fmaxf(mA, __shfl_xor_sync(0xffffffffu, mA, o));
                    mB = fmaxf(mB, __shfl_xor_sync(0xffffffffu, mB, o));
                }
                const float nA = fmaxf(m_run[nt][0], mA), nB = fmaxf(m_run[nt][1], mB);
                const float aA = ex2(m_run[nt][0] - nA), aB = ex2(m_run[nt][1] - nB);
                m_run[nt][0] = nA;
                m_run[nt][1] = nB;
                const float p0 = ex2(x0 - nA), p1 = ex2(x1 - nB), p2 = ex2(x2 - nA), p3 = ex2(x3 - nB);
                l_run[nt][0] = l_run[nt][0] * aA + p0 + p2;
                l_run[nt][1] = l_run[nt][1] * aB + p1 + p3;
#pragma unroll
                for (int mt = 0; mt < KS; ++mt) {
                    acc[nt][mt][0] *= aA;
                    acc[nt][mt][1] *= aB;
                    acc[nt][mt][2] *= aA;
                    acc[nt][mt][3] *= aB;
                }
                pb[nt][0] = movm_t(pack_half2(p0, p1));
                pb[nt][1] = movm_t(pack_half2(p2, p3));
            }

            // O^T[D x 8 heads] += V^T P^T
            const int vt0 = (lane & 3) * 2;  // first token held in a[0]/a[1]
#pragma unroll
            for (int mt = 0; mt < KS; ++mt) {
                const int tok = rr + (mi >> 1) * 8;
                const int d = mt * 16 + (mi & 1) * 8;
                uint32_t a[4];
                ldsm_x4_t(a, sb + (d >> 6) * (2 * P * 128) + swz128(P + tok, (d & 63) >> 3));
                if (valid < P) {  // zero V of unwritten slots (they may hold any bits)
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const int t = vt0 + (r >= 2 ? 8 : 0);
                        const uint32_t keep = (t < valid ? 0x0000ffffu : 0u) | (t + 1 < valid ? 0xffff0000u : 0u);
                        a[r] &= keep;
                    }
                }
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma16816(acc[nt][mt], a, pb[nt][0], pb[nt][1]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&empty[st]));
        }
        if constexpr (FMT == 1) {  // back to this kernel's state, acc in true units
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    m_run[nt][j] = st8.m[nt][j];
                    l_run[nt][j] = st8.l[nt][j];
                }
#pragma unroll
                for (int mt = 0; mt < KS; ++mt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[nt][mt][e] = st8.acc[nt][mt][e] * st8.vf;
            }
        }
        // Row sums: reduce over the 8 lanes sharing lane&3.
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) l_run[nt][j] += __shfl_xor_sync(0xffffffffu, l_run[nt][j], o);
    }

    __syncthreads();  // every page consumed: the ring can be reused for the combine

    float* cm = reinterpret_cast<float*>(smem);                 // [4][NH]
    float* cl = cm + kDecodeConsumers * NH;                      // [4][NH]
    float* co = cl + kDecodeConsumers * NH;                      // [4][D][NH]
    if (warp < kDecodeConsumers) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int h0 = nt * 8 + (lane & 3) * 2;
            if (lane < 4) {
                cm[warp * NH + h0] = m_run[nt][0];
                cm[warp * NH + h0 + 1] = m_run[nt][1];
                cl[warp * NH + h0] = l_run[nt][0];
                cl[warp * NH + h0 + 1] = l_run[nt][1];
            }
#pragma unroll
            for (int mt = 0; mt < KS; ++mt) {
                const int d = mt * 16 + (lane >> 2);
                float* o = co + (warp * D) * NH;
                o[d * NH + h0] = acc[nt][mt][0];
                o[d * NH + h0 + 1] = acc[nt][mt][1];
                o[(d + 8) * NH + h0] = acc[nt][mt][2];
                o[(d + 8) * NH + h0 + 1] = acc[nt][mt][3];
            }
        }
    }
    __syncthreads();

    const int64_t head0 = static_cast<int64_t>(b) * p.Hq + hkv * p.G;
    for (int idx = threadIdx.x; idx < p.G * D; idx += blockDim.x) {
        const int h = idx / D, d = idx % D;
        float mx = -INFINITY;
#pragma unroll
        for (int w = 0; w < kDecodeConsumers; ++w) mx = fmaxf(mx, cm[w * NH + h]);
        float num = 0.f, den = 0.f;
#pragma unroll
        for (int w = 0; w < kDecodeConsumers; ++w) {
            const float f = ex2(cm[w * NH + h] - mx);
            num += f * co[(w * D + d) * NH + h];
            den += f * cl[w * NH + h];
        }
        const float o = num / den;
        if (nsplit == 1) {
            p.out[(head0 + h) * D + d] = __float2half(o);
        } else {
            const int64_t slot = (head0 + h) * p.max_splits + split;
            p.ws_o[slot * D + d] = o;
            if (d == 0) p.ws_lse[slot] = mx + __log2f(den);
        }
    }
}

// Combines split partials: out = sum_s 2^(lse_s - max) o_s / sum_s 2^(lse_s - max).
template <int D>
__global__ void __launch_bounds__(D) merge_kernel(const DecodeParams p) {
    const int bh = blockIdx.x;
    const int b = bh / p.Hq;
    const int seq_len = checked_len(p, b, false);
    const int npages = (seq_len + kPageTokens - 1) / kPageTokens;
    const int nsplit = (npages + p.pps - 1) / p.pps;
    if (nsplit <= 1) return;
    const float* lse = p.ws_lse + static_cast<int64_t>(bh) * p.max_splits;
    const float* o = p.ws_o + static_cast<int64_t>(bh) * p.max_splits * D;
    float mx = -INFINITY;
    for (int s = 0; s < nsplit; ++s) mx = fmaxf(mx, lse[s]);
    float num = 0.f, den = 0.f;
    for (int s = 0; s < nsplit; ++s) {
        const float f = ex2(lse[s] - mx);
        num += f * o[s * D + threadIdx.x];
        den += f;
    }
    p.out[static_cast<int64_t>(bh) * D + threadIdx.x] = __float2half(num / den);
}

int decode_pages_per_split(const vk_pool* pool, int B, int max_seq_len) {
    if (!pool || !pool->kv || B <= 0 || max_seq_len < 0) return 0;
    if (pool->split_override > 0) return pool->split_override;
    const int max_pages = std::max(1, (max_seq_len + kPageTokens - 1) / kPageTokens);
    // Aim for ~8 CTAs per SM of real work assuming lengths average half the
    // maximum; chunks of 8..64 pages (128..1024 tokens).
    const double est_pages = 0.5 * static_cast<double>(B) * pool->cfg.num_kv_heads * max_pages;
    const double per_cta = est_pages / (8.0 * pool->num_sms);
    int pps = 8;
    while (pps < 64 && pps < per_cta) pps <<= 1;
    return pps;
}

template <int D, int NT, int FMT>
static vk_status launch_decode_t(vk_pool* pool, const DecodeParams& p, int B, cudaStream_t st) {
    constexpr int smem = decode_smem_bytes<D, FMT>();
    static uint64_t attr_set = 0;  // one bit per device ordinal
    const uint64_t bit = 1ull << (pool->device & 63);
    if (!(attr_set & bit)) {
        cudaError_t e = cudaFuncSetAttribute(decode_kernel<D, NT, FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(decode)");
        attr_set |= bit;
    }
    dim3 grid(p.max_splits, p.Hkv, B);
    decode_kernel<D, NT, FMT><<<grid, kDecodeThreads, smem, st>>>(pool->tmap, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "decode_kernel launch");
    if (p.max_splits > 1) {
        merge_kernel<D><<<B * p.Hq, D, 0, st>>>(p);
        e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_fail(e, "merge_kernel launch");
    }
    return VK_OK;
}

static int decode_max_splits(int pps, int max_seq_len) {
    const int max_pages = std::max(1, (max_seq_len + kPageTokens - 1) / kPageTokens);
    return (max_pages + pps - 1) / pps;
}

}  // namespace vk

using namespace vk;

extern "C" {

int32_t vk_decode_pages_per_split(const vk_pool* pool, int32_t batch, int32_t max_seq_len) {
    return decode_pages_per_split(pool, batch, max_seq_len);
}

vk_status vk_set_decode_split(vk_pool* pool, int32_t pages_per_split) {
    if (!pool || pages_per_split < 0) return fail(VK_INVALID_ARG, "bad split override");
    pool->split_override = pages_per_split;
    return VK_OK;
}

size_t vk_decode_workspace_size(const vk_pool* pool, int32_t batch, int32_t num_q_heads,
                                int32_t max_seq_len) {
    const int pps = decode_pages_per_split(pool, batch, max_seq_len);
    if (pps <= 0 || num_q_heads <= 0) return 0;
    const int ms = decode_max_splits(pps, max_seq_len);
    if (ms <= 1) return 0;
    return static_cast<size_t>(batch) * num_q_heads * ms * (pool->cfg.head_dim + 1) * sizeof(float);
}

vk_status vk_decode(vk_pool* pool, int32_t layer, const void* q, void* out,
                    const int32_t* block_tables, int32_t bt_stride, const int32_t* seq_lens,
                    int32_t batch, int32_t num_q_heads, int32_t max_seq_len, float scale,
                    void* workspace, size_t workspace_bytes, void* stream) {
    if (!pool) return fail(VK_INVALID_ARG, "pool is NULL");
    if (!pool->kv) return fail(VK_UNSUPPORTED, "decode needs a KV pool (page_bytes == 0)");
    const bool fp8 = pool->kv_format == VK_KV_FP8;
    if (!fp8 && !pool->tmap_ok) return fail(VK_UNSUPPORTED, "pool too large for 32-bit TMA row coordinates");
    if (pool->cfg.page_tokens != kPageTokens) return fail(VK_UNSUPPORTED, "decode supports page_tokens == 16");
    const int D = pool->cfg.head_dim, Hkv = pool->cfg.num_kv_heads;
    if (D != 64 && D != 128 && D != 256) return fail(VK_UNSUPPORTED, "decode supports head_dim 64, 128, 256");
    if (layer < 0 || layer >= pool->cfg.num_layers) return fail(VK_INVALID_ARG, "layer out of range");
    if (batch < 0 || bt_stride <= 0 || max_seq_len < 0) return fail(VK_INVALID_ARG, "bad batch/bt_stride/max_seq_len");
    if (num_q_heads <= 0 || num_q_heads % Hkv) return fail(VK_INVALID_ARG, "num_q_heads must be a positive multiple of num_kv_heads");
    if (max_seq_len > bt_stride * kPageTokens) return fail(VK_INVALID_ARG, "max_seq_len exceeds the block table capacity");
    if (batch == 0) return VK_OK;
    if (batch > 65535 || Hkv > 65535) return fail(VK_INVALID_ARG, "batch and num_kv_heads must be <= 65535");
    if (!q || !out || !block_tables || !seq_lens) return fail(VK_INVALID_ARG, "NULL array");
    if ((reinterpret_cast<uintptr_t>(q) & 3) || (reinterpret_cast<uintptr_t>(out) & 1))
        return fail(VK_INVALID_ARG, "q must be 4-byte aligned, out 2-byte aligned");
    const int G = num_q_heads / Hkv;
    if (G > 16) return fail(VK_UNSUPPORTED, "decode supports up to 16 query heads per KV head");

    DecodeParams p;
    p.q = static_cast<const __half*>(q);
    p.out = static_cast<__half*>(out);
    p.bt = block_tables;
    p.seq_lens = seq_lens;
    p.err = pool->d_err;
    p.bt_stride = bt_stride;
    p.Hq = num_q_heads;
    p.Hkv = Hkv;
    p.G = G;
    p.L = pool->cfg.num_layers;
    p.layer = layer;
    p.num_pages = pool->num_pages;
    p.pps = decode_pages_per_split(pool, batch, max_seq_len);
    p.max_splits = decode_max_splits(p.pps, max_seq_len);
    if (p.max_splits > 65535) return fail(VK_INVALID_ARG, "too many splits");
    const float sc = scale > 0.f ? scale : 1.0f / sqrtf(static_cast<float>(D));
    p.scale_log2 = sc * 1.4426950408889634f;
    p.rope_freq = pool->rope_freq;
    p.pool_base = pool->base;
    p.seg_bytes = pool->seg_bytes;
    p.layer_off = static_cast<uint64_t>(layer) * pool->seg_stride;
    p.head_bytes = pool->head_bytes;
    p.ws_o = nullptr;
    p.ws_lse = nullptr;
    if (p.max_splits > 1) {
        const size_t need = vk_decode_workspace_size(pool, batch, num_q_heads, max_seq_len);
        if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15))
            return fail(VK_INVALID_ARG, "workspace missing, too small or not 16-byte aligned");
        p.ws_o = static_cast<float*>(workspace);
        p.ws_lse = p.ws_o + static_cast<size_t>(batch) * num_q_heads * p.max_splits * D;
    }
    DeviceGuard g(pool->device);
    cudaStream_t st = as_stream(stream);
    if (fp8)  // FP8 pools have head_dim 128
        return G <= 8 ? launch_decode_t<128, 1, 1>(pool, p, batch, st) : launch_decode_t<128, 2, 1>(pool, p, batch, st);
    if (D == 128)
        return G <= 8 ? launch_decode_t<128, 1, 0>(pool, p, batch, st) : launch_decode_t<128, 2, 0>(pool, p, batch, st);
    if (D == 64) return G <= 8 ? launch_decode_t<64, 1, 0>(pool, p, batch, st) : launch_decode_t<64, 2, 0>(pool, p, batch, st);
    return G <= 8 ? launch_decode_t<256, 1, 0>(pool, p, batch, st) : launch_decode_t<256, 2, 0>(pool, p, batch, st);
}

}  // extern "C"
