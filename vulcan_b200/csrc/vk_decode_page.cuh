// Per-page decode update shared by the decode kernels: one warp folds one
// 16-token page of K and V (already in shared memory, two 128-byte-swizzled TMA
// boxes per 64 columns) into its running softmax state for up to 8*NT query
// heads of one KV head.
//
//   S^T[16 tokens x 8 heads] = K Q^T         mma.m16n8k16, Q as the B operand
//   online softmax per head over the tokens  shuffles across the 8 token lanes
//   O^T[D x 8 heads] += V^T P^T              ldmatrix.trans of V, movmatrix.trans of P
//
// Fragment ownership (lane = 4*g + c):
//   S^T: tokens g and g+8, heads 2c and 2c+1 of each 8-head tile
//   O^T: rows d = 16*mt + g (+8), heads 2c, 2c+1
#pragma once

#include "vk_ptx.cuh"
#include "vk_rope.cuh"

namespace vk {

template <int D, int NT>
struct WarpSoftmaxState {
    float m[NT][2];
    float l[NT][2];
    float acc[NT][D / 16][4];
    float vf;  // FP8 pages: acc holds the true sums divided by vf (a power of two)

    __device__ __forceinline__ void reset() {
        vf = 1.f;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            m[nt][0] = m[nt][1] = -INFINITY;
            l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
            for (int mt = 0; mt < D / 16; ++mt) acc[nt][mt][0] = acc[nt][mt][1] = acc[nt][mt][2] = acc[nt][mt][3] = 0.f;
        }
    }
};

// Q of heads [head0, head0 + G) of one sequence as mma B fragments; heads at
// or beyond G are zero.
template <int D, int NT>
__device__ __forceinline__ void load_q_frags(uint32_t (&qf)[NT][D / 16][2], const __half* q_seq, int G, int lane) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int hl = nt * 8 + (lane >> 2);
        const bool ok = hl < G;
        const __half* qrow = q_seq + (ok ? hl : 0) * D;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
            const int d = ks * 16 + (lane & 3) * 2;
            qf[nt][ks][0] = ok ? __ldg(reinterpret_cast<const unsigned int*>(qrow + d)) : 0u;
            qf[nt][ks][1] = ok ? __ldg(reinterpret_cast<const unsigned int*>(qrow + d + 8)) : 0u;
        }
    }
}

// Fused RoPE of the q fragments loaded by load_q_frags (every query head of a
// unit at the new token's position pos); freq == nullptr: no rotation.
template <int D, int NT>
__device__ __forceinline__ void rope_q_frags(uint32_t (&qf)[NT][D / 16][2], int pos, const float* freq, int lane) {
    if (freq == nullptr) return;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
            const int d = ks * 16 + (lane & 3) * 2;
            qf[nt][ks][0] = rope_word(qf[nt][ks][0], d, pos, freq);
            qf[nt][ks][1] = rope_word(qf[nt][ks][1], d + 8, pos, freq);
        }
}

// Folds one page held at shared address `sb` (valid tokens 1..16) into `st`.
template <int D, int NT>
__device__ __forceinline__ void page_update(uint32_t sb, int valid, const uint32_t (&qf)[NT][D / 16][2],
                                            WarpSoftmaxState<D, NT>& st, float scale_log2, int lane) {
    constexpr int P = 16;
    constexpr int KS = D / 16;
    const int g8 = lane >> 2;
    const int mi = lane >> 3, rr = lane & 7;

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

    uint32_t pb[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const bool v0 = g8 < valid, v1 = g8 + 8 < valid;
        const float x0 = v0 ? s[nt][0] * scale_log2 : -INFINITY;
        const float x1 = v0 ? s[nt][1] * scale_log2 : -INFINITY;
        const float x2 = v1 ? s[nt][2] * scale_log2 : -INFINITY;
        const float x3 = v1 ? s[nt][3] * scale_log2 : -INFINITY;
        float mA = fmaxf(x0, x2), mB = fmaxf(x1, x3);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            mA = fmaxf(mA, __shfl_xor_sync(0xffffffffu, mA, o));
            mB = fmaxf(mB, __shfl_xor_sync(0xffffffffu, mB, o));
        }
        const float nA = fmaxf(st.m[nt][0], mA), nB = fmaxf(st.m[nt][1], mB);
        const float aA = ex2(st.m[nt][0] - nA), aB = ex2(st.m[nt][1] - nB);
        st.m[nt][0] = nA;
        st.m[nt][1] = nB;
        const float p0 = ex2(x0 - nA), p1 = ex2(x1 - nB), p2 = ex2(x2 - nA), p3 = ex2(x3 - nB);
        st.l[nt][0] = st.l[nt][0] * aA + p0 + p2;
        st.l[nt][1] = st.l[nt][1] * aB + p1 + p3;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
            st.acc[nt][mt][0] *= aA;
            st.acc[nt][mt][1] *= aB;
            st.acc[nt][mt][2] *= aA;
            st.acc[nt][mt][3] *= aB;
        }
        pb[nt][0] = movm_t(pack_half2(p0, p1));
        pb[nt][1] = movm_t(pack_half2(p2, p3));
    }

    const int vt0 = (lane & 3) * 2;
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
        const int tok = rr + (mi >> 1) * 8;
        const int d = mt * 16 + (mi & 1) * 8;
        uint32_t a[4];
        ldsm_x4_t(a, sb + (d >> 6) * (2 * P * 128) + swz128(P + tok, (d & 63) >> 3));
        if (valid < P) {  // unwritten slots may hold any bits: zero their V
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int t = vt0 + (r >= 2 ? 8 : 0);
                const uint32_t keep = (t < valid ? 0x0000ffffu : 0u) | (t + 1 < valid ? 0xffff0000u : 0u);
                a[r] &= keep;
            }
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma16816(st.acc[nt][mt], a, pb[nt][0], pb[nt][1]);
    }
}

// Sums the per-lane partial row sums over the 8 lanes that share lane&3.
template <int D, int NT>
__device__ __forceinline__ void reduce_l(WarpSoftmaxState<D, NT>& st) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) st.l[nt][j] += __shfl_xor_sync(0xffffffffu, st.l[nt][j], o);
}

}  // namespace vk
