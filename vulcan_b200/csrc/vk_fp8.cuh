// FP8 (e4m3) KV pages: the group-wise symmetric quantisation of VULCAN's
// ADR-003 (docs/ADRs/003-quantization-format.md:11-18: one fp32 scale per
// group, scale = max|group| / qmax, value = code * scale) with an e4m3 element
// (qmax = 448) in place of int4, and the group = one token's K or V row of one
// head (head_dim = 128 values, ADR-003's group size).
//
// Block of one (layer, page, head), 2*16*D + 128 bytes:
//   K codes  [16 tokens][D]   row t's 16-byte chunks rotated by XOR (t & 7), so
//                             the 8 rows an ldmatrix reads sit in 8 bank groups
//   V codes  [D][16 tokens]   token order 0,1,8,9 | 2,3,10,11 | 4,5,12,13 |
//                             6,7,14,15: the four tokens an mma lane holds for
//                             one element are one 32-bit word
//   K scales [16] fp32, V scales [16] fp32
//
// Quantisation of a row x (fp32): amax = max|x|; amax below the smallest
// normal fp32 gives scale 0 and zero codes; otherwise code = e4m3(x * (448 /
// amax)) rounded to nearest even and saturated to +-448, scale = amax / 448,
// each division and product rounded once (IEEE).
//
// Decode: K codes become the A operand of S^T = K Q^T through ldmatrix and a
// conversion, with the contraction index permuted inside each 16-element step
// (lane c holds elements 4c..4c+3; q fragments are loaded in the same order),
// and each token's K scale multiplies its score.  V codes become V^T fragments
// through ldmatrix (no transpose: the block stores V element-major), unscaled;
// each token's V scale multiplies its probability instead, relative to a power
// of two per page (the largest scale's exponent) so that the fp16 P stays in
// range, and that power of two is carried in the accumulator's rescale.
#pragma once

#include "vk_decode_page.cuh"
#include "vk_internal.h"

namespace vk {

constexpr int kFp8Dim = 128;  // head_dim of FP8 pools

__host__ __device__ constexpr int fp8_head_bytes(int D) { return 2 * kPageTokens * D + 2 * kPageTokens * 4; }
// byte offset of the K code of (token t, element d) in the block
__host__ __device__ constexpr int fp8_k_off(int t, int d, int D) {
    return t * D + ((((d >> 4) ^ (t & 7))) << 4) + (d & 15);
}
// position of token t inside a V row
__host__ __device__ constexpr int fp8_v_pos(int t) { return ((t & 7) >> 1) * 4 + (t & 1) + ((t >> 3) << 1); }
__host__ __device__ constexpr int fp8_v_off(int t, int d, int D) { return kPageTokens * D + d * kPageTokens + fp8_v_pos(t); }
// byte offset of the scale of (K or V, token t)
__host__ __device__ constexpr int fp8_scale_off(int kv, int t, int D) { return 2 * kPageTokens * D + (kv * kPageTokens + t) * 4; }

// e4m3 codes of (lo, hi), nearest even, saturated: lo in bits 0-7.
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}

// Four e4m3 codes (bytes 0..3 of w) as two fp16 pairs: bytes 0,1 -> lo, 2,3 -> hi.
__device__ __forceinline__ void e4m3x4_to_h2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
    asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
        : "=r"(lo), "=r"(hi)
        : "r"(w));
}

// Quantises one row held by a warp, elements 4*lane + i in x[i]: returns the
// lane's four codes (element 4*lane in bits 0-7) and the row's scale.
__device__ __forceinline__ uint32_t fp8_quant_row(const float (&x)[4], float& scale) {
    float a = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    if (!(a >= 1.17549435e-38f)) {
        scale = 0.f;
        return 0u;
    }
    const float inv = __fdiv_rn(448.f, a);
    scale = __fdiv_rn(a, 448.f);
    return e4m3x2(__fmul_rn(x[0], inv), __fmul_rn(x[1], inv)) |
           (e4m3x2(__fmul_rn(x[2], inv), __fmul_rn(x[3], inv)) << 16);
}

// Writes a quantised token (K codes kc, V codes vc of the lane's four
// elements, scales) into a block at `blk` (generic address: global or shared).
__device__ __forceinline__ void fp8_store_token(char* blk, int t, int lane, uint32_t kc, uint32_t vc, float ks,
                                                float vs) {
    constexpr int D = kFp8Dim;
    *reinterpret_cast<uint32_t*>(blk + fp8_k_off(t, 4 * lane, D)) = kc;
#pragma unroll
    for (int i = 0; i < 4; ++i) blk[fp8_v_off(t, 4 * lane + i, D)] = static_cast<char>((vc >> (8 * i)) & 0xffu);
    if (lane == 0) {
        *reinterpret_cast<float*>(blk + fp8_scale_off(0, t, D)) = ks;
        *reinterpret_cast<float*>(blk + fp8_scale_off(1, t, D)) = vs;
    }
}

// Q of heads [head0, head0 + G) as mma B fragments in the FP8 contraction
// order: step ks, lane c holds elements 16ks + 4c .. 4c+3.
template <int D, int NT>
__device__ __forceinline__ void load_q_frags_fp8(uint32_t (&qf)[NT][D / 16][2], const __half* q_seq, int G, int lane) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int hl = nt * 8 + (lane >> 2);
        const bool ok = hl < G;
        const __half* qrow = q_seq + (ok ? hl : 0) * D;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
            const int d = ks * 16 + (lane & 3) * 4;
            qf[nt][ks][0] = ok ? __ldg(reinterpret_cast<const unsigned int*>(qrow + d)) : 0u;
            qf[nt][ks][1] = ok ? __ldg(reinterpret_cast<const unsigned int*>(qrow + d + 2)) : 0u;
        }
    }
}

template <int D, int NT>
__device__ __forceinline__ void rope_q_frags_fp8(uint32_t (&qf)[NT][D / 16][2], int pos, const float* freq, int lane) {
    if (freq == nullptr) return;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
            const int d = ks * 16 + (lane & 3) * 4;
            qf[nt][ks][0] = rope_word(qf[nt][ks][0], d, pos, freq);
            qf[nt][ks][1] = rope_word(qf[nt][ks][1], d + 2, pos, freq);
        }
}

__device__ __forceinline__ float lds_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}

// Folds one FP8 block held at shared address `sb` (valid tokens 1..16) into
// `st`; the softmax steps are those of page_update.
template <int D, int NT>
__device__ __forceinline__ void page_update_fp8(uint32_t sb, int valid, const uint32_t (&qf)[NT][D / 16][2],
                                                WarpSoftmaxState<D, NT>& st, float scale_log2, int lane) {
    static_assert(D == kFp8Dim, "FP8 blocks are defined for head_dim 128");
    constexpr int P = kPageTokens;
    constexpr int KS = D / 16;
    const int g8 = lane >> 2;
    const int mi = lane >> 3, rr = lane & 7;

    float s[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
    for (int i = 0; i < D / 32; ++i) {
        // matrices: tokens 0-7 / 8-15 of chunk 2i, then of chunk 2i+1
        const int tok = rr + (mi & 1) * 8;
        const int ch = 2 * i + (mi >> 1);
        uint32_t r[4];
        ldsm_x4(r, sb + tok * D + ((ch ^ (tok & 7)) << 4));
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint32_t a[4];
            e4m3x4_to_h2x2(r[2 * h], a[0], a[2]);
            e4m3x4_to_h2x2(r[2 * h + 1], a[1], a[3]);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) mma16816(s[nt], a, qf[nt][2 * i + h][0], qf[nt][2 * i + h][1]);
        }
    }

    // scales of the lane's tokens g8 and g8+8; unwritten tokens (any bits)
    // count as V scale 0.  V scales are used relative to 2^e, e the exponent of
    // the page's largest; acc is kept in units of the current 2^e (st.vf),
    // folded into each page's rescale factor.
    const bool v0 = g8 < valid, v1 = g8 + 8 < valid;
    const uint32_t sk = sb + fp8_scale_off(0, 0, D), sv = sb + fp8_scale_off(1, 0, D);
    const float kA = scale_log2 * lds_f32(sk + g8 * 4), kB = scale_log2 * lds_f32(sk + (g8 + 8) * 4);
    const float vA = v0 ? lds_f32(sv + g8 * 4) : 0.f, vB = v1 ? lds_f32(sv + (g8 + 8) * 4) : 0.f;
    float vmax = fmaxf(vA, vB);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
    const int e = min(60, max(-60, static_cast<int>((__float_as_uint(vmax) >> 23) & 0xffu) - 127));
    const float inv_f = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);  // 2^-e
    const float ratio = st.vf * inv_f;                                             // exact
    st.vf = __uint_as_float(static_cast<uint32_t>(127 + e) << 23);
    const float rA = vA * inv_f, rB = vB * inv_f;  // in [0, 2)

    uint32_t pb[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const float x0 = v0 ? s[nt][0] * kA : -INFINITY;
        const float x1 = v0 ? s[nt][1] * kA : -INFINITY;
        const float x2 = v1 ? s[nt][2] * kB : -INFINITY;
        const float x3 = v1 ? s[nt][3] * kB : -INFINITY;
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
        // unconditional: a warp vote to skip it when no max moved measured 3% slower
        const float cA = aA * ratio, cB = aB * ratio;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
            st.acc[nt][mt][0] *= cA;
            st.acc[nt][mt][1] *= cB;
            st.acc[nt][mt][2] *= cA;
            st.acc[nt][mt][3] *= cB;
        }
        // p of token g8 (heads 2c, 2c+1) and g8+8, times the token's V scale
        pb[nt][0] = movm_t(pack_half2(p0 * rA, p1 * rA));
        pb[nt][1] = movm_t(pack_half2(p2 * rB, p3 * rB));
    }

    const int t0 = (lane & 3) * 2;
#pragma unroll
    for (int i = 0; i < D / 32; ++i) {
        // matrices: element rows 32i + 8*mi + 0..7 (16 bytes each)
        uint32_t r[4];
        ldsm_x4(r, sb + P * D + (32 * i + 8 * mi + rr) * P);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int mt = 2 * i + h;
            uint32_t a[4];
            e4m3x4_to_h2x2(r[2 * h], a[0], a[2]);      // element 16mt + g: tokens (2c, 2c+1), (2c+8, 2c+9)
            e4m3x4_to_h2x2(r[2 * h + 1], a[1], a[3]);  // element 16mt + g + 8
            if (valid < P) {  // unwritten slots may hold any bits (NaN codes): zero them
                const uint32_t keepA = (t0 < valid ? 0x0000ffffu : 0u) | (t0 + 1 < valid ? 0xffff0000u : 0u);
                const uint32_t keepB = (t0 + 8 < valid ? 0x0000ffffu : 0u) | (t0 + 9 < valid ? 0xffff0000u : 0u);
                a[0] &= keepA;
                a[1] &= keepA;
                a[2] &= keepB;
                a[3] &= keepB;
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) mma16816(st.acc[nt][mt], a, pb[nt][0], pb[nt][1]);
        }
    }
}

}  // namespace vk
