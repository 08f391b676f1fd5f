// Rotary position embedding fused into the kernels that read Q or write K:
// the rotation of VULCAN's rope kernel (cuda/rope.cu:34-60, golden cpu_rope in
// tests/test_kernels.cu:697-716): pair i = (x[2i], x[2i+1]) at position pos
// turns by pos * freq[i], freq[i] = 1 / theta_base^(2i / head_dim).  The
// frequencies come from a table the host computes with the same float steps
// as cpu_rope (vk_set_rope), so the angle is the CPU's bit for bit; the
// rotation uses CUDA's sincosf and no fused multiply-adds.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

namespace vk {

__device__ __forceinline__ float2 rope_pair(float x0, float x1, int i, int pos, const float* freq) {
    const float ang = __fmul_rn(static_cast<float>(pos), __ldg(freq + i));
    float s, c;
    sincosf(ang, &s, &c);
    return make_float2(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s)), __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c)));
}

// One 32-bit word of two fp16 at even element index d (the pair d/2).
__device__ __forceinline__ uint32_t rope_word(uint32_t w, int d, int pos, const float* freq) {
    __half2 h = *reinterpret_cast<const __half2*>(&w);
    const float2 x = __half22float2(h);
    const float2 y = rope_pair(x.x, x.y, d >> 1, pos, freq);
    h = __floats2half2_rn(y.x, y.y);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Eight fp16 (16 bytes) starting at element d0 (a multiple of 8).
__device__ __forceinline__ uint4 rope_uint4(uint4 v, int d0, int pos, const float* freq) {
    v.x = rope_word(v.x, d0, pos, freq);
    v.y = rope_word(v.y, d0 + 2, pos, freq);
    v.z = rope_word(v.z, d0 + 4, pos, freq);
    v.w = rope_word(v.w, d0 + 6, pos, freq);
    return v;
}

}  // namespace vk
