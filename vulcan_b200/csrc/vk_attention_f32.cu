// Compatibility entry: contiguous fp32 causal attention with the contract of
// VULCAN's vulcan::cuda::launch_attention (cuda/attention.cu:119-131):
// Q, K, V, O are [batch, heads, seq_len, head_dim]; row i attends keys 0..i
// with scale 1/sqrt(head_dim).
//
// The reference runs one thread per row with three recompute passes.  Here one
// warp owns a query row: each lane scores one key of a 32-key chunk, the warp
// keeps an online softmax (running max and sum), and lanes accumulate the
// output across the head dimension with coalesced V reads.  One pass over K
// and V per row, asynchronous on the caller's stream.
#include "vk_internal.h"

namespace vk {

constexpr int kAttnWarps = 4;
constexpr int kAttnMaxD = 256;

__global__ void __launch_bounds__(kAttnWarps * 32) attention_f32_kernel(const float* __restrict__ Q,
                                                                        const float* __restrict__ K,
                                                                        const float* __restrict__ V,
                                                                        float* __restrict__ O, int H,
                                                                        int S, int D, float scale) {
    __shared__ float qs[kAttnWarps][kAttnMaxD];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * kAttnWarps + warp;
    const int h = blockIdx.y, b = blockIdx.z;
    if (row >= S) return;
    const int64_t bh = (static_cast<int64_t>(b) * H + h) * S * D;
    const float* q = Q + bh + static_cast<int64_t>(row) * D;
    for (int d = lane; d < D; d += 32) qs[warp][d] = q[d];
    __syncwarp();

    float m = -INFINITY, l = 0.f;
    float acc[kAttnMaxD / 32];
#pragma unroll
    for (int k = 0; k < kAttnMaxD / 32; ++k) acc[k] = 0.f;

    for (int j0 = 0; j0 <= row; j0 += 32) {
        const int j = j0 + lane;
        float s = -INFINITY;
        if (j <= row) {
            const float* kr = K + bh + static_cast<int64_t>(j) * D;
            float dot = 0.f;
            for (int d = 0; d < D; ++d) dot += qs[warp][d] * kr[d];
            s = dot * scale;
        }
        float cmax = s;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, o));
        const float mn = fmaxf(m, cmax);
        const float alpha = expf(m - mn);
        const float pj = (j <= row) ? expf(s - mn) : 0.f;
        float psum = pj;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
        l = l * alpha + psum;
        m = mn;
#pragma unroll
        for (int k = 0; k < kAttnMaxD / 32; ++k) acc[k] *= alpha;
        const int cnt = min(32, row + 1 - j0);
        for (int t = 0; t < cnt; ++t) {
            const float w = __shfl_sync(0xffffffffu, pj, t);
            const float* vr = V + bh + static_cast<int64_t>(j0 + t) * D;
#pragma unroll
            for (int k = 0; k < kAttnMaxD / 32; ++k) {
                const int d = lane + 32 * k;
                if (d < D) acc[k] += w * vr[d];
            }
        }
    }
    float* o = O + bh + static_cast<int64_t>(row) * D;
    const float inv = 1.f / l;
#pragma unroll
    for (int k = 0; k < kAttnMaxD / 32; ++k) {
        const int d = lane + 32 * k;
        if (d < D) o[d] = acc[k] * inv;
    }
}

}  // namespace vk

using namespace vk;

extern "C" vk_status vk_attention_f32(const float* Q, const float* K, const float* V, float* O,
                                      int32_t batch, int32_t heads, int32_t seq_len,
                                      int32_t head_dim, void* stream) {
    if (batch < 0 || heads < 0 || seq_len < 0 || head_dim <= 0)
        return fail(VK_INVALID_ARG, "bad attention shape");
    if (head_dim > kAttnMaxD) return fail(VK_UNSUPPORTED, "head_dim > 256");
    if (batch == 0 || heads == 0 || seq_len == 0) return VK_OK;
    if (!Q || !K || !V || !O) return fail(VK_INVALID_ARG, "NULL array");
    if (heads > 65535 || batch > 65535) return fail(VK_INVALID_ARG, "batch/heads must be <= 65535");
    dim3 grid((seq_len + kAttnWarps - 1) / kAttnWarps, heads, batch);
    const float scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    attention_f32_kernel<<<grid, kAttnWarps * 32, 0, as_stream(stream)>>>(Q, K, V, O, heads, seq_len,
                                                                          head_dim, scale);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? VK_OK : cuda_fail(e, "attention_f32_kernel launch");
}
