#pragma once

// The attention entry of VULCAN's kernel library (include/cuda/kernels.h:
// 99-101) over libvulcan_kv.so.  Same signature and contract: Q, K, V, output
// are [batch, heads, seq_len, head_dim] fp32 device arrays, causal, scale
// 1/sqrt(head_dim); the call returns after the kernel has finished, as the
// reference's does.  A CUDA error is reported on stderr and leaves output
// unwritten instead of exiting the process.

namespace vulcan {
namespace cuda {

void launch_attention(const float* Q, const float* K, const float* V, float* output, int batch, int heads,
                      int seq_len, int head_dim);

}  // namespace cuda
}  // namespace vulcan
