// Exposes the reference's golden RoPE helper from its kernel test file
// (tests/test_kernels.cu: random_floats :30-37, cpu_rope :697-716) with C
// linkage, for pinning the oracle's RoPE and generating golden fixtures.
// Test infrastructure only.  VK_REF_TEST_KERNELS is set by oracle/Makefile.
#include VK_REF_TEST_KERNELS

#include <cstring>

extern "C" void ref_kernels_random_floats(int n, float lo, float hi, int seed, float* out) {
    std::vector<float> v = random_floats(n, lo, hi, seed);
    std::memcpy(out, v.data(), sizeof(float) * static_cast<size_t>(n));
}

extern "C" void ref_cpu_rope(const float* in, int head_dim, int pos, float theta_base, float* out) {
    std::vector<float> x(in, in + head_dim);
    std::vector<float> y = cpu_rope(x, pos, head_dim, theta_base);
    std::memcpy(out, y.data(), sizeof(float) * static_cast<size_t>(head_dim));
}
