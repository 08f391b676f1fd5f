// Exposes the reference's own golden helpers from its attention test file
// (tests/test_attention.cu: random_floats :19-26, cpu_attention :53-103) with
// C linkage, for pinning the oracle and generating golden fixtures.
// Test infrastructure only.  VK_REF_TEST_ATTENTION is set by oracle/Makefile.
#include VK_REF_TEST_ATTENTION

#include <cstring>

extern "C" void ref_random_floats(int n, float lo, float hi, int seed, float* out) {
    std::vector<float> v = random_floats(n, lo, hi, seed);
    std::memcpy(out, v.data(), sizeof(float) * static_cast<size_t>(n));
}

extern "C" void ref_cpu_attention(const float* Q, const float* K, const float* V, float* O,
                                  int batch, int heads, int seq_len, int head_dim) {
    const size_t n = static_cast<size_t>(batch) * heads * seq_len * head_dim;
    std::vector<float> q(Q, Q + n), k(K, K + n), v(V, V + n);
    std::vector<float> o = cpu_attention(q, k, v, batch, heads, seq_len, head_dim);
    std::memcpy(O, o.data(), sizeof(float) * n);
}
