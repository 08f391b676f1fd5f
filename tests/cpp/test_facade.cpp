// C++ tests of the VULCAN-compatible facade (include/vulcan/kv_cache.h,
// include/cuda/memory.h, include/cuda/kernels.h) linked against
// libvulcan_kv.so.  They follow the reference's own tests
// (tests/test_memory.cpp:21-286 and the attention cases of
// tests/test_attention.cu:107-264) with a small assertion macro in place of
// GoogleTest.  Exit status 0 when every check passes.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <vector>

#include "cuda/kernels.h"
#include "cuda/memory.h"
#include "vulcan/kv_cache.h"

static int g_failures = 0;
static int g_checks = 0;
#define CHECK(cond)                                                                 \
    do {                                                                            \
        ++g_checks;                                                                 \
        if (!(cond)) {                                                              \
            ++g_failures;                                                           \
            std::fprintf(stderr, "FAILED %s:%d: %s\n", __FILE__, __LINE__, #cond);  \
        }                                                                           \
    } while (0)

using vulcan::cuda::GPUBuffer;
using vulcan::cuda::MemoryManager;

static std::vector<float> uniform(int n, float lo, float hi, int seed) {
    std::mt19937 rng(seed);
    std::uniform_real_distribution<float> dist(lo, hi);
    std::vector<float> v(n);
    for (auto& x : v) x = dist(rng);
    return v;
}

// double-precision causal attention over [B, H, S, D]
static std::vector<float> cpu_causal(const std::vector<float>& Q, const std::vector<float>& K,
                                     const std::vector<float>& V, int B, int H, int S, int D) {
    std::vector<float> O(Q.size());
    const double scale = 1.0 / std::sqrt(static_cast<double>(D));
    std::vector<double> s(S);
    for (int bh = 0; bh < B * H; ++bh) {
        const size_t off = static_cast<size_t>(bh) * S * D;
        for (int r = 0; r < S; ++r) {
            double mx = -1e300, sum = 0;
            for (int j = 0; j <= r; ++j) {
                double dot = 0;
                for (int d = 0; d < D; ++d) dot += static_cast<double>(Q[off + r * D + d]) * K[off + j * D + d];
                s[j] = dot * scale;
                mx = std::max(mx, s[j]);
            }
            for (int j = 0; j <= r; ++j) sum += (s[j] = std::exp(s[j] - mx));
            for (int d = 0; d < D; ++d) {
                double v = 0;
                for (int j = 0; j <= r; ++j) v += s[j] / sum * V[off + j * D + d];
                O[off + r * D + d] = static_cast<float>(v);
            }
        }
    }
    return O;
}

static void test_gpubuffer() {
    GPUBuffer a;
    CHECK(!a.is_valid() && a.size() == 0 && a.data() == nullptr);
    GPUBuffer b(1024 * sizeof(float));
    CHECK(b.is_valid() && b.size() == 1024 * sizeof(float) && b.data() != nullptr);
    GPUBuffer z(0);
    CHECK(!z.is_valid() && z.size() == 0);
    GPUBuffer orig(4096);
    void* p = orig.data();
    GPUBuffer moved(std::move(orig));
    CHECK(moved.data() == p && moved.size() == 4096 && !orig.is_valid() && orig.size() == 0);
    GPUBuffer b1(1024), b2(2048);
    void* p2 = b2.data();
    b1 = std::move(b2);
    CHECK(b1.data() == p2 && b1.size() == 2048 && !b2.is_valid());
    GPUBuffer r(1024);
    void* rp = r.data();
    void* rel = r.release();
    CHECK(rel == rp && !r.is_valid());
    cudaFree(rel);
    GPUBuffer t(256 * sizeof(float));
    std::vector<float> h(256, 3.14f), o(256, 0.f);
    cudaMemcpy(t.as<float>(), h.data(), 256 * sizeof(float), cudaMemcpyHostToDevice);
    cudaMemcpy(o.data(), t.as<float>(), 256 * sizeof(float), cudaMemcpyDeviceToHost);
    CHECK(o[0] == 3.14f && o[255] == 3.14f);
}

static void test_memory_manager() {
    {
        MemoryManager m(4096, 16);
        CHECK(m.blocks_in_use() == 0 && m.blocks_available() == 16 && m.total_allocated_bytes() == 0);
    }
    {
        MemoryManager m(4096, 8);
        int id = m.allocate_block();
        CHECK(id >= 0 && m.blocks_in_use() == 1 && m.blocks_available() == 7 && m.get_block_ptr(id) != nullptr);
        m.free_block(id);
        CHECK(m.blocks_in_use() == 0 && m.blocks_available() == 8);
    }
    {
        MemoryManager m(1024, 4);
        std::vector<int> ids;
        for (int i = 0; i < 4; ++i) ids.push_back(m.allocate_block());
        CHECK(ids[0] == 0 && ids[3] == 3 && m.blocks_in_use() == 4 && m.blocks_available() == 0);
        CHECK(m.allocate_block() == -1);
        m.free_block(ids[0]);
        CHECK(m.blocks_available() == 1 && m.allocate_block() >= 0);
    }
    {
        MemoryManager m(4096, 8);
        int a = m.allocate_block(), b = m.allocate_block();
        auto* pa = static_cast<uint8_t*>(m.get_block_ptr(a));
        auto* pb = static_cast<uint8_t*>(m.get_block_ptr(b));
        CHECK(pa != pb && pa && pb && std::abs(pb - pa) == 4096);
    }
    {
        MemoryManager m(1024, 4);
        int id = m.allocate_block();
        std::vector<uint8_t> data(1024), back(1024);
        for (int i = 0; i < 1024; ++i) data[i] = static_cast<uint8_t>(i % 256);
        cudaMemcpy(m.get_block_ptr(id), data.data(), 1024, cudaMemcpyHostToDevice);
        CHECK(m.swap_to_cpu(id) && m.blocks_in_use() == 0);
        CHECK(m.swap_to_gpu(id) && m.blocks_in_use() == 1);
        cudaMemcpy(back.data(), m.get_block_ptr(id), 1024, cudaMemcpyDeviceToHost);
        CHECK(std::memcmp(back.data(), data.data(), 1024) == 0);
        // the reference test's sequence: freeing the reused id drops the copy
        CHECK(m.swap_to_cpu(id));
        int t = m.allocate_block();
        CHECK(t == id);
        m.free_block(t);
        CHECK(!m.swap_to_gpu(id) && m.blocks_in_use() == 0);
    }
    {
        MemoryManager m(1024, 4);
        CHECK(m.get_block_ptr(-1) == nullptr && m.get_block_ptr(999) == nullptr);
        CHECK(!m.swap_to_cpu(-1) && !m.swap_to_gpu(999));
    }
}

static void test_kvcache() {
    {
        vulcan::KVCache c(4, 128, 64, 2);
        CHECK(c.current_length() == 0 && c.max_seq_len() == 128 && c.memory_usage() > 0);
    }
    {
        const int H = 2, S = 32, D = 64;
        vulcan::KVCache c(H, S, D, 1);
        std::vector<float> k(H * D), v(H * D);
        for (int i = 0; i < H * D; ++i) {
            k[i] = static_cast<float>(i + 1);
            v[i] = static_cast<float>(i + 100);
        }
        float *dk, *dv;
        cudaMalloc(&dk, k.size() * 4);
        cudaMalloc(&dv, v.size() * 4);
        cudaMemcpy(dk, k.data(), k.size() * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(dv, v.data(), v.size() * 4, cudaMemcpyHostToDevice);
        c.append(0, dk, dv, 0, 1);
        CHECK(c.current_length() == 1);
        const float *ko, *vo;
        c.get(0, &ko, &vo);
        CHECK(ko != nullptr && vo != nullptr);
        // read the appended rows back: page of token 0, every head, slot 0
        int32_t page = -1;
        cudaMemcpy(&page, c.block_table(), 4, cudaMemcpyDeviceToHost);
        for (int h = 0; h < H; ++h) {
            std::vector<__half> row(D), vrow(D);
            const size_t off = (static_cast<size_t>(page) * H + h) * 2 * 16 * D * 2;
            cudaMemcpy(row.data(), reinterpret_cast<const char*>(ko) + off, D * 2, cudaMemcpyDeviceToHost);
            cudaMemcpy(vrow.data(), reinterpret_cast<const char*>(vo) + off, D * 2, cudaMemcpyDeviceToHost);
            bool ok = true;
            for (int d = 0; d < D; ++d)
                ok = ok && __half2float(row[d]) == k[h * D + d] && __half2float(vrow[d]) == v[h * D + d];
            CHECK(ok);
        }
        c.append(5, dk, dv, 1, 1);   // bad layer: ignored
        c.append(0, dk, dv, 32, 1);  // overflow: ignored
        CHECK(c.current_length() == 1);
        cudaFree(dk);
        cudaFree(dv);
    }
    {
        vulcan::KVCache c(4, 64, 32, 1);
        c.set_length(42);
        CHECK(c.current_length() == 42);
        c.reset();
        CHECK(c.current_length() == 0);
    }
    {
        vulcan::KVCache a(4, 64, 32, 2);
        a.set_length(10);
        vulcan::KVCache b(std::move(a));
        CHECK(b.current_length() == 10 && b.max_seq_len() == 64 && a.current_length() == 0);
    }
    {
        vulcan::KVCache c(8, 2048, 128, 32);
        CHECK(c.memory_usage() == 2ull * 32 * 8 * 2048 * 128 * 2);
    }
}

static void test_kvcache_decode() {
    // 37 tokens, 2 KV heads, 8 query heads (G = 4): decode vs double-precision attention
    const int Hkv = 2, Hq = 8, D = 128, T = 37;
    vulcan::KVCache c(Hkv, 100, D, 2);
    auto k = uniform(T * Hkv * D, -1.f, 1.f, 11), v = uniform(T * Hkv * D, -1.f, 1.f, 12);
    auto q = uniform(Hq * D, -1.f, 1.f, 13);
    for (auto* x : {&k, &v, &q})
        for (auto& e : *x) e = __half2float(__float2half(e));  // fp16-representable inputs
    float *dk, *dv;
    cudaMalloc(&dk, k.size() * 4);
    cudaMalloc(&dv, v.size() * 4);
    cudaMemcpy(dk, k.data(), k.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dv, v.data(), v.size() * 4, cudaMemcpyHostToDevice);
    c.append(1, dk, dv, 0, T);
    std::vector<__half> qh(q.size()), oh(q.size());
    for (size_t i = 0; i < q.size(); ++i) qh[i] = __float2half(q[i]);
    void *dq, *dout;
    cudaMalloc(&dq, qh.size() * 2);
    cudaMalloc(&dout, oh.size() * 2);
    cudaMemcpy(dq, qh.data(), qh.size() * 2, cudaMemcpyHostToDevice);
    CHECK(c.decode(1, dq, dout, Hq));
    cudaMemcpy(oh.data(), dout, oh.size() * 2, cudaMemcpyDeviceToHost);
    double worst = 0;
    for (int h = 0; h < Hq; ++h) {
        const int kv = h / (Hq / Hkv);
        std::vector<float> Q(T * D, 0.f), K(T * D), V(T * D);
        for (int d = 0; d < D; ++d) Q[(T - 1) * D + d] = q[h * D + d];
        for (int t = 0; t < T; ++t)
            for (int d = 0; d < D; ++d) {
                K[t * D + d] = k[(t * Hkv + kv) * D + d];
                V[t * D + d] = v[(t * Hkv + kv) * D + d];
            }
        auto ref = cpu_causal(Q, K, V, 1, 1, T, D);
        for (int d = 0; d < D; ++d) {
            const double r = ref[(T - 1) * D + d], g = __half2float(oh[h * D + d]);
            worst = std::max(worst, std::abs(g - r) - (2e-3 + 1e-2 * std::abs(r)));
        }
    }
    CHECK(worst <= 0);
    cudaFree(dk);
    cudaFree(dv);
    cudaFree(dq);
    cudaFree(dout);
}

static void test_launch_attention() {
    struct Case { int B, H, S, D; float lo, hi; int seed; float tol; };
    const Case cases[] = {{1, 1, 4, 8, -1.f, 1.f, 2000, 1e-4f}, {1, 4, 8, 16, -.5f, .5f, 2010, 1e-3f},
                          {1, 2, 32, 32, -.3f, .3f, 2030, 1e-3f}, {2, 4, 8, 16, -.5f, .5f, 2040, 1e-3f},
                          {2, 3, 300, 128, -.5f, .5f, 2060, 1e-3f}};
    for (const auto& cs : cases) {
        const int n = cs.B * cs.H * cs.S * cs.D;
        auto Q = uniform(n, cs.lo, cs.hi, cs.seed), K = uniform(n, cs.lo, cs.hi, cs.seed + 1),
             V = uniform(n, cs.lo, cs.hi, cs.seed + 2);
        auto ref = cpu_causal(Q, K, V, cs.B, cs.H, cs.S, cs.D);
        float *dq, *dk, *dv, *dout;
        cudaMalloc(&dq, n * 4);
        cudaMalloc(&dk, n * 4);
        cudaMalloc(&dv, n * 4);
        cudaMalloc(&dout, n * 4);
        cudaMemcpy(dq, Q.data(), n * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(dk, K.data(), n * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(dv, V.data(), n * 4, cudaMemcpyHostToDevice);
        vulcan::cuda::launch_attention(dq, dk, dv, dout, cs.B, cs.H, cs.S, cs.D);
        std::vector<float> O(n);
        cudaMemcpy(O.data(), dout, n * 4, cudaMemcpyDeviceToHost);
        float err = 0;
        for (int i = 0; i < n; ++i) err = std::max(err, std::abs(O[i] - ref[i]));
        CHECK(err < cs.tol);
        if (cs.S >= 4) {  // CausalMask_FirstRow: row 0 equals V[0]
            bool ok = true;
            for (int d = 0; d < cs.D; ++d) ok = ok && std::abs(O[d] - V[d]) < 1e-5f;
            CHECK(ok);
        }
        cudaFree(dq);
        cudaFree(dk);
        cudaFree(dv);
        cudaFree(dout);
    }
}

int main() {
    test_gpubuffer();
    test_memory_manager();
    test_kvcache();
    test_kvcache_decode();
    test_launch_attention();
    std::printf("%d checks, %d failures\n", g_checks, g_failures);
    return g_failures == 0 ? 0 : 1;
}
