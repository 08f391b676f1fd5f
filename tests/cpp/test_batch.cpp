// Engine-shaped driver of vulcan::PagedAttention (include/vulcan/paged_attention.h)
// linked against libvulcan_kv.so.  It plays the role of the reference's
// TransformerBlock::self_attention (src/transformer.cpp:86-197) under
// Engine::forward / forward_one (src/engine.cpp:70-127) for several sequences
// at once: prompt chunks (prefill steps) and one-token decode steps through
// every layer, a sequence released mid-run and a new one admitted into its
// pages.  The projections are stood in for by seeded N(0, 0.5^2) fp16 rows.
//
//   test_batch <dump file> <fp16|fp8> <rope theta (0 = off)>
//
// Every step's inputs, block tables, positions and outputs are written to the
// dump file, which tests/test_gpu_facade.py replays through the CPU oracle.
// Exit status 0 when every call succeeded.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "vk_paged_kv.h"
#include "vulcan/paged_attention.h"

namespace {

// Dump records: u32 name length, name, u32 dtype (0 f16, 1 i32, 2 u8), u32 ndim,
// i64 dims, then the raw bytes.
struct Dump {
    FILE* f = nullptr;
    void put(const std::string& name, int dtype, const std::vector<int64_t>& dims, const void* data, size_t bytes) {
        const uint32_t n = static_cast<uint32_t>(name.size()), dt = dtype, nd = static_cast<uint32_t>(dims.size());
        std::fwrite(&n, 4, 1, f);
        std::fwrite(name.data(), 1, n, f);
        std::fwrite(&dt, 4, 1, f);
        std::fwrite(&nd, 4, 1, f);
        std::fwrite(dims.data(), 8, dims.size(), f);
        std::fwrite(data, 1, bytes, f);
    }
};

int g_errors = 0;
#define REQUIRE(cond)                                                          \
    do {                                                                       \
        if (!(cond)) {                                                         \
            ++g_errors;                                                        \
            std::fprintf(stderr, "FAILED %s:%d: %s\n", __FILE__, __LINE__, #cond); \
        }                                                                      \
    } while (0)

std::vector<__half> normal_rows(std::mt19937_64& rng, size_t n) {
    std::normal_distribution<float> dist(0.f, 0.5f);
    std::vector<__half> v(n);
    for (auto& x : v) x = __float2half(dist(rng));
    return v;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc != 4) {
        std::fprintf(stderr, "usage: test_batch <dump> <fp16|fp8> <rope theta>\n");
        return 2;
    }
    const bool fp8 = std::strcmp(argv[2], "fp8") == 0;
    const float theta = static_cast<float>(std::atof(argv[3]));
    vulcan::PagedAttentionConfig cfg;
    cfg.num_heads = 16;
    cfg.num_kv_heads = 2;
    cfg.head_dim = 128;
    cfg.num_layers = 3;
    cfg.max_seq_len = 1024;
    cfg.max_sequences = 6;
    cfg.num_pages = 160;
    cfg.fp8_pages = fp8;
    cfg.rope_theta = theta;
    const int H = cfg.num_heads, Hkv = cfg.num_kv_heads, D = cfg.head_dim, L = cfg.num_layers;

    Dump dump;
    dump.f = std::fopen(argv[1], "wb");
    if (!dump.f) return 2;
    vulcan::PagedAttention attn(cfg);
    REQUIRE(attn.ok());
    if (!attn.ok()) return 1;
    const int64_t geom[] = {L, Hkv, D, cfg.num_pages, attn.block_table_width(), fp8 ? 1 : 0};
    dump.put("geom", 1, {6}, std::vector<int32_t>(geom, geom + 6).data(), 6 * 4);
    const float th[] = {theta};
    dump.put("theta", 1, {1}, th, 4);  // bits of the fp32 theta

    std::mt19937_64 rng(20240917);
    std::vector<int> seqs;
    for (int i = 0; i < 4; ++i) seqs.push_back(attn.add_sequence());
    REQUIRE(seqs[3] == 3);

    // the engine's schedule: prompts, decodes, a release and a new admission
    struct Step { std::vector<int> ids; int tokens; };
    std::vector<Step> plan = {
        {{0, 1, 2, 3}, 37},           // prompt chunk of every sequence
        {{0, 1, 2, 3}, 1},            // decode
        {{0, 1, 2, 3}, 1},
        {{2, 0}, 100},                // a second chunk for two of them (other order)
        {{0, 1, 2, 3}, 1},
        {{-1}, 20},                   // sequence 1 released, sequence 4 admitted: its prompt
        {{0, 2, 3, 4}, 1},
        {{4, 3, 2, 0}, 1},
    };
    void* d_q = nullptr;
    void* d_k = nullptr;
    void* d_v = nullptr;
    void* d_o = nullptr;
    const size_t max_rows = 4 * 100;
    REQUIRE(cudaMalloc(&d_q, max_rows * H * D * 2) == cudaSuccess);
    REQUIRE(cudaMalloc(&d_k, max_rows * Hkv * D * 2) == cudaSuccess);
    REQUIRE(cudaMalloc(&d_v, max_rows * Hkv * D * 2) == cudaSuccess);
    REQUIRE(cudaMalloc(&d_o, max_rows * H * D * 2) == cudaSuccess);
    int step_no = 0;
    for (Step st : plan) {
        if (st.ids.size() == 1 && st.ids[0] == -1) {
            REQUIRE(attn.release_sequence(1));
            REQUIRE(attn.length(1) == -1);
            const int s4 = attn.add_sequence();
            REQUIRE(s4 == 1);  // the freed id is reused
            st.ids = {s4};
            // later steps name the new sequence 4 in the schedule: map it
            for (auto& later : plan)
                for (auto& id : later.ids)
                    if (id == 4) id = s4;
        }
        const int B = static_cast<int>(st.ids.size()), T = st.tokens;
        std::vector<int32_t> pos(B);
        for (int b = 0; b < B; ++b) pos[b] = attn.length(st.ids[b]);
        REQUIRE(attn.begin_step(st.ids, T));
        std::vector<int32_t> table(static_cast<size_t>(B) * attn.block_table_width());
        REQUIRE(cudaMemcpy(table.data(), attn.block_tables(), table.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess);
        const std::string pre = "s" + std::to_string(step_no) + ".";
        dump.put(pre + "ids", 1, {B}, std::vector<int32_t>(st.ids.begin(), st.ids.end()).data(), B * 4);
        dump.put(pre + "pos", 1, {B}, pos.data(), B * 4);
        dump.put(pre + "bt", 1, {B, attn.block_table_width()}, table.data(), table.size() * 4);
        for (int l = 0; l < L; ++l) {
            const size_t nq = static_cast<size_t>(B) * T * H * D, nk = static_cast<size_t>(B) * T * Hkv * D;
            auto q = normal_rows(rng, nq), k = normal_rows(rng, nk), v = normal_rows(rng, nk);
            REQUIRE(cudaMemcpy(d_q, q.data(), nq * 2, cudaMemcpyHostToDevice) == cudaSuccess);
            REQUIRE(cudaMemcpy(d_k, k.data(), nk * 2, cudaMemcpyHostToDevice) == cudaSuccess);
            REQUIRE(cudaMemcpy(d_v, v.data(), nk * 2, cudaMemcpyHostToDevice) == cudaSuccess);
            REQUIRE(attn.attend(l, d_q, d_k, d_v, d_o));
            std::vector<__half> o(nq);
            REQUIRE(cudaMemcpy(o.data(), d_o, nq * 2, cudaMemcpyDeviceToHost) == cudaSuccess);
            const std::string lp = pre + "l" + std::to_string(l) + ".";
            dump.put(lp + "q", 0, {B, T, H, D}, q.data(), nq * 2);
            dump.put(lp + "k", 0, {B, T, Hkv, D}, k.data(), nk * 2);
            dump.put(lp + "v", 0, {B, T, Hkv, D}, v.data(), nk * 2);
            dump.put(lp + "out", 0, {B, T, H, D}, o.data(), nq * 2);
        }
        REQUIRE(attn.end_step());
        for (int b = 0; b < B; ++b) REQUIRE(attn.length(st.ids[b]) == pos[b] + T);
        ++step_no;
    }
    const int32_t nsteps[] = {step_no};
    dump.put("steps", 1, {1}, nsteps, 4);
    // argument checks: nothing changes on a refused step
    REQUIRE(!attn.begin_step({0, 0}, 1));                 // repeated id
    REQUIRE(!attn.begin_step({5}, 1));                    // never added
    REQUIRE(!attn.begin_step({0}, cfg.max_seq_len));      // beyond max_seq_len
    REQUIRE(!attn.attend(0, d_q, d_k, d_v, d_o));          // outside a step
    const int avail = attn.pages_available();
    REQUIRE(!attn.begin_step({0, 2, 3}, 810));            // 153 more pages than the 137 free
    REQUIRE(attn.pages_available() == avail);
    uint32_t bits = 0;
    REQUIRE(vk_pool_check(attn.pool(), &bits) == VK_OK && bits == 0);
    // the final pool image (fp16 values or FP8 block bytes) for the byte-exact check
    const size_t pool_bytes = static_cast<size_t>(vk_pool_page_bytes(attn.pool())) * cfg.num_pages;
    std::vector<uint8_t> img(pool_bytes);
    REQUIRE(cudaMemcpy(img.data(), vk_pool_base(attn.pool()), pool_bytes, cudaMemcpyDeviceToHost) == cudaSuccess);
    dump.put("pool", 2, {static_cast<int64_t>(pool_bytes)}, img.data(), pool_bytes);
    std::fclose(dump.f);
    cudaFree(d_q);
    cudaFree(d_k);
    cudaFree(d_v);
    cudaFree(d_o);
    std::printf("%d steps, %d errors\n", step_no, g_errors);
    return g_errors == 0 ? 0 : 1;
}
