#pragma once

// vulcan::PagedAttention — the attention step of an engine over the B200 paged
// KV cache, for many sequences at once.
//
// In the reference, TransformerBlock::self_attention (src/transformer.cpp:86-197)
// holds one sequence: it appends the step's K/V to a contiguous fp32 cache
// (src/kv_cache.cpp:84-128), fetches the cache with KVCache::get and launches
// launch_attention once per query head (src/transformer.cpp:157-189), and
// Engine::forward / forward_one (src/engine.cpp:70-127) drive it through the
// layers for a prompt or one new token.  This class is the part of that path
// between the projections (plus RoPE) and the output projection, batched:
//
//   PagedAttention attn(cfg);                      // Engine::load_model
//   int s = attn.add_sequence();                   // a new request
//   attn.begin_step({s, ...}, T);                  // prompt chunk (T > 1) or decode (T = 1)
//   for (layer ...) attn.attend(layer, q, k, v, out);   // self_attention's cache + attention
//   attn.end_step();                               // lengths advance by T
//
// A step with T = 1 is one planned-decode launch per layer (the new token's
// K/V appended inside the launch); T > 1 appends the chunk and runs the
// chunked prefill.  With cfg.rope_theta > 0, q and k are passed before RoPE and
// rotated on load (the reference rotates them first, src/transformer.cpp:114-128).
// The pages of all sequences come from one pool; a sequence takes pages as it
// grows and returns them when released.
//
// Calls are host-side and not thread-safe (one engine thread, like the
// reference).  begin_step may allocate device memory (the step's plan
// workspace, grown to the largest step seen); attend only launches.  Errors
// print the library's message and return false; nothing exits the process.

#include <cstddef>
#include <cstdint>
#include <vector>

struct vk_pool;
struct vk_decode_plan;

namespace vulcan {

struct PagedAttentionConfig {
    int num_heads = 0;        // query heads (ModelConfig::num_heads)
    int num_kv_heads = 0;     // KV heads (ModelConfig::num_kv_heads)
    int head_dim = 0;         // hidden_dim / num_heads: 64, 128 or 256 (128 for FP8 pages)
    int num_layers = 0;       // ModelConfig::num_layers
    int max_seq_len = 0;      // longest sequence, prompt included (block-table width)
    int max_sequences = 0;    // sequences held at once
    int num_pages = 0;        // 16-token pages shared by all sequences
    int device = -1;          // CUDA device; -1: the current one
    bool fp8_pages = false;   // e4m3 pages with one fp32 scale per row (half the bytes)
    float rope_theta = 0.f;   // > 0: RoPE fused into append, decode and prefill
};

class PagedAttention {
public:
    explicit PagedAttention(const PagedAttentionConfig& cfg);
    ~PagedAttention();

    PagedAttention(PagedAttention&& other) noexcept;
    PagedAttention& operator=(PagedAttention&& other) noexcept;
    PagedAttention(const PagedAttention&) = delete;
    PagedAttention& operator=(const PagedAttention&) = delete;

    /// True when construction succeeded.
    bool ok() const;

    /// A new empty sequence: its id (>= 0), or -1 when max_sequences are held.
    int add_sequence();
    /// Frees the sequence's pages; false for an unknown id or during a step
    /// that includes it.
    bool release_sequence(int id);
    /// Tokens cached for the sequence, -1 for an unknown id.
    int length(int id) const;
    /// Physical pages not held by any sequence.
    int pages_available() const;

    /// Starts a step in which each sequence of `ids` (distinct, in this order:
    /// row b of the step's tensors is ids[b]) gains `tokens` tokens at its end.
    /// Takes the pages the new tokens need (all or nothing: false, and nothing
    /// changes, when the pool or max_seq_len cannot hold them), writes the
    /// step's block tables on `stream` and, for tokens == 1, builds and uploads
    /// the decode plan.  `stream` is a cudaStream_t (nullptr: legacy default).
    bool begin_step(const std::vector<int>& ids, int tokens, void* stream = nullptr);

    /// One layer of the step, on the step's stream, asynchronous.  Device fp16
    /// arrays: q [B, T, num_heads, head_dim], k_new / v_new
    /// [B, T, num_kv_heads, head_dim] (the reference's token-major K_new/V_new
    /// rows per sequence), out [B, T, num_heads, head_dim]; B = ids.size(),
    /// T = tokens.  Row t of sequence b sits at position length(ids[b]) + t and
    /// attends keys 0 .. that position.
    bool attend(int layer, const void* q, const void* k_new, const void* v_new, void* out);

    /// Ends the step: every sequence of the step has grown by `tokens`.
    bool end_step();

    /// The pool and the current step's device block tables [B, width] (int32).
    vk_pool* pool() const;
    const int32_t* block_tables() const;
    int block_table_width() const;
    /// Host page ids of a sequence (empty for an unknown id).
    std::vector<int32_t> pages(int id) const;

private:
    void release();

    PagedAttentionConfig cfg_{};
    int width_ = 0;                       // block-table entries per sequence
    vk_pool* pool_ = nullptr;
    int32_t* d_tables_ = nullptr;         // device [max_sequences, width]
    int32_t* d_positions_ = nullptr;      // device [max_sequences]
    void* d_ws_ = nullptr;                // decode-plan workspace
    size_t ws_bytes_ = 0;
    vk_decode_plan* plan_ = nullptr;
    std::vector<std::vector<int32_t>> seq_pages_;  // per sequence id
    std::vector<int> seq_len_;            // -1: id free
    std::vector<int> step_ids_;
    int step_tokens_ = 0;
    bool in_step_ = false;
    void* stream_ = nullptr;
};

}  // namespace vulcan
