#pragma once

// vulcan::KVCache over the B200 paged KV-cache library (libvulcan_kv.so).
//
// Same class name, constructor, methods and move-only semantics as VULCAN's
// include/vulcan/kv_cache.h:34-92, so code using the class compiles against it.
// Storage differs: the cache is a paged fp16 pool (16-token pages, taken on
// demand by append) instead of contiguous fp32 [heads, max_seq, head_dim]
// buffers.  append() still takes fp32 rows and rounds them to fp16.
//
// What changes for the engine: get() no longer hands out contiguous fp32
// [num_kv_heads, max_seq_len, head_dim] arrays, so the reference's
// self_attention loop that strides them that way and calls launch_attention
// per head (src/transformer.cpp:142, 157-189) must not be kept: it would read
// paged fp16 bytes as fp32.  Replace that loop by decode() below (one
// sequence) or by vulcan::PagedAttention (include/vulcan/paged_attention.h,
// many sequences, one launch per layer).

#include <cstddef>
#include <cstdint>
#include <vector>

struct vk_pool;

namespace vulcan {

class KVCache {
public:
    /// @param num_kv_heads  KV heads (may differ from query heads in GQA)
    /// @param max_seq_len   longest sequence the cache will hold
    /// @param head_dim      dimension per head (multiple of 8)
    /// @param num_layers    transformer layers
    KVCache(int num_kv_heads, int max_seq_len, int head_dim, int num_layers);
    ~KVCache();

    KVCache(KVCache&& other) noexcept;
    KVCache& operator=(KVCache&& other) noexcept;
    KVCache(const KVCache&) = delete;
    KVCache& operator=(const KVCache&) = delete;

    /// Appends num_tokens rows of K and V ([num_tokens, num_kv_heads*head_dim]
    /// fp32, device memory) at positions start_pos.. of layer `layer`.  As in
    /// the reference, a bad layer is ignored and an overflow past max_seq_len
    /// prints a message and writes nothing.  Synchronous, like the reference.
    void append(int layer, const float* k_new, const float* v_new, int start_pos, int num_tokens);

    /// Device addresses of layer `layer`'s K and V blocks of physical page 0.
    /// The pool is paged fp16: element (page, head, slot, d) of the layer is at
    /// k + (page*num_kv_heads + head)*2*16*head_dim*2 bytes + (slot*head_dim + d)*2
    /// (V: the same offsets from v).  nullptr for a bad layer.  Unlike the
    /// reference, these are not fp32 [num_kv_heads, max_seq_len, head_dim]
    /// arrays: attention over the cache goes through decode() or the C ABI.
    void get(int layer, const float** k_out, const float** v_out) const;

    int current_length() const;
    void set_length(int len);
    void reset();
    int max_seq_len() const;

    /// Bytes of fp16 page storage for max_seq_len tokens:
    /// 2 * layers * kv_heads * ceil(max_seq_len/16)*16 * head_dim * 2.
    size_t memory_usage() const;

    // ---- paged extensions ---------------------------------------------------

    /// Attention of one query token per head (q: [num_q_heads, head_dim] fp16,
    /// device) over the current_length() cached tokens of `layer`; writes
    /// out: [num_q_heads, head_dim] fp16 (device).  Synchronous.
    /// Returns false on a bad argument.
    bool decode(int layer, const void* q_f16, void* out_f16, int num_q_heads);

    /// Device block table of this sequence (int32, one entry per page) and
    /// the underlying pool handle, for the C ABI.
    const int32_t* block_table() const;
    vk_pool* pool() const;

private:
    void release();
    bool ensure_pages(int tokens);

    int num_kv_heads_ = 0;
    int max_seq_len_ = 0;
    int head_dim_ = 0;
    int num_layers_ = 0;
    int current_len_ = 0;
    vk_pool* pool_ = nullptr;
    int32_t* d_block_table_ = nullptr;   // device [max_pages]
    int32_t* d_scalars_ = nullptr;       // device: positions / lengths scratch
    void* d_workspace_ = nullptr;
    size_t workspace_bytes_ = 0;
    std::vector<int32_t> pages_;         // host copy of the block table
};

}  // namespace vulcan
