// Internal definitions shared by the translation units of libvulcan_kv.so.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "vk_paged_kv.h"

namespace vk {

constexpr int kPageTokens = 16;     // tokens per page for the attention kernels
constexpr int kNumSmsDefault = 148;

struct Allocator {
    // free_bits[w] bit i set <=> page 64*w+i is free.  `hint` is a lower bound
    // on the first word that may hold a free bit, so lowest-id allocation is
    // amortised O(1) and every id order matches a first-fit scan.
    std::vector<uint64_t> free_bits;
    size_t hint = 0;
    int32_t num_pages = 0;
    int32_t used = 0;

    void reset(int32_t n);
    int32_t take_lowest();           // -1 when full
    bool is_used(int32_t id) const;
    void set_used(int32_t id);
    void set_free(int32_t id);
};

}  // namespace vk

struct vk_pool {
    vk_pool_cfg cfg{};
    bool kv = false;           // KV geometry present (attention entry points allowed)
    bool owns_mem = false;
    int device = 0;
    char* base = nullptr;
    uint64_t page_bytes = 0;   // bytes of one page over all its segments
    uint64_t seg_bytes = 0;    // bytes of one page in one layer (the whole page for byte pools)
    uint64_t seg_stride = 0;   // distance between a page's consecutive layer segments
    int32_t nseg = 1;          // segments per page: num_layers (KV pools) or 1 (byte pools)
    uint64_t head_bytes = 0;   // K block + V block of one (page, layer, head)
    int32_t num_pages = 0;
    uint32_t* d_err = nullptr;  // device error word (VK_ERR_* bits)
    alignas(64) CUtensorMap tmap;    // 2-D view: rows of head_dim fp16, boxes of 64 x 32 rows (K+V)
    alignas(64) CUtensorMap tmap16;  // same view, boxes of 64 x 16 rows (K or V of one page)
    bool tmap_ok = false;
    int32_t kv_format = VK_KV_FP16;  // page format of a KV pool (VK_KV_FP16 / VK_KV_FP8)
    int32_t prefill_path = 0;        // 0 auto, 1 mma.sync kernel, 2 tcgen05 kernel
    int32_t split_override = 0;
    int32_t plan_workers = 0;        // cap on planned-decode workers (0 = resident warps)
    float rope_theta = 0.f;          // fused RoPE base (0 = off)
    float* rope_freq = nullptr;      // device [head_dim/2] frequencies when RoPE is on
    int32_t num_sms = vk::kNumSmsDefault;
    vk::Allocator alloc;
};

namespace vk {

// Error reporting (thread-local last error string).
vk_status fail(vk_status s, const std::string& msg);
vk_status cuda_fail(cudaError_t e, const char* what);
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Device guard: makes the pool's device current for the scope.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) cudaSetDevice(dev);
        else prev = -1;
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

// cuTensorMapEncodeTiled from the driver (NULL when unavailable).
PFN_cuTensorMapEncodeTiled_v12000 tmap_encode_fn();

// Kernel launchers (defined in the .cu files).
vk_status launch_append(vk_pool* pool, int layer, const void* k, const void* v, bool f32,
                        const int32_t* bt, int bt_stride, const int32_t* pos, int B, int T,
                        cudaStream_t st);
vk_status launch_append_fp8(vk_pool* pool, int layer, const void* k, const void* v, bool f32,
                            const int32_t* bt, int bt_stride, const int32_t* pos, int B, int T,
                            cudaStream_t st);
vk_status launch_copy_pages(vk_pool* pool, const int32_t* src, const int32_t* dst, int n,
                            cudaStream_t st);
vk_status launch_remap(int32_t* bt, int64_t entries, const int32_t* map, int map_len,
                       cudaStream_t st);
int decode_pages_per_split(const vk_pool* pool, int B, int max_seq_len);

// Device-side description of a bound output gather (vk_gather), passed by value
// in kernel parameters.  Allocation of every rank: [slots][world][slice] fp16
// receive slices, then flags [slots][world] u32 (column r written only by rank
// r, with step epochs), then [slots] u32 epochs already signalled by this rank
// (local), then an error word (waits outside a pool).
constexpr int kMaxGatherRanks = 8;
struct GatherView {
    char* base[kMaxGatherRanks];  // receive allocations of all ranks, own included
    uint64_t slice_bytes = 0, slot_bytes = 0, flags_off = 0, sig_off = 0, err_off = 0;
    int rank = 0, world = 0, slots = 0;
};
// Fills `v` if every peer is imported; false otherwise.
bool gather_view(const vk_gather* g, GatherView* v);
int gather_device(const vk_gather* g);
uint32_t gather_next_epoch(vk_gather* g);
vk_status prefill_tc(vk_pool* pool, int layer, const void* q, void* out, const int32_t* bt, int bt_stride,
                     const int32_t* positions, int B, int T, int Hq, float scale, cudaStream_t st);

}  // namespace vk
