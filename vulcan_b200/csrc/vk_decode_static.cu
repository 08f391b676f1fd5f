// vk_decode_static: paged decode whose split-K scratch lives in a fixed device
// array of this library, for callers that cannot allocate device memory (a
// host engine that owns all device memory and passes operators only their
// inputs and outputs, a serving loop that must not call cudaMalloc, an FFI host
// without a CUDA allocator).  No counterpart in the reference.
//
// The array is a file-scope __device__ object.  Host code must not pass its
// name to a kernel: on the host that name is only a stand-in, not a device
// address.  The device address is looked up here with cudaGetSymbolAddress,
// once per device with that device current, and handed to vk_decode as its
// workspace.
#include <cstdio>
#include <mutex>

#include "vk_internal.h"

namespace {

static __device__ __align__(256) unsigned char g_decode_scratch[VK_DECODE_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on `device` (which must be current).
vk_status scratch_address(int device, void** out) {
    if (device < 0 || device >= kMaxDevices)
        return vk::fail(VK_INVALID_ARG, "vk_decode_static: device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (e != cudaSuccess) return vk::cuda_fail(e, "vk_decode_static: cudaGetSymbolAddress");
        g_scratch_addr[device] = p;
    }
    *out = g_scratch_addr[device];
    return VK_OK;
}

}  // namespace

extern "C" vk_status vk_decode_static(vk_pool* pool, int32_t layer, const void* q, void* out,
                                      const int32_t* block_tables, int32_t bt_stride,
                                      const int32_t* seq_lens, int32_t batch, int32_t num_q_heads,
                                      int32_t max_seq_len, float scale, void* stream) {
    if (!pool) return vk::fail(VK_INVALID_ARG, "pool is NULL");
    const size_t need = vk_decode_workspace_size(pool, batch, num_q_heads, max_seq_len);
    if (need > VK_DECODE_STATIC_SCRATCH_BYTES) {
        char msg[200];
        std::snprintf(msg, sizeof msg,
                      "vk_decode_static: this shape needs %zu bytes of split-K scratch, more than the "
                      "fixed %u-byte array; use vk_decode with a caller workspace",
                      need, VK_DECODE_STATIC_SCRATCH_BYTES);
        return vk::fail(VK_INVALID_ARG, msg);
    }
    void* scratch = nullptr;
    if (need > 0) {
        vk::DeviceGuard g(pool->device);
        vk_status s = scratch_address(pool->device, &scratch);
        if (s != VK_OK) return s;
    }
    return vk_decode(pool, layer, q, out, block_tables, bt_stride, seq_lens, batch, num_q_heads,
                     max_seq_len, scale, scratch, need > 0 ? VK_DECODE_STATIC_SCRATCH_BYTES : 0, stream);
}
