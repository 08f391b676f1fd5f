// Receive buffers and flags of the fused head-shard output gather (C ABI).
// The peer stores, the flag signals and the waits are issued by the planned
// decode (vk_decode_planned.cu).
//
// Each rank allocates one device region with cudaMalloc and shares it with the
// other processes of the node through CUDA IPC handles; peers map it with
// cudaIpcOpenMemHandle and write into it with ordinary stores over NVLink.
#include <cstring>

#include "vk_gather.cuh"
#include "vk_internal.h"

struct vk_gather {
    int device = 0, rank = 0, world = 0, slots = 0;
    uint64_t slice_bytes = 0, slot_bytes = 0, flags_off = 0, sig_off = 0, err_off = 0, total = 0;
    uint32_t epoch = 0;  // steps uploaded with this gather bound (host counter)
    char* own = nullptr;
    char* peer[vk::kMaxGatherRanks] = {};
    bool imported[vk::kMaxGatherRanks] = {};
    bool local[vk::kMaxGatherRanks] = {};  // peer is a gather of this process (not an IPC mapping)
};

namespace vk {

static uint64_t round256(uint64_t x) { return (x + 255) & ~uint64_t(255); }

bool gather_view(const vk_gather* g, GatherView* v) {
    if (!g) return false;
    for (int r = 0; r < g->world; ++r)
        if (r != g->rank && !g->imported[r]) return false;
    for (int r = 0; r < kMaxGatherRanks; ++r) v->base[r] = r < g->world ? (r == g->rank ? g->own : g->peer[r]) : nullptr;
    v->slice_bytes = g->slice_bytes;
    v->slot_bytes = g->slot_bytes;
    v->flags_off = g->flags_off;
    v->sig_off = g->sig_off;
    v->err_off = g->err_off;
    v->rank = g->rank;
    v->world = g->world;
    v->slots = g->slots;
    return true;
}

int gather_device(const vk_gather* g) { return g ? g->device : -1; }

uint32_t gather_next_epoch(vk_gather* g) { return ++g->epoch; }

}  // namespace vk

using namespace vk;

extern "C" {

vk_status vk_gather_create(int32_t device, int32_t rank, int32_t world, uint64_t slice_bytes, int32_t slots,
                           vk_gather** out_gather) {
    if (!out_gather) return fail(VK_INVALID_ARG, "out_gather is NULL");
    *out_gather = nullptr;
    if (world < 1 || world > kMaxGatherRanks) return fail(VK_UNSUPPORTED, "gather supports 1..8 ranks");
    if (rank < 0 || rank >= world) return fail(VK_INVALID_ARG, "rank outside [0, world)");
    if (slice_bytes == 0 || (slice_bytes & 15) || slots < 1)
        return fail(VK_INVALID_ARG, "slice_bytes must be a positive multiple of 16 and slots >= 1");
    auto* g = new vk_gather();
    g->device = device;
    g->rank = rank;
    g->world = world;
    g->slots = slots;
    g->slice_bytes = slice_bytes;
    g->slot_bytes = round256(slice_bytes * static_cast<uint64_t>(world));
    g->flags_off = g->slot_bytes * static_cast<uint64_t>(slots);
    g->sig_off = g->flags_off + round256(static_cast<uint64_t>(slots) * world * sizeof(uint32_t));
    g->err_off = g->sig_off + round256(static_cast<uint64_t>(slots) * sizeof(uint32_t));
    g->total = g->err_off + 256;
    DeviceGuard dg(device);
    cudaError_t e = cudaMalloc(&g->own, g->total);
    if (e != cudaSuccess) {
        delete g;
        return cuda_fail(e, "cudaMalloc(gather buffers)");
    }
    e = cudaMemset(g->own, 0, g->total);
    if (e != cudaSuccess) {
        cudaFree(g->own);
        delete g;
        return cuda_fail(e, "cudaMemset(gather buffers)");
    }
    *out_gather = g;
    return VK_OK;
}

vk_status vk_gather_release_peers(vk_gather* g) {
    if (!g) return fail(VK_INVALID_ARG, "gather is NULL");
    DeviceGuard dg(g->device);
    cudaError_t e = cudaDeviceSynchronize();
    for (int r = 0; r < g->world; ++r)
        if (g->imported[r]) {
            if (!g->local[r]) {
                cudaError_t c = cudaIpcCloseMemHandle(g->peer[r]);
                if (e == cudaSuccess) e = c;
            }
            g->imported[r] = false;
            g->local[r] = false;
            g->peer[r] = nullptr;
        }
    return e == cudaSuccess ? VK_OK : cuda_fail(e, "closing peer mappings");
}

vk_status vk_gather_destroy(vk_gather* g) {
    if (!g) return VK_OK;
    vk_status s = vk_gather_release_peers(g);
    DeviceGuard dg(g->device);
    cudaError_t e = cudaFree(g->own);
    delete g;
    if (s != VK_OK) return s;
    return e == cudaSuccess ? VK_OK : cuda_fail(e, "cudaFree(gather buffers)");
}

vk_status vk_gather_export(const vk_gather* g, void* handle_out) {
    static_assert(sizeof(cudaIpcMemHandle_t) == VK_GATHER_HANDLE_BYTES, "IPC handle size");
    if (!g || !handle_out) return fail(VK_INVALID_ARG, "gather or handle is NULL");
    DeviceGuard dg(g->device);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, g->own);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
    std::memcpy(handle_out, &h, sizeof(h));
    return VK_OK;
}

vk_status vk_gather_import(vk_gather* g, int32_t peer, const void* handle) {
    if (!g || !handle) return fail(VK_INVALID_ARG, "gather or handle is NULL");
    if (peer < 0 || peer >= g->world || peer == g->rank) return fail(VK_INVALID_ARG, "peer outside [0, world) or own rank");
    if (g->imported[peer]) return fail(VK_INVALID_ARG, "peer already imported");
    DeviceGuard dg(g->device);
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    g->peer[peer] = static_cast<char*>(p);
    g->imported[peer] = true;
    return VK_OK;
}

vk_status vk_gather_import_local(vk_gather* g, int32_t peer, const vk_gather* pg) {
    if (!g || !pg) return fail(VK_INVALID_ARG, "gather or peer gather is NULL");
    if (peer < 0 || peer >= g->world || peer == g->rank) return fail(VK_INVALID_ARG, "peer outside [0, world) or own rank");
    if (g->imported[peer]) return fail(VK_INVALID_ARG, "peer already imported");
    if (pg->rank != peer || pg->world != g->world || pg->slots != g->slots || pg->slice_bytes != g->slice_bytes)
        return fail(VK_INVALID_ARG, "peer gather has another rank, world, slot count or slice size");
    if (pg->device != g->device) {
        DeviceGuard dg(g->device);
        int ok = 0;
        cudaError_t e = cudaDeviceCanAccessPeer(&ok, g->device, pg->device);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceCanAccessPeer");
        if (!ok) return fail(VK_UNSUPPORTED, "no peer access between the two devices");
        e = cudaDeviceEnablePeerAccess(pg->device, 0);
        if (e == cudaErrorPeerAccessAlreadyEnabled) {
            cudaGetLastError();  // not an error here: drop it from the runtime's last-error state
        } else if (e != cudaSuccess) {
            return cuda_fail(e, "cudaDeviceEnablePeerAccess");
        }
    }
    g->peer[peer] = pg->own;
    g->imported[peer] = true;
    g->local[peer] = true;
    return VK_OK;
}

void* vk_gather_buffer(const vk_gather* g, int32_t slot) {
    if (!g || slot < 0 || slot >= g->slots) return nullptr;
    return g->own + static_cast<uint64_t>(slot) * g->slot_bytes;
}

vk_status vk_gather_check(vk_gather* g) {
    if (!g) return fail(VK_INVALID_ARG, "gather is NULL");
    DeviceGuard dg(g->device);
    uint32_t bits = 0;
    cudaError_t e = cudaMemcpy(&bits, g->own + g->err_off, sizeof(bits), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(gather error word)");
    if (bits == 0) return VK_OK;
    e = cudaMemset(g->own + g->err_off, 0, sizeof(bits));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(gather error word)");
    return fail(VK_TIMEOUT, "a gather wait gave up: a rank's slice did not arrive within 1 s");
}

}  // extern "C"
