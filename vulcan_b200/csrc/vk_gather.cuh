// Device helpers of the fused head-shard output gather: system-scope flag
// loads and stores over NVLink and a bounded wait on one slot's flags.
#pragma once

#include "vk_internal.h"

namespace vk {

constexpr uint64_t kGatherWaitNs = 1000000000ull;  // 1 s bound on a cross-GPU wait

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t* gather_flag(const GatherView& g, int on_rank, int slot, int from_rank) {
    return reinterpret_cast<uint32_t*>(g.base[on_rank] + g.flags_off) + slot * g.world + from_rank;
}

// One thread: waits until every rank's flag of `slot` in this rank's block has
// reached `target` (flags carry step epochs and only grow, mod 2^32).  False,
// with VK_ERR_TIMEOUT, after kGatherWaitNs, or at once when another wait on
// the same error word has already given up (so a failed step costs one bound,
// not one per waiting warp).
__device__ __forceinline__ bool gather_wait_slot(const GatherView& g, int slot, uint32_t target, uint32_t* err) {
    const uint64_t t0 = global_ns();
    for (int r = 0; r < g.world; ++r) {
        const uint32_t* f = gather_flag(g, g.rank, slot, r);
        while (static_cast<int32_t>(ld_acquire_sys(f) - target) < 0) {
            if ((*reinterpret_cast<volatile uint32_t*>(err) & VK_ERR_TIMEOUT) || global_ns() - t0 > kGatherWaitNs) {
                atomicOr(err, VK_ERR_TIMEOUT);
                return false;
            }
            __nanosleep(64);
        }
    }
    return true;
}

// One thread, once every store of this rank into `slot` is visible to it (the
// grid that made them has completed: griddepcontrol.wait or stream order):
// raises this rank's flag of the slot on every rank to `epoch`.  One
// system-scope fence, then relaxed stores: a release pattern, so the peers
// that acquire a flag see those stores.
__device__ __forceinline__ void gather_signal(const GatherView& g, int slot, uint32_t epoch) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (int r = 0; r < g.world; ++r)
        asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(gather_flag(g, r, slot, g.rank)), "r"(epoch)
                     : "memory");
}

}  // namespace vk
