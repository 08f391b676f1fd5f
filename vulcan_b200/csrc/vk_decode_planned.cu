// Planned paged GQA decode: a persistent kernel over a host-built balanced
// schedule, with the new token's K/V append and the split merge fused in.
//
// Same arithmetic and result as vk_decode (one causal row of the reference's
// cpu_attention per query head, tests/test_attention.cu:66-97, over the paged
// cache; GQA mapping of src/transformer.cpp:173-179), organised for the B200:
//
//  * The plan (host, once per decode step since every layer of a step has the
//    same lengths) lays the pages of all (sequence, KV head) units end to end
//    and cuts that list into W contiguous ranges of equal cost, one per warp
//    ("worker"), with W = resident warps of the GPU: a page costs 1 and the end
//    of a unit inside a range (fused append, partial, next q) costs 6, so no
//    worker is a straggler; there is no tail of long sequences and no
//    per-split CTA prologue; ranges cross unit boundaries freely.
//  * Each worker warp prefetches its own pages kPlanStages ahead with 2-D TMA
//    loads (one mbarrier per stage; the block-table entries of the next 32
//    pages read in one coalesced round trip) and folds each page into its
//    softmax state with the tensor-core page update shared with vk_decode.
//  * Append fused: the last page of a unit is loaded as it is; when new K/V
//    rows were given, the consuming warp stores them into the pool and patches
//    them into the staged copy before folding the page in, so no load waits for
//    the new rows.
//  * Merge fused: a unit covered by one worker writes its fp16 output directly;
//    otherwise each piece writes its normalised partial and log2-sum-exp and
//    counts itself on the unit.  When workers have long ranges (>= 64 pages),
//    a unit of at most 8 pieces is merged by its last piece at once.  Other
//    units (and all of them for small per-GPU shares, where every piece ends
//    at the same time) are merged by tasks of (unit, group of query heads)
//    dealt to all warps of the grid by the plan; a warp runs its tasks after
//    its own page range, each once the unit's pieces are all counted
//    (bounded wait).  The merge of a unit split into many pieces is thus
//    spread over up to G warps.
//  * Gather fused (optional, head-sharded multi-GPU): each finished output is
//    also stored into every rank's receive slice over NVLink with plain peer
//    stores.  The next run on the stream, which starts after this grid has
//    completed, raises this rank's flag of that slot on every rank (step
//    epoch, one system fence); in strict order a run first waits for all
//    ranks' flags of the previous layer's slot.
//  * RoPE fused (optional): q and the new K rows are rotated in registers as
//    they are loaded (vk_rope.cuh).
//  * FP8 pools (FMT = 1, vk_fp8.cuh): a page block (codes and scales, 4,224
//    bytes at D=128) arrives in one bulk copy; the appended token is quantised
//    by the consuming warp, stored to the pool and patched into the stage.
#include <algorithm>
#include <vector>

#include "vk_decode_page.cuh"
#include "vk_fp8.cuh"
#include "vk_gather.cuh"
#include "vk_internal.h"

namespace vk {

constexpr int kPlanWarps = 2;      // worker warps per CTA
constexpr int kPlanStages = 4;     // TMA stages per worker (8 KiB each at D=128)
// Small per-GPU shares (few pages per worker, fp16 pages, head_dim 128): 3
// stages per worker and 4 CTAs per SM, i.e. 8 worker warps per SM instead of 6;
// measured on the 8-GPU share of the 70B layer (10 pages per worker).
constexpr int kSmallStages = 3;
constexpr int kSmallSharePages = 16;  // pages per worker below which the small-share kernel runs
constexpr int kMinPagesPerWorker = 8;
constexpr int64_t kUnitEndPages = 6;  // cost of a unit end inside a worker range, in pages (measured best of 0-16)
constexpr int kLastMergeMax = 8;   // large shares: units of up to this many pieces merge in their last piece
constexpr int kLastMergeMinPages = 64;  // ... when workers have at least this many pages
// Merge counters are polled by many warps at once: one 128-byte line each, so
// the pollers of one unit do not queue behind those of its neighbours.
constexpr int kCtrStride = 32;

struct PlanParams {
    const int32_t* wb;     // [W+1] first global page of each worker
    const int32_t* wfu;    // [W]   unit holding the worker's first page
    const int32_t* uoff;   // [U+1] first global page of each unit
    const int32_t* ulen;   // [U]   tokens of the unit's sequence
    const int32_t* ufw;    // [U]   first worker touching the unit
    const int32_t* unp;    // [U]   workers touching the unit (pieces)
    const int32_t* uslot;  // [U]   first partial slot of the unit (-1 if one piece)
    const int32_t* tunits; // [ntasks / S] unit of each merge task group
    const int32_t* zunits; // [Z]   units without pages (zero output)
    uint32_t* counters;    // [2U lines of kCtrStride] pieces finished, merge tasks finished (reset by the merger / last task)
    float* part_o;         // [slots, G, D]
    float* part_lse;       // [slots, G]
    const __half* q;
    __half* out;
    const __half* k_new;   // [B, Hkv, D] or null
    const __half* v_new;
    const int32_t* bt;
    uint32_t* err;
    char* pool_base;
    uint64_t seg_bytes, layer_off, head_bytes;
    int bt_stride, Hq, Hkv, G, L, layer, num_pages, W, Z, U;
    int ntasks, S;   // merge tasks, tasks (head groups) per split unit
    int lmm;         // units of up to lmm pieces merge in their last piece (others: tasks)
    const float* rope_freq;  // non-null: q and the new K rotated (RoPE) at the new token's position
    float scale_log2;
    // fused output gather (g.world == 0: none)
    GatherView g;
    const uint32_t* gepoch;  // step epoch of the uploaded plan (flag value)
    int gslot;       // slot this layer writes
    int gsig_slot;   // slot of the preceding run (its stores are complete): signal it (-1: none)
    int gwait_slot;  // slot to wait for before reading inputs (-1: none)
    int out_own;     // out is this rank's own slice (skip the local copy)
};

// bytes of one stage: the K and V rows of one (page, head), fp16 or FP8 block
template <int D, int FMT>
__host__ __device__ constexpr int plan_stage_bytes() {
    return FMT ? fp8_head_bytes(D) : 2 * kPageTokens * D * 2;
}

template <int D, int FMT, int NS = kPlanStages>
__host__ __device__ constexpr int plan_smem_bytes() {
    return kPlanWarps * NS * plan_stage_bytes<D, FMT>() + kPlanWarps * NS * 8 + 1024;
}

// Programmatic dependent launch: let the next kernel on the stream start
// launching, and wait for the previous one to complete (no-ops when the launch
// did not opt in).
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Writes zeros for a unit without pages (a sequence of length 0).
template <int D>
__device__ __forceinline__ void zero_unit(const PlanParams& p, int u, int lane) {
    __half* o = p.out + (static_cast<int64_t>(u / p.Hkv) * p.Hq + (u % p.Hkv) * p.G) * D;
    for (int e = lane; e < p.G * D; e += 32) o[e] = __float2half(0.f);
}

__device__ __forceinline__ void atom_add_release_gpu(unsigned int* p, unsigned int v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned int atom_add_acq_rel_gpu(unsigned int* p, unsigned int v) {
    unsigned int old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Fused gather: the warp that finished `nh` query heads of unit u starting at
// head h (their [nh, D] outputs are in p.out) copies them in 16-byte pieces
// into every rank's receive slice.  No fence: the slot is signalled by the
// next run on the stream, once this grid has completed.
template <int D>
__device__ __forceinline__ void publish_heads(const PlanParams& p, int u, int h, int nh, int lane) {
    if (p.g.world == 0) return;
    __syncwarp();
    const int64_t head0 = static_cast<int64_t>(u / p.Hkv) * p.Hq + (u % p.Hkv) * p.G + h;
    const uint4* src = reinterpret_cast<const uint4*>(p.out + head0 * D);
    const uint64_t off = static_cast<uint64_t>(p.gslot) * p.g.slot_bytes +
                         static_cast<uint64_t>(p.g.rank) * p.g.slice_bytes + static_cast<uint64_t>(head0) * D * 2;
    const int n16 = nh * D / 8;
    for (int c = lane; c < n16; c += 32) {
        const uint4 v = __ldcg(src + c);  // written by other lanes of this warp
        for (int r = 0; r < p.g.world; ++r) {
            if (r == p.g.rank && p.out_own) continue;
            reinterpret_cast<uint4*>(p.g.base[r] + off)[c] = v;
        }
    }
}

template <int D>
__device__ __forceinline__ void publish_unit(const PlanParams& p, int u, int lane) {
    publish_heads<D>(p, u, 0, p.G, lane);
}

// Fused gather, after griddepcontrol.wait.  Strict order (a wait slot): warp 0
// raises this rank's flags for the preceding run's slot, then every warp waits
// until all ranks' slices of that slot have arrived.  Otherwise the flags are
// raised at the end (gather_epilogue), off the critical path.
__device__ __forceinline__ void gather_prologue(const PlanParams& p, int w, int lane) {
    if (p.g.world == 0 || p.gwait_slot < 0) return;
    const uint32_t epoch = *p.gepoch;
    if (w == 0 && lane == 0 && p.gsig_slot >= 0) gather_signal(p.g, p.gsig_slot, epoch);
    if (lane == 0) gather_wait_slot(p.g, p.gwait_slot, epoch, p.err);
    __syncwarp();
}

// Fused gather without the strict order: the first warp to finish its work
// raises this rank's flags for the preceding run's slot (each slot records the
// epoch it was last raised with, so exactly one warp does it).
__device__ __forceinline__ void gather_epilogue(const PlanParams& p, int lane) {
    if (p.g.world == 0 || p.gwait_slot >= 0 || p.gsig_slot < 0 || lane != 0) return;
    const uint32_t epoch = *p.gepoch;
    unsigned int* sig = reinterpret_cast<unsigned int*>(p.g.base[p.g.rank] + p.g.sig_off) + p.gsig_slot;
    if (static_cast<int32_t>(atomicMax(sig, epoch) - epoch) < 0) gather_signal(p.g, p.gsig_slot, epoch);
}

// Iterator over (unit, page-in-unit) along the concatenated page list.
struct PageIt {
    int u, p, np;
    __device__ __forceinline__ void next(const int32_t* uoff) {
        if (++p == np) {
            p = 0;
            do {
                ++u;
                np = uoff[u + 1] - uoff[u];
            } while (np == 0);
        }
    }
};


// One merge task: heads [h0, h0 + hs) of unit u from its np piece partials,
// out = sum_k 2^(lse_k - m) o_k / sum_k 2^(lse_k - m), written as fp16, in one
// streaming pass with a running max.  IT = float4 items per lane (items
// f = lane + 32 i, i < IT, of the task's [hs, D] block); the loads of KB
// pieces (partials and their lse) are issued together.  FP8 pools (FMT 1)
// batch fewer pieces: the kernel then runs 6 CTAs per SM on fewer registers.
template <int D, int NT, int IT, int FMT>
__device__ __forceinline__ void merge_task(const PlanParams& p, int u, int h0, int hs, int np, int lane) {
    constexpr int KB = FMT ? (IT == 1 ? 8 : (IT >= 8 ? 1 : 8 / IT)) : (IT == 1 ? 32 : (IT >= 16 ? 1 : 16 / IT));
    const int base = p.uslot[u];
    const int nf = hs * D / 4;
    float m[IT], den[IT];
    int hi[IT];
    float4 acc[IT];
#pragma unroll
    for (int i = 0; i < IT; ++i) {
        const int f = lane + 32 * i;
        hi[i] = f < nf ? (f * 4) / D : 0;
        m[i] = -INFINITY;
        den[i] = 0.f;
        acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const float4* os = reinterpret_cast<const float4*>(p.part_o);
    const int64_t row = static_cast<int64_t>(p.G) * D / 4;  // float4 per piece partial
    for (int k0 = 0; k0 < np; k0 += KB) {
        float4 ov[KB][IT];
        float lw[KB][IT];
#pragma unroll
        for (int b = 0; b < KB; ++b)
#pragma unroll
            for (int i = 0; i < IT; ++i) {
                const int f = lane + 32 * i;
                const bool live = f < nf && k0 + b < np;
                const int64_t k = base + min(k0 + b, np - 1);
                ov[b][i] = live ? __ldcg(os + k * row + static_cast<int64_t>(h0) * (D / 4) + f)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
                lw[b][i] = live ? __ldcg(p.part_lse + k * p.G + h0 + hi[i]) : -INFINITY;
            }
#pragma unroll
        for (int i = 0; i < IT; ++i) {
            float mb = m[i];
#pragma unroll
            for (int b = 0; b < KB; ++b) mb = fmaxf(mb, lw[b][i]);
            if (mb == -INFINITY) continue;  // no piece for this item yet
            const float a = ex2(m[i] - mb);  // 0 while m is -inf
            den[i] *= a;
            acc[i].x *= a;
            acc[i].y *= a;
            acc[i].z *= a;
            acc[i].w *= a;
#pragma unroll
            for (int b = 0; b < KB; ++b) {
                const float wgt = ex2(lw[b][i] - mb);
                den[i] += wgt;
                acc[i].x += wgt * ov[b][i].x;
                acc[i].y += wgt * ov[b][i].y;
                acc[i].z += wgt * ov[b][i].z;
                acc[i].w += wgt * ov[b][i].w;
            }
            m[i] = mb;
        }
    }
    const int64_t head0 = static_cast<int64_t>(u / p.Hkv) * p.Hq + (u % p.Hkv) * p.G + h0;
#pragma unroll
    for (int i = 0; i < IT; ++i) {
        const int f = lane + 32 * i;
        if (f < nf) {
            const float inv = 1.f / den[i];
            const __half2 lo = __floats2half2_rn(acc[i].x * inv, acc[i].y * inv);
            const __half2 hi2 = __floats2half2_rn(acc[i].z * inv, acc[i].w * inv);
            uint2 v;
            v.x = *reinterpret_cast<const uint32_t*>(&lo);
            v.y = *reinterpret_cast<const uint32_t*>(&hi2);
            *reinterpret_cast<uint2*>(p.out + head0 * D + f * 4) = v;
            // fused gather: the same 8 bytes into every rank's receive slice
            const uint64_t off = static_cast<uint64_t>(p.gslot) * p.g.slot_bytes +
                                 static_cast<uint64_t>(p.g.rank) * p.g.slice_bytes +
                                 (static_cast<uint64_t>(head0) * D + f * 4) * 2;
            for (int r = 0; r < p.g.world; ++r)
                if (!(r == p.g.rank && p.out_own)) *reinterpret_cast<uint2*>(p.g.base[r] + off) = v;
        }
    }
}

// The merge tasks dealt to warp w (w, w + Wtot, ...): each waits, bounded,
// until its unit's pieces are all counted, merges its heads and publishes them.
template <int D, int NT, int FMT>
__device__ __forceinline__ void run_merge_tasks(const PlanParams& p, int w, int Wtot, int lane) {
    for (int k = w; k < p.ntasks; k += Wtot) {
        const int u = p.tunits[k / p.S];
        const int hs = p.G / p.S;
        const int h0 = (k % p.S) * hs;
        const int np = p.unp[u];
        int ok = 1;
        if (lane == 0) {
            const uint64_t t0 = global_ns();
            while (ld_acquire_gpu(&p.counters[u * kCtrStride]) < static_cast<unsigned int>(np)) {
                // give up at once if a piece's warp already gave up on a wait
                if ((*reinterpret_cast<volatile uint32_t*>(p.err) & VK_ERR_TIMEOUT) ||
                    global_ns() - t0 > kGatherWaitNs) {
                    atomicOr(p.err, VK_ERR_TIMEOUT);
                    ok = 0;
                    break;
                }
                __nanosleep(32);
            }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (ok) {
            const int ni = (hs * D / 4 + 31) / 32;  // float4 items per lane
            if (ni <= 1) merge_task<D, NT, 1, FMT>(p, u, h0, hs, np, lane);
            else if (ni <= 2) merge_task<D, NT, 2, FMT>(p, u, h0, hs, np, lane);
            else if (ni <= 4) merge_task<D, NT, 4, FMT>(p, u, h0, hs, np, lane);
            else if (ni <= 8) merge_task<D, NT, 8, FMT>(p, u, h0, hs, np, lane);
            else merge_task<D, NT, 16, FMT>(p, u, h0, hs, np, lane);
        }
        __syncwarp();
        if (lane == 0 && atomicAdd(&p.counters[(p.U + u) * kCtrStride], 1u) == static_cast<unsigned int>(p.S - 1)) {
            p.counters[u * kCtrStride] = 0u;  // every task of the unit has passed its wait
            p.counters[(p.U + u) * kCtrStride] = 0u;
        }
    }
}

// FP8 pools: 6 CTAs (12 worker warps) per SM, measured 9% faster than 4 CTAs
// on fewer registers (the FP8 page update is bound by per-warp latency, not by
// bytes in flight).
template <int D, int NT, int FMT, int NS>
__global__ void __launch_bounds__(kPlanWarps * 32, FMT ? 6 : (NS == kSmallStages ? 4 : 1)) planned_decode_kernel(const __grid_constant__ CUtensorMap tmap,
                                                                         const PlanParams p) {
    constexpr int P = kPageTokens;
    constexpr int SB = plan_stage_bytes<D, FMT>();
    constexpr int NB = D / 64;
    constexpr int KS = D / 16;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPlanWarps * NS * SB);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int w = blockIdx.x * kPlanWarps + warp;

    griddep_launch_dependents();

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPlanWarps * NS; ++s) mbar_init(smem_u32(&bars[s]), 1);
        mbar_fence_init();
    }
    __syncthreads();
    // Before griddep_wait only the plan tables, block tables and pool pages are
    // read (not written by the preceding kernel); q, k_new, v_new, out and the
    // merge scratch are touched after it.
    const int g0 = w < p.W ? p.wb[w] : 0;
    const int n = w < p.W ? p.wb[w + 1] - g0 : 0;
    if (n <= 0) {
        griddep_wait();
        gather_prologue(p, w, lane);
        for (int i = w; i < p.Z; i += gridDim.x * kPlanWarps) {
            zero_unit<D>(p, p.zunits[i], lane);
            publish_unit<D>(p, p.zunits[i], lane);
        }
        run_merge_tasks<D, NT, FMT>(p, w, gridDim.x * kPlanWarps, lane);
        gather_epilogue(p, lane);
        return;
    }

    uint8_t* my_stages = smem + warp * NS * SB;
    uint64_t* full = bars + warp * NS;
    if (FMT == 0 && lane == 0) prefetch_tmap(&tmap);
    const uint64_t pol = l2_evict_first_policy();

    const int u0 = p.wfu[w];
    PageIt pf{u0, g0 - p.uoff[u0], p.uoff[u0 + 1] - p.uoff[u0]};  // prefetch cursor
    PageIt cu = pf;                                                // consume cursor

    // Block-table entries of the next 32 pages of the range, one per lane, read
    // in one coalesced round trip instead of one dependent load per page.
    int nissued = 0;  // pages of the range issued so far
    int win = -1;     // page id of range page (nissued & ~31) + lane; -1 bad or past the end
    auto load_window = [&]() {
        win = -1;
        if (nissued + lane < n) {
            PageIt c = pf;
            int adv = lane;
            while (adv > 0) {
                const int left = c.np - 1 - c.p;
                if (adv <= left) {
                    c.p += adv;
                    adv = 0;
                } else {
                    adv -= left + 1;
                    c.p = 0;
                    do {
                        ++c.u;
                        c.np = p.uoff[c.u + 1] - p.uoff[c.u];
                    } while (c.np == 0);
                }
            }
            const int page = p.bt[static_cast<int64_t>(c.u / p.Hkv) * p.bt_stride + c.p];
            if (page < 0 || page >= p.num_pages) atomicOr(p.err, VK_ERR_PAGE_ID);
            else win = page;
        }
    };

    // Loads page `pf` into stage s (whole warp; lane 0 issues the TMA).  The
    // page that receives the new token is loaded as it is in memory; the new
    // rows are patched into the stage when it is consumed.
    uint32_t bad_stages = 0;  // bit s: stage s holds a stand-in for a bad page id
    auto issue = [&](int s) {
        const int hkv = pf.u % p.Hkv;
        if ((nissued & 31) == 0) load_window();
        int page = __shfl_sync(0xffffffffu, win, nissued & 31);
        ++nissued;
        bad_stages &= ~(1u << s);
        if (page < 0) {
            page = 0;  // recorded in the error word; read a valid page instead
            bad_stages |= 1u << s;
        }
        if (lane == 0) {
            const uint32_t bar = smem_u32(&full[s]);
            mbar_expect_tx(bar, SB);
            const uint32_t dst = smem_u32(my_stages + s * SB);
            if constexpr (FMT == 1) {
                bulk_load(dst, p.pool_base + p.layer_off + static_cast<uint64_t>(page) * p.seg_bytes +
                                   static_cast<uint64_t>(hkv) * p.head_bytes,
                          SB, bar, pol);
            } else {
                const int row = ((p.layer * p.num_pages + page) * p.Hkv + hkv) * (2 * P);
#pragma unroll
                for (int hb = 0; hb < NB; ++hb) tma_load_2d(dst + hb * (2 * P * 128), &tmap, hb * 64, row, bar, pol);
            }
        }
        pf.next(p.uoff);
    };

    // Prefetch the first stages (block tables and pages only: nothing the
    // preceding kernel writes).
    const int pre = min(n, NS);
    int issued = 0;
    while (issued < pre) issue(issued++);
    griddep_wait();
    gather_prologue(p, w, lane);
    for (int i = w; i < p.Z; i += gridDim.x * kPlanWarps) {
        zero_unit<D>(p, p.zunits[i], lane);
        publish_unit<D>(p, p.zunits[i], lane);
    }

    uint32_t qf[NT][KS][2];
    WarpSoftmaxState<D, NT> st;
    auto load_q = [&]() {
        const __half* qs = p.q + (static_cast<int64_t>(cu.u / p.Hkv) * p.Hq + (cu.u % p.Hkv) * p.G) * D;
        if constexpr (FMT == 1) {
            load_q_frags_fp8<D, NT>(qf, qs, p.G, lane);
            rope_q_frags_fp8<D, NT>(qf, p.ulen[cu.u] - 1, p.rope_freq, lane);
        } else {
            load_q_frags<D, NT>(qf, qs, p.G, lane);
            rope_q_frags<D, NT>(qf, p.ulen[cu.u] - 1, p.rope_freq, lane);
        }
    };
    load_q();
    st.reset();

    for (int j = 0; j < n; ++j) {
        const int s = j % NS;
        // Fused append: the unit's last page takes the new token at slot
        // (len-1) % P; its K and V rows are read now (in flight during the
        // stage wait), stored to the pool and patched into the stage.
        const bool app = p.k_new != nullptr && cu.p == cu.np - 1 && !((bad_stages >> s) & 1u);
        constexpr int NCH = D / 8;  // 16-byte chunks per row
        uint4 row_val[(2 * NCH + 31) / 32];
        int app_page = 0, app_slot = 0;
        uint32_t q8k = 0u, q8v = 0u;  // FP8: the lane's codes of the new K and V rows
        float q8ks = 0.f, q8vs = 0.f;
        if (FMT == 1 && app) {
            const int b = cu.u / p.Hkv, hkv = cu.u % p.Hkv;
            app_page = p.bt[static_cast<int64_t>(b) * p.bt_stride + cu.p];
            const int pos = p.ulen[cu.u] - 1;
            app_slot = pos % P;
            const int64_t src = (static_cast<int64_t>(b) * p.Hkv + hkv) * D + 4 * lane;
            const uint2 kw = __ldg(reinterpret_cast<const uint2*>(p.k_new + src));
            const uint2 vw = __ldg(reinterpret_cast<const uint2*>(p.v_new + src));
            float xk[4], xv[4];
            float2 f;
            f = __half22float2(*reinterpret_cast<const __half2*>(&kw.x)); xk[0] = f.x; xk[1] = f.y;
            f = __half22float2(*reinterpret_cast<const __half2*>(&kw.y)); xk[2] = f.x; xk[3] = f.y;
            f = __half22float2(*reinterpret_cast<const __half2*>(&vw.x)); xv[0] = f.x; xv[1] = f.y;
            f = __half22float2(*reinterpret_cast<const __half2*>(&vw.y)); xv[2] = f.x; xv[3] = f.y;
            if (p.rope_freq != nullptr) {
                f = rope_pair(xk[0], xk[1], 2 * lane, pos, p.rope_freq); xk[0] = f.x; xk[1] = f.y;
                f = rope_pair(xk[2], xk[3], 2 * lane + 1, pos, p.rope_freq); xk[2] = f.x; xk[3] = f.y;
            }
            q8k = fp8_quant_row(xk, q8ks);
            q8v = fp8_quant_row(xv, q8vs);
        } else if (app) {
            const int b = cu.u / p.Hkv, hkv = cu.u % p.Hkv;
            app_page = p.bt[static_cast<int64_t>(b) * p.bt_stride + cu.p];
            app_slot = (p.ulen[cu.u] - 1) % P;
            const int64_t src = (static_cast<int64_t>(b) * p.Hkv + hkv) * D;
#pragma unroll
            for (int i = 0; i < (2 * NCH + 31) / 32; ++i) {
                const int v = lane + 32 * i;
                const bool is_v = v >= NCH;
                row_val[i] = v < 2 * NCH ? __ldg(reinterpret_cast<const uint4*>((is_v ? p.v_new : p.k_new) + src) +
                                                 (is_v ? v - NCH : v))
                                         : make_uint4(0, 0, 0, 0);
                if (v < NCH && p.rope_freq != nullptr)  // the new K row, rotated at its position
                    row_val[i] = rope_uint4(row_val[i], v * 8, p.ulen[cu.u] - 1, p.rope_freq);
            }
        }
        if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&full[s]), (j / NS) & 1, p.err))) return;
        if (FMT == 1 && app) {
            char* blk = p.pool_base + p.layer_off + static_cast<uint64_t>(app_page) * p.seg_bytes +
                        static_cast<uint64_t>(cu.u % p.Hkv) * p.head_bytes;
            fp8_store_token(blk, app_slot, lane, q8k, q8v, q8ks, q8vs);
            fp8_store_token(reinterpret_cast<char*>(my_stages + s * SB), app_slot, lane, q8k, q8v, q8ks, q8vs);
            __syncwarp();
        } else if (app) {
            const int hkv = cu.u % p.Hkv;
            char* dk = p.pool_base + p.layer_off + static_cast<uint64_t>(app_page) * p.seg_bytes +
                       static_cast<uint64_t>(hkv) * p.head_bytes + static_cast<uint64_t>(app_slot) * D * 2;
            const uint32_t sb = smem_u32(my_stages + s * SB);
#pragma unroll
            for (int i = 0; i < (2 * NCH + 31) / 32; ++i) {
                const int v = lane + 32 * i;
                if (v < 2 * NCH) {
                    const bool is_v = v >= NCH;
                    const int vi = is_v ? v - NCH : v;
                    reinterpret_cast<uint4*>(dk + (is_v ? P * D * 2 : 0))[vi] = row_val[i];
                    const int r = (is_v ? P : 0) + app_slot, d0 = vi * 8;
                    const uint32_t a = sb + (d0 >> 6) * (2 * P * 128) + swz128(r, (d0 & 63) >> 3);
                    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(row_val[i].x),
                                 "r"(row_val[i].y), "r"(row_val[i].z), "r"(row_val[i].w)
                                 : "memory");
                }
            }
            __syncwarp();
        }
        const int valid = min(P, p.ulen[cu.u] - cu.p * P);
        if constexpr (FMT == 1) page_update_fp8<D, NT>(smem_u32(my_stages + s * SB), valid, qf, st, p.scale_log2, lane);
        else page_update<D, NT>(smem_u32(my_stages + s * SB), valid, qf, st, p.scale_log2, lane);
        // Every lane's ldmatrix results for stage s have been consumed by its MMAs
        // before __syncwarp returns, so the stage can be refilled.
        __syncwarp();
        if (app) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // patch before the next TMA write
        if (j + NS < n) issue(s);

        const bool unit_done = (cu.p == cu.np - 1) || (j == n - 1);
        if (unit_done) {
            // ------------------------------------------------ finish this piece of unit cu.u
            reduce_l<D, NT>(st);
            const int u = cu.u;
            const int64_t head0 = static_cast<int64_t>(u / p.Hkv) * p.Hq + (u % p.Hkv) * p.G;
            const int npieces = p.unp[u];
            if (npieces == 1) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const int h0 = nt * 8 + (lane & 3) * 2;
                    const float i0 = (FMT ? st.vf : 1.f) / st.l[nt][0], i1 = (FMT ? st.vf : 1.f) / st.l[nt][1];
#pragma unroll
                    for (int mt = 0; mt < KS; ++mt) {
                        const int d = mt * 16 + (lane >> 2);
                        if (h0 < p.G) {
                            p.out[(head0 + h0) * D + d] = __float2half(st.acc[nt][mt][0] * i0);
                            p.out[(head0 + h0) * D + d + 8] = __float2half(st.acc[nt][mt][2] * i0);
                        }
                        if (h0 + 1 < p.G) {
                            p.out[(head0 + h0 + 1) * D + d] = __float2half(st.acc[nt][mt][1] * i1);
                            p.out[(head0 + h0 + 1) * D + d + 8] = __float2half(st.acc[nt][mt][3] * i1);
                        }
                    }
                }
                publish_unit<D>(p, u, lane);
            } else {
                const int slot = p.uslot[u] + (w - p.ufw[u]);
                float* po = p.part_o + static_cast<int64_t>(slot) * p.G * D;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const int h0 = nt * 8 + (lane & 3) * 2;
                    const float i0 = (FMT ? st.vf : 1.f) / st.l[nt][0], i1 = (FMT ? st.vf : 1.f) / st.l[nt][1];
#pragma unroll
                    for (int mt = 0; mt < KS; ++mt) {
                        const int d = mt * 16 + (lane >> 2);
                        if (h0 < p.G) {
                            po[h0 * D + d] = st.acc[nt][mt][0] * i0;
                            po[h0 * D + d + 8] = st.acc[nt][mt][2] * i0;
                        }
                        if (h0 + 1 < p.G) {
                            po[(h0 + 1) * D + d] = st.acc[nt][mt][1] * i1;
                            po[(h0 + 1) * D + d + 8] = st.acc[nt][mt][3] * i1;
                        }
                    }
                    if (lane < 4) {
                        if (h0 < p.G) p.part_lse[static_cast<int64_t>(slot) * p.G + h0] = st.m[nt][0] + __log2f(st.l[nt][0]);
                        if (h0 + 1 < p.G) p.part_lse[static_cast<int64_t>(slot) * p.G + h0 + 1] = st.m[nt][1] + __log2f(st.l[nt][1]);
                    }
                }
                __syncwarp();  // every lane's partial stores precede lane 0's release
                if (npieces > p.lmm) {
                    if (lane == 0) atom_add_release_gpu(&p.counters[u * kCtrStride], 1u);
                } else {
                    // few pieces: the last to finish merges the unit at once
                    unsigned int prev = 0;
                    if (lane == 0) prev = atom_add_acq_rel_gpu(&p.counters[u * kCtrStride], 1u);
                    prev = __shfl_sync(0xffffffffu, prev, 0);
                    if (prev == static_cast<unsigned int>(npieces - 1)) {
                        __syncwarp();  // lane 0's acquire precedes every lane's loads
                        // head groups of at most 8 float4 items per lane
                        constexpr int HG = 1024 / D;
                        for (int hg = 0; hg < p.G; hg += HG)
                            merge_task<D, NT, (HG * D / 128 < NT * 8 * D / 128 ? HG * D / 128 : NT * 8 * D / 128), FMT>(
                                p, u, hg, min(HG, p.G - hg), npieces, lane);
                        if (lane == 0) p.counters[u * kCtrStride] = 0u;
                    }
                }
            }
            if (j + 1 < n) {
                cu.next(p.uoff);
                load_q();
                st.reset();
            }
        } else {
            cu.next(p.uoff);
        }
    }
    run_merge_tasks<D, NT, FMT>(p, w, gridDim.x * kPlanWarps, lane);
    gather_epilogue(p, lane);
}

// Signals this rank's stores of `slot` (the preceding run on the stream has
// completed) and waits until every rank's have arrived.
__global__ void plan_gather_wait_kernel(const GatherView g, int slot, const uint32_t* epoch_p, uint32_t* err) {
    if (threadIdx.x == 0) {
        const uint32_t epoch = *epoch_p;
        gather_signal(g, slot, epoch);
        gather_wait_slot(g, slot, epoch, err);
    }
}

template <int D, int NT, int FMT, int NS>
static int plan_occupancy(int device, int* occ_out) {
    static int cache[64] = {};
    if (device < 0 || device >= 64) return -1;
    if (cache[device] == 0) {
        constexpr int smem = plan_smem_bytes<D, FMT, NS>();
        if (cudaFuncSetAttribute(planned_decode_kernel<D, NT, FMT, NS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
            return -1;
        int occ = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, planned_decode_kernel<D, NT, FMT, NS>, kPlanWarps * 32, smem) !=
                cudaSuccess ||
            occ <= 0)
            return -1;
        cache[device] = occ;
    }
    *occ_out = cache[device];
    return 0;
}

static int occupancy_for(int D, int NT, int fmt, int ns, int device, int* occ) {
    constexpr int S = kPlanStages, s3 = kSmallStages;
    if (fmt == VK_KV_FP8)  // FP8 pools: head_dim 128 only
        return NT == 1 ? plan_occupancy<128, 1, 1, S>(device, occ) : plan_occupancy<128, 2, 1, S>(device, occ);
    if (D == 128 && ns == s3)
        return NT == 1 ? plan_occupancy<128, 1, 0, s3>(device, occ) : plan_occupancy<128, 2, 0, s3>(device, occ);
    if (D == 128) return NT == 1 ? plan_occupancy<128, 1, 0, S>(device, occ) : plan_occupancy<128, 2, 0, S>(device, occ);
    if (D == 64) return NT == 1 ? plan_occupancy<64, 1, 0, S>(device, occ) : plan_occupancy<64, 2, 0, S>(device, occ);
    return NT == 1 ? plan_occupancy<256, 1, 0, S>(device, occ) : plan_occupancy<256, 2, 0, S>(device, occ);
}

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace vk

struct vk_decode_plan {
    int device = 0, B = 0, Hq = 0, Hkv = 0, G = 0, D = 0, NT = 1, fmt = VK_KV_FP16, ns = vk::kPlanStages;
    int W = 0, U = 0, Z = 0, slots = 0, grid = 0, max_unit_pages = 0, total_pages = 0;
    mutable std::vector<int32_t> tables;
    size_t o_wb = 0, o_wfu = 0, o_uoff = 0, o_ulen = 0, o_ufw = 0, o_unp = 0, o_uslot = 0, o_tu = 0, o_z = 0;
    int ntasks = 0, S = 1, lmm = 1;
    int last_merge_units = 0, max_pieces = 0;  // units merged by their last piece; most pieces of one unit
    size_t o_hdr = 0;  // [0]: step epoch written at upload (fused gather)
    size_t tables_bytes = 0, counters_off = 0, part_o_off = 0, part_lse_off = 0, ws_bytes = 0;
    bool early_start = false;
    vk_gather* gather = nullptr;
    int gather_slot_base = 0;
    bool gather_wait_prev = false;
};

using namespace vk;

extern "C" {

vk_status vk_decode_plan_create(const vk_pool* pool, const int32_t* seq_lens_host, int32_t batch,
                                int32_t num_q_heads, vk_decode_plan** out_plan) {
    if (!out_plan) return fail(VK_INVALID_ARG, "out_plan is NULL");
    *out_plan = nullptr;
    if (!pool || !pool->kv) return fail(VK_INVALID_ARG, "plan needs a KV pool");
    if (pool->cfg.page_tokens != kPageTokens) return fail(VK_UNSUPPORTED, "plan supports page_tokens == 16");
    const int D = pool->cfg.head_dim, Hkv = pool->cfg.num_kv_heads;
    if (D != 64 && D != 128 && D != 256) return fail(VK_UNSUPPORTED, "plan supports head_dim 64, 128, 256");
    if (batch < 0 || (batch > 0 && !seq_lens_host)) return fail(VK_INVALID_ARG, "bad batch / seq_lens");
    if (num_q_heads <= 0 || num_q_heads % Hkv) return fail(VK_INVALID_ARG, "num_q_heads must be a positive multiple of num_kv_heads");
    const int G = num_q_heads / Hkv;
    if (G > 16) return fail(VK_UNSUPPORTED, "plan supports up to 16 query heads per KV head");
    auto* pl = new vk_decode_plan();
    pl->device = pool->device;
    pl->B = batch;
    pl->Hq = num_q_heads;
    pl->Hkv = Hkv;
    pl->G = G;
    pl->D = D;
    pl->NT = G <= 8 ? 1 : 2;
    pl->fmt = pool->kv_format;
    const int U = batch * Hkv;
    pl->U = U;
    std::vector<int64_t> uoff(static_cast<size_t>(U) + 1, 0);
    std::vector<int32_t> ulen(U), zunits;
    for (int b = 0; b < batch; ++b) {
        if (seq_lens_host[b] < 0) {
            delete pl;
            return fail(VK_INVALID_ARG, "negative sequence length");
        }
        const int np = (seq_lens_host[b] + kPageTokens - 1) / kPageTokens;
        pl->max_unit_pages = std::max(pl->max_unit_pages, np);
        for (int h = 0; h < Hkv; ++h) {
            const int u = b * Hkv + h;
            ulen[u] = seq_lens_host[b];
            uoff[u + 1] = uoff[u] + np;
            if (np == 0) zunits.push_back(u);
        }
    }
    const int64_t T = uoff[U];
    if (T >= (1ll << 31)) {
        delete pl;
        return fail(VK_INVALID_ARG, "too many pages in one step");
    }
    pl->total_pages = static_cast<int>(T);
    pl->Z = static_cast<int>(zunits.size());
    int occ = 1;
    int64_t cap = 0, W = 0;
    auto size_workers = [&]() -> bool {
        DeviceGuard g(pool->device);
        if (occupancy_for(D, pl->NT, pl->fmt, pl->ns, pool->device, &occ) != 0) return false;
        cap = static_cast<int64_t>(pool->num_sms) * occ * kPlanWarps;
        if (pool->plan_workers > 0) cap = std::min<int64_t>(cap, pool->plan_workers);
        W = T > 0 ? std::min<int64_t>(cap, (T + kMinPagesPerWorker - 1) / kMinPagesPerWorker) : 0;
        W = std::max<int64_t>(W, T > 0 ? 1 : 0);
        return true;
    };
    bool sized = size_workers();
    if (sized && pl->fmt == VK_KV_FP16 && D == 128 && W > 0 && T / W < kSmallSharePages) {
        pl->ns = kSmallStages;  // small share: more, shallower workers
        sized = size_workers();
    }
    if (!sized) {
        delete pl;
        return fail(VK_CUDA_ERROR, "occupancy query for the planned decode kernel failed");
    }
    pl->W = static_cast<int>(W);
    // with long worker ranges a unit's few pieces end at different times: the
    // last merges at once; with short ranges (small per-GPU shares) all pieces
    // end together and the merges are spread over the grid as tasks
    pl->lmm = (W > 0 && T / W >= kLastMergeMinPages) ? kLastMergeMax : 1;
    const int zero_ctas = (pl->Z + kPlanWarps - 1) / kPlanWarps;
    pl->grid = static_cast<int>(std::max<int64_t>((W + kPlanWarps - 1) / kPlanWarps, std::min<int64_t>(zero_ctas, cap / kPlanWarps)));
    if (pl->grid == 0 && pl->Z > 0) pl->grid = 1;

    // worker ranges and the unit each starts in
    std::vector<int32_t> wb(static_cast<size_t>(W) + 1), wfu(static_cast<size_t>(W));
    // Equal cost rather than equal pages: the end of a unit inside a range
    // (the fused append, the piece's partial and the next unit's q) costs
    // about kUnitEndPages pages of streaming, so ranges that hold unit ends get
    // fewer pages.  Every range keeps at least one page.
    if (W > 0) {
        std::vector<int64_t> uend;  // page index just past each non-empty unit
        for (int u = 0; u < U; ++u)
            if (uoff[u + 1] > uoff[u]) uend.push_back(uoff[u + 1]);
        auto cost_before = [&](int64_t g) {  // pages before g plus ends of units finished before g
            const int64_t ends = std::upper_bound(uend.begin(), uend.end(), g) - uend.begin();
            return g + ends * kUnitEndPages;
        };
        const int64_t total = cost_before(T);
        for (int64_t w = 0; w <= W; ++w) {
            const int64_t target = total * w / W;
            int64_t lo = 0, hi = T;  // smallest g with cost_before(g) >= target
            while (lo < hi) {
                const int64_t mid = (lo + hi) / 2;
                if (cost_before(mid) >= target) hi = mid; else lo = mid + 1;
            }
            wb[w] = static_cast<int32_t>(lo);
        }
        wb[0] = 0;
        wb[W] = static_cast<int32_t>(T);
        for (int64_t w = 1; w < W; ++w) wb[w] = std::max<int32_t>(wb[w], wb[w - 1] + 1);
        for (int64_t w = W - 1; w >= 1; --w) wb[w] = std::min<int32_t>(wb[w], wb[w + 1] - 1);
    }
    {
        int u = 0;
        for (int64_t w = 0; w < W; ++w) {
            while (u < U && uoff[u + 1] <= wb[w]) ++u;
            wfu[w] = u;
        }
    }
    // pieces per unit
    std::vector<int32_t> ufw(U, 0), unp(U, 0), uslot(U, -1), tunits;
    auto worker_of = [&](int64_t g) {  // largest w with wb[w] <= g
        int64_t lo = 0, hi = W - 1;
        while (lo < hi) {
            const int64_t mid = (lo + hi + 1) / 2;
            if (wb[mid] <= g) lo = mid; else hi = mid - 1;
        }
        return static_cast<int32_t>(lo);
    };
    int slots = 0;
    for (int u = 0; u < U; ++u) {
        if (uoff[u + 1] == uoff[u]) continue;
        const int32_t f = worker_of(uoff[u]), l = worker_of(uoff[u + 1] - 1);
        ufw[u] = f;
        unp[u] = l - f + 1;
        pl->max_pieces = std::max(pl->max_pieces, unp[u]);
        if (unp[u] > 1) {
            uslot[u] = slots;
            slots += unp[u];
            if (unp[u] > pl->lmm) tunits.push_back(u);  // merged by dealt tasks
            else ++pl->last_merge_units;
        }
    }
    pl->slots = slots;
    // merge tasks: each split unit's G query heads in S groups, S as large as
    // the grid's warps allow (a power of two dividing G)
    {
        const int64_t nmulti = static_cast<int64_t>(tunits.size());
        const int64_t wtot = static_cast<int64_t>(pl->grid) * kPlanWarps;
        int S = 1;
        while (S * 2 <= G && G % (S * 2) == 0 && nmulti * S * 2 <= wtot) S *= 2;
        pl->S = S;
        pl->ntasks = static_cast<int>(nmulti * S);
    }

    // packed int32 tables
    auto& t = pl->tables;
    auto put = [&](const auto& v, size_t* off) {
        *off = t.size();
        for (auto x : v) t.push_back(static_cast<int32_t>(x));
        while (t.size() % 64) t.push_back(0);  // keep each array 256-byte aligned
    };
    put(std::vector<int32_t>{0}, &pl->o_hdr);
    put(wb, &pl->o_wb);
    put(wfu, &pl->o_wfu);
    std::vector<int32_t> uoff32(uoff.begin(), uoff.end());
    uoff32.push_back(uoff32.back() + 1);  // sentinel so the page iterator can run one unit past the end
    put(uoff32, &pl->o_uoff);
    put(ulen, &pl->o_ulen);
    put(ufw, &pl->o_ufw);
    put(unp, &pl->o_unp);
    put(uslot, &pl->o_uslot);
    put(tunits, &pl->o_tu);
    put(zunits, &pl->o_z);
    pl->tables_bytes = t.size() * sizeof(int32_t);
    pl->counters_off = align256(pl->tables_bytes);
    pl->part_o_off = align256(pl->counters_off + static_cast<size_t>(2 * U) * kCtrStride * sizeof(uint32_t));
    pl->part_lse_off = align256(pl->part_o_off + static_cast<size_t>(slots) * G * D * sizeof(float));
    pl->ws_bytes = align256(pl->part_lse_off + static_cast<size_t>(slots) * G * sizeof(float));
    *out_plan = pl;
    return VK_OK;
}

vk_status vk_decode_plan_destroy(vk_decode_plan* plan) {
    delete plan;
    return VK_OK;
}

size_t vk_decode_plan_workspace_size(const vk_decode_plan* plan) { return plan ? plan->ws_bytes : 0; }

vk_status vk_decode_plan_upload(const vk_decode_plan* plan, void* workspace, size_t workspace_bytes,
                                void* stream) {
    if (!plan || !workspace || workspace_bytes < plan->ws_bytes || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return fail(VK_INVALID_ARG, "workspace missing, too small or not 256-byte aligned");
    DeviceGuard g(plan->device);
    cudaStream_t st = as_stream(stream);
    // each upload with a gather bound starts a new step epoch (flag value)
    if (plan->gather) plan->tables[plan->o_hdr] = static_cast<int32_t>(gather_next_epoch(plan->gather));
    cudaError_t e = cudaMemcpyAsync(workspace, plan->tables.data(), plan->tables_bytes, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(plan tables)");
    if (plan->U > 0) {
        e = cudaMemsetAsync(static_cast<char*>(workspace) + plan->counters_off, 0,
                            static_cast<size_t>(2 * plan->U) * kCtrStride * sizeof(uint32_t), st);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(plan counters)");
    }
    return VK_OK;
}

vk_status vk_decode_plan_set_early_start(vk_decode_plan* plan, int32_t enable) {
    if (!plan) return fail(VK_INVALID_ARG, "plan is NULL");
    plan->early_start = enable != 0;
    return VK_OK;
}

vk_status vk_set_decode_workers(vk_pool* pool, int32_t max_workers) {
    if (!pool || max_workers < 0) return fail(VK_INVALID_ARG, "pool NULL or negative worker cap");
    pool->plan_workers = max_workers;
    return VK_OK;
}

vk_status vk_decode_plan_set_gather(vk_decode_plan* plan, vk_gather* g, int32_t slot_base, int32_t wait_prev) {
    if (!plan) return fail(VK_INVALID_ARG, "plan is NULL");
    if (slot_base < 0) return fail(VK_INVALID_ARG, "negative slot_base");
    if (g) {
        GatherView v;
        if (!gather_view(g, &v)) return fail(VK_INVALID_ARG, "gather has peers not imported");
        if (gather_device(g) != plan->device) return fail(VK_INVALID_ARG, "gather lives on another device");
        const uint64_t need = static_cast<uint64_t>(plan->B) * plan->Hq * plan->D * 2;
        if (v.slice_bytes < need) return fail(VK_INVALID_ARG, "gather slice smaller than the plan's [B, Hq, D] output");
    }
    plan->gather = g;
    plan->gather_slot_base = slot_base;
    plan->gather_wait_prev = g && wait_prev != 0;
    return VK_OK;
}

vk_status vk_decode_plan_gather_wait(const vk_decode_plan* plan, void* workspace, int32_t layer, void* stream) {
    if (!plan || !plan->gather || !workspace) return fail(VK_INVALID_ARG, "plan without a gather, or no workspace");
    GatherView gv;
    if (!gather_view(plan->gather, &gv)) return fail(VK_INVALID_ARG, "gather has peers not imported");
    if (layer < 0) return fail(VK_INVALID_ARG, "negative layer");
    const int slot = (plan->gather_slot_base + layer) % gv.slots;
    DeviceGuard g(plan->device);
    const uint32_t* epoch = reinterpret_cast<const uint32_t*>(static_cast<const int32_t*>(workspace) + plan->o_hdr);
    uint32_t* err = reinterpret_cast<uint32_t*>(gv.base[gv.rank] + gv.err_off);
    plan_gather_wait_kernel<<<1, 32, 0, as_stream(stream)>>>(gv, slot, epoch, err);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? VK_OK : cuda_fail(e, "plan_gather_wait_kernel launch");
}

int32_t vk_decode_plan_info(const vk_decode_plan* plan, int32_t what) {
    if (!plan) return -1;
    switch (what) {
        case 0: return plan->W;
        case 1: return plan->grid;
        case 2: return plan->slots;
        case 3: return plan->total_pages;
        case 4: return plan->max_unit_pages;
        case 5: return plan->lmm;
        case 6: return plan->last_merge_units;
        case 7: return plan->ntasks / plan->S;
        case 8: return plan->max_pieces;
        case 9: return plan->ntasks;
        default: return -1;
    }
}

vk_status vk_decode_run(vk_pool* pool, const vk_decode_plan* plan, int32_t layer, const void* q, void* out,
                        const int32_t* block_tables, int32_t bt_stride, const void* k_new, const void* v_new,
                        float scale, void* workspace, void* stream) {
    if (!pool || !plan) return fail(VK_INVALID_ARG, "pool or plan is NULL");
    if (!pool->kv || (pool->kv_format == VK_KV_FP16 && !pool->tmap_ok))
        return fail(VK_UNSUPPORTED, "decode needs a KV pool addressable by TMA");
    if (pool->cfg.head_dim != plan->D || pool->cfg.num_kv_heads != plan->Hkv || pool->device != plan->device ||
        pool->kv_format != plan->fmt)
        return fail(VK_INVALID_ARG, "plan was made for another pool shape, format or device");
    if (layer < 0 || layer >= pool->cfg.num_layers) return fail(VK_INVALID_ARG, "layer out of range");
    if (plan->B == 0) return VK_OK;
    GatherView gv{};
    if (plan->gather) {
        if (!gather_view(plan->gather, &gv)) return fail(VK_INVALID_ARG, "gather has peers not imported");
        if (out && (reinterpret_cast<uintptr_t>(out) & 15)) return fail(VK_INVALID_ARG, "out must be 16-byte aligned with a gather");
    } else if (!out) {
        return fail(VK_INVALID_ARG, "NULL out");
    }
    const int gslot = plan->gather ? (plan->gather_slot_base + layer) % gv.slots : -1;
    const bool out_own = plan->gather && !out;
    if (out_own) out = gv.base[gv.rank] + static_cast<uint64_t>(gslot) * gv.slot_bytes +
                       static_cast<uint64_t>(gv.rank) * gv.slice_bytes;
    if (!q || !block_tables || !workspace) return fail(VK_INVALID_ARG, "NULL array");
    if (bt_stride < plan->max_unit_pages) return fail(VK_INVALID_ARG, "block table narrower than the longest sequence");
    if ((k_new == nullptr) != (v_new == nullptr)) return fail(VK_INVALID_ARG, "give both k_new and v_new or neither");
    if (k_new && ((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new)) & 15))
        return fail(VK_INVALID_ARG, "k_new/v_new must be 16-byte aligned");
    if ((reinterpret_cast<uintptr_t>(q) & 3) || (reinterpret_cast<uintptr_t>(out) & 1) ||
        (reinterpret_cast<uintptr_t>(workspace) & 255))
        return fail(VK_INVALID_ARG, "misaligned q/out/workspace");
    const int D = plan->D;
    char* ws = static_cast<char*>(workspace);
    PlanParams p;
    const int32_t* t = reinterpret_cast<const int32_t*>(ws);
    p.wb = t + plan->o_wb;
    p.wfu = t + plan->o_wfu;
    p.uoff = t + plan->o_uoff;
    p.ulen = t + plan->o_ulen;
    p.ufw = t + plan->o_ufw;
    p.unp = t + plan->o_unp;
    p.uslot = t + plan->o_uslot;
    p.tunits = t + plan->o_tu;
    p.ntasks = plan->ntasks;
    p.S = plan->S;
    p.lmm = plan->lmm;
    p.rope_freq = pool->rope_freq;
    p.zunits = t + plan->o_z;
    p.counters = reinterpret_cast<uint32_t*>(ws + plan->counters_off);
    p.part_o = reinterpret_cast<float*>(ws + plan->part_o_off);
    p.part_lse = reinterpret_cast<float*>(ws + plan->part_lse_off);
    p.q = static_cast<const __half*>(q);
    p.out = static_cast<__half*>(out);
    p.k_new = static_cast<const __half*>(k_new);
    p.v_new = static_cast<const __half*>(v_new);
    p.bt = block_tables;
    p.err = pool->d_err;
    p.pool_base = pool->base;
    p.seg_bytes = pool->seg_bytes;
    p.layer_off = static_cast<uint64_t>(layer) * pool->seg_stride;
    p.head_bytes = pool->head_bytes;
    p.bt_stride = bt_stride;
    p.Hq = plan->Hq;
    p.Hkv = plan->Hkv;
    p.G = plan->G;
    p.L = pool->cfg.num_layers;
    p.layer = layer;
    p.num_pages = pool->num_pages;
    p.W = plan->W;
    p.Z = plan->Z;
    p.U = plan->U;
    p.g = gv;
    p.gslot = gslot;
    p.gepoch = reinterpret_cast<const uint32_t*>(t + plan->o_hdr);
    // run l > 0 signals run l-1's slot; layer 0 follows the previous step's
    // vk_decode_plan_gather_wait on the stream, which already waited
    p.gsig_slot = plan->gather && layer > 0 ? (gslot + gv.slots - 1) % gv.slots : -1;
    p.gwait_slot = plan->gather_wait_prev && layer > 0 ? (gslot + gv.slots - 1) % gv.slots : -1;
    p.out_own = out_own ? 1 : 0;
    const float sc = scale > 0.f ? scale : 1.0f / sqrtf(static_cast<float>(D));
    p.scale_log2 = sc * 1.4426950408889634f;
    if (plan->grid <= 0) return VK_OK;
    DeviceGuard g(pool->device);
    cudaStream_t st = as_stream(stream);
    int occ = 0;
    if (occupancy_for(D, plan->NT, plan->fmt, plan->ns, pool->device, &occ) != 0) return fail(VK_CUDA_ERROR, "kernel attribute setup failed");
    const dim3 grid(plan->grid), block(kPlanWarps * 32);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = plan->early_start ? 1 : 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t le = cudaSuccess;
#define VK_LAUNCH(DD, NN, FF, SS)                                                               \
    do {                                                                                        \
        cfg.dynamicSmemBytes = plan_smem_bytes<DD, FF, SS>();                                   \
        le = cudaLaunchKernelEx(&cfg, planned_decode_kernel<DD, NN, FF, SS>, pool->tmap, p);    \
    } while (0)
    constexpr int S4 = kPlanStages, S3 = kSmallStages;
    if (plan->fmt == VK_KV_FP8) { if (plan->NT == 1) VK_LAUNCH(128, 1, 1, S4); else VK_LAUNCH(128, 2, 1, S4); }
    else if (D == 128 && plan->ns == S3) { if (plan->NT == 1) VK_LAUNCH(128, 1, 0, S3); else VK_LAUNCH(128, 2, 0, S3); }
    else if (D == 128) { if (plan->NT == 1) VK_LAUNCH(128, 1, 0, S4); else VK_LAUNCH(128, 2, 0, S4); }
    else if (D == 64) { if (plan->NT == 1) VK_LAUNCH(64, 1, 0, S4); else VK_LAUNCH(64, 2, 0, S4); }
    else { if (plan->NT == 1) VK_LAUNCH(256, 1, 0, S4); else VK_LAUNCH(256, 2, 0, S4); }
#undef VK_LAUNCH
    if (le != cudaSuccess) return cuda_fail(le, "planned_decode_kernel launch");
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? VK_OK : cuda_fail(e, "planned_decode_kernel launch");
}

}  // extern "C"
