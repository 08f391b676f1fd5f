/*
 * vk_paged_kv.h — C ABI of the B200 paged KV-cache subsystem for VULCAN.
 *
 * One shared library (libvulcan_kv.so) exports every function declared here.
 * Signatures use plain pointers, integers and sizes only, so any FFI (ctypes,
 * cgo, JNI, N-API) can bind them.  Streams are passed as `void*` holding a
 * cudaStream_t (NULL = the legacy default stream).  Every device-side entry
 * point is asynchronous on the given stream and performs no implicit device
 * synchronisation; functions that must read device state say so.
 *
 * Memory layout of a KV pool (fp16, layer-major):
 *
 *   layer l, page p, kv head h, K-or-V kv, slot s, element d lives at byte
 *     base + l*layer_stride + p*seg_bytes + h*head_bytes
 *          + kv*(page_tokens*head_dim*2) + (s*head_dim + d)*2
 *   head_bytes   = 2 * page_tokens * head_dim * 2     (K block then V block)
 *   seg_bytes    = num_kv_heads * head_bytes          (one page, one layer)
 *   layer_stride = num_pages * seg_bytes              (one layer, all pages)
 *   page_bytes   = num_layers * seg_bytes             (one page, all layers)
 *
 * One block-table entry addresses a page in every layer.  One layer's pages
 * form one contiguous region, so a decode launch (one layer) touches a region
 * of num_pages*seg_bytes rather than the whole pool.  Swap and copy move a page
 * as num_layers strided segments; a host swap buffer holds page_bytes per page
 * with the page's layer segments in layer order.  A raw byte pool
 * (cfg.page_bytes != 0) is one contiguous page after another.
 *
 * Error convention: every function returns a vk_status (VK_OK = 0) and never
 * exits the process; vk_last_error_string() describes the last failure on the
 * calling thread.  Kernels that find a bad block-table entry, position or
 * sequence length skip the access and record a bit in the pool's device error
 * word; vk_pool_check() reads and clears it.
 */
#ifndef VK_PAGED_KV_H
#define VK_PAGED_KV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct vk_pool vk_pool;

typedef enum vk_status {
    VK_OK = 0,
    VK_INVALID_ARG = 1,      /* bad argument detected on the host              */
    VK_OUT_OF_PAGES = 2,     /* allocation could not be satisfied              */
    VK_CUDA_ERROR = 3,       /* a CUDA runtime call failed                     */
    VK_TIMEOUT = 4,          /* a bounded device-side wait gave up             */
    VK_BAD_BLOCK_TABLE = 5,  /* a kernel met an out-of-range page/position     */
    VK_NOT_FOUND = 6,        /* no such page / nothing swapped for this id     */
    VK_UNSUPPORTED = 7       /* shape or mode the library does not implement   */
} vk_status;

/* Device error-word bits reported by vk_pool_check(). */
#define VK_ERR_PAGE_ID      0x1  /* block-table entry outside [0, num_pages)     */
#define VK_ERR_TABLE_INDEX  0x2  /* position beyond the block table's capacity   */
#define VK_ERR_SEQ_LEN      0x4  /* sequence length < 0 or beyond capacity       */
#define VK_ERR_TIMEOUT      0x8  /* bounded mbarrier wait expired                */

typedef struct vk_pool_cfg {
    int32_t  num_layers;     /* L                                                */
    int32_t  num_kv_heads;   /* KV heads held by this pool (this GPU's shard)    */
    int32_t  head_dim;       /* D: 64, 128 or 256 for attention entry points     */
    int32_t  page_tokens;    /* tokens per page: 16 for attention entry points   */
    int32_t  num_pages;      /* physical pages                                   */
    int32_t  device;         /* CUDA device ordinal                              */
    uint64_t page_bytes;     /* 0: derived from the KV shape above.  Non-zero:   */
                             /* a raw byte-page pool (allocator, copy and swap   */
                             /* only), the MemoryManager(page_size, max_pages)   */
                             /* form; the KV shape fields are then ignored.      */
} vk_pool_cfg;

/* ---- pool lifetime --------------------------------------------------------
 * Replaces KVCache::KVCache / ~KVCache (src/kv_cache.cpp:23-53) and
 * MemoryManager::MemoryManager / ~MemoryManager (cuda/memory.cu:73-125):
 * one device allocation carved into fixed-size pages, zero-filled. */
vk_status vk_pool_create(const vk_pool_cfg* cfg, vk_pool** out_pool);

/* As vk_pool_create, but the pool lives in caller-owned device memory
 * (`bytes` >= num_pages*page_bytes, 256-byte aligned); the library neither
 * frees nor zero-fills it. */
vk_status vk_pool_create_in(const vk_pool_cfg* cfg, void* device_mem, size_t bytes,
                            vk_pool** out_pool);

/* ---- quantised KV pages ---------------------------------------------------
 * VK_KV_FP16: the fp16 layout above (vk_pool_create, vk_pool_create_in).
 * VK_KV_FP8: e4m3 codes with one fp32 scale per group of head_dim values (one
 * token's K or V row of one head), the group-wise symmetric format of the
 * reference's ADR-003 (docs/ADRs/003-quantization-format.md:11-18: scale =
 * max|group| / qmax, value = code * scale) with qmax = 448.  Each (layer,
 * page, head) block is 2*16*D + 128 bytes: K codes [16][D] with the 16-byte
 * chunks of token t's row rotated by XOR (t & 7), V codes [D][16] with the
 * tokens of a row in the order 0,1,8,9,2,3,10,11,4,5,12,13,6,7,14,15, then 16
 * K and 16 V scales.  head_dim 128 and page_tokens 16 only.  FP8 pools take
 * vk_append, vk_append_f32 (quantising), the planned decode (vk_decode_plan_*,
 * vk_decode_run, fused append included), vk_decode and vk_decode_static,
 * vk_prefill (the tcgen05 kernel with FP8-to-fp16 converter warps, or the
 * mma.sync kernel with prefill path 1), allocation,
 * copy and swap. */
#define VK_KV_FP16 0
#define VK_KV_FP8  1

/* vk_pool_create (device_mem NULL) or vk_pool_create_in (device_mem given)
 * with a page format; cfg->page_bytes must be 0. */
vk_status vk_pool_create_fmt(const vk_pool_cfg* cfg, int32_t kv_format, void* device_mem, size_t bytes,
                             vk_pool** out_pool);
/* VK_KV_FP16 or VK_KV_FP8; -1 for a byte-page pool or NULL. */
int32_t   vk_pool_kv_format(const vk_pool* pool);

vk_status vk_pool_destroy(vk_pool* pool);

/* Base device pointer, bytes per page and page count of the pool. */
void*    vk_pool_base(const vk_pool* pool);
uint64_t vk_pool_page_bytes(const vk_pool* pool);
int32_t  vk_pool_num_pages(const vk_pool* pool);

/* Reads (synchronously) and clears the pool's device error word.
 * VK_OK when it was zero, VK_BAD_BLOCK_TABLE or VK_TIMEOUT otherwise. */
vk_status vk_pool_check(vk_pool* pool, uint32_t* out_bits);

/* ---- page allocator (host side, not thread-safe, like the reference) ------
 * vk_alloc_pages replaces MemoryManager::allocate_block (cuda/memory.cu:127-135):
 * lowest free id first.  All-or-nothing: on VK_OUT_OF_PAGES no page is taken
 * and every out_ids[i] is set to -1 (the reference's -1 on exhaustion). */
vk_status vk_alloc_pages(vk_pool* pool, int32_t n, int32_t* out_ids);

/* MemoryManager::free_block (cuda/memory.cu:137-143): ids outside the pool or
 * already free are ignored.  (Host swap buffers belong to the caller, who drops
 * the copy of a freed id, as the reference's free_block does.) */
vk_status vk_free_pages(vk_pool* pool, const int32_t* ids, int32_t n);

/* MemoryManager::get_block_ptr (cuda/memory.cu:145-150): NULL on a bad id.
 * Byte pools: base + id*page_bytes.  KV pools: the page's layer-0 segment. */
void* vk_page_ptr(const vk_pool* pool, int32_t id);

/* MemoryManager::blocks_in_use / blocks_available / total_allocated_bytes
 * (cuda/memory.cu:193-207), O(1). */
int32_t  vk_pages_in_use(const vk_pool* pool);
int32_t  vk_pages_available(const vk_pool* pool);
uint64_t vk_allocated_bytes(const vk_pool* pool);
/* 1 if the id is allocated, 0 if free, -1 if outside the pool. */
int32_t  vk_page_in_use(const vk_pool* pool, int32_t id);

/* ---- K1: append ------------------------------------------------------------
 * Replaces KVCache::append (src/kv_cache.cpp:84-128).  Token t of sequence b
 * (position positions[b]+t) is written for every KV head to page
 * block_tables[b*bt_stride + pos/page_tokens], slot pos%page_tokens.
 * k_new, v_new: [batch, tokens, num_kv_heads, head_dim] fp16 device arrays
 * (token-major with heads interleaved, the reference's [T, Hkv*D]).
 * block_tables: int32 [batch, bt_stride]; positions: int32 [batch]. */
vk_status vk_append(vk_pool* pool, int32_t layer, const void* k_new, const void* v_new,
                    const int32_t* block_tables, int32_t bt_stride,
                    const int32_t* positions, int32_t batch, int32_t tokens,
                    void* stream);

/* As vk_append with fp32 inputs rounded to fp16 (round-to-nearest-even), the
 * element type of the reference's KVCache::append(const float*, ...). */
vk_status vk_append_f32(vk_pool* pool, int32_t layer, const float* k_new, const float* v_new,
                        const int32_t* block_tables, int32_t bt_stride,
                        const int32_t* positions, int32_t batch, int32_t tokens,
                        void* stream);

/* ---- K2: paged GQA decode (split-K + merge) --------------------------------
 * Replaces the decode use of launch_attention (cuda/attention.cu:38-131 as
 * called per head from src/transformer.cpp:157-189).  For sequence b and query
 * head h (KV head h / (num_q_heads/num_kv_heads)) it attends the first
 * seq_lens[b] cached tokens:
 *   out[b,h,:] = softmax_j(scale * q[b,h,:] . K_j) @ V
 * q, out: [batch, num_q_heads, head_dim] fp16.  seq_lens: int32 [batch] device
 * array (a length of 0 yields zeros).  max_seq_len (host) bounds every
 * seq_lens[b] and sizes the split-K schedule and workspace.
 * scale <= 0 selects 1/sqrt(head_dim), the reference's scale.
 * workspace: device scratch of at least vk_decode_workspace_size() bytes. */
size_t vk_decode_workspace_size(const vk_pool* pool, int32_t batch, int32_t num_q_heads,
                                int32_t max_seq_len);

vk_status vk_decode(vk_pool* pool, int32_t layer, const void* q, void* out,
                    const int32_t* block_tables, int32_t bt_stride,
                    const int32_t* seq_lens, int32_t batch, int32_t num_q_heads,
                    int32_t max_seq_len, float scale,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Pages per split-K chunk that vk_decode will use for this shape (0 if the
 * shape is invalid); vk_set_decode_split overrides it for the pool (0 = auto). */
int32_t   vk_decode_pages_per_split(const vk_pool* pool, int32_t batch, int32_t max_seq_len);
vk_status vk_set_decode_split(vk_pool* pool, int32_t pages_per_split);

/* ---- K2, planned: persistent load-balanced decode with fused append -------
 * The same computation as vk_decode (and the append of vk_append for one new
 * token per sequence), organised by a host-side plan.  A decode step's
 * sequence lengths are known on the host and are the same for every layer, so
 * the plan is built once per step:
 *   vk_decode_plan_create(pool, seq_lens_host, B, Hq, &plan)   host only
 *   vk_decode_plan_upload(plan, ws, ws_bytes, stream)          tables -> ws
 *   for each layer: vk_decode_run(pool, plan, layer, ...)      one launch
 * The plan cuts the pages of all (sequence, KV head) pairs into equal
 * contiguous ranges, one per resident warp of the GPU.  seq_lens_host[b] is
 * the number of tokens to attend, including the token being appended.
 * k_new, v_new: [B, Hkv, D] fp16 rows of the token at position
 * seq_lens_host[b]-1, written into the pool before it is read; pass NULL for
 * both to attend without appending.  The page receiving the new token must not
 * be shared with another sequence.  The workspace passed to vk_decode_run must
 * hold the uploaded plan; runs on it must not overlap on the GPU. */
typedef struct vk_decode_plan vk_decode_plan;

vk_status vk_decode_plan_create(const vk_pool* pool, const int32_t* seq_lens_host, int32_t batch,
                                int32_t num_q_heads, vk_decode_plan** out_plan);
vk_status vk_decode_plan_destroy(vk_decode_plan* plan);
size_t    vk_decode_plan_workspace_size(const vk_decode_plan* plan);
/* Copies the plan's tables into the workspace (256-byte aligned) and zeroes its
 * merge counters, asynchronously on `stream`. */
vk_status vk_decode_plan_upload(const vk_decode_plan* plan, void* workspace,
                                size_t workspace_bytes, void* stream);
/* Early start (programmatic dependent launch): when enabled, vk_decode_run's
 * grid may begin while the preceding kernel on the stream is still running; it
 * reads the plan tables, block tables and pool pages early, and waits for that
 * kernel to finish before it reads q, k_new, v_new or writes out and the merge
 * scratch.  Enable only when the preceding kernel writes none of the block
 * tables or pool pages this run reads (for example back-to-back layers of one
 * step).  Default off. */
vk_status vk_decode_plan_set_early_start(vk_decode_plan* plan, int32_t enable);

/* Caps the workers of plans made after the call (0 = one per resident warp,
 * the default); a tuning aid for small per-GPU shares. */
vk_status vk_set_decode_workers(vk_pool* pool, int32_t max_workers);

/* Plan facts: 0 workers, 1 CTAs, 2 partial slots, 3 total pages, 4 longest
 * sequence in pages, 5 most pieces of a unit that its last piece merges (1:
 * every split unit is merged by dealt tasks), 6 units merged by their last
 * piece, 7 units merged by dealt tasks, 8 most pieces of any unit, 9 merge
 * tasks; -1 for an unknown query. */
int32_t   vk_decode_plan_info(const vk_decode_plan* plan, int32_t what);
vk_status vk_decode_run(vk_pool* pool, const vk_decode_plan* plan, int32_t layer, const void* q,
                        void* out, const int32_t* block_tables, int32_t bt_stride,
                        const void* k_new, const void* v_new, float scale, void* workspace,
                        void* stream);

/* ---- Head-sharded output all-gather fused into the planned decode ---------
 * KV-head sharding over `world` GPUs of one node (one process per GPU): rank r
 * owns a contiguous block of KV heads and their query heads, and every rank
 * needs the whole [B, Hq, D] output of each layer.  Instead of a separate
 * collective, the planned decode bound to a gather stores each finished output
 * straight into every rank's receive buffer over NVLink (plain peer stores, no
 * multicast), and the next run on the stream, which starts only once this one
 * has completed, raises this rank's flag of the slot on every rank.
 *
 * Receive buffer of each rank: `slots` slots of [world][slice_bytes]; rank r's
 * slice of a slot holds its [B, Hq/world, D] fp16 output of one layer (the
 * layout ncclAllGather gives).  Setup (host):
 *   vk_gather_create(device, rank, world, slice_bytes, slots, &g)
 *   vk_gather_export(g, handle)            VK_GATHER_HANDLE_BYTES opaque bytes
 *   ... exchange handles between the ranks (any host transport) ...
 *   vk_gather_import(g, peer, peer_handle) for every peer != rank
 * Per step of L layers (same plan, one stream):
 *   vk_decode_plan_set_gather(plan, g, slot_base, wait_prev)
 *   vk_decode_plan_upload(...)                       starts a new step epoch
 *   vk_decode_run(layer 0), ..., vk_decode_run(layer L-1)
 *   vk_decode_plan_gather_wait(plan, ws, L-1, stream)
 * Run l writes slot (slot_base + l) % slots; run l > 0 raises the flags of run
 * l-1's slot, so the runs of a step must be issued in layer order on one
 * stream (other kernels may sit between them).  vk_decode_plan_gather_wait
 * raises the flags of its layer's slot (its run must precede it on the stream)
 * and makes the stream wait until all ranks' slices of that slot have arrived;
 * since every rank signals its slots in layer order, the wait on the last
 * layer covers the whole step.  With a gather bound, vk_decode_run's `out` may
 * be NULL (the rank's own slice of the slot is written), else it must be
 * 16-byte aligned and is written as well.  With wait_prev = 1, every run of a
 * layer l > 0 waits before it reads q, k_new or v_new until all ranks' slices
 * of layer l-1's slot have arrived (layer 0 follows the previous step's
 * vk_decode_plan_gather_wait): the order of a model whose next layer consumes
 * the gathered output; with wait_prev = 0 the gather of layer l overlaps layer l+1
 * (the order of an all-gather on a side stream).  Waits are bounded (1 s) and
 * record VK_ERR_TIMEOUT (vk_pool_check for runs, vk_gather_check for
 * vk_decode_plan_gather_wait); until that check clears it, later waits that
 * record into the same error word give up at once.  The library does not order a slot's reuse
 * against the readers of a receive buffer: callers rewrite a slot only after a
 * wait that follows its readers on every rank (for example slot_base 0 and L
 * on alternate steps of L layers, with 2L slots).  No reference counterpart:
 * the reference runs on one GPU. */
#define VK_GATHER_HANDLE_BYTES 64
typedef struct vk_gather vk_gather;

vk_status vk_gather_create(int32_t device, int32_t rank, int32_t world, uint64_t slice_bytes,
                           int32_t slots, vk_gather** out_gather);
/* Teardown in two phases: every rank calls vk_gather_release_peers (waits
 * for the device, closes its mappings of the peers' buffers), the ranks meet
 * at a host barrier, then each calls vk_gather_destroy (frees its own buffer,
 * which no peer maps any more).  vk_gather_destroy alone releases first. */
vk_status vk_gather_release_peers(vk_gather* g);
vk_status vk_gather_destroy(vk_gather* g);
vk_status vk_gather_export(const vk_gather* g, void* handle_out);
vk_status vk_gather_import(vk_gather* g, int32_t peer, const void* handle);
/* For a host that drives several ranks from one process (CUDA IPC cannot map
 * a buffer into the process that allocated it): rank `peer` is the gather
 * `peer_gather` of this process, on this device or another one with peer
 * access (enabled here).  Both must have the same world, slots and
 * slice_bytes, and peer_gather must be rank `peer`. */
vk_status vk_gather_import_local(vk_gather* g, int32_t peer, const vk_gather* peer_gather);
/* This rank's receive buffer of one slot: [world][slice_bytes] (NULL if bad). */
void*     vk_gather_buffer(const vk_gather* g, int32_t slot);
/* Synchronous: VK_TIMEOUT if a vk_decode_plan_gather_wait gave up since the
 * last check (timeouts inside vk_decode_run are reported by vk_pool_check). */
vk_status vk_gather_check(vk_gather* g);
/* Binds (g != NULL) or unbinds (g == NULL) a gather; slice_bytes must cover
 * the plan's [B, Hq, D] fp16 output, and every peer must be imported. */
vk_status vk_decode_plan_set_gather(vk_decode_plan* plan, vk_gather* g, int32_t slot_base,
                                    int32_t wait_prev);
vk_status vk_decode_plan_gather_wait(const vk_decode_plan* plan, void* workspace, int32_t layer,
                                     void* stream);

/* ---- output projection fused with its reduce-scatter -----------------------
 * The `wo` matmul after attention (reference src/transformer.cpp:191-194:
 * launch_matmul(attn_output, wo, output, T, hidden, hidden), cuda/matmul.cu:42-103,
 * C = A * B) for KV-head sharding over `world` GPUs.  Rank r holds x_r, the
 * attention output of its heads ([tokens, k_local] fp16: the [B, Hq/world, D]
 * decode output), and the same rows of wo; y = sum_r x_r * wo[rows of r].  A
 * run leaves on rank r the output features [r*n_out/world, (r+1)*n_out/world)
 * of y ([tokens, n_out/world] fp16, row stride ldy, a multiple of 4, y 8-byte
 * aligned): a reduce-scatter over
 * features in the same launch as the tcgen05 GEMM, partial tiles stored into
 * their owner's memory over NVLink as they finish (no NCCL call).  fp16 inputs,
 * fp32 accumulation and fp32 partial sums, summed in rank order.
 *
 * Weights: this rank's rows of wo, packed once (per model load) into the
 * kernel's layout, vk_oproj_packed_bytes(k_local, n_out) bytes: 16 KiB blocks
 * of 128 output features x 64 k, each in the 128-byte-swizzled order the
 * tensor cores read, so every pipeline stage streams one contiguous block.
 * vk_oproj_pack_weight packs the reference's fp32 wo rows ([k_rows, n], row
 * stride ldw); vk_oproj_pack_weight_t16 packs fp16 rows of wo transposed
 * ([n, k_rows], row stride ldw: an nn.Linear [out, in] weight or its column
 * slice for this rank).
 *
 * Setup mirrors the gather (vk_gather_*): create on every rank with the same
 * world, max_tokens, k_local and n_out; export / import the handles (or
 * import_local for ranks driven by one process).  Every rank makes the same
 * sequence of runs on one stream; runs wait for one another across ranks
 * (bounded, 1 s; vk_oproj_check reports VK_TIMEOUT), so all ranks must run.
 * Limits: max_tokens <= 256, k_local a multiple of 64, n_out a multiple of
 * 128 * world, n_out / 128 tiles resident at once (n_out <= 18,944 on a B200).
 * No reference counterpart for the collective: the reference runs on one GPU
 * (world = 1 is the plain projection). */
typedef struct vk_oproj vk_oproj;
vk_status vk_oproj_create(int32_t device, int32_t rank, int32_t world, int32_t max_tokens,
                          int32_t k_local, int32_t n_out, vk_oproj** out);
vk_status vk_oproj_export(const vk_oproj* h, void* handle_out);   /* VK_GATHER_HANDLE_BYTES */
vk_status vk_oproj_import(vk_oproj* h, int32_t peer, const void* handle);
vk_status vk_oproj_import_local(vk_oproj* h, int32_t peer, const vk_oproj* peer_h);
vk_status vk_oproj_release_peers(vk_oproj* h);
vk_status vk_oproj_destroy(vk_oproj* h);
/* k splits per tile the runs use (CTAs = n_out/128 * splits); -1 for NULL. */
int32_t   vk_oproj_splits(const vk_oproj* h);
vk_status vk_oproj_run(vk_oproj* h, const void* x, int32_t ldx, const void* w_packed,
                       void* y, int32_t ldy, int32_t tokens, void* stream);
/* Synchronous: VK_TIMEOUT if a run's wait gave up since the last check. */
vk_status vk_oproj_check(vk_oproj* h);
/* Bytes of a packed weight (0 unless k_rows % 64 == 0 and n % 128 == 0). */
size_t    vk_oproj_packed_bytes(int32_t k_rows, int32_t n);
vk_status vk_oproj_pack_weight(const float* w, int32_t ldw, int32_t k_rows, int32_t n, void* w_packed,
                               void* stream);
vk_status vk_oproj_pack_weight_t16(const void* w_t, int32_t ldw, int32_t n, int32_t k_rows,
                                   void* w_packed, void* stream);

/* ---- K3: chunked prefill -------------------------------------------------
 * The prefill use of launch_attention (src/transformer.cpp:136-189 with
 * num_tokens = chunk, src/engine.cpp:70-101): query token t of sequence b sits
 * at position positions[b]+t and attends cached keys 0..positions[b]+t
 * (causal).  The chunk's own K/V must already be appended.
 * q, out: [batch, tokens, num_q_heads, head_dim] fp16. */
vk_status vk_prefill(vk_pool* pool, int32_t layer, const void* q, void* out,
                     const int32_t* block_tables, int32_t bt_stride,
                     const int32_t* positions, int32_t batch, int32_t tokens,
                     int32_t num_q_heads, float scale, void* stream);

/* Fused RoPE (VULCAN's rope kernel, cuda/rope.cu:34-60, applied to Q and to
 * K_new before the append at src/transformer.cpp:114-128): with theta_base > 0
 * the pool's kernels rotate each pair (2i, 2i+1) by
 * pos / theta_base^(2i / head_dim) as they read it: vk_append and
 * vk_append_f32 rotate K rows at their positions (V unchanged); vk_decode and
 * vk_decode_run rotate q, and vk_decode_run its k_new, at the new token's
 * position seq_len - 1; vk_prefill rotates q at positions[b] + t.  Callers
 * then pass unrotated projections.  0 (the default) turns it off; head_dim
 * must be even. */
vk_status vk_set_rope(vk_pool* pool, float theta_base);

/* Selects the prefill kernel for the pool: 0 = automatic (the tcgen05/TMEM
 * kernel for head_dim 128, fp16 or FP8 pages; the mma.sync kernel otherwise),
 * 1 = the mma.sync kernel, 2 = the tcgen05 kernel (VK_UNSUPPORTED from
 * vk_prefill for other head dims). */
vk_status vk_set_prefill_path(vk_pool* pool, int32_t path);

/* ---- K4: page copy (fork / compaction; no reference counterpart) -----------
 * dst_ids[i] <- src_ids[i] byte-exactly, whole pages, every layer.  Both are
 * int32 device arrays of n ids; no id may appear in both arrays. */
vk_status vk_copy_pages(vk_pool* pool, const int32_t* src_ids, const int32_t* dst_ids,
                        int32_t n, void* stream);

/* Rewrites block-table entries through a page-id map: every entry e with
 * 0 <= e < map_len becomes page_map[e].  block_tables: int32 device array of
 * `entries` ids; page_map: int32 device array. */
vk_status vk_remap_block_tables(int32_t* block_tables, int64_t entries,
                                const int32_t* page_map, int32_t map_len, void* stream);

/* Host-side compaction plan: moves the highest in-use pages into the lowest
 * free ids so that in-use ids become 0..in_use-1.  Writes up to `cap` (src,
 * dst) pairs, their count to *out_n, and updates the allocator (dst in use,
 * src free).  Follow with vk_copy_pages and vk_remap_block_tables. */
vk_status vk_compact_plan(vk_pool* pool, int32_t* src_ids, int32_t* dst_ids, int32_t cap,
                          int32_t* out_n);

/* ---- K5: pinned-host swap -------------------------------------------------
 * MemoryManager::swap_to_cpu (cuda/memory.cu:152-169): copies pages ids[0..n)
 * into host_buf (page i at host_buf + i*page_bytes, its layer segments in layer
 * order; page-locked memory for an asynchronous copy) on `stream`, then frees
 * the ids.  The ids may be handed
 * out again at once; work that writes them must be ordered after `stream`. */
vk_status vk_swap_out(vk_pool* pool, const int32_t* ids, int32_t n, void* host_buf,
                      void* stream);

/* MemoryManager::swap_to_gpu (cuda/memory.cu:171-191), batched: allocates n
 * new pages (lowest free ids, written to out_ids) and copies host_buf into them
 * on `stream`.  The new ids may differ from the swapped-out ones; callers
 * rewrite their block tables with them. */
vk_status vk_swap_in(vk_pool* pool, const void* host_buf, int32_t n, int32_t* out_ids,
                     void* stream);

/* Swap-in into the given ids, which must be free (the reference's same-id
 * swap_to_gpu).  VK_INVALID_ARG if any id is in use or out of range. */
vk_status vk_swap_in_to(vk_pool* pool, const void* host_buf, const int32_t* ids, int32_t n,
                        void* stream);

/* ---- compatibility entry: contiguous fp32 causal attention ----------------
 * Same contract as vulcan::cuda::launch_attention (cuda/attention.cu:119-131,
 * include/cuda/kernels.h:99-101): Q, K, V, O are [batch, heads, seq_len,
 * head_dim] fp32 device arrays; row i attends keys 0..i; scale 1/sqrt(D).
 * Asynchronous on `stream` (the reference synchronises after each launch). */
vk_status vk_attention_f32(const float* Q, const float* K, const float* V, float* O,
                           int32_t batch, int32_t heads, int32_t seq_len, int32_t head_dim,
                           void* stream);

/* ---- decode without any device allocation ---------------------------------
 * No counterpart in the reference.  Same computation and result as vk_decode
 * (it runs vk_decode with the same split-K schedule), but the split-K scratch
 * comes from a fixed array compiled into the library instead of a caller
 * workspace.  It is meant for callers that cannot allocate device memory: a
 * host engine or plugin framework that owns all device memory and hands an
 * operator only its inputs and outputs, a serving loop that must not call
 * cudaMalloc (which can synchronise the device), or an FFI host (cgo, JNI)
 * with no CUDA allocator.  The caller still passes q, out, block tables and
 * lengths.
 *
 * Limit: the shape must need at most VK_DECODE_STATIC_SCRATCH_BYTES of scratch
 * (vk_decode_workspace_size() for the same arguments); larger shapes return
 * VK_INVALID_ARG with a message, and nothing is launched.  The array is part
 * of the library's device code: under CUDA's default lazy module loading a
 * GPU holds it from this entry point's first call there until the process
 * exits; with CUDA_MODULE_LOADING=EAGER every GPU on which the process creates
 * a context holds it, whether it calls this entry point or not.
 *
 * The first call on a device looks up the array's device address (once per
 * device, with that device current) and keeps it for the life of the
 * process; make that first call before any stream capture.  After
 * cudaDeviceReset on a device (which unloads the library's device code there)
 * do not call this entry point on that device again.  All calls on a device share the one array and it keeps the last
 * call's contents; nothing in it needs to start at zero, because every split
 * writes its partial result before the merge reads it.  Calls that overlap on
 * the GPU (different streams, or concurrent host threads) race on the array:
 * order them on one stream.  The function never calls cudaMalloc, cudaFree or
 * any allocating library routine. */
#define VK_DECODE_STATIC_SCRATCH_BYTES (32u << 20)

vk_status vk_decode_static(vk_pool* pool, int32_t layer, const void* q, void* out,
                           const int32_t* block_tables, int32_t bt_stride,
                           const int32_t* seq_lens, int32_t batch, int32_t num_q_heads,
                           int32_t max_seq_len, float scale, void* stream);

/* ---- diagnostics ----------------------------------------------------------- */
const char* vk_last_error_string(void);
const char* vk_status_string(vk_status s);
/* Library version as major*10000 + minor*100 + patch. */
int32_t vk_version(void);

#ifdef __cplusplus
}
#endif

#endif /* VK_PAGED_KV_H */
