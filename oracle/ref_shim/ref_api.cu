// C-linkage handles onto the reference library's own MemoryManager, KVCache,
// launch_attention and launch_matmul (cuda/memory.cu, src/kv_cache.cpp,
// cuda/attention.cu, cuda/matmul.cu), so
// GPU tests can run the reference implementation beside the new library.
// Test infrastructure only.  Note: the reference's CUDA_CHECK exits the
// process on a CUDA error.
#include "cuda/kernels.h"
#include "cuda/memory.h"
#include "vulcan/kv_cache.h"

using vulcan::KVCache;
using vulcan::cuda::MemoryManager;

extern "C" {

void* ref_mm_create(size_t page_size, int max_pages) { return new MemoryManager(page_size, max_pages); }
void ref_mm_destroy(void* m) { delete static_cast<MemoryManager*>(m); }
int ref_mm_allocate(void* m) { return static_cast<MemoryManager*>(m)->allocate_block(); }
void ref_mm_free(void* m, int id) { static_cast<MemoryManager*>(m)->free_block(id); }
void* ref_mm_ptr(void* m, int id) { return static_cast<MemoryManager*>(m)->get_block_ptr(id); }
int ref_mm_swap_to_cpu(void* m, int id) { return static_cast<MemoryManager*>(m)->swap_to_cpu(id) ? 1 : 0; }
int ref_mm_swap_to_gpu(void* m, int id) { return static_cast<MemoryManager*>(m)->swap_to_gpu(id) ? 1 : 0; }
int ref_mm_in_use(void* m) { return static_cast<MemoryManager*>(m)->blocks_in_use(); }
int ref_mm_available(void* m) { return static_cast<MemoryManager*>(m)->blocks_available(); }
size_t ref_mm_total_bytes(void* m) { return static_cast<MemoryManager*>(m)->total_allocated_bytes(); }

void* ref_kv_create(int heads, int max_seq, int head_dim, int layers) {
    return new KVCache(heads, max_seq, head_dim, layers);
}
void ref_kv_destroy(void* c) { delete static_cast<KVCache*>(c); }
void ref_kv_append(void* c, int layer, const float* k, const float* v, int start, int n) {
    static_cast<KVCache*>(c)->append(layer, k, v, start, n);
}
void ref_kv_get(void* c, int layer, const float** k, const float** v) {
    static_cast<KVCache*>(c)->get(layer, k, v);
}
int ref_kv_len(void* c) { return static_cast<KVCache*>(c)->current_length(); }
size_t ref_kv_memory(void* c) { return static_cast<KVCache*>(c)->memory_usage(); }

void ref_launch_attention(const float* Q, const float* K, const float* V, float* O, int b, int h,
                          int s, int d) {
    vulcan::cuda::launch_attention(Q, K, V, O, b, h, s, d);
}

void ref_launch_matmul(const float* A, const float* B, float* C, int m, int k, int n) {
    vulcan::cuda::launch_matmul(A, B, C, m, k, n);
}

}  // extern "C"
