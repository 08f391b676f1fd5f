// C++ facade with VULCAN's class and function names (include/vulcan/kv_cache.h,
// include/cuda/memory.h, include/cuda/kernels.h) implemented over the C ABI of
// this library.  Host code only; every device operation goes through vk_*.
//
// Error behaviour follows the reference where it has one (-1 / nullptr / false,
// silent return on a bad layer, a message on overflow) and otherwise prints the
// library's error string instead of exiting the process.
#include <cstdio>
#include <iostream>
#include <utility>

#include "cuda/kernels.h"
#include "cuda/memory.h"
#include "vk_internal.h"
#include "vulcan/kv_cache.h"

namespace {

int current_device() {
    int d = 0;
    cudaGetDevice(&d);
    return d;
}

void report(const char* what, vk_status s) {
    std::fprintf(stderr, "[VULCAN] %s: %s (%s)\n", what, vk_status_string(s), vk_last_error_string());
}

}  // namespace

namespace vulcan {

// ============================================================== KVCache

KVCache::KVCache(int num_kv_heads, int max_seq_len, int head_dim, int num_layers)
    : num_kv_heads_(num_kv_heads), max_seq_len_(max_seq_len), head_dim_(head_dim), num_layers_(num_layers) {
    const int pages = (max_seq_len + vk::kPageTokens - 1) / vk::kPageTokens;
    vk_pool_cfg cfg{};
    cfg.num_layers = num_layers;
    cfg.num_kv_heads = num_kv_heads;
    cfg.head_dim = head_dim;
    cfg.page_tokens = vk::kPageTokens;
    cfg.num_pages = pages > 0 ? pages : 1;
    cfg.device = current_device();
    vk_status s = vk_pool_create(&cfg, &pool_);
    if (s != VK_OK) {
        report("KVCache pool", s);
        pool_ = nullptr;
        return;
    }
    if (cudaMalloc(&d_block_table_, sizeof(int32_t) * cfg.num_pages) != cudaSuccess ||
        cudaMemset(d_block_table_, 0xff, sizeof(int32_t) * cfg.num_pages) != cudaSuccess ||
        cudaMalloc(&d_scalars_, sizeof(int32_t) * 2) != cudaSuccess) {
        std::fprintf(stderr, "[VULCAN] KVCache: device allocation failed\n");
        release();
    }
}

KVCache::~KVCache() { release(); }

void KVCache::release() {
    if (d_block_table_) cudaFree(d_block_table_);
    if (d_scalars_) cudaFree(d_scalars_);
    if (d_workspace_) cudaFree(d_workspace_);
    if (pool_) vk_pool_destroy(pool_);
    d_block_table_ = nullptr;
    d_scalars_ = nullptr;
    d_workspace_ = nullptr;
    workspace_bytes_ = 0;
    pool_ = nullptr;
    pages_.clear();
}

KVCache::KVCache(KVCache&& o) noexcept
    : num_kv_heads_(o.num_kv_heads_), max_seq_len_(o.max_seq_len_), head_dim_(o.head_dim_),
      num_layers_(o.num_layers_), current_len_(o.current_len_), pool_(o.pool_), d_block_table_(o.d_block_table_),
      d_scalars_(o.d_scalars_), d_workspace_(o.d_workspace_), workspace_bytes_(o.workspace_bytes_),
      pages_(std::move(o.pages_)) {
    o.pool_ = nullptr;
    o.d_block_table_ = nullptr;
    o.d_scalars_ = nullptr;
    o.d_workspace_ = nullptr;
    o.workspace_bytes_ = 0;
    o.current_len_ = 0;
}

KVCache& KVCache::operator=(KVCache&& o) noexcept {
    if (this != &o) {
        release();
        num_kv_heads_ = o.num_kv_heads_;
        max_seq_len_ = o.max_seq_len_;
        head_dim_ = o.head_dim_;
        num_layers_ = o.num_layers_;
        current_len_ = o.current_len_;
        pool_ = o.pool_;
        d_block_table_ = o.d_block_table_;
        d_scalars_ = o.d_scalars_;
        d_workspace_ = o.d_workspace_;
        workspace_bytes_ = o.workspace_bytes_;
        pages_ = std::move(o.pages_);
        o.pool_ = nullptr;
        o.d_block_table_ = nullptr;
        o.d_scalars_ = nullptr;
        o.d_workspace_ = nullptr;
        o.workspace_bytes_ = 0;
        o.current_len_ = 0;
    }
    return *this;
}

bool KVCache::ensure_pages(int tokens) {
    const int need = (tokens + vk::kPageTokens - 1) / vk::kPageTokens;
    const int have = static_cast<int>(pages_.size());
    if (need <= have) return true;
    std::vector<int32_t> ids(need - have);
    vk_status s = vk_alloc_pages(pool_, need - have, ids.data());
    if (s != VK_OK) {
        report("KVCache pages", s);
        return false;
    }
    pages_.insert(pages_.end(), ids.begin(), ids.end());
    return cudaMemcpy(d_block_table_ + have, ids.data(), sizeof(int32_t) * ids.size(), cudaMemcpyHostToDevice) ==
           cudaSuccess;
}

void KVCache::append(int layer, const float* k_new, const float* v_new, int start_pos, int num_tokens) {
    if (layer < 0 || layer >= num_layers_ || !pool_) return;  // src/kv_cache.cpp:86
    if (start_pos + num_tokens > max_seq_len_) {               // src/kv_cache.cpp:87-92
        std::cerr << "[VULCAN] KV Cache overflow: pos=" << start_pos << " + tokens=" << num_tokens
                  << " > max_seq=" << max_seq_len_ << std::endl;
        return;
    }
    if (num_tokens <= 0 || !ensure_pages(start_pos + num_tokens)) return;
    const int32_t pos = start_pos;
    if (cudaMemcpy(d_scalars_, &pos, sizeof pos, cudaMemcpyHostToDevice) != cudaSuccess) return;
    const int width = static_cast<int>((max_seq_len_ + vk::kPageTokens - 1) / vk::kPageTokens);
    vk_status s = vk_append_f32(pool_, layer, k_new, v_new, d_block_table_, width, d_scalars_, 1, num_tokens,
                                nullptr);
    if (s != VK_OK) {
        report("KVCache::append", s);
        return;
    }
    cudaStreamSynchronize(nullptr);
    if (start_pos + num_tokens > current_len_) current_len_ = start_pos + num_tokens;
}

void KVCache::get(int layer, const float** k_out, const float** v_out) const {
    if (layer < 0 || layer >= num_layers_ || !pool_) {
        *k_out = nullptr;
        *v_out = nullptr;
        return;
    }
    const uint64_t seg = static_cast<uint64_t>(num_kv_heads_) * 2 * vk::kPageTokens * head_dim_ * 2;
    const char* k = static_cast<const char*>(vk_pool_base(pool_)) + layer * seg * vk_pool_num_pages(pool_);
    *k_out = reinterpret_cast<const float*>(k);
    *v_out = reinterpret_cast<const float*>(k + static_cast<uint64_t>(vk::kPageTokens) * head_dim_ * 2);
}

int KVCache::current_length() const { return current_len_; }
void KVCache::set_length(int len) { current_len_ = len; }
void KVCache::reset() { current_len_ = 0; }
int KVCache::max_seq_len() const { return max_seq_len_; }

size_t KVCache::memory_usage() const {
    const size_t tokens = static_cast<size_t>((max_seq_len_ + vk::kPageTokens - 1) / vk::kPageTokens) * vk::kPageTokens;
    return 2ull * num_layers_ * num_kv_heads_ * tokens * head_dim_ * 2;
}

bool KVCache::decode(int layer, const void* q_f16, void* out_f16, int num_q_heads) {
    if (!pool_ || layer < 0 || layer >= num_layers_) return false;
    const int32_t len = current_len_;
    if (len > static_cast<int>(pages_.size()) * vk::kPageTokens) return false;
    if (cudaMemcpy(d_scalars_ + 1, &len, sizeof len, cudaMemcpyHostToDevice) != cudaSuccess) return false;
    const size_t need = vk_decode_workspace_size(pool_, 1, num_q_heads, max_seq_len_);
    if (need > workspace_bytes_) {
        if (d_workspace_) cudaFree(d_workspace_);
        d_workspace_ = nullptr;
        workspace_bytes_ = 0;
        if (cudaMalloc(&d_workspace_, need) != cudaSuccess) return false;
        workspace_bytes_ = need;
    }
    const int width = static_cast<int>((max_seq_len_ + vk::kPageTokens - 1) / vk::kPageTokens);
    vk_status s = vk_decode(pool_, layer, q_f16, out_f16, d_block_table_, width, d_scalars_ + 1, 1, num_q_heads,
                            max_seq_len_, 0.f, d_workspace_, workspace_bytes_, nullptr);
    if (s != VK_OK) {
        report("KVCache::decode", s);
        return false;
    }
    return cudaStreamSynchronize(nullptr) == cudaSuccess;
}

const int32_t* KVCache::block_table() const { return d_block_table_; }
vk_pool* KVCache::pool() const { return pool_; }

namespace cuda {

// ============================================================== GPUBuffer

GPUBuffer::GPUBuffer() : data_(nullptr), size_(0) {}

GPUBuffer::GPUBuffer(size_t size_bytes) : data_(nullptr), size_(size_bytes) {
    if (size_bytes > 0 && cudaMalloc(&data_, size_bytes) != cudaSuccess) {
        std::fprintf(stderr, "[VULCAN] GPUBuffer: cudaMalloc(%zu) failed\n", size_bytes);
        data_ = nullptr;
        size_ = 0;
    }
}

GPUBuffer::~GPUBuffer() {
    if (data_) cudaFree(data_);
}

GPUBuffer::GPUBuffer(GPUBuffer&& o) noexcept : data_(o.data_), size_(o.size_) {
    o.data_ = nullptr;
    o.size_ = 0;
}

GPUBuffer& GPUBuffer::operator=(GPUBuffer&& o) noexcept {
    if (this != &o) {
        if (data_) cudaFree(data_);
        data_ = o.data_;
        size_ = o.size_;
        o.data_ = nullptr;
        o.size_ = 0;
    }
    return *this;
}

void* GPUBuffer::data() { return data_; }
const void* GPUBuffer::data() const { return data_; }
size_t GPUBuffer::size() const { return size_; }
bool GPUBuffer::is_valid() const { return data_ != nullptr; }

void* GPUBuffer::release() {
    void* p = data_;
    data_ = nullptr;
    size_ = 0;
    return p;
}

// ============================================================== MemoryManager

MemoryManager::MemoryManager(size_t page_size, int max_pages) : page_size_(page_size), max_pages_(max_pages) {
    // Like the reference (cuda/memory.cu:84-104): on an allocation failure try
    // half as many pages until one fits.
    int pages = max_pages;
    while (pages > 0) {
        vk_pool_cfg cfg{};
        cfg.num_pages = pages;
        cfg.page_bytes = page_size;
        cfg.device = current_device();
        vk_status s = vk_pool_create(&cfg, &pool_);
        if (s == VK_OK) break;
        pool_ = nullptr;
        if (s != VK_CUDA_ERROR) break;
        cudaGetLastError();
        pages /= 2;
        if (pages > 0)
            std::fprintf(stderr, "[VULCAN] Warning: Reduced page pool to %d pages\n", pages);
    }
    max_pages_ = pool_ ? pages : 0;
    if (!pool_) std::fprintf(stderr, "[VULCAN] Error: Cannot allocate page pool.\n");
}

MemoryManager::~MemoryManager() {
    if (pool_) vk_pool_destroy(pool_);
    cpu_swap_.clear();
}

int MemoryManager::allocate_block() {
    int32_t id = -1;
    if (!pool_ || vk_alloc_pages(pool_, 1, &id) != VK_OK) return -1;
    return id;
}

void MemoryManager::free_block(int block_id) {
    if (!pool_) return;
    const int32_t id = block_id;
    vk_free_pages(pool_, &id, 1);
    if (block_id >= 0 && block_id < max_pages_) cpu_swap_.erase(block_id);
}

void* MemoryManager::get_block_ptr(int block_id) const { return pool_ ? vk_page_ptr(pool_, block_id) : nullptr; }

bool MemoryManager::swap_to_cpu(int block_id) {
    if (!pool_ || vk_page_in_use(pool_, block_id) != 1) return false;
    std::vector<uint8_t> buf(page_size_);
    const int32_t id = block_id;
    if (vk_swap_out(pool_, &id, 1, buf.data(), nullptr) != VK_OK) return false;
    if (cudaStreamSynchronize(nullptr) != cudaSuccess) return false;
    cpu_swap_[block_id] = std::move(buf);
    return true;
}

bool MemoryManager::swap_to_gpu(int block_id) {
    if (!pool_ || block_id < 0 || block_id >= max_pages_) return false;
    auto it = cpu_swap_.find(block_id);
    if (it == cpu_swap_.end()) return false;
    const int32_t id = block_id;
    if (vk_swap_in_to(pool_, it->second.data(), &id, 1, nullptr) != VK_OK) return false;
    if (cudaStreamSynchronize(nullptr) != cudaSuccess) return false;
    cpu_swap_.erase(it);
    return true;
}

int MemoryManager::blocks_in_use() const { return pool_ ? vk_pages_in_use(pool_) : 0; }
int MemoryManager::blocks_available() const { return pool_ ? vk_pages_available(pool_) : 0; }
size_t MemoryManager::total_allocated_bytes() const { return pool_ ? vk_allocated_bytes(pool_) : 0; }

// ============================================================== launch_attention

void launch_attention(const float* Q, const float* K, const float* V, float* output, int batch, int heads,
                      int seq_len, int head_dim) {
    vk_status s = vk_attention_f32(Q, K, V, output, batch, heads, seq_len, head_dim, nullptr);
    if (s != VK_OK) {
        report("launch_attention", s);
        return;
    }
    cudaError_t e = cudaStreamSynchronize(nullptr);
    if (e != cudaSuccess) std::fprintf(stderr, "[VULCAN] launch_attention: %s\n", cudaGetErrorString(e));
}

}  // namespace cuda
}  // namespace vulcan
