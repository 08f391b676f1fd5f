#pragma once

// vulcan::cuda::GPUBuffer and MemoryManager over the B200 paged KV-cache
// library (libvulcan_kv.so).  Same names, signatures and return conventions as
// VULCAN's include/cuda/memory.h:18-128: allocate_block returns -1 when the
// pool is full, get_block_ptr returns nullptr for a bad id, swap_* return false
// on failure, and free_block drops a swapped-out copy of the id.  Pages live in
// one device allocation (contiguous, page_size apart); the allocator is O(1)
// per call and hands out the lowest free id first, as the reference's scan does.
//
// Difference: swap_to_gpu refuses (returns false) an id that was reallocated
// after its swap-out; the reference would overwrite the new owner's data.

#include <cstddef>
#include <cstdint>
#include <unordered_map>
#include <vector>

struct vk_pool;

namespace vulcan {
namespace cuda {

class GPUBuffer {
public:
    GPUBuffer();
    explicit GPUBuffer(size_t size_bytes);
    ~GPUBuffer();

    GPUBuffer(GPUBuffer&& other) noexcept;
    GPUBuffer& operator=(GPUBuffer&& other) noexcept;
    GPUBuffer(const GPUBuffer&) = delete;
    GPUBuffer& operator=(const GPUBuffer&) = delete;

    void* data();
    const void* data() const;

    template <typename T>
    T* as() { return static_cast<T*>(data_); }

    template <typename T>
    const T* as() const { return static_cast<const T*>(data_); }

    size_t size() const;
    bool is_valid() const;

    /// Releases ownership; the caller must cudaFree the pointer.
    void* release();

private:
    void* data_;
    size_t size_;
};

constexpr size_t DEFAULT_PAGE_SIZE = 16 * 1024;

struct MemoryBlock {
    void* ptr;
    size_t size;
    bool in_use;
    int block_id;
};

class MemoryManager {
public:
    explicit MemoryManager(size_t page_size = DEFAULT_PAGE_SIZE, int max_pages = 1024);
    ~MemoryManager();

    MemoryManager(const MemoryManager&) = delete;
    MemoryManager& operator=(const MemoryManager&) = delete;

    int allocate_block();
    void free_block(int block_id);
    void* get_block_ptr(int block_id) const;
    bool swap_to_cpu(int block_id);
    bool swap_to_gpu(int block_id);

    int blocks_in_use() const;
    int blocks_available() const;
    size_t total_allocated_bytes() const;

    /// The underlying pool handle, for the C ABI.
    vk_pool* pool() const { return pool_; }

private:
    size_t page_size_;
    int max_pages_;
    vk_pool* pool_ = nullptr;
    std::unordered_map<int, std::vector<uint8_t>> cpu_swap_;
};

}  // namespace cuda
}  // namespace vulcan
