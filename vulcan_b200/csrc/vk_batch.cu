// vulcan::PagedAttention (include/vulcan/paged_attention.h): the multi-sequence
// attention step an engine calls from TransformerBlock::self_attention's place
// (reference src/transformer.cpp:130-189, driven by src/engine.cpp:70-127).
// Host code over the C ABI; every device operation goes through vk_*.
#include <cstdio>
#include <utility>

#include "vk_internal.h"
#include "vulcan/paged_attention.h"

namespace {

void report(const char* what, vk_status s) {
    std::fprintf(stderr, "[VULCAN] %s: %s (%s)\n", what, vk_status_string(s), vk_last_error_string());
}

bool fail_msg(const char* what) {
    std::fprintf(stderr, "[VULCAN] PagedAttention: %s\n", what);
    return false;
}

}  // namespace

namespace vulcan {

PagedAttention::PagedAttention(const PagedAttentionConfig& cfg) : cfg_(cfg) {
    if (cfg.num_heads <= 0 || cfg.num_kv_heads <= 0 || cfg.num_heads % cfg.num_kv_heads || cfg.head_dim <= 0 ||
        cfg.num_layers <= 0 || cfg.max_seq_len <= 0 || cfg.max_sequences <= 0 || cfg.num_pages <= 0) {
        fail_msg("bad configuration");
        return;
    }
    if (cfg_.device < 0 && cudaGetDevice(&cfg_.device) != cudaSuccess) {
        fail_msg("no current CUDA device");
        return;
    }
    width_ = (cfg.max_seq_len + vk::kPageTokens - 1) / vk::kPageTokens;
    vk_pool_cfg pc{};
    pc.num_layers = cfg.num_layers;
    pc.num_kv_heads = cfg.num_kv_heads;
    pc.head_dim = cfg.head_dim;
    pc.page_tokens = vk::kPageTokens;
    pc.num_pages = cfg.num_pages;
    pc.device = cfg_.device;
    vk_status s = vk_pool_create_fmt(&pc, cfg.fp8_pages ? VK_KV_FP8 : VK_KV_FP16, nullptr, 0, &pool_);
    if (s != VK_OK) {
        report("PagedAttention pool", s);
        pool_ = nullptr;
        return;
    }
    if (cfg.rope_theta > 0.f && (s = vk_set_rope(pool_, cfg.rope_theta)) != VK_OK) {
        report("PagedAttention RoPE", s);
        release();
        return;
    }
    vk::DeviceGuard g(cfg_.device);
    const size_t tb = sizeof(int32_t) * static_cast<size_t>(cfg.max_sequences) * width_;
    if (cudaMalloc(&d_tables_, tb) != cudaSuccess || cudaMemset(d_tables_, 0xff, tb) != cudaSuccess ||
        cudaMalloc(&d_positions_, sizeof(int32_t) * cfg.max_sequences) != cudaSuccess) {
        fail_msg("device allocation failed");
        release();
        return;
    }
    seq_pages_.assign(cfg.max_sequences, {});
    seq_len_.assign(cfg.max_sequences, -1);
}

PagedAttention::~PagedAttention() { release(); }

void PagedAttention::release() {
    if (plan_) vk_decode_plan_destroy(plan_);
    if (d_tables_ || d_positions_ || d_ws_) {
        vk::DeviceGuard g(cfg_.device);
        if (d_tables_) cudaFree(d_tables_);
        if (d_positions_) cudaFree(d_positions_);
        if (d_ws_) cudaFree(d_ws_);
    }
    if (pool_) vk_pool_destroy(pool_);
    plan_ = nullptr;
    d_tables_ = nullptr;
    d_positions_ = nullptr;
    d_ws_ = nullptr;
    ws_bytes_ = 0;
    pool_ = nullptr;
    seq_pages_.clear();
    seq_len_.clear();
    step_ids_.clear();
    in_step_ = false;
}

PagedAttention::PagedAttention(PagedAttention&& o) noexcept { *this = std::move(o); }

PagedAttention& PagedAttention::operator=(PagedAttention&& o) noexcept {
    if (this != &o) {
        release();
        cfg_ = o.cfg_;
        width_ = o.width_;
        pool_ = std::exchange(o.pool_, nullptr);
        d_tables_ = std::exchange(o.d_tables_, nullptr);
        d_positions_ = std::exchange(o.d_positions_, nullptr);
        d_ws_ = std::exchange(o.d_ws_, nullptr);
        ws_bytes_ = std::exchange(o.ws_bytes_, 0);
        plan_ = std::exchange(o.plan_, nullptr);
        seq_pages_ = std::move(o.seq_pages_);
        seq_len_ = std::move(o.seq_len_);
        step_ids_ = std::move(o.step_ids_);
        step_tokens_ = o.step_tokens_;
        in_step_ = std::exchange(o.in_step_, false);
        stream_ = o.stream_;
    }
    return *this;
}

bool PagedAttention::ok() const { return pool_ != nullptr; }

int PagedAttention::add_sequence() {
    for (size_t i = 0; i < seq_len_.size(); ++i)
        if (seq_len_[i] < 0) {
            seq_len_[i] = 0;
            seq_pages_[i].clear();
            return static_cast<int>(i);
        }
    return -1;
}

bool PagedAttention::release_sequence(int id) {
    if (id < 0 || id >= static_cast<int>(seq_len_.size()) || seq_len_[id] < 0) return false;
    if (in_step_)
        for (int s : step_ids_)
            if (s == id) return fail_msg("release_sequence during a step that includes it");
    auto& pg = seq_pages_[id];
    if (!pg.empty()) {
        vk_status s = vk_free_pages(pool_, pg.data(), static_cast<int32_t>(pg.size()));
        if (s != VK_OK) {
            report("PagedAttention free", s);
            return false;
        }
    }
    pg.clear();
    seq_len_[id] = -1;
    return true;
}

int PagedAttention::length(int id) const {
    return id < 0 || id >= static_cast<int>(seq_len_.size()) ? -1 : seq_len_[id];
}

int PagedAttention::pages_available() const { return pool_ ? vk_pages_available(pool_) : 0; }

bool PagedAttention::begin_step(const std::vector<int>& ids, int tokens, void* stream) {
    if (!pool_) return fail_msg("not constructed");
    if (in_step_) return fail_msg("begin_step inside a step");
    if (ids.empty() || tokens <= 0) return fail_msg("a step needs sequences and tokens > 0");
    const int B = static_cast<int>(ids.size());
    std::vector<char> seen(seq_len_.size(), 0);
    int64_t need = 0;
    for (int id : ids) {
        if (id < 0 || id >= static_cast<int>(seq_len_.size()) || seq_len_[id] < 0 || seen[id])
            return fail_msg("unknown or repeated sequence id");
        seen[id] = 1;
        const int64_t len = static_cast<int64_t>(seq_len_[id]) + tokens;
        if (len > cfg_.max_seq_len) return fail_msg("a sequence would exceed max_seq_len");
        need += (len + vk::kPageTokens - 1) / vk::kPageTokens - static_cast<int64_t>(seq_pages_[id].size());
    }
    // pages for the new tokens, all or nothing
    std::vector<int32_t> fresh(static_cast<size_t>(need));
    if (need > 0) {
        vk_status s = vk_alloc_pages(pool_, static_cast<int32_t>(need), fresh.data());
        if (s != VK_OK) {
            report("PagedAttention pages", s);
            return false;
        }
    }
    size_t next = 0;
    std::vector<int32_t> table(static_cast<size_t>(B) * width_, -1), pos(B), lens(B);
    for (int b = 0; b < B; ++b) {
        const int id = ids[b];
        const int len = seq_len_[id] + tokens;
        auto& pg = seq_pages_[id];
        while (static_cast<int>(pg.size()) * vk::kPageTokens < len) pg.push_back(fresh[next++]);
        std::copy(pg.begin(), pg.end(), table.begin() + static_cast<size_t>(b) * width_);
        pos[b] = seq_len_[id];
        lens[b] = len;
    }
    vk::DeviceGuard g(cfg_.device);
    cudaStream_t st = vk::as_stream(stream);
    // pageable sources: each copy has read its host buffer when the call returns
    cudaError_t e = cudaMemcpyAsync(d_tables_, table.data(), sizeof(int32_t) * table.size(), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(d_positions_, pos.data(), sizeof(int32_t) * B, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) {
        std::fprintf(stderr, "[VULCAN] PagedAttention: %s\n", cudaGetErrorString(e));
        return false;
    }
    if (plan_) {
        vk_decode_plan_destroy(plan_);
        plan_ = nullptr;
    }
    if (tokens == 1) {
        vk_status s = vk_decode_plan_create(pool_, lens.data(), B, cfg_.num_heads, &plan_);
        if (s != VK_OK) {
            report("PagedAttention plan", s);
            return false;
        }
        const size_t bytes = vk_decode_plan_workspace_size(plan_);
        if (bytes > ws_bytes_) {
            // the old workspace may still be read by earlier launches on the stream
            if (d_ws_ && (e = cudaStreamSynchronize(st)) == cudaSuccess) e = cudaFree(d_ws_);
            d_ws_ = nullptr;
            ws_bytes_ = 0;
            if (e == cudaSuccess) e = cudaMalloc(&d_ws_, bytes);
            if (e != cudaSuccess) {
                std::fprintf(stderr, "[VULCAN] PagedAttention workspace: %s\n", cudaGetErrorString(e));
                d_ws_ = nullptr;
                return false;
            }
            ws_bytes_ = bytes;
        }
        s = vk_decode_plan_upload(plan_, d_ws_, ws_bytes_, stream);
        if (s != VK_OK) {
            report("PagedAttention plan upload", s);
            return false;
        }
    }
    step_ids_ = ids;
    step_tokens_ = tokens;
    stream_ = stream;
    in_step_ = true;
    return true;
}

bool PagedAttention::attend(int layer, const void* q, const void* k_new, const void* v_new, void* out) {
    if (!in_step_) return fail_msg("attend outside a step");
    const int B = static_cast<int>(step_ids_.size());
    vk_status s;
    if (step_tokens_ == 1) {
        s = vk_decode_run(pool_, plan_, layer, q, out, d_tables_, width_, k_new, v_new, 0.f, d_ws_, stream_);
        if (s != VK_OK) report("PagedAttention decode", s);
        return s == VK_OK;
    }
    s = vk_append(pool_, layer, k_new, v_new, d_tables_, width_, d_positions_, B, step_tokens_, stream_);
    if (s != VK_OK) {
        report("PagedAttention append", s);
        return false;
    }
    s = vk_prefill(pool_, layer, q, out, d_tables_, width_, d_positions_, B, step_tokens_, cfg_.num_heads, 0.f,
                   stream_);
    if (s != VK_OK) report("PagedAttention prefill", s);
    return s == VK_OK;
}

bool PagedAttention::end_step() {
    if (!in_step_) return fail_msg("end_step outside a step");
    for (int id : step_ids_) seq_len_[id] += step_tokens_;
    in_step_ = false;
    return true;
}

vk_pool* PagedAttention::pool() const { return pool_; }
const int32_t* PagedAttention::block_tables() const { return d_tables_; }
int PagedAttention::block_table_width() const { return width_; }

std::vector<int32_t> PagedAttention::pages(int id) const {
    if (id < 0 || id >= static_cast<int>(seq_len_.size()) || seq_len_[id] < 0) return {};
    return seq_pages_[id];
}

}  // namespace vulcan
