// K3: chunked-prefill attention over the paged cache (placeholder until the
// tensor-core kernel lands).
#include "vk_internal.h"

using namespace vk;

extern "C" vk_status vk_prefill(vk_pool* pool, int32_t layer, const void* q, void* out,
                                const int32_t* block_tables, int32_t bt_stride,
                                const int32_t* positions, int32_t batch, int32_t tokens,
                                int32_t num_q_heads, float scale, void* stream) {
    (void)pool; (void)layer; (void)q; (void)out; (void)block_tables; (void)bt_stride;
    (void)positions; (void)batch; (void)tokens; (void)num_q_heads; (void)scale; (void)stream;
    return fail(VK_UNSUPPORTED, "prefill not built yet");
}
