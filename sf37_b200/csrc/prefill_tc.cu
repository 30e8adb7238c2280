// Tensor-core chunked prefill for f16 caches (placeholder until the tile
// kernel lands: reports "not handled" so the query-per-job path runs).
#include "kv_internal.cuh"

namespace sf37kv {

int prefill_tc(const sf37kv_cache *, const void *, int, const float *, float *, uint32_t, uint32_t,
               uint32_t, uint32_t, cudaStream_t, bool *handled) {
    *handled = false;
    return SF37KV_OK;
}

}  // namespace sf37kv
