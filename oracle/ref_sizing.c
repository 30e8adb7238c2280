/*
 * Test infrastructure only: re-exports the reference engine's CUDA cache
 * sizing helpers, which are static functions of sf37.c compiled only with
 * SF37_USE_CUDA (sf37.c:2358-4446).  The translation unit is the reference's
 * own sf37.c built with that define; its sf37_cuda_* calls resolve against
 * _ref/libsf37ref_cuda.so (the reference's sf37_cuda.cu).  Only the pure
 * sizing functions are called; nothing here touches a GPU.
 *
 * Re-exported (reference file:line):
 *   cuda_sliding_cache_cap          sf37.c:3067-3081
 *   cuda_sliding_cache_prefill_cap  sf37.c:3083-3091
 *   cuda_decode_kv_bytes_for_cap    sf37.c:3093-3096
 *   layer_is_full                   sf37.c:1983-1985
 */
#define SF37_USE_CUDA 1
#include "sf37.c"

uint32_t sf37ref_sliding_cache_cap(uint32_t ctx_size, uint32_t prefill_cap) {
    return cuda_sliding_cache_cap(ctx_size, prefill_cap);
}
uint32_t sf37ref_sliding_prefill_cap(uint32_t ctx_size, uint32_t cache_cap) {
    return cuda_sliding_cache_prefill_cap(ctx_size, cache_cap);
}
uint64_t sf37ref_decode_kv_bytes_for_cap(uint32_t cap) { return cuda_decode_kv_bytes_for_cap(cap); }
int sf37ref_layer_is_full(uint32_t il) { return layer_is_full(il) ? 1 : 0; }
