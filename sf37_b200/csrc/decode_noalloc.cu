// Allocation-free decode entry point: sf37kv_decode_noalloc().
//
// Some callers cannot call cudaMalloc at the moment they decode: an engine
// running inside a host allocator or memory pool that owns every device
// byte (and treats any other allocation as a budget violation), a process
// whose allocations are frozen after start-up, or a latency-critical loop
// where a first-use cudaMalloc (which also synchronizes the device) is not
// acceptable.  sf37kv_decode() grows a scratch buffer with cudaMalloc when a
// bigger split-K plan needs it; this entry point instead keeps its split-K
// partials and counters in the fixed array below, which every GPU that loads
// the library holds until the process exits.
//
// Set-up: the first call on each device looks up the array's device address
// with cudaGetSymbolAddress while that device is current (the host-side name
// of a __device__ array is only a stand-in and must not be passed to a
// kernel).  Make that first call before any CUDA stream capture.
//
// Sharing: all calls on a device use the same array, which keeps the last
// call's contents; the split counters are cleared on the stream at the start
// of every call.  Calls that overlap on the GPU (different streams, or
// several host threads) race on the array: serialize them.
#include "kv_internal.cuh"

namespace sf37kv {

constexpr uint64_t kCounterBytes = 16384;  // 4096 split counters
static_assert(SF37KV_NOALLOC_SCRATCH_BYTES > kCounterBytes, "scratch too small");

static __device__ __align__(256) unsigned char g_noalloc_scratch[SF37KV_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
static void *g_noalloc_addr[kMaxDevices];

static int noalloc_scratch(void **out) {
    int dev = 0;
    if (int rc = check_cuda(cudaGetDevice(&dev), "decode_noalloc get device")) return rc;
    if (dev < 0 || dev >= kMaxDevices)
        return set_error(SF37KV_EUNSUPPORTED, "decode_noalloc: device %d out of range", dev);
    if (!g_noalloc_addr[dev]) {
        void *p = nullptr;
        if (int rc = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch),
                                "decode_noalloc cudaGetSymbolAddress"))
            return rc;
        g_noalloc_addr[dev] = p;
    }
    *out = g_noalloc_addr[dev];
    return SF37KV_OK;
}

}  // namespace sf37kv

using namespace sf37kv;

extern "C" int sf37kv_decode_noalloc(const sf37kv_decode_layer *layers, uint32_t n_layers,
                                     uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                                     int dtype, void *stream) {
    if (!layers && n_layers) return set_error(SF37KV_EINVAL, "decode_noalloc: layers is NULL");
    if (n_layers > (uint32_t)kMaxJobs)
        return set_error(SF37KV_EINVAL, "decode_noalloc: %u layers exceed the maximum of %d per call",
                         n_layers, kMaxJobs);
    cudaStream_t s = stream ? (cudaStream_t)stream : current_stream();
    // Every check runs before the first launch, so a rejected call leaves
    // the caches untouched.  The appended row is stored by the attention
    // kernel itself (the same pipelined kernels sf37kv_decode uses), so a
    // call is one counter clear plus one launch.
    AttnJob jobs[kMaxJobs];
    for (uint32_t i = 0; i < n_layers; i++) {
        const sf37kv_decode_layer &L = layers[i];
        if (L.cache.cap == 0) return set_error(SF37KV_EINVAL, "decode_noalloc: layer %u cap 0", i);
        if ((L.k_new != nullptr) != (L.v_new != nullptr))
            return set_error(SF37KV_EINVAL, "decode_noalloc: layer %u has only one of k_new/v_new", i);
        if (L.k_new && (((uintptr_t)L.k_new | (uintptr_t)L.v_new) & 15u))
            return set_error(SF37KV_EINVAL, "decode_noalloc: layer %u k_new/v_new must be 16-byte aligned", i);
        jobs[i] = AttnJob{L.cache.k_cache, L.cache.v_cache, L.q, L.gate, L.out,
                          start_at(L.pos, L.cache.cap, L.cache.sliding, L.cache.window), L.pos + 1u,
                          L.cache.cap, L.k_new, L.v_new};
    }
    void *scratch = nullptr;
    if (int rc = noalloc_scratch(&scratch)) return rc;
    unsigned char *base = static_cast<unsigned char *>(scratch);
    return attention_jobs_prealloc(jobs, n_layers, q_heads, kv_heads, head_dim, dtype, s,
                                   reinterpret_cast<float *>(base + kCounterBytes),
                                   SF37KV_NOALLOC_SCRATCH_BYTES - kCounterBytes,
                                   reinterpret_cast<uint32_t *>(base), kCounterBytes / 4u);
}
