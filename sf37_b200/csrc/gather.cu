// Multi-GPU output gather over peer memory (KV-head sharding).
//
// GPU r of N owns KV heads [r*K/N, (r+1)*K/N) of every layer.  Instead of a
// separate all-gather after the decode kernel, the decode kernel's epilogue
// stores each final output directly into the gather buffer of every rank
// (plain NVLink stores to CUDA-IPC-mapped buffers, layout
// [epoch & 1][rank][layer][q_heads_local][head_dim]) and the last (layer, KV head) group
// of the launch raises this rank's step epoch in every rank's flag array.
// sf37kv_gather_wait() then waits -- bounded, on this GPU -- until all ranks'
// flags reach the epoch, after which the local buffer holds every head.
// Two halves alternate by epoch parity: a rank can run at most one step ahead
// of any other (it waits for everyone's flag of the previous epoch), so the
// half it writes was consumed by every reader before that reader's own
// previous decode launch (stream order).
#include <algorithm>
#include <cstring>

#include "kv_internal.cuh"

namespace sf37kv {

extern unsigned long long g_launches;

// Launched with programmatic stream serialization right behind the decode
// kernel (which triggers its dependents at its start), so it is resident and
// polling while the decode runs.  It returns only after griddepcontrol.wait,
// i.e. after the decode kernel has completed, so work after it on the stream
// sees a finished step.  It triggers its own dependents at once: the next
// step's decode CTAs then launch into free SMs and wait in their own
// griddepcontrol.wait for this kernel, hiding that launch (measured at 8
// GPUs: 150 -> 147-149 us per step).
__global__ void gather_wait_kernel(const uint32_t *flags, uint32_t world, uint32_t epoch, int *err) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const uint32_t p = threadIdx.x;
    bool ok = true;
    if (p < world) {
        const long long t0 = clock64();
        for (;;) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + p) : "memory");
            if ((int32_t)(v - epoch) >= 0) break;
            if (clock64() - t0 > 4000000000ll) {  // about 2 s: a peer never finished
                ok = false;
                break;
            }
            __nanosleep(200);
        }
    }
    if (!ok) atomicExch(err, 2);
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

}  // namespace sf37kv

using namespace sf37kv;

extern "C" void *sf37kv_dev_alloc(uint64_t bytes) {
    void *p = nullptr;
    if (check_cuda(cudaMalloc(&p, bytes ? bytes : 1), "device alloc")) return nullptr;
    if (check_cuda(cudaMemset(p, 0, bytes ? bytes : 1), "device alloc clear")) {
        cudaFree(p);
        return nullptr;
    }
    return p;
}

extern "C" void sf37kv_dev_free(void *p) {
    if (p) cudaFree(p);
}

extern "C" int sf37kv_ipc_handle(void *dev_ptr, void *handle_out) {
    cudaIpcMemHandle_t h;
    if (int rc = check_cuda(cudaIpcGetMemHandle(&h, dev_ptr), "ipc get handle")) return rc;
    memcpy(handle_out, &h, sizeof(h));
    return SF37KV_OK;
}

extern "C" void *sf37kv_ipc_open(const void *handle) {
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void *p = nullptr;
    if (check_cuda(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "ipc open")) return nullptr;
    return p;
}

extern "C" void sf37kv_ipc_close(void *p) {
    if (p) cudaIpcCloseMemHandle(p);
}

namespace sf37kv {
int gather_dev(const sf37kv_peer_gather *g, uint32_t epoch, GatherDev *d) {
    if (!g || g->world < 1 || g->world > 8 || g->rank >= g->world)
        return set_error(SF37KV_EINVAL, "gather: world must be 1..8 and rank < world");
    memset(d, 0, sizeof(*d));
    for (uint32_t p = 0; p < g->world; p++) {
        if (!g->peer_buf[p] || !g->peer_flags[p])
            return set_error(SF37KV_EINVAL, "gather: peer %u buffer is NULL", p);
        d->peer[p] = (float *)g->peer_buf[p];
        d->peer_flags[p] = (uint32_t *)g->peer_flags[p];
    }
    d->world = g->world;
    d->rank = g->rank;
    d->epoch = epoch;
    d->done = (uint32_t *)g->done_counter;
    if (!d->done) return set_error(SF37KV_EINVAL, "gather: done_counter is NULL");
    return SF37KV_OK;
}
}  // namespace sf37kv

extern "C" int sf37kv_decode_gather(const sf37kv_decode_layer *layers, uint32_t n_layers, uint32_t q_heads,
                                    uint32_t kv_heads, uint32_t head_dim, int dtype,
                                    const sf37kv_peer_gather *g, uint32_t epoch, void *stream) {
    if (!layers && n_layers) return set_error(SF37KV_EINVAL, "decode_gather: layers is NULL");
    if (n_layers > (uint32_t)kMaxJobs)
        return set_error(SF37KV_EINVAL, "decode_gather: at most %d layers per call", kMaxJobs);
    GatherDev d;
    if (int rc = gather_dev(g, epoch, &d)) return rc;
    AttnJob jobs[kMaxJobs];
    uint64_t off[kMaxJobs];
    for (uint32_t i = 0; i < n_layers; i++) {
        const sf37kv_decode_layer &L = layers[i];
        if (L.cache.cap == 0) return set_error(SF37KV_EINVAL, "decode_gather: layer %u cap 0", i);
        if ((L.k_new != nullptr) != (L.v_new != nullptr))
            return set_error(SF37KV_EINVAL, "decode_gather: layer %u has only one of k_new/v_new", i);
        off[i] = ((((uint64_t)(epoch & 1u) * g->world + g->rank) * n_layers) + i) * q_heads * head_dim;
        jobs[i] = AttnJob{L.cache.k_cache, L.cache.v_cache, L.q, L.gate, (float *)g->peer_buf[g->rank] + off[i],
                          start_at(L.pos, L.cache.cap, L.cache.sliding, L.cache.window), L.pos + 1u, L.cache.cap,
                          L.k_new, L.v_new};
    }
    cudaStream_t s = stream ? (cudaStream_t)stream : current_stream();
    return attention_jobs_gather(jobs, n_layers, q_heads, kv_heads, head_dim, dtype, s, &d, off);
}

extern "C" int sf37kv_gather_wait(const sf37kv_peer_gather *g, uint32_t epoch, void *stream) {
    if (!g || !g->my_flags || g->world < 1 || g->world > 8)
        return set_error(SF37KV_EINVAL, "gather_wait: bad gather descriptor");
    int *err = device_error_flag();
    if (!err) return set_error(SF37KV_ECUDA, "gather_wait: no device error flag");
    cudaStream_t s = stream ? (cudaStream_t)stream : current_stream();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    (void)cudaLaunchKernelEx(&cfg, gather_wait_kernel, (const uint32_t *)g->my_flags, g->world, epoch, err);
    g_launches++;
    return check_cuda(cudaGetLastError(), "gather wait launch");
}

// ---------------------------------------------------------------- reduce
// Sum of the world partial vectors that sf37kv_oproj_q8_0_shard stored into
// this rank's buffer half: every CTA first waits (bounded, as
// gather_wait_kernel) for all ranks' epoch flags, then adds the slots in rank
// order 0..world-1, so every rank gets the same bits.
namespace sf37kv {
__global__ void reduce_slots_kernel(const float *half_base, const uint32_t *flags, uint32_t world, uint32_t epoch,
                                    uint64_t n4, float *out, int *err) {
    __shared__ int ok;
    if (threadIdx.x < 32) {
        bool fine = true;
        if (threadIdx.x < world) {
            const long long t0 = clock64();
            for (;;) {
                uint32_t v;
                asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + threadIdx.x) : "memory");
                if ((int32_t)(v - epoch) >= 0) break;
                if (clock64() - t0 > 4000000000ll) {
                    fine = false;
                    break;
                }
                __nanosleep(200);
            }
        }
        fine = __all_sync(0xffffffffu, fine);
        if (threadIdx.x == 0) ok = fine;
    }
    __syncthreads();
    if (!ok) {
        if (threadIdx.x == 0) atomicExch(err, 2);
        return;
    }
    const float4 *src = reinterpret_cast<const float4 *>(half_base);
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (uint64_t)gridDim.x * blockDim.x) {
        float4 s = src[i];
        for (uint32_t p = 1; p < world; p++) {
            const float4 v = src[p * n4 + i];
            s.x += v.x;
            s.y += v.y;
            s.z += v.z;
            s.w += v.w;
        }
        reinterpret_cast<float4 *>(out)[i] = s;
    }
}
}  // namespace sf37kv

extern "C" int sf37kv_oproj_reduce(const sf37kv_peer_gather *g, uint32_t n_layers, uint32_t out_dim, uint32_t epoch,
                                   float *out, void *stream) {
    GatherDev d;
    if (int rc = gather_dev(g, epoch, &d)) return rc;
    if (!out || !g->my_flags) return set_error(SF37KV_EINVAL, "oproj_reduce: NULL output or flags");
    if (out_dim % 4u || ((uintptr_t)out & 15u))
        return set_error(SF37KV_EINVAL, "oproj_reduce: out_dim must be a multiple of 4 and out 16-byte aligned");
    int *err = device_error_flag();
    if (!err) return set_error(SF37KV_ECUDA, "oproj_reduce: no device error flag");
    const uint64_t n = (uint64_t)n_layers * out_dim;
    const float *half = (const float *)g->peer_buf[g->rank] + (uint64_t)(epoch & 1u) * g->world * n;
    cudaStream_t s = stream ? (cudaStream_t)stream : current_stream();
    const uint64_t n4 = n / 4u;
    unsigned grid = (unsigned)std::min<uint64_t>((n4 + 255u) / 256u, (uint64_t)num_sms() * 2u);
    if (grid == 0) grid = 1;
    reduce_slots_kernel<<<grid, 256, 0, s>>>(half, (const uint32_t *)g->my_flags, g->world, epoch, n4, out, err);
    g_launches++;
    return check_cuda(cudaGetLastError(), "oproj reduce launch");
}
