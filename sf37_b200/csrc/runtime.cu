// Library runtime: error reporting, the library stream, the split-K scratch,
// the reference-compatible tensor API (sf37_cuda.cu:32-35, 1742-1834) and
// the managed-cache policy (sf37_cuda.cu:1766-1800).
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "kv_internal.cuh"
#include "../../include/sf37_cuda_kv.h"

namespace sf37kv {

static thread_local char g_err[512];
static cudaStream_t g_stream = nullptr;  // nullptr = legacy default stream
static Scratch g_scratch;
static int g_num_sms = 0;
unsigned long long g_launches = 0;

int set_error(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

int check_cuda(cudaError_t err, const char *what) {
    if (err == cudaSuccess) return SF37KV_OK;
    (void)cudaGetLastError();
    return set_error(SF37KV_ECUDA, "CUDA %s failed: %s", what ? what : "operation",
                     cudaGetErrorString(err));
}

cudaStream_t current_stream() { return g_stream; }

int num_sms() {
    if (g_num_sms <= 0) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev) !=
                cudaSuccess || g_num_sms <= 0) {
            (void)cudaGetLastError();
            g_num_sms = 148;
        }
    }
    return g_num_sms;
}

// The scratch is process-wide, like the reference's cuda_tmp_alloc
// (sf37_cuda.cu:1579-1592): grow-only, freed at cleanup.  Growing
// synchronizes the device first because in-flight kernels may still use it.
int scratch_get(uint64_t part_bytes, uint64_t n_counters, Scratch *out) {
    if (part_bytes > g_scratch.part_bytes) {
        if (g_scratch.part) {
            (void)cudaDeviceSynchronize();
            cudaFree(g_scratch.part);
            g_scratch.part = nullptr;
            g_scratch.part_bytes = 0;
        }
        uint64_t want = part_bytes + (part_bytes >> 2);
        if (int rc = check_cuda(cudaMalloc(&g_scratch.part, want), "scratch alloc")) return rc;
        g_scratch.part_bytes = want;
    }
    if (n_counters > g_scratch.n_counters) {
        if (g_scratch.counters) {
            (void)cudaDeviceSynchronize();
            cudaFree(g_scratch.counters);
            g_scratch.counters = nullptr;
            g_scratch.n_counters = 0;
        }
        uint64_t want = n_counters < 4096 ? 4096 : n_counters * 2;
        if (int rc = check_cuda(cudaMalloc(&g_scratch.counters, want * 4), "counter alloc"))
            return rc;
        if (int rc = check_cuda(cudaMemset(g_scratch.counters, 0, want * 4), "counter clear"))
            return rc;
        g_scratch.n_counters = want;
    }
    *out = g_scratch;
    return SF37KV_OK;
}

// One device int that kernels set when a bounded wait gives up.
static int *g_err_flag = nullptr;
int *device_error_flag() {
    if (!g_err_flag) {
        if (cudaMalloc(&g_err_flag, sizeof(int)) != cudaSuccess ||
            cudaMemset(g_err_flag, 0, sizeof(int)) != cudaSuccess) {
            (void)cudaGetLastError();
            g_err_flag = nullptr;
        }
    }
    return g_err_flag;
}

void scratch_release() {
    if (g_scratch.part) cudaFree(g_scratch.part);
    if (g_scratch.counters) cudaFree(g_scratch.counters);
    g_scratch = Scratch();
}

}  // namespace sf37kv

using namespace sf37kv;

extern "C" {

const char *sf37kv_last_error(void) { return g_err; }
const char *sf37kv_version(void) { return "sf37kv 0.1 (sm_100a)"; }

int sf37kv_set_stream(void *stream) {
    g_stream = (cudaStream_t)stream;
    return SF37KV_OK;
}
void *sf37kv_get_stream(void) { return (void *)g_stream; }
uint64_t sf37kv_launch_count(void) { return g_launches; }

int sf37kv_device_error(int clear) {
    int *f = device_error_flag();
    if (!f) return -1;
    int v = 0;
    if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpy(&v, f, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
        (void)cudaGetLastError();
        return -1;
    }
    if (clear && v) cudaMemset(f, 0, sizeof(int));
    return v;
}

void *sf37kv_host_alloc(uint64_t bytes) {
    void *p = nullptr;
    if (cudaHostAlloc(&p, bytes ? bytes : 1, cudaHostAllocMapped) != cudaSuccess) {
        check_cuda(cudaGetLastError(), "host alloc");
        return nullptr;
    }
    return p;
}
void sf37kv_host_free(void *p) {
    if (p) cudaFreeHost(p);
}

// ------------------------------------------------------------------------
// Reference-compatible runtime entry points (sf37_cuda.h:12-50).  Errors go
// to stderr with the reference's wording style and return 0.
static int dropin_ok(cudaError_t err, const char *what) {
    if (err == cudaSuccess) return 1;
    fprintf(stderr, "sf37: CUDA %s failed: %s\n", what ? what : "operation",
            cudaGetErrorString(err));
    (void)cudaGetLastError();
    return 0;
}

int sf37_cuda_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        (void)cudaGetLastError();
        return -1;
    }
    return n;
}

int sf37_cuda_init(void) {
    // The reference pins device 0 (sf37_cuda.cu:1618); a multi-GPU host
    // program selects its device before calling in, so keep the current one.
    int dev = 0;
    if (!dropin_ok(cudaGetDevice(&dev), "get device")) return 0;
    if (!dropin_ok(cudaFree(nullptr), "context init")) return 0;
    (void)num_sms();
    return 1;
}

void sf37_cuda_cleanup(void) {
    (void)cudaDeviceSynchronize();
    scratch_release();
    staging_release();
}

int sf37_cuda_synchronize(void) { return dropin_ok(cudaDeviceSynchronize(), "synchronize"); }

int sf37_cuda_memory_info(uint64_t *free_bytes, uint64_t *total_bytes) {
    size_t f = 0, t = 0;
    if (!dropin_ok(cudaMemGetInfo(&f, &t), "memory info")) return 0;
    if (free_bytes) *free_bytes = f;
    if (total_bytes) *total_bytes = t;
    return 1;
}

sf37_cuda_tensor *sf37_cuda_tensor_alloc(uint64_t bytes) {
    if (bytes == 0) bytes = 1;
    sf37_cuda_tensor *t = (sf37_cuda_tensor *)calloc(1, sizeof(*t));
    if (!t) return nullptr;
    if (!dropin_ok(cudaMalloc(&t->ptr, (size_t)bytes), "tensor alloc")) {
        free(t);
        return nullptr;
    }
    t->bytes = bytes;
    return t;
}

sf37_cuda_tensor *sf37_cuda_tensor_alloc_managed(uint64_t bytes) {
    if (bytes == 0) bytes = 1;
    sf37_cuda_tensor *t = (sf37_cuda_tensor *)calloc(1, sizeof(*t));
    if (!t) return nullptr;
    if (!dropin_ok(cudaMallocManaged(&t->ptr, (size_t)bytes), "managed tensor alloc")) {
        free(t);
        return nullptr;
    }
    t->bytes = bytes;
    return t;
}

void sf37_cuda_tensor_free(sf37_cuda_tensor *tensor) {
    if (!tensor) return;
    if (tensor->ptr) (void)cudaFree(tensor->ptr);
    free(tensor);
}

uint64_t sf37_cuda_tensor_bytes(const sf37_cuda_tensor *tensor) {
    return tensor ? tensor->bytes : 0;
}

// Synchronous like the reference (sf37_cuda.cu:1809-1822), but ordered
// after the library stream's work so a non-default library stream is safe.
int sf37_cuda_tensor_write(sf37_cuda_tensor *tensor, uint64_t offset, const void *data,
                           uint64_t bytes) {
    if (!tensor || !data || offset > tensor->bytes || bytes > tensor->bytes - offset) return 0;
    if (!dropin_ok(cudaMemcpyAsync((char *)tensor->ptr + offset, data, (size_t)bytes,
                                   cudaMemcpyHostToDevice, g_stream), "tensor write"))
        return 0;
    return dropin_ok(cudaStreamSynchronize(g_stream), "tensor write sync");
}

int sf37_cuda_tensor_read(const sf37_cuda_tensor *tensor, uint64_t offset, void *data,
                          uint64_t bytes) {
    if (!tensor || !data || offset > tensor->bytes || bytes > tensor->bytes - offset) return 0;
    if (!dropin_ok(cudaMemcpyAsync(data, (const char *)tensor->ptr + offset, (size_t)bytes,
                                   cudaMemcpyDeviceToHost, g_stream), "tensor read"))
        return 0;
    return dropin_ok(cudaStreamSynchronize(g_stream), "tensor read sync");
}

int sf37_cuda_tensor_copy(sf37_cuda_tensor *dst, uint64_t dst_offset, const sf37_cuda_tensor *src,
                          uint64_t src_offset, uint64_t bytes) {
    if (!dst || !src || dst_offset > dst->bytes || bytes > dst->bytes - dst_offset ||
        src_offset > src->bytes || bytes > src->bytes - src_offset)
        return 0;
    return dropin_ok(cudaMemcpyAsync((char *)dst->ptr + dst_offset,
                                     (const char *)src->ptr + src_offset, (size_t)bytes,
                                     cudaMemcpyDeviceToDevice, g_stream),
                     "tensor copy");
}

}  // extern "C"

__global__ static void fill_f32_kernel(float *x, uint64_t n, float v) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = v;
}

extern "C" int sf37_cuda_tensor_fill_f32(sf37_cuda_tensor *tensor, float value, uint64_t count) {
    if (!tensor || count > tensor->bytes / sizeof(float)) return 0;
    if (count == 0) return 1;
    fill_f32_kernel<<<(unsigned)((count + 255u) / 256u), 256, 0, g_stream>>>((float *)tensor->ptr,
                                                                           count, value);
    g_launches++;
    return dropin_ok(cudaGetLastError(), "fill f32 launch");
}

// Policy of sf37_cuda.cu:1766-1800 (managed memory once the KV cache
// reaches 8 GiB, or when a >= 8 GiB context would leave less than the
// reserve, total/4 clamped to [8, 40] GiB, free), with the device's free and
// total memory from cudaMemGetInfo; the arithmetic is
// sf37kv_managed_kv_policy (sizing.cu).  A failed query answers 0, as the
// reference does.
extern "C" int sf37_cuda_should_use_managed_kv_cache(uint64_t kv_cache_bytes,
                                                     uint64_t context_bytes) {
    if (kv_cache_bytes == 0) return 0;
    const uint64_t gib = 1073741824ull;
    if (kv_cache_bytes < 8ull * gib && context_bytes < 8ull * gib) return 0;
    size_t free_b = 0, total_b = 0;
    if (kv_cache_bytes < 8ull * gib && cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    return sf37kv_managed_kv_policy(kv_cache_bytes, context_bytes, free_b, total_b);
}
