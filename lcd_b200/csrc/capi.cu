// Host-side helpers shared by every entry point: error text, status block I/O.
#include <stdio.h>
#include <string.h>

#include "common.cuh"

namespace lcd {

static thread_local char g_cuda_error[512] = "";

void set_cuda_error(cudaError_t e, const char *where) {
    snprintf(g_cuda_error, sizeof g_cuda_error, "%s: %s (%s)", cudaGetErrorName(e),
             cudaGetErrorString(e), where);
}

int reset_status(int32_t *status_dev, cudaStream_t stream) {
    LCD_CUDA_TRY(cudaMemsetAsync(status_dev, 0, LCD_STATUS_WORDS * sizeof(int32_t), stream));
    return LCD_OK;
}

int finish(int32_t *status_dev, cudaStream_t stream, int *status_host) {
    if (!status_host) return LCD_OK;
    int32_t node = -1;
    const int rc = lcd_read_status(status_dev, stream, &node);
    *status_host = rc;
    return rc;
}

static long long *g_trace = nullptr;
long long *debug_trace() { return g_trace; }
void set_debug_trace(long long *p) { g_trace = p; }

int sm_count() {
    static int cached = 0;
    if (!cached) {
        int dev = 0, sms = 0;
        if (cudaGetDevice(&dev) == cudaSuccess &&
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
            cached = sms;
        else
            return 148;
    }
    return cached;
}

// 128-bit order-sensitive checksum of an int32 array: every element is mixed with
// its position (splitmix64 finaliser) and the mixes are combined by sum and xor.
__device__ __forceinline__ unsigned long long mix64(unsigned long long z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void checksum_i32_kernel(const int *__restrict__ data, long long count,
                                    unsigned long long *out) {
    unsigned long long sum = 0, fold = 0;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < count; k += stride) {
        const unsigned long long m =
            mix64(((unsigned long long)k << 32) ^ (unsigned long long)(unsigned)data[k]);
        sum += m;
        fold ^= mix64(m + (unsigned long long)k);
    }
    for (int off = 16; off > 0; off >>= 1) {
        sum += __shfl_xor_sync(0xffffffffu, sum, off);
        fold ^= __shfl_xor_sync(0xffffffffu, fold, off);
    }
    if ((threadIdx.x & 31) == 0) {
        atomicAdd(out, sum);
        atomicXor(out + 1, fold);
    }
}

}  // namespace lcd

using namespace lcd;

extern "C" int lcd_checksum_i32(const int32_t *data, int64_t count, uint64_t *out_dev,
                                uint64_t *out_host, void *stream) {
    if (count < 0 || !out_dev || (count > 0 && !data)) return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    LCD_CUDA_TRY(cudaMemsetAsync(out_dev, 0, 2 * sizeof(uint64_t), st));
    if (count > 0) {
        long long blocks = (count + 1023) / 1024;
        if (blocks > 148 * 8) blocks = 148 * 8;
        checksum_i32_kernel<<<(unsigned)blocks, 256, 0, st>>>(
            data, count, reinterpret_cast<unsigned long long *>(out_dev));
        LCD_CUDA_TRY(cudaGetLastError());
    }
    if (out_host) {
        LCD_CUDA_TRY(cudaMemcpyAsync(out_host, out_dev, 2 * sizeof(uint64_t),
                                     cudaMemcpyDeviceToHost, st));
        LCD_CUDA_TRY(cudaStreamSynchronize(st));
    }
    return LCD_OK;
}

// Profiling aid: when set, the one-lane-per-row and chain solvers store the SM cycle
// counter at which each row was published into trace[node] (n 64-bit words).
extern "C" int lcd_debug_set_trace(long long *trace_dev) {
    set_debug_trace(trace_dev);
    return LCD_OK;
}

extern "C" const char *lcd_error_string(int code) {
    switch (code) {
        case LCD_OK: return "success";
        case LCD_ERR_INVALID_ARGUMENT: return "invalid argument";
        case LCD_ERR_CUDA: return "CUDA runtime error";
        case LCD_ERR_WORKSPACE: return "workspace too small";
        case LCD_ERR_TIMEOUT: return "a bounded device wait expired (dependency never satisfied)";
        case LCD_ERR_UNSORTED: return "segment violates the sorted-segment property";
        case LCD_ERR_BAD_POINTERS: return "pointer array is not monotone or out of range";
        case LCD_ERR_INDEX_RANGE: return "index out of range or on the wrong side of the diagonal";
        case LCD_ERR_CYCLE: return "dependence graph is not acyclic";
        case LCD_ERR_MISSING_DIAGONAL: return "a required diagonal entry is not stored";
        case LCD_ERR_TOO_LARGE: return "size exceeds a documented limit";
        case LCD_ERR_LEVEL_CAP: return "level propagation stopped at the requested cap";
        default: return "unknown lcd_b200 error";
    }
}

extern "C" const char *lcd_last_cuda_error(void) { return g_cuda_error; }

extern "C" int lcd_version(void) { return 100; }

extern "C" int lcd_read_status(const int32_t *status_dev, void *stream, int32_t *node) {
    if (!status_dev) return LCD_ERR_INVALID_ARGUMENT;
    int32_t words[2] = {0, -1};
    cudaStream_t st = (cudaStream_t)stream;
    LCD_CUDA_TRY(cudaMemcpyAsync(words, status_dev, sizeof words, cudaMemcpyDeviceToHost, st));
    LCD_CUDA_TRY(cudaStreamSynchronize(st));
    if (node) *node = words[1];
    return words[0];
}

extern "C" int lcd_device_sm_count(int *count) {
    if (!count) return LCD_ERR_INVALID_ARGUMENT;
    *count = sm_count();
    return LCD_OK;
}

// ---- peer-visible buffers for the multi-GPU partitioned solve --------------------
// One process per GPU: a rank allocates its x array here, exports an IPC handle, and
// the other ranks of the node map it.  These are the only entry points that allocate.
extern "C" int lcd_peer_alloc(int64_t bytes, void **ptr, unsigned char *handle64) {
    if (bytes <= 0 || !ptr || !handle64) return LCD_ERR_INVALID_ARGUMENT;
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    LCD_CUDA_TRY(cudaMalloc(ptr, (size_t)bytes));
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, *ptr);
    if (e != cudaSuccess) {
        set_cuda_error(e, "cudaIpcGetMemHandle");
        cudaFree(*ptr);
        *ptr = nullptr;
        return LCD_ERR_CUDA;
    }
    memcpy(handle64, &h, 64);
    return LCD_OK;
}

extern "C" int lcd_peer_open(const unsigned char *handle64, void **ptr) {
    if (!handle64 || !ptr) return LCD_ERR_INVALID_ARGUMENT;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, 64);
    LCD_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return LCD_OK;
}

extern "C" int lcd_peer_close(void *ptr) {
    if (!ptr) return LCD_OK;
    LCD_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
    return LCD_OK;
}

extern "C" int lcd_peer_free(void *ptr) {
    if (!ptr) return LCD_OK;
    LCD_CUDA_TRY(cudaFree(ptr));
    return LCD_OK;
}
