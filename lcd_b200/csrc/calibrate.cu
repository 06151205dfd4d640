// On-device measurement of the machine constants the scheduler's cost model uses (sm_100a):
// kernel launch latency, the cost of a hand-off between two thread blocks through L2, between
// two warps of a block through shared memory, of a block barrier, of a grid-wide barrier, of an
// atomic on one contended address, and the copy bandwidth.  Counterpart of the reference's
// measure_arch_constants (compiler/scheduler.py:714-775), which times empty launches and an
// atomic kernel with Numba.  Every wait in here is bounded.
#include <algorithm>

#include "common.cuh"

namespace lcd {

__global__ void calib_empty_kernel() {}

// Two blocks bounce a counter through global memory: block 0 waits for an even value and makes
// it odd, block 1 the other way round.  2 * rounds hand-offs in total.
__global__ void calib_pingpong_kernel(int *flag, int rounds, unsigned long long budget_ns,
                                      unsigned long long *elapsed_ns, int32_t *status) {
    if (threadIdx.x != 0) return;
    const int me = blockIdx.x;
    const unsigned long long t0 = global_timer();
    Deadline dl;
    dl.start(budget_ns);
    for (int r = 0; r < rounds; ++r) {
        const int want = 2 * r + me;
        while (ld_relaxed_s32(flag) != want)
            if (dl.tick(status, me)) return;
        asm volatile("st.relaxed.gpu.global.s32 [%0], %1;" ::"l"(flag), "r"(want + 1) : "memory");
    }
    if (me == 1) *elapsed_ns = global_timer() - t0;
}

// The same bounce between two warps of one block through shared memory, and a run of
// __syncthreads() by a block of 512 threads.
__global__ void calib_block_kernel(int rounds, unsigned long long *out_ns) {
    __shared__ volatile int s_flag;
    if (threadIdx.x == 0) s_flag = 0;
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned long long t0 = global_timer();
    if (warp < 2 && lane == 0) {
        for (int r = 0; r < rounds; ++r) {
            const int want = 2 * r + warp;
            unsigned spins = 0;
            while (s_flag != want && ++spins < (1u << 22)) {}
            s_flag = want + 1;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) out_ns[0] = global_timer() - t0;
    t0 = global_timer();
    for (int r = 0; r < rounds; ++r) __syncthreads();
    if (threadIdx.x == 0) out_ns[1] = global_timer() - t0;
}

// Every thread of a full grid adds to one address.
__global__ void calib_atomic_kernel(int *target, int per_thread) {
    for (int k = 0; k < per_thread; ++k) atomicAdd(target, 1);
}

// Grid-wide barrier on a monotone counter (cooperative launch), as the level-synchronous
// kernels do it.
__global__ void calib_gridbar_kernel(unsigned long long *counter, int rounds, unsigned long long budget_ns,
                                     unsigned long long *elapsed_ns, int32_t *status) {
    const unsigned long long t0 = global_timer();
    unsigned long long target = 0;
    for (int r = 0; r < rounds; ++r) {
        __syncthreads();
        if (threadIdx.x == 0) {
            target += gridDim.x;
            __threadfence();
            atomicAdd(counter, 1ull);
            Deadline dl;
            dl.start(budget_ns);
            while (ld_relaxed_u64(counter) < target)
                if (dl.tick(status, -1)) break;
        }
        __syncthreads();
        if (aborted(status)) return;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) *elapsed_ns = global_timer() - t0;
}

// Dependent loads through L2: a chain of kChaseSteps addresses 128 bytes apart spread over 32 MB
// (resident in L2 after the first walk), each loaded with ld.relaxed.gpu as the polls are.
constexpr int kChaseSteps = 4096;
constexpr int kChaseSlots = 1 << 18;       // x 128 B = 32 MB
__global__ void calib_chase_init_kernel(unsigned long long *buf) {
    const unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (unsigned)kChaseSlots)
        buf[(size_t)i * 16] = (i * 1664525u + 1013904223u) & (unsigned)(kChaseSlots - 1);
}
__global__ void calib_chase_kernel(const unsigned long long *buf, int passes, unsigned *cycles) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    for (int pass = 0; pass < passes; ++pass) {
        unsigned long long at = 0;
        for (int k = 0; k < kChaseSteps; ++k) {
            const long long t0 = clock64();
            unsigned long long next;
            asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(next) : "l"(buf + at * 16) : "memory");
            at = next;
            const long long t1 = clock64() + (long long)(at >> 40);   // (waits for the value)
            if (pass == passes - 1) cycles[k] = (unsigned)(t1 - t0);
        }
    }
}

__global__ void calib_copy_kernel(const double4 *__restrict__ src, double4 *__restrict__ dst, long long count) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < count; k += stride) dst[k] = src[k];
}

}  // namespace lcd

using namespace lcd;

extern "C" int lcd_calibrate(void *workspace, int64_t workspace_bytes, void *stream, double *out_host) {
    if (!workspace || !out_host || workspace_bytes < (64 << 20) || ((uintptr_t)workspace & 255))
        return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    for (int k = 0; k < LCD_CALIBRATION_VALUES; ++k) out_host[k] = 0.0;
    // scratch words at the start of the workspace
    int32_t *status = static_cast<int32_t *>(workspace);
    int *flag = reinterpret_cast<int *>(status + 64);
    unsigned long long *words = reinterpret_cast<unsigned long long *>(status + 128);   // 8 words
    LCD_CUDA_TRY(cudaMemsetAsync(workspace, 0, 4096, st));
    cudaEvent_t e0, e1;
    LCD_CUDA_TRY(cudaEventCreate(&e0));
    LCD_CUDA_TRY(cudaEventCreate(&e1));
    float ms = 0.f;
    int rc = LCD_OK;
    auto fail = [&](int code) { cudaEventDestroy(e0); cudaEventDestroy(e1); return code; };
    // 1. launch latency: back-to-back empty kernels
    const int launches = 2000;
    for (int k = 0; k < 50; ++k) calib_empty_kernel<<<1, 32, 0, st>>>();
    cudaEventRecord(e0, st);
    for (int k = 0; k < launches; ++k) calib_empty_kernel<<<1, 32, 0, st>>>();
    cudaEventRecord(e1, st);
    if (cudaEventSynchronize(e1) != cudaSuccess) return fail(LCD_ERR_CUDA);
    cudaEventElapsedTime(&ms, e0, e1);
    out_host[LCD_CAL_LAUNCH_S] = ms * 1e-3 / launches;
    // 2. hand-off through L2 between two blocks
    const int rounds = 2000;
    calib_pingpong_kernel<<<2, 32, 0, st>>>(flag, rounds, timeout_ns(1000), words, status);
    // 3. hand-off through shared memory, block barrier
    calib_block_kernel<<<1, 512, 0, st>>>(rounds, words + 1);
    unsigned long long host_words[8] = {0};
    if (cudaMemcpyAsync(host_words, words, sizeof host_words, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return fail(LCD_ERR_CUDA);
    rc = lcd_read_status(status, st, nullptr);
    if (rc) return fail(rc);
    out_host[LCD_CAL_L2_HANDOFF_S] = (double)host_words[0] * 1e-9 / (2.0 * rounds);
    out_host[LCD_CAL_SMEM_HANDOFF_S] = (double)host_words[1] * 1e-9 / (2.0 * rounds);
    out_host[LCD_CAL_BLOCK_BARRIER_S] = (double)host_words[2] * 1e-9 / rounds;
    // 4. contended atomic
    const int blocks = sm_count() * 4, per_thread = 16;
    cudaEventRecord(e0, st);
    calib_atomic_kernel<<<blocks, 256, 0, st>>>(flag + 16, per_thread);
    cudaEventRecord(e1, st);
    if (cudaEventSynchronize(e1) != cudaSuccess) return fail(LCD_ERR_CUDA);
    cudaEventElapsedTime(&ms, e0, e1);
    out_host[LCD_CAL_ATOMIC_S] = ms * 1e-3 / ((double)blocks * 256 * per_thread);
    // 5. grid barrier (cooperative launch over every SM)
    {
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, calib_gridbar_kernel, 512, 0) == cudaSuccess &&
            per_sm >= 1) {
            unsigned long long *counter = words + 4, *elapsed = words + 5;
            int bar_rounds = 500;
            unsigned long long budget = timeout_ns(1000);
            void *args[] = {(void *)&counter, (void *)&bar_rounds, (void *)&budget, (void *)&elapsed,
                            (void *)&status};
            if (cudaLaunchCooperativeKernel((void *)calib_gridbar_kernel, dim3((unsigned)sm_count()), dim3(512),
                                            args, 0, st) == cudaSuccess &&
                cudaMemcpyAsync(host_words, words, sizeof host_words, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
                cudaStreamSynchronize(st) == cudaSuccess && lcd_read_status(status, st, nullptr) == LCD_OK)
                out_host[LCD_CAL_GRID_BARRIER_S] = (double)host_words[5] * 1e-9 / bar_rounds;
            else
                cudaGetLastError();
        }
    }
    // 6. copy bandwidth over the two halves of the workspace (read + write bytes)
    {
        const long long half = ((workspace_bytes - 4096) / 2) & ~1023ll;
        const double4 *src = reinterpret_cast<const double4 *>(static_cast<char *>(workspace) + 4096);
        double4 *dst = reinterpret_cast<double4 *>(static_cast<char *>(workspace) + 4096 + half);
        const long long count = half / (long long)sizeof(double4);
        calib_copy_kernel<<<sm_count() * 8, 512, 0, st>>>(src, dst, count);
        cudaEventRecord(e0, st);
        for (int k = 0; k < 3; ++k) calib_copy_kernel<<<sm_count() * 8, 512, 0, st>>>(src, dst, count);
        cudaEventRecord(e1, st);
        if (cudaEventSynchronize(e1) != cudaSuccess) return fail(LCD_ERR_CUDA);
        cudaEventElapsedTime(&ms, e0, e1);
        out_host[LCD_CAL_COPY_BYTES_PER_S] = 3.0 * 2.0 * (double)half / (ms * 1e-3);
    }
    // 7. latency of a dependent L2 load (what one poll of a waiting row costs)
    if (workspace_bytes >= (40ll << 20)) {
        unsigned long long *buf = reinterpret_cast<unsigned long long *>(static_cast<char *>(workspace) + 8192);
        unsigned *cycles = reinterpret_cast<unsigned *>(static_cast<char *>(workspace) + (36ll << 20));
        calib_chase_init_kernel<<<kChaseSlots / 256, 256, 0, st>>>(buf);
        calib_chase_kernel<<<1, 32, 0, st>>>(buf, 2, cycles);
        static unsigned host_cycles[kChaseSteps];
        int clock_khz = 0;
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&clock_khz, cudaDevAttrClockRate, dev);
        if (cudaMemcpyAsync(host_cycles, cycles, sizeof host_cycles, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
            cudaStreamSynchronize(st) == cudaSuccess && clock_khz > 0) {
            std::sort(host_cycles, host_cycles + kChaseSteps);
            double sum = 0.0;
            for (int k = 0; k < kChaseSteps; ++k) sum += host_cycles[k];
            const double to_s = 1.0 / (clock_khz * 1e3);
            out_host[LCD_CAL_L2_LOAD_S] = sum / kChaseSteps * to_s;
            out_host[LCD_CAL_L2_LOAD_P10_S] = host_cycles[kChaseSteps / 10] * to_s;
            out_host[LCD_CAL_L2_LOAD_P90_S] = host_cycles[kChaseSteps * 9 / 10] * to_s;
        }
    }
    if (cudaGetLastError() != cudaSuccess) return fail(LCD_ERR_CUDA);
    return fail(LCD_OK);
}
