// Shared device/host helpers of the lcd_b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "lcd_b200.h"

namespace lcd {

// Reserved bit pattern that marks "not produced yet" in solution vectors.  It is
// a NaN that no arithmetic instruction produces on its own (results that happen
// to carry it are replaced by the canonical NaN before being published).
constexpr unsigned long long kPendingBits = 0xFFFFFFFFFFFFFFFFull;
constexpr long long kCanonicalNaN = 0x7FF8000000000000ll;

constexpr int kDefaultTimeoutMs = 4000;

// status block layout (int32 words)
constexpr int kStatusCode = 0;
constexpr int kStatusNode = 1;
constexpr int kStatusTicket = 2;
constexpr int kStatusBarrier = 4;  // 64-bit barrier counter lives in words 4..5

void set_cuda_error(cudaError_t e, const char *where);

#define LCD_CUDA_TRY(expr)                                   \
    do {                                                     \
        cudaError_t _e = (expr);                             \
        if (_e != cudaSuccess) {                             \
            ::lcd::set_cuda_error(_e, #expr);                \
            return LCD_ERR_CUDA;                             \
        }                                                    \
    } while (0)

int finish(int32_t *status_dev, cudaStream_t stream, int *status_host);
int reset_status(int32_t *status_dev, cudaStream_t stream);
inline unsigned long long timeout_ns(int32_t timeout_ms) {
    return (unsigned long long)(timeout_ms > 0 ? timeout_ms : kDefaultTimeoutMs) * 1000000ull;
}
int sm_count();
void set_debug_trace(long long *p);
int set_chain_cluster_limit(int blocks);  // LCD_TUNE_CHAIN_CLUSTER
int set_ordered_pause(int ns);           // LCD_TUNE_ORDERED_PAUSE_NS
int set_ordered_min_lanes(int lanes);    // LCD_TUNE_ORDERED_MIN_LANES
int set_small_threads(int threads);      // LCD_TUNE_SMALL_THREADS
int set_ilu0_lookahead(int on);          // LCD_TUNE_ILU0_LOOKAHEAD
long long *debug_trace();  // profiling aid set by lcd_debug_set_trace (NULL = off)

#ifdef __CUDACC__

__device__ __forceinline__ unsigned long long global_timer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// L2-coherent 8-byte load / store: the value itself is the hand-off, so relaxed
// gpu-scope accesses are enough.
__device__ __forceinline__ double ld_relaxed_f64(const double *p) {
    double v;
    asm volatile("ld.relaxed.gpu.global.f64 %0, [%1];" : "=d"(v) : "l"(p) : "memory");
    return v;
}
// system scope: the value may have been stored by another GPU through a peer mapping
__device__ __forceinline__ double ld_relaxed_sys_f64(const double *p) {
    double v;
    asm volatile("ld.relaxed.sys.global.f64 %0, [%1];" : "=d"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_f64(double *p, double v) {
    asm volatile("st.relaxed.gpu.global.f64 [%0], %1;" ::"l"(p), "d"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys_f64(double *p, double v) {
    asm volatile("st.relaxed.sys.global.f64 [%0], %1;" ::"l"(p), "d"(v) : "memory");
}
__device__ __forceinline__ int ld_relaxed_s32(const int *p) {
    int v;
    asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int ld_acquire_s32(const int *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_s32(int *p, int v) {
    asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_add_s32(int *p, int v) {
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_relaxed_add_f64(double *p, double v) {
    asm volatile("red.relaxed.gpu.global.add.f64 [%0], %1;" ::"l"(p), "d"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Flags are polled with relaxed loads (an acquire load on every failed poll costs an
// ordering operation each time); the acquire ordering is established once, by this
// fence, after the poll that observed the released value.
__device__ __forceinline__ void acquire_fence() {
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

__device__ __forceinline__ bool is_pending(double v) {
    return (unsigned long long)__double_as_longlong(v) == kPendingBits;
}
__device__ __forceinline__ double publishable(double v) {
    return is_pending(v) ? __longlong_as_double(kCanonicalNaN) : v;
}

// First error wins; word 0 doubles as the abort flag every waiter polls.
__device__ __forceinline__ void raise_error(int32_t *status, int code, int node) {
    if (atomicCAS(&status[kStatusCode], 0, code) == 0) status[kStatusNode] = node;
}
__device__ __forceinline__ bool aborted(const int32_t *status) {
    return ld_relaxed_s32(&status[kStatusCode]) != 0;
}

// Bounded wait bookkeeping: call tick() once per failed poll.  Returns true when
// the wait must be abandoned (deadline passed or another thread raised an error).
struct Deadline {
    unsigned long long end;
    unsigned polls;
    __device__ __forceinline__ void start(unsigned long long budget_ns) {
        end = global_timer() + budget_ns;
        polls = 0;
    }
    __device__ __forceinline__ bool tick(int32_t *status, int node) {
        if ((++polls & 127u) != 0) return false;
        if (aborted(status)) return true;
        if (global_timer() > end) {
            raise_error(status, LCD_ERR_TIMEOUT, node);
            return true;
        }
        return false;
    }
};

// Arguments of the CSR triangular solvers (sync-free and wavefront).
struct CsrSolveParams {
    int n;
    long long nnz;
    const int *__restrict__ Ap;
    const int *__restrict__ Ai;
    const double *__restrict__ Ax;
    const int *__restrict__ dpos;
    const double *__restrict__ b;
    double *x;
    int flags;
    int nrhs;
    long long ld;
    int32_t *status;
    unsigned long long budget_ns;
    long long *trace;  // optional: per-row SM cycle counter at publication (profiling aid)
    // block-row partition across GPUs: this launch owns the nodes [task_begin, task_end);
    // a published value is also stored into the x arrays of the ranks whose bit is set in
    // need_mask[row] (peer-mapped pointers, indexed by rank)
    int task_begin;
    int task_end;
    const unsigned char *__restrict__ need_mask;
    double *peers[8];
};

// Off-diagonal range [lo, hi) and diagonal position d (-1: implicit unit) of a row.
// Returns false when the row's pointers are inconsistent.
__device__ __forceinline__ bool csr_row_range(const CsrSolveParams &p, int r, int &lo, int &hi,
                                              int &d) {
    const int s = __ldg(p.Ap + r), e = __ldg(p.Ap + r + 1);
    if (s < 0 || e < s || (long long)e > p.nnz) return false;
    const bool upper = p.flags & LCD_SOLVE_UPPER;
    if (p.flags & LCD_SOLVE_OF_FULL) {
        const int dp = __ldg(p.dpos + r);
        if (dp < s || dp >= e) return false;
        if (upper) { lo = dp + 1; hi = e; d = dp; }
        else { lo = s; hi = dp; d = (p.flags & LCD_SOLVE_UNIT_DIAG) ? -1 : dp; }
    } else {
        if (e == s) return false;
        if (upper) { lo = s + 1; hi = e; d = s; }
        else { lo = s; hi = e - 1; d = e - 1; }
    }
    return true;
}

#endif  // __CUDACC__

}  // namespace lcd
