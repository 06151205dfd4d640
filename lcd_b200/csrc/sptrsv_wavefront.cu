// Level-synchronous (wavefront) sparse triangular solves for sm_100a.
//
// Two drivers over the same per-node code:
//   * per-level launches on a stream (suited to capture in a CUDA graph),
//   * one cooperative launch that walks all levels; levels wide enough for the
//     whole grid end in a grid-wide barrier, while a run of consecutive levels
//     that each fit one thread block is executed by block 0 alone with
//     block-level barriers, so a long tail of narrow levels costs a
//     __syncthreads() per level instead of a grid barrier or a launch.
// x is read with L2-coherent loads (nodes of earlier levels were produced by other
// blocks).  The grid barrier's wait is bounded like every other wait here.
#include "common.cuh"

namespace lcd {

struct WavefrontParams {
    CsrSolveParams m;   // matrix, b, x, flags, status, budget
    int csc;            // 0: row form (pull), 1: column form (push with atomics)
    const int *__restrict__ wavefronts;
    const int *__restrict__ wavefront_ptr;
    int n_levels;
    int lanes;          // lanes per node, power of two <= 32
    // Band chains (band_width > 1 of the reference's warp tasks): when set, the items of a
    // level are tasks, task t being the nodes wavefronts[task_ptr[t] .. task_ptr[t + 1]) that
    // one lane group solves one after another; levels are then bands of such tasks.
    const int *__restrict__ task_ptr;
};

__device__ __forceinline__ void solve_node(const WavefrontParams &w, int node, bool active,
                                           int lane, int lanes);

// One item of a level: a node, or a chain of nodes solved in order by the same lane group.
// Must be called by all 32 lanes of the warp.
__device__ __forceinline__ void solve_item(const WavefrontParams &w, int t, bool active, int lane,
                                           int lanes) {
    if (!w.task_ptr) {
        const int node = active ? __ldg(w.wavefronts + t) : 0;
        solve_node(w, node, active && (unsigned)node < (unsigned)w.m.n, lane, lanes);
        return;
    }
    const int first = active ? __ldg(w.task_ptr + t) : 0;
    const int count = active ? __ldg(w.task_ptr + t + 1) - first : 0;
    const int longest = __reduce_max_sync(0xffffffffu, count);
    for (int k = 0; k < longest; ++k) {
        const bool on = k < count;
        const int node = on ? __ldg(w.wavefronts + first + k) : 0;
        solve_node(w, node, on && (unsigned)node < (unsigned)w.m.n, lane, lanes);
        // the next node of the chain reads what this one wrote (stores and atomics to L2)
        __threadfence();
        __syncwarp();
    }
}

// One node handled by `lanes` consecutive lanes of a warp.  Must be called by
// all 32 lanes of the warp (inactive groups pass active = false).
__device__ __forceinline__ void solve_node(const WavefrontParams &w, int node, bool active,
                                           int lane, int lanes) {
    const CsrSolveParams &p = w.m;
    const bool upper = p.flags & LCD_SOLVE_UPPER;
    const int lane_in_warp = threadIdx.x & 31;
    if (!w.csc) {
        int lo = 0, hi = 0, d = -1, r = 0;
        if (active) {
            r = upper ? p.n - 1 - node : node;
            if (!csr_row_range(p, r, lo, hi, d)) {
                if (lane == 0)
                    raise_error(p.status, (p.flags & LCD_SOLVE_OF_FULL) ? LCD_ERR_MISSING_DIAGONAL
                                                                       : LCD_ERR_BAD_POINTERS, r);
                active = false;
            }
        }
        const bool exact = (p.flags & LCD_SOLVE_EXACT) && lanes == 1;
        double acc = 0.0;
        if (active) {
            if (exact) acc = __ldg(p.b + r);
            for (int j = lo + lane; j < hi; j += lanes) {
                const int c = __ldg(p.Ai + j);
                if ((unsigned)c >= (unsigned)p.n) { raise_error(p.status, LCD_ERR_INDEX_RANGE, r); continue; }
                const double xv = __ldcg(p.x + c);
                const double a = __ldg(p.Ax + j);
                acc = exact ? __dsub_rn(acc, __dmul_rn(a, xv)) : fma(a, xv, acc);
            }
        }
        for (int off = lanes >> 1; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (active && lane == 0) {
            double s = exact ? acc : __ldg(p.b + r) - acc;
            if (d >= 0) s = s / __ldg(p.Ax + d);
            __stcg(p.x + r, s);
        }
    } else {
        int lo = 0, hi = 0, d = 0, i = 0;
        if (active) {
            i = upper ? p.n - 1 - node : node;
            const int s = __ldg(p.Ap + i), e = __ldg(p.Ap + i + 1);
            if (s < 0 || e <= s || (long long)e > p.nnz) {
                if (lane == 0) raise_error(p.status, LCD_ERR_BAD_POINTERS, i);
                active = false;
            }
            d = upper ? e - 1 : s;
            lo = upper ? s : s + 1;
            hi = upper ? e - 1 : e;
        }
        double xi = 0.0;
        if (active && lane == 0) {
            xi = (__ldg(p.b + i) - __ldcg(p.x + i)) / __ldg(p.Ax + d);
            __stcg(p.x + i, xi);
        }
        xi = __shfl_sync(0xffffffffu, xi, lane_in_warp & ~(lanes - 1));
        if (active) {
            for (int j = lo + lane; j < hi; j += lanes) {
                const int r = __ldg(p.Ai + j);
                const bool ok = upper ? (r >= 0 && r < i) : (r > i && r < p.n);
                if (!ok) { raise_error(p.status, LCD_ERR_INDEX_RANGE, i); continue; }
                red_relaxed_add_f64(p.x + r, __dmul_rn(__ldg(p.Ax + j), xi));
            }
        }
    }
}

__global__ void __launch_bounds__(256)
wavefront_level_kernel(const WavefrontParams w, int wave_start, int wave_end) {
    const int gtid = blockIdx.x * blockDim.x + threadIdx.x;
    const int t = wave_start + gtid / w.lanes;
    solve_item(w, t, t < wave_end, gtid % w.lanes, w.lanes);
}

constexpr int kCoopThreads = 512;

// Grid-wide barrier on a monotone 64-bit counter.  Returns false when the solve
// has been aborted (every block then leaves the kernel).
__device__ __forceinline__ bool grid_barrier(const WavefrontParams &w, unsigned long long &target,
                                             int *s_ok) {
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long *counter =
            reinterpret_cast<unsigned long long *>(w.m.status + kStatusBarrier);
        target += gridDim.x;
        int ok = 1;
        __threadfence();
        atomicAdd(counter, 1ull);
        Deadline dl;
        dl.start(w.m.budget_ns);
        while (ld_relaxed_u64(counter) < target) {
            if (dl.tick(w.m.status, -1)) { ok = 0; break; }
        }
        acquire_fence();
        if (aborted(w.m.status)) ok = 0;
        *s_ok = ok;
    }
    __syncthreads();
    return *s_ok != 0;
}

__global__ void __launch_bounds__(kCoopThreads) wavefront_coop_kernel(const WavefrontParams w) {
    __shared__ int s_ok;
    const int lanes = w.lanes;
    const int rows_per_block = kCoopThreads / lanes;
    const int local = threadIdx.x / lanes, lane = threadIdx.x % lanes;
    unsigned long long target = 0;
    int l = 0;
    while (l < w.n_levels) {
        const int ws = __ldg(w.wavefront_ptr + l), we = __ldg(w.wavefront_ptr + l + 1);
        if (we - ws <= rows_per_block) {
            // run of levels that each fit one block: block 0 walks them alone
            int end = l + 1;
            while (end < w.n_levels &&
                   __ldg(w.wavefront_ptr + end + 1) - __ldg(w.wavefront_ptr + end) <= rows_per_block)
                ++end;
            if (blockIdx.x == 0) {
                for (int k = l; k < end; ++k) {
                    const int s = __ldg(w.wavefront_ptr + k), e = __ldg(w.wavefront_ptr + k + 1);
                    const int t = s + local;
                    solve_item(w, t, t < e, lane, lanes);
                    __syncthreads();
                }
            }
            l = end;
        } else {
            const int total_rows = gridDim.x * rows_per_block;
            for (int base = ws + blockIdx.x * rows_per_block; base < we; base += total_rows) {
                const int t = base + local;
                solve_item(w, t, t < we, lane, lanes);
            }
            ++l;
        }
        if (l < w.n_levels && gridDim.x > 1) {
            if (!grid_barrier(w, target, &s_ok)) return;
        } else {
            __syncthreads();
        }
    }
}

// ---- multi-RHS, level-synchronous ---------------------------------------------
// Row-major blocks of right-hand sides: a warp owns a row, lane l owns the columns
// l, l + 32, ...  Every gather of x is a coalesced row segment and there is nothing to
// wait for inside a level, so wide levels stream at memory speed.
template <int KR>
__device__ __forceinline__ void solve_node_multi(const WavefrontParams &w, int node) {
    const CsrSolveParams &p = w.m;
    const int lane = threadIdx.x & 31;
    const bool upper = p.flags & LCD_SOLVE_UPPER;
    const int r = upper ? p.n - 1 - node : node;
    int lo = 0, hi = 0, d = -1;
    if (!csr_row_range(p, r, lo, hi, d)) {
        if (lane == 0)
            raise_error(p.status, (p.flags & LCD_SOLVE_OF_FULL) ? LCD_ERR_MISSING_DIAGONAL
                                                               : LCD_ERR_BAD_POINTERS, r);
        return;
    }
    double acc[KR];
#pragma unroll
    for (int k = 0; k < KR; ++k) {
        const int q = lane + 32 * k;
        acc[k] = q < p.nrhs ? __ldg(p.b + (long long)r * p.ld + q) : 0.0;
    }
    for (int j = lo; j < hi; ++j) {
        const int c = __ldg(p.Ai + j);
        if ((unsigned)c >= (unsigned)p.n) {
            if (lane == 0) raise_error(p.status, LCD_ERR_INDEX_RANGE, r);
            continue;
        }
        const double a = __ldg(p.Ax + j);
        const double *src = p.x + (long long)c * p.ld;
#pragma unroll
        for (int k = 0; k < KR; ++k) {
            const int q = lane + 32 * k;
            if (q < p.nrhs) acc[k] = fma(-a, __ldcg(src + q), acc[k]);
        }
    }
    const double rinv = d >= 0 ? 1.0 / __ldg(p.Ax + d) : 1.0;
#pragma unroll
    for (int k = 0; k < KR; ++k) {
        const int q = lane + 32 * k;
        if (q < p.nrhs) __stcg(p.x + (long long)r * p.ld + q, acc[k] * rinv);
    }
}

template <int KR>
__global__ void __launch_bounds__(kCoopThreads) wavefront_multi_coop_kernel(const WavefrontParams w) {
    __shared__ int s_ok;
    constexpr int rows_per_block = kCoopThreads / 32;
    const int warp = threadIdx.x >> 5;
    unsigned long long target = 0;
    int l = 0;
    while (l < w.n_levels) {
        const int ws = __ldg(w.wavefront_ptr + l), we = __ldg(w.wavefront_ptr + l + 1);
        if (we - ws <= rows_per_block) {
            int end = l + 1;
            while (end < w.n_levels &&
                   __ldg(w.wavefront_ptr + end + 1) - __ldg(w.wavefront_ptr + end) <= rows_per_block)
                ++end;
            if (blockIdx.x == 0) {
                for (int k = l; k < end; ++k) {
                    const int t = __ldg(w.wavefront_ptr + k) + warp;
                    if (t < __ldg(w.wavefront_ptr + k + 1)) {
                        const int node = __ldg(w.wavefronts + t);
                        if ((unsigned)node < (unsigned)w.m.n) solve_node_multi<KR>(w, node);
                    }
                    __syncthreads();
                }
            }
            l = end;
        } else {
            const int total_rows = gridDim.x * rows_per_block;
            for (int t = ws + blockIdx.x * rows_per_block + warp; t < we; t += total_rows) {
                const int node = __ldg(w.wavefronts + t);
                if ((unsigned)node < (unsigned)w.m.n) solve_node_multi<KR>(w, node);
            }
            ++l;
        }
        if (l < w.n_levels && gridDim.x > 1) {
            if (!grid_barrier(w, target, &s_ok)) return;
        } else {
            __syncthreads();
        }
    }
}

template <int KR>
static int launch_multi_coop(WavefrontParams &w, cudaStream_t st) {
    int per_sm = 0;
    LCD_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, wavefront_multi_coop_kernel<KR>,
                                                              kCoopThreads, 0));
    if (per_sm < 1) return LCD_ERR_CUDA;
    long long grid = (long long)per_sm * sm_count();
    const long long useful = ((long long)w.m.n + 15) / 16;
    if (grid > useful) grid = useful;
    if (grid < 1) grid = 1;
    void *args[] = {(void *)&w};
    LCD_CUDA_TRY(cudaLaunchCooperativeKernel((void *)wavefront_multi_coop_kernel<KR>,
                                             dim3((unsigned)grid), dim3(kCoopThreads), args, 0, st));
    return LCD_OK;
}

}  // namespace lcd

using namespace lcd;

static int wavefront_solve(int op, int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                           const double *Ax, const int32_t *diag_pos, const double *b, double *x,
                           int flags, const int32_t *wavefronts, const int32_t *task_ptr_dev,
                           const int32_t *wavefront_ptr_dev, const int32_t *wavefront_ptr_host,
                           int32_t n_levels, int mode, int lanes_per_row, int32_t *status_dev,
                           int32_t timeout_ms, void *stream, int *status_host) {
    if (n < 0 || nnz < 0 || n_levels < 0 || !status_dev) return LCD_ERR_INVALID_ARGUMENT;
    const bool csc = (op == LCD_OP_CSC_LOWER || op == LCD_OP_CSC_UPPER);
    const bool csr = (op == LCD_OP_CSR_LOWER || op == LCD_OP_CSR_UPPER);
    if (!csc && !csr) return LCD_ERR_INVALID_ARGUMENT;
    if (op == LCD_OP_CSR_UPPER || op == LCD_OP_CSC_UPPER) flags |= LCD_SOLVE_UPPER;
    if (csc && (flags & (LCD_SOLVE_OF_FULL | LCD_SOLVE_UNIT_DIAG))) return LCD_ERR_INVALID_ARGUMENT;
    if ((flags & LCD_SOLVE_OF_FULL) && !diag_pos) return LCD_ERR_INVALID_ARGUMENT;
    if ((flags & LCD_SOLVE_UNIT_DIAG) && !(flags & LCD_SOLVE_OF_FULL)) return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && (!Ap || !b || !x || x == b || !wavefronts || !wavefront_ptr_dev))
        return LCD_ERR_INVALID_ARGUMENT;
    if (mode == LCD_WAVEFRONT_PER_LEVEL && n_levels > 0 && !wavefront_ptr_host)
        return LCD_ERR_INVALID_ARGUMENT;
    int lanes = lanes_per_row > 0 ? lanes_per_row : 1;
    if (lanes > 32 || (lanes & (lanes - 1))) return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    int rc = reset_status(status_dev, st);
    if (rc) return rc;
    if (n > 0 && n_levels > 0) {
        if (csc) LCD_CUDA_TRY(cudaMemsetAsync(x, 0, (size_t)n * sizeof(double), st));
        WavefrontParams w;
        w.m = CsrSolveParams{n, nnz, Ap, Ai, Ax, diag_pos, b, x, flags, 1, 1, status_dev,
                             timeout_ns(timeout_ms), nullptr, 0, n, nullptr, {nullptr}};
        w.csc = csc ? 1 : 0;
        w.wavefronts = wavefronts;
        w.wavefront_ptr = wavefront_ptr_dev;
        w.n_levels = n_levels;
        w.lanes = lanes;
        w.task_ptr = task_ptr_dev;
        if (mode == LCD_WAVEFRONT_PER_LEVEL) {
            for (int l = 0; l < n_levels; ++l) {
                const int ws = wavefront_ptr_host[l], we = wavefront_ptr_host[l + 1];
                if (we <= ws) continue;
                const long long threads = (long long)(we - ws) * lanes;
                wavefront_level_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(w, ws, we);
            }
            LCD_CUDA_TRY(cudaGetLastError());
        } else if (mode == LCD_WAVEFRONT_COOPERATIVE) {
            int per_sm = 0;
            LCD_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, wavefront_coop_kernel,
                                                                      kCoopThreads, 0));
            if (per_sm < 1) return LCD_ERR_CUDA;
            const int rows_per_block = kCoopThreads / lanes;
            long long grid = (long long)per_sm * sm_count();
            const long long useful = ((long long)n + rows_per_block - 1) / rows_per_block;
            if (grid > useful) grid = useful;
            if (grid < 1) grid = 1;
            void *args[] = {(void *)&w};
            LCD_CUDA_TRY(cudaLaunchCooperativeKernel((void *)wavefront_coop_kernel, dim3((unsigned)grid),
                                                     dim3(kCoopThreads), args, 0, st));
        } else {
            return LCD_ERR_INVALID_ARGUMENT;
        }
    }
    return finish(status_dev, st, status_host);
}

extern "C" int lcd_sptrsv_wavefront(int op, int32_t n, int64_t nnz, const int32_t *Ap,
                                    const int32_t *Ai, const double *Ax, const int32_t *diag_pos,
                                    const double *b, double *x, int flags,
                                    const int32_t *wavefronts, const int32_t *wavefront_ptr_dev,
                                    const int32_t *wavefront_ptr_host, int32_t n_levels, int mode,
                                    int lanes_per_row, int32_t *status_dev, int32_t timeout_ms,
                                    void *stream, int *status_host) {
    return wavefront_solve(op, n, nnz, Ap, Ai, Ax, diag_pos, b, x, flags, wavefronts, nullptr,
                           wavefront_ptr_dev, wavefront_ptr_host, n_levels, mode, lanes_per_row,
                           status_dev, timeout_ms, stream, status_host);
}

extern "C" int lcd_sptrsv_wavefront_tasks(int op, int32_t n, int64_t nnz, const int32_t *Ap,
                                          const int32_t *Ai, const double *Ax,
                                          const int32_t *diag_pos, const double *b, double *x,
                                          int flags, const int32_t *task_nodes,
                                          const int32_t *task_ptr_dev, const int32_t *band_ptr_dev,
                                          const int32_t *band_ptr_host, int32_t n_bands, int mode,
                                          int lanes_per_row, int32_t *status_dev,
                                          int32_t timeout_ms, void *stream, int *status_host) {
    if (n > 0 && !task_ptr_dev) return LCD_ERR_INVALID_ARGUMENT;
    return wavefront_solve(op, n, nnz, Ap, Ai, Ax, diag_pos, b, x, flags, task_nodes, task_ptr_dev,
                           band_ptr_dev, band_ptr_host, n_bands, mode, lanes_per_row, status_dev,
                           timeout_ms, stream, status_host);
}

extern "C" int lcd_sptrsv_wavefront_multi(int32_t n, int64_t nnz, int32_t nrhs, const int32_t *Ap,
                                          const int32_t *Ai, const double *Ax,
                                          const int32_t *diag_pos, const double *B, double *X,
                                          int64_t ld, int flags, const int32_t *wavefronts,
                                          const int32_t *wavefront_ptr_dev, int32_t n_levels,
                                          int32_t *status_dev, int32_t timeout_ms, void *stream,
                                          int *status_host) {
    if (n < 0 || nnz < 0 || nrhs < 1 || nrhs > 64 || ld < nrhs || n_levels < 0 || !status_dev)
        return LCD_ERR_INVALID_ARGUMENT;
    if ((flags & LCD_SOLVE_OF_FULL) && !diag_pos) return LCD_ERR_INVALID_ARGUMENT;
    if ((flags & LCD_SOLVE_UNIT_DIAG) && !(flags & LCD_SOLVE_OF_FULL)) return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && (!Ap || !B || !X || X == B || !wavefronts || !wavefront_ptr_dev))
        return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    int rc = reset_status(status_dev, st);
    if (rc) return rc;
    if (n > 0 && n_levels > 0) {
        WavefrontParams w;
        w.m = CsrSolveParams{n, nnz, Ap, Ai, Ax, diag_pos, B, X, flags, nrhs, ld, status_dev,
                             timeout_ns(timeout_ms), nullptr, 0, n, nullptr, {nullptr}};
        w.csc = 0;
        w.wavefronts = wavefronts;
        w.wavefront_ptr = wavefront_ptr_dev;
        w.n_levels = n_levels;
        w.lanes = 32;
        w.task_ptr = nullptr;
        rc = nrhs <= 32 ? launch_multi_coop<1>(w, st) : launch_multi_coop<2>(w, st);
        if (rc) return rc;
    }
    return finish(status_dev, st, status_host);
}
