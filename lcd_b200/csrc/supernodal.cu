// Sync-free supernodal lower-triangular solve on column-major panels (sm_100a).
//
// Work is cut into tasks handed out by ticket in dependence-level order (a topological
// order): task (s, 0) waits until every update into the columns of supernode s has arrived
// (pending[s] == 0), solves the dense w x w diagonal block - by one product with its inverse
// when lcd_supernodal_prepare was run (independent loads and multiply-adds), else in
// 32-column steps (a warp solves the 32 x 32 triangle with shuffles, the block then applies
// the 32 solved values to the rows below) - and publishes x_s into a second vector whose
// reserved-NaN pre-fill makes each value its own ready flag; tasks (s, q) wait for those
// values, stream one strip of the off-diagonal panel (coalesced down the columns, sixteen
// loads in flight per thread, the strip pulled towards L2 while the task waits), subtract
// the strip's product from x with fp64 atomics and release the target supernodes' counters,
// one decrement per distinct target per warp.  Every panel value is read exactly once; what
// keeps the solve below the HBM roofline is the critical path through the supernode DAG.
#include "common.cuh"

namespace lcd {

constexpr int kSnThreads = 256;
constexpr int kSnMaxWidth = 1024;  // x_s lives in shared memory

struct SupernodalParams {
    int n_super;
    int n_tasks;
    const int *__restrict__ task_super;
    const int *__restrict__ task_strip;
    const int *__restrict__ sn;
    const int *__restrict__ Lip;
    const int *__restrict__ Li;
    const long long *__restrict__ Lp;
    const double *__restrict__ Lx;
    const int *__restrict__ col_to_super;
    int *pending;
    double *solved;   // x_s as published for the strips (pre-filled with the reserved NaN)
    double *x;
    int n;
    int32_t *status;
    unsigned long long budget_ns;
    const double *__restrict__ inv;        // inverses of the diagonal blocks (column-major w x w), or NULL
    const long long *__restrict__ inv_ptr; // where each supernode's inverse starts
};

__device__ __forceinline__ void prefetch_l2(const void *ptr) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr));
}

__global__ void __launch_bounds__(kSnThreads, 4) supernodal_kernel(const SupernodalParams p) {
    __shared__ double xs[kSnMaxWidth];
    __shared__ double ys[kSnMaxWidth];   // product with the inverse diagonal block
    __shared__ double tri[32][33];  // current 32 x 32 diagonal sub-block, row-major, padded
    double *part = &tri[0][0];      // ... or the partial sums of the threads that share a row
    __shared__ int s_task;
    __shared__ int s_ok;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) s_task = atomicAdd(&p.status[kStatusTicket], 1);
    __syncthreads();
    const int task = s_task;
    if (task >= p.n_tasks) return;
    const int s = __ldg(p.task_super + task);
    const int strip = __ldg(p.task_strip + task);
    const int c0 = __ldg(p.sn + s), w = __ldg(p.sn + s + 1) - c0;
    const int row_begin = __ldg(p.Lip + s);
    const int len = __ldg(p.Lip + s + 1) - row_begin;
    const double *M = p.Lx + __ldg(p.Lp + c0);
    if (w <= 0 || w > kSnMaxWidth || len < w) {
        if (tid == 0) raise_error(p.status, w > kSnMaxWidth ? LCD_ERR_TOO_LARGE : LCD_ERR_BAD_POINTERS, s);
        return;
    }
    // ---- while the inputs are not there yet: pull this task's panel strip (and, for the
    // task that solves the diagonal block, that block) towards L2, so that the dependence
    // wait overlaps the HBM stream instead of preceding it
    {
        const int rows = len - w;
        const int j0 = strip * kSnThreads;
        const int nrow = min(kSnThreads, rows - j0);
        if (nrow > 0) {
            // one prefetch per 32-byte sector: 4 consecutive rows share a sector per column
            const double *P = M + w + j0;
            for (int idx = tid; idx < ((nrow + 3) >> 2) * w; idx += kSnThreads) {
                const int c = idx / ((nrow + 3) >> 2), q = idx % ((nrow + 3) >> 2);
                prefetch_l2(P + (long long)c * len + 4 * q);
            }
        }
        if (strip == 0 && p.inv) {
            const double *inv = p.inv + __ldg(p.inv_ptr + s);
            for (int idx = tid * 4; idx < w * w; idx += kSnThreads * 4) prefetch_l2(inv + idx);
        } else if (strip == 0) {
            for (int idx = tid; idx < ((w + 3) >> 2) * w; idx += kSnThreads) {
                const int c = idx / ((w + 3) >> 2), q = idx % ((w + 3) >> 2);
                prefetch_l2(M + (long long)c * len + 4 * q);
            }
        }
    }
    // ---- wait for the inputs of this task --------------------------------
    // Strip 0 waits for the last update into its columns (a counter, then the values); the
    // other strips wait for x_s itself: the solved values are published into a second vector
    // that was pre-filled with a reserved NaN, so a value is its own ready flag and a strip
    // needs one round trip to L2 instead of two (flag, then values) and no fence.
    if (strip == 0) {
        if (tid == 0) {
            Deadline dl;
            dl.start(p.budget_ns);
            int ok = 1;
            for (;;) {
                if (ld_relaxed_s32(p.pending + s) == 0) { acquire_fence(); break; }
                if (dl.tick(p.status, s)) { ok = 0; break; }
            }
            s_ok = ok;
        }
        __syncthreads();
        if (!s_ok) return;
        for (int c = tid; c < w; c += kSnThreads) xs[c] = ld_relaxed_f64(p.x + c0 + c);
    } else {
        if (tid == 0) s_ok = 1;
        __syncthreads();
        Deadline dl;
        dl.start(p.budget_ns);
        for (int c = tid; c < w; c += kSnThreads) {
            double v;
            while (is_pending(v = ld_relaxed_f64(p.solved + c0 + c)))
                if (dl.tick(p.status, s)) { s_ok = 0; break; }
            xs[c] = v;
        }
        __syncthreads();
        if (!s_ok) return;
    }
    __syncthreads();
    if (strip == 0 && p.inv) {
        // ---- x_s = T^-1 v with the inverse of the diagonal block (lcd_supernodal_prepare): one
        // pass of independent loads and multiply-adds instead of a chain of w dependent steps.
        // A row is shared by 256 / w' threads (w' = w rounded up to a power of two) that take
        // every (256 / w')-th column; wide blocks give every thread several rows.
        const double *inv = p.inv + __ldg(p.inv_ptr + s);
        int wp = 16;
        while (wp < w && wp < kSnThreads) wp <<= 1;
        const int tpr = kSnThreads / wp;              // threads per row (1 when w >= 256)
        const int sub = tid / wp;
        for (int r = tid % wp; r < w; r += wp) {       // (one trip unless w > 256)
            double y0 = 0.0, y1 = 0.0;
            int c = sub;
            for (; c <= r; c += 16 * tpr) {            // sixteen loads in flight, the tail masked
                double m[16];
#pragma unroll
                for (int u = 0; u < 16; ++u)
                    m[u] = c + u * tpr <= r ? __ldg(inv + (long long)(c + u * tpr) * w + r) : 0.0;
#pragma unroll
                for (int u = 0; u < 16; u += 2) {
                    y0 = fma(m[u], xs[min(c + u * tpr, w - 1)], y0);
                    y1 = fma(m[u + 1], xs[min(c + (u + 1) * tpr, w - 1)], y1);
                }
            }
            if (tpr == 1) ys[r] = y0 + y1;
            else part[sub * wp + r] = y0 + y1;
        }
        __syncthreads();
        if (tpr > 1) {
            if (tid < w) {
                double y = 0.0;
                for (int q = 0; q < tpr; ++q) y += part[q * wp + tid];
                ys[tid] = y;
            }
            __syncthreads();
        }
        for (int c = tid; c < w; c += kSnThreads) xs[c] = ys[c];
        __syncthreads();
    } else if (strip == 0) {
        // ---- dense triangular solve, 32 columns at a time --------------------
        for (int cb = 0; cb < w; cb += 32) {
            const int bw = min(32, w - cb);
            // stage the 32 x 32 triangle (coalesced down the columns), then warp 0 solves it
            for (int idx = tid; idx < 32 * bw; idx += kSnThreads) {
                const int c = idx >> 5, rr = idx & 31;
                if (rr < bw && rr >= c) tri[rr][c] = __ldg(M + (long long)(cb + c) * len + cb + rr);
            }
            __syncthreads();
            if (warp == 0) {
                const int r = cb + lane;  // row of this lane inside the diagonal block
                double v = lane < bw ? xs[r] : 0.0;
                // the 32 reciprocals are taken at once, off the 32-step dependent chain (a
                // division per step would cost about 100 cycles each)
                const double rinv = lane < bw ? 1.0 / tri[lane][lane] : 0.0;
                for (int c = 0; c < bw; ++c) {
                    if (lane == c) v = v * rinv;
                    const double xc = __shfl_sync(0xffffffffu, v, c);
                    if (lane > c && lane < bw) v = fma(-tri[lane][c], xc, v);
                }
                if (lane < bw) xs[r] = v;
            }
            __syncthreads();
            for (int r = cb + 32 + tid; r < w; r += kSnThreads) {
                double v0 = xs[r], v1 = 0.0;
                int c = 0;
                for (; c + 16 <= bw; c += 16) {
                    double m[16];
#pragma unroll
                    for (int u = 0; u < 16; ++u) m[u] = __ldg(M + (long long)(cb + c + u) * len + r);
#pragma unroll
                    for (int u = 0; u < 16; u += 2) {
                        v0 = fma(-m[u], xs[cb + c + u], v0);
                        v1 = fma(-m[u + 1], xs[cb + c + u + 1], v1);
                    }
                }
                for (; c < bw; ++c) v0 = fma(-__ldg(M + (long long)(cb + c) * len + r), xs[cb + c], v0);
                xs[r] = v0 + v1;
            }
            __syncthreads();
        }
    }
    if (strip == 0) {
        for (int c = tid; c < w; c += kSnThreads) {
            st_relaxed_f64(p.solved + c0 + c, publishable(xs[c]));   // what the strips wait for
            st_relaxed_f64(p.x + c0 + c, xs[c]);
        }
    }
    // ---- one strip of the off-diagonal panel -------------------------------
    const int rows = len - w;
    const int j = strip * kSnThreads + tid;
    const bool active = j < rows;
    int target = -1;
    if (active) {
        const double *P = M + w + j;
        double acc0 = 0.0, acc1 = 0.0, acc2 = 0.0, acc3 = 0.0;
        int c = 0;
        // sixteen loads in flight per thread: the strip's latency is w / 16 round trips to
        // L2 or HBM instead of w / 4, and a strip sits on the critical path of its level
        for (; c + 16 <= w; c += 16) {
            double v[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) v[u] = __ldg(P + (long long)(c + u) * len);
#pragma unroll
            for (int u = 0; u < 16; u += 4) {
                acc0 = fma(v[u + 0], xs[c + u + 0], acc0);
                acc1 = fma(v[u + 1], xs[c + u + 1], acc1);
                acc2 = fma(v[u + 2], xs[c + u + 2], acc2);
                acc3 = fma(v[u + 3], xs[c + u + 3], acc3);
            }
        }
        for (; c + 4 <= w; c += 4) {
            acc0 = fma(__ldg(P + (long long)(c + 0) * len), xs[c + 0], acc0);
            acc1 = fma(__ldg(P + (long long)(c + 1) * len), xs[c + 1], acc1);
            acc2 = fma(__ldg(P + (long long)(c + 2) * len), xs[c + 2], acc2);
            acc3 = fma(__ldg(P + (long long)(c + 3) * len), xs[c + 3], acc3);
        }
        for (; c < w; ++c) acc0 = fma(__ldg(P + (long long)c * len), xs[c], acc0);
        const int row = __ldg(p.Li + row_begin + w + j);
        if ((unsigned)row >= (unsigned)p.n || row < c0 + w) {
            raise_error(p.status, LCD_ERR_INDEX_RANGE, s);
        } else {
            red_relaxed_add_f64(p.x + row, -((acc0 + acc1) + (acc2 + acc3)));
            target = __ldg(p.col_to_super + row);
        }
    }
    // one counter decrement per distinct target supernode per warp
    const unsigned peers = __match_any_sync(0xffffffffu, target);
    __syncwarp();
    if (target >= 0 && (peers & ((1u << lane) - 1u)) == 0)
        red_release_add_s32(p.pending + target, -__popc(peers));
}

// Inverse of every supernode's w x w lower-triangular diagonal block, column-major with
// leading dimension w at inv[inv_ptr[s]]: thread c computes column c by forward substitution
// (entries above the diagonal are stored as zeros).
__global__ void __launch_bounds__(128)
supernodal_inverse_kernel(int n_super, const int *__restrict__ sn, const int *__restrict__ Lip,
                          const long long *__restrict__ Lp, const double *__restrict__ Lx,
                          const long long *__restrict__ inv_ptr, double *inv,
                          unsigned long long *growth) {
    const int s = blockIdx.x;
    if (s >= n_super) return;
    const int c0 = sn[s], w = sn[s + 1] - c0;
    const int len = Lip[s + 1] - Lip[s];
    const double *M = Lx + Lp[c0];
    double *out = inv + inv_ptr[s];
    // growth of the explicit inverse: largest |entry| of the inverse times largest |diagonal
    // entry| of the block (about 1 for diagonally dominant blocks; NaN counts as inf)
    double inv_max = 0.0, diag_max = 0.0;
    auto absmax = [](double m, double v) {
        v = fabs(v);
        return (v != v) ? (double)INFINITY : (v > m ? v : m);
    };
    for (int c = threadIdx.x; c < w; c += blockDim.x) {
        double *col = out + (long long)c * w;
        for (int r = 0; r < c; ++r) col[r] = 0.0;
        for (int r = c; r < w; ++r) {
            double acc = (r == c) ? 1.0 : 0.0;
            for (int k = c; k < r; ++k) acc = fma(-M[(long long)k * len + r], col[k], acc);
            col[r] = acc / M[(long long)r * len + r];
            inv_max = absmax(inv_max, col[r]);
        }
        diag_max = absmax(diag_max, M[(long long)c * len + c]);
    }
    if (growth) {
        __shared__ unsigned long long s_inv, s_diag;
        if (threadIdx.x == 0) { s_inv = 0ull; s_diag = 0ull; }
        __syncthreads();
        // non-negative doubles order like their bit patterns
        atomicMax(&s_inv, (unsigned long long)__double_as_longlong(inv_max));
        atomicMax(&s_diag, (unsigned long long)__double_as_longlong(diag_max));
        __syncthreads();
        if (threadIdx.x == 0) {
            const double g = __longlong_as_double((long long)s_inv) * __longlong_as_double((long long)s_diag);
            atomicMax(growth, (unsigned long long)__double_as_longlong(g != g ? (double)INFINITY : g));
        }
    }
}

__global__ void supernodal_pending_kernel(int n_super, const int *__restrict__ sn,
                                          const int *__restrict__ Lip, const int *__restrict__ Li,
                                          const int *__restrict__ col_to_super, int *pending) {
    // one warp per supernode, lanes over its off-diagonal rows
    const int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (s >= n_super) return;
    const int w = sn[s + 1] - sn[s];
    for (int j = Lip[s] + w + lane; j < Lip[s + 1]; j += 32) atomicAdd(pending + col_to_super[Li[j]], 1);
}

}  // namespace lcd

using namespace lcd;

extern "C" int lcd_supernodal_pending(int32_t n_super, const int32_t *sn, const int32_t *Lip,
                                      const int32_t *Li, const int32_t *col_to_super,
                                      int32_t *pending, void *stream) {
    if (n_super < 0 || (n_super > 0 && (!sn || !Lip || !Li || !col_to_super || !pending)))
        return LCD_ERR_INVALID_ARGUMENT;
    if (n_super == 0) return LCD_OK;
    cudaStream_t st = (cudaStream_t)stream;
    LCD_CUDA_TRY(cudaMemsetAsync(pending, 0, (size_t)n_super * sizeof(int32_t), st));
    const long long threads = (long long)n_super * 32;
    supernodal_pending_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
        n_super, sn, Lip, Li, col_to_super, pending);
    LCD_CUDA_TRY(cudaGetLastError());
    return LCD_OK;
}

extern "C" int lcd_supernodal_prepare(int32_t n_super, const int32_t *sn, const int32_t *Lip,
                                      const int64_t *Lp, const double *Lx, const int64_t *inv_ptr,
                                      double *inv, double *growth_dev, void *stream) {
    if (n_super < 0 || (n_super > 0 && (!sn || !Lip || !Lp || !Lx || !inv_ptr || !inv)))
        return LCD_ERR_INVALID_ARGUMENT;
    if (growth_dev) LCD_CUDA_TRY(cudaMemsetAsync(growth_dev, 0, sizeof(double), (cudaStream_t)stream));
    if (n_super == 0) return LCD_OK;
    supernodal_inverse_kernel<<<n_super, 128, 0, (cudaStream_t)stream>>>(
        n_super, sn, Lip, reinterpret_cast<const long long *>(Lp), Lx,
        reinterpret_cast<const long long *>(inv_ptr), inv,
        reinterpret_cast<unsigned long long *>(growth_dev));
    LCD_CUDA_TRY(cudaGetLastError());
    return LCD_OK;
}

extern "C" int lcd_supernodal_strip_rows(void) { return kSnThreads; }

extern "C" int lcd_sptrsv_supernodal(int32_t n, int32_t n_super, int32_t n_tasks,
                                     const int32_t *task_super, const int32_t *task_strip,
                                     const int32_t *sn, const int32_t *Lip, const int32_t *Li,
                                     const int64_t *Lp, const double *Lx,
                                     const int32_t *col_to_super, int32_t *pending,
                                     double *solved, double *x, const int64_t *inv_ptr,
                                     const double *inv, int32_t *status_dev, int32_t timeout_ms,
                                     void *stream, int *status_host) {
    if (n < 0 || n_super < 0 || n_tasks < 0 || !status_dev) return LCD_ERR_INVALID_ARGUMENT;
    if (n_super > 0 && (!task_super || !task_strip || !sn || !Lip || !Li || !Lp || !Lx ||
                        !col_to_super || !pending || !solved || !x))
        return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    int rc = reset_status(status_dev, st);
    if (rc) return rc;
    if (n_super > 0 && n_tasks > 0) {
        LCD_CUDA_TRY(cudaMemsetAsync(solved, 0xFF, (size_t)n * sizeof(double), st));
        SupernodalParams p{n_super, n_tasks, task_super, task_strip, sn, Lip, Li,
                           reinterpret_cast<const long long *>(Lp), Lx, col_to_super, pending,
                           solved, x, n, status_dev, timeout_ns(timeout_ms), inv_ptr ? inv : nullptr,
                           reinterpret_cast<const long long *>(inv_ptr)};
        supernodal_kernel<<<n_tasks, kSnThreads, 0, st>>>(p);
        LCD_CUDA_TRY(cudaGetLastError());
    }
    return finish(status_dev, st, status_host);
}
