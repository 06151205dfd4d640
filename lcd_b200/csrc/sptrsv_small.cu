// Triangular solves small enough for one thread block (sm_100a), CSR (pull) and CSC (push).
//
// A solve with a few hundred levels of a few hundred rows each is bound by the hand-off
// between levels, not by bandwidth: through L2 (polling or a grid barrier) a level costs
// 0.5 - 2 us, whatever the kernel.  Here one block walks the level sets with a
// __syncthreads() per level (about 0.1 us) and keeps the recent part of x in shared memory:
//
//   * positions.  Rows are renumbered by their place t in the level order.  x lives in a
//     ring of kRing doubles indexed by t mod kRing; an operand at most kRing / 2 places
//     back (always the case for grid-like matrices) is a shared-memory read, anything
//     further back comes from a position-ordered copy in global memory.
//   * no pointer chasing on the critical path.  Per pattern (once): an ELL image of the
//     matrix in level order - entry e of task t at [e * n + t]: the operand's position and
//     where its value sits in Ax.  Per solve a fully parallel pass gathers values, right-hand
//     side and reciprocal diagonals into that order; the walking kernel then loads everything
//     of a task with independent, coalesced loads whose addresses follow from t alone, issued
//     two turns (several levels) before the task's level comes up.
//   * CSC (the push form of compiler/demo/sptrsv.py:37-43): the ring holds the accumulators
//     of the next kRing / 2 positions, updated with shared-memory atomics; a column reads
//     and clears its slot when its level comes up.
// Nothing spins: the only synchronisation is the block barrier.
#include "common.cuh"

namespace lcd {

constexpr int kRing = 16384;       // doubles of x (or accumulators) kept in shared memory
constexpr int kWptrChunk = 4096;   // level offsets staged per refill
constexpr int kSmallMaxEntries = 8;

struct SmallLayout {
    int n;
    const int *__restrict__ ell_pc;    // [E * n] position of the operand / target, -1: padding
    const int *__restrict__ ell_src;   // [E * n] index into Ax, -1: padding
    const int *__restrict__ row_of;    // [n] matrix row (column) of task t
    const int *__restrict__ diag_src;  // [n] index of the diagonal in Ax, -1: unit diagonal
};

struct SmallSolveParams {
    SmallLayout lay;
    const int *__restrict__ wptr;
    int n_levels;
    int max_width;
    int has_far;
    const double *__restrict__ ell_val;  // [E * n]
    const double *__restrict__ bp;       // [n] right-hand side in level order
    const double *__restrict__ dinv;     // [n] reciprocal diagonals
    double *xp;                          // [n] CSR: x by position; CSC: far accumulators
    double *x;
};

// ---- per pattern -------------------------------------------------------------------
struct SmallOp {
    int op, flags, n;
    long long nnz;
    const int *__restrict__ Ap;
    const int *__restrict__ Ai;
    const int *__restrict__ dpos;
};

// off-diagonal range [lo, hi) and diagonal position of node v's row / column
__device__ __forceinline__ bool small_range(const SmallOp &q, int v, int &i, int &lo, int &hi, int &d) {
    const bool upper = q.op == LCD_OP_CSR_UPPER || q.op == LCD_OP_CSC_UPPER;
    const bool csc = q.op == LCD_OP_CSC_LOWER || q.op == LCD_OP_CSC_UPPER;
    i = upper ? q.n - 1 - v : v;
    if (!csc) {
        CsrSolveParams p{};
        p.n = q.n; p.nnz = q.nnz; p.Ap = q.Ap; p.dpos = q.dpos;
        p.flags = q.flags | (upper ? LCD_SOLVE_UPPER : 0);
        return csr_row_range(p, i, lo, hi, d);
    }
    const int s = q.Ap[i], e = q.Ap[i + 1];
    if (s < 0 || e <= s || (long long)e > q.nnz) return false;
    d = upper ? e - 1 : s;       // lower: diagonal first; upper: diagonal last
    lo = upper ? s : s + 1;
    hi = upper ? e - 1 : e;
    return true;
}

__global__ void small_measure_kernel(const SmallOp q, const int *__restrict__ order,
                                     const int *__restrict__ wptr, int n_levels, int *pos,
                                     int *info, int32_t *status) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < n_levels) atomicMax(info + 1, wptr[t + 1] - wptr[t]);
    if (t >= q.n) return;
    const int v = order[t];
    if ((unsigned)v >= (unsigned)q.n) { raise_error(status, LCD_ERR_INDEX_RANGE, t); return; }
    pos[v] = t;
    int i, lo, hi, d;
    if (!small_range(q, v, i, lo, hi, d)) {
        raise_error(status, (q.flags & LCD_SOLVE_OF_FULL) ? LCD_ERR_MISSING_DIAGONAL : LCD_ERR_BAD_POINTERS, i);
        return;
    }
    atomicMax(info + 0, hi - lo);
}

__global__ void small_fill_kernel(const SmallOp q, const int *__restrict__ order,
                                  const int *__restrict__ pos, int E, int *ell_pc, int *ell_src,
                                  int *row_of, int *diag_src, int *info, int32_t *status) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= q.n) return;
    const bool upper = q.op == LCD_OP_CSR_UPPER || q.op == LCD_OP_CSC_UPPER;
    const bool csc = q.op == LCD_OP_CSC_LOWER || q.op == LCD_OP_CSC_UPPER;
    const int v = order[t];
    int i = 0, lo = 0, hi = 0, d = -1;
    const bool ok = (unsigned)v < (unsigned)q.n && small_range(q, v, i, lo, hi, d);
    if (!ok) { lo = hi = 0; d = -1; }
    row_of[t] = ok ? i : 0;
    diag_src[t] = ok ? d : -1;
    for (int e = 0; e < E; ++e) {
        int pc = -1, src = -1;
        if (lo + e < hi) {
            const int c = q.Ai[lo + e];
            // the other end must lie strictly on the dependent side of the diagonal
            const bool side = (unsigned)c < (unsigned)q.n && ((upper != csc) ? c > i : c < i);
            if (!side) {
                raise_error(status, LCD_ERR_INDEX_RANGE, i);
            } else {
                const int other = pos[upper ? q.n - 1 - c : c];
                // pull: operands stand before the task; push: targets stand after it
                if (csc ? other <= t : other >= t) raise_error(status, LCD_ERR_CYCLE, i);
                else {
                    pc = other;
                    src = lo + e;
                    if ((csc ? other - t : t - other) > kRing / 2) atomicAdd(info + 2, 1);
                }
            }
        }
        ell_pc[(size_t)e * q.n + t] = pc;
        ell_src[(size_t)e * q.n + t] = src;
    }
}

// ---- per solve ------------------------------------------------------------------------
__global__ void small_pack_kernel(const SmallLayout lay, int E, const double *__restrict__ Ax,
                                  const double *__restrict__ b, double *ell_val, double *bp,
                                  double *dinv, double *xp) {
    const int stride = gridDim.x * blockDim.x;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < lay.n; t += stride) {
        bp[t] = b[lay.row_of[t]];
        const int d = lay.diag_src[t];
        dinv[t] = d >= 0 ? 1.0 / Ax[d] : 1.0;
        xp[t] = 0.0;
        for (int e = 0; e < E; ++e) {
            const int s = lay.ell_src[(size_t)e * lay.n + t];
            ell_val[(size_t)e * lay.n + t] = s >= 0 ? Ax[s] : 0.0;
        }
    }
}

template <int E>
struct SmallTask {
    double val[E];
    int pc[E];
    double bb, dinv;
    int row;
};

template <int E>
__device__ __forceinline__ void small_load(SmallTask<E> &q, const SmallSolveParams &p, int t) {
    if (t < p.lay.n) {
#pragma unroll
        for (int e = 0; e < E; ++e) {
            q.val[e] = __ldg(p.ell_val + (size_t)e * p.lay.n + t);
            q.pc[e] = __ldg(p.lay.ell_pc + (size_t)e * p.lay.n + t);
        }
        q.bb = __ldg(p.bp + t);
        q.dinv = __ldg(p.dinv + t);
        q.row = __ldg(p.lay.row_of + t);
    }
}

template <int E, bool CSC, int T, int DEPTH>
__global__ void __launch_bounds__(T, 1) sptrsv_small_kernel(const SmallSolveParams p) {
    extern __shared__ __align__(16) double ring[];  // kRing doubles
    __shared__ int s_wptr[kWptrChunk + 1];
    const int tid = threadIdx.x;
    if (CSC)
        for (int k = tid; k < kRing; k += T) ring[k] = 0.0;
    const bool use_ring = p.max_width <= kRing / 2;
    // two register sets used in turn: a set is reloaded right after its task and not touched
    // again until two turns later, so its loads have several levels to arrive
    SmallTask<E> q0, q1;
    int t = tid;
    int phase = 0;
    small_load(q0, p, t);
    if (DEPTH > 1) small_load(q1, p, t + T);
    auto run = [&](SmallTask<E> &c) {
        const int slot = t & (kRing - 1);
        if (!CSC) {
            double acc = c.bb;
#pragma unroll
            for (int e = 0; e < E; ++e) {
                const int pc = c.pc[e];
                if (pc >= 0) {
                    const double xv = (use_ring && t - pc <= kRing / 2) ? ring[pc & (kRing - 1)]
                                                                        : ld_relaxed_f64(p.xp + pc);
                    acc = fma(-c.val[e], xv, acc);
                }
            }
            const double xi = acc * c.dinv;
            ring[slot] = xi;
            if (p.has_far || !use_ring) st_relaxed_f64(p.xp + t, xi);
            p.x[c.row] = xi;
        } else {
            double accv = ring[slot];
            ring[slot] = 0.0;
            if (p.has_far || !use_ring) accv += ld_relaxed_f64(p.xp + t);
            const double xi = (c.bb - accv) * c.dinv;
            p.x[c.row] = xi;
#pragma unroll
            for (int e = 0; e < E; ++e) {
                const int pt = c.pc[e];
                if (pt >= 0) {
                    const double v = c.val[e] * xi;
                    if (use_ring && pt - t <= kRing / 2) atomicAdd(&ring[pt & (kRing - 1)], v);
                    else red_relaxed_add_f64(p.xp + pt, v);
                }
            }
        }
        small_load(c, p, t + DEPTH * T);
        t += T;
    };
    for (int base = 0; base < p.n_levels; base += kWptrChunk) {
        const int count = min(kWptrChunk, p.n_levels - base);
        __syncthreads();  // the previous chunk of offsets is no longer read (and the ring is cleared)
        for (int k = tid; k <= count; k += T) s_wptr[k] = __ldg(p.wptr + base + k);
        __syncthreads();
        for (int l = 0; l < count; ++l) {
            const int we = s_wptr[l + 1];
            while (t < we) {
                if (DEPTH == 1 || phase == 0) run(q0);
                else run(q1);
                phase ^= 1;
            }
            __syncthreads();
        }
    }
}

template <int E, bool CSC, int T, int DEPTH>
static int launch_small_t(const SmallSolveParams &p, cudaStream_t st) {
    static bool configured = false;
    const int smem = kRing * (int)sizeof(double);
    if (!configured) {
        LCD_CUDA_TRY(cudaFuncSetAttribute(sptrsv_small_kernel<E, CSC, T, DEPTH>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        configured = true;
    }
    sptrsv_small_kernel<E, CSC, T, DEPTH><<<1, T, smem, st>>>(p);
    LCD_CUDA_TRY(cudaGetLastError());
    return LCD_OK;
}

static int g_small_threads = 0;  // LCD_TUNE_SMALL_THREADS: 0 = by level width

template <int E, bool CSC>
static int launch_small_e(const SmallSolveParams &p, cudaStream_t st) {
    int threads = g_small_threads;
    if (threads == 0) threads = p.max_width <= 512 ? 512 : 1024;
    if (threads == 256) return launch_small_t<E, CSC, 256, 2>(p, st);
    if (threads == 512) return launch_small_t<E, CSC, 512, 2>(p, st);
    return launch_small_t<E, CSC, 1024, (E > 4 ? 1 : 2)>(p, st);
}

template <bool CSC>
static int launch_small(const SmallSolveParams &p, int E, cudaStream_t st) {
    if (E <= 2) return launch_small_e<2, CSC>(p, st);
    if (E <= 4) return launch_small_e<4, CSC>(p, st);
    return launch_small_e<8, CSC>(p, st);
}

int set_small_threads(int threads) {
    if (threads != 0 && threads != 256 && threads != 512 && threads != 1024) return LCD_ERR_INVALID_ARGUMENT;
    g_small_threads = threads;
    return LCD_OK;
}

static inline size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

}  // namespace lcd

using namespace lcd;

extern "C" int lcd_small_max_entries(void) { return kSmallMaxEntries; }

extern "C" int lcd_small_plan_measure(int op, int flags, int32_t n, int64_t nnz, const int32_t *Ap,
                                      const int32_t *diag_pos, const int32_t *order,
                                      const int32_t *wavefront_ptr_dev, int32_t n_levels,
                                      int32_t *pos, int32_t *info_dev, int32_t *status_dev,
                                      void *stream, int32_t *info_host) {
    if (n < 0 || nnz < 0 || n_levels < 0 || !info_dev || !status_dev || !info_host)
        return LCD_ERR_INVALID_ARGUMENT;
    if (op != LCD_OP_CSR_LOWER && op != LCD_OP_CSR_UPPER && op != LCD_OP_CSC_LOWER && op != LCD_OP_CSC_UPPER)
        return LCD_ERR_INVALID_ARGUMENT;
    const bool csc = op == LCD_OP_CSC_LOWER || op == LCD_OP_CSC_UPPER;
    if (csc && (flags & (LCD_SOLVE_OF_FULL | LCD_SOLVE_UNIT_DIAG))) return LCD_ERR_INVALID_ARGUMENT;
    if ((flags & LCD_SOLVE_OF_FULL) && !diag_pos) return LCD_ERR_INVALID_ARGUMENT;
    if ((flags & LCD_SOLVE_UNIT_DIAG) && !(flags & LCD_SOLVE_OF_FULL)) return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && (!Ap || !order || !wavefront_ptr_dev || !pos)) return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    int rc = reset_status(status_dev, st);
    if (rc) return rc;
    LCD_CUDA_TRY(cudaMemsetAsync(info_dev, 0, 4 * sizeof(int32_t), st));
    if (n > 0) {
        LCD_CUDA_TRY(cudaMemsetAsync(pos, 0xFF, (size_t)n * sizeof(int32_t), st));
        const SmallOp q{op, flags & (LCD_SOLVE_OF_FULL | LCD_SOLVE_UNIT_DIAG), n, nnz, Ap, nullptr, diag_pos};
        const int m = n > n_levels ? n : n_levels;
        small_measure_kernel<<<(m + 255) / 256, 256, 0, st>>>(q, order, wavefront_ptr_dev, n_levels, pos,
                                                              info_dev, status_dev);
        LCD_CUDA_TRY(cudaGetLastError());
    }
    LCD_CUDA_TRY(cudaMemcpyAsync(info_host, info_dev, 4 * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    int host = 0;
    return finish(status_dev, st, &host);
}

extern "C" int lcd_small_plan_fill(int op, int flags, int32_t n, int64_t nnz, const int32_t *Ap,
                                   const int32_t *Ai, const int32_t *diag_pos, const int32_t *order,
                                   const int32_t *pos, int32_t entries, int32_t *ell_pc,
                                   int32_t *ell_src, int32_t *row_of, int32_t *diag_src,
                                   int32_t *info_dev, int32_t *status_dev, void *stream,
                                   int32_t *far_host) {
    if (n < 0 || nnz < 0 || entries < 1 || entries > kSmallMaxEntries || !info_dev || !status_dev ||
        !far_host)
        return LCD_ERR_INVALID_ARGUMENT;
    if (op != LCD_OP_CSR_LOWER && op != LCD_OP_CSR_UPPER && op != LCD_OP_CSC_LOWER && op != LCD_OP_CSC_UPPER)
        return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && (!Ap || (nnz > 0 && !Ai) || !order || !pos || !ell_pc || !ell_src || !row_of || !diag_src))
        return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    int rc = reset_status(status_dev, st);
    if (rc) return rc;
    LCD_CUDA_TRY(cudaMemsetAsync(info_dev + 2, 0, sizeof(int32_t), st));
    if (n > 0) {
        const SmallOp q{op, flags & (LCD_SOLVE_OF_FULL | LCD_SOLVE_UNIT_DIAG), n, nnz, Ap, Ai, diag_pos};
        small_fill_kernel<<<(n + 255) / 256, 256, 0, st>>>(q, order, pos, entries, ell_pc, ell_src, row_of,
                                                           diag_src, info_dev, status_dev);
        LCD_CUDA_TRY(cudaGetLastError());
    }
    LCD_CUDA_TRY(cudaMemcpyAsync(far_host, info_dev + 2, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    int host = 0;
    return finish(status_dev, st, &host);
}

extern "C" int lcd_small_scratch_bytes(int32_t n, int32_t entries, int64_t *bytes) {
    if (n < 0 || entries < 1 || entries > kSmallMaxEntries || !bytes) return LCD_ERR_INVALID_ARGUMENT;
    const size_t m = (size_t)(n > 0 ? n : 1);
    *bytes = (int64_t)(align256(m * entries * 8) + 3 * align256(m * 8) + 256);
    return LCD_OK;
}

extern "C" int lcd_sptrsv_small(int csc, int32_t n, int32_t entries, const double *Ax, const double *b,
                                double *x, const int32_t *ell_pc, const int32_t *ell_src,
                                const int32_t *row_of, const int32_t *diag_src,
                                const int32_t *wavefront_ptr_dev, int32_t n_levels, int32_t max_width,
                                int32_t has_far, void *scratch, int64_t scratch_bytes, void *stream) {
    if (n < 0 || n_levels < 0 || entries < 1 || entries > kSmallMaxEntries) return LCD_ERR_INVALID_ARGUMENT;
    if (n == 0) return LCD_OK;
    if (!Ax || !b || !x || x == b || !ell_pc || !ell_src || !row_of || !diag_src || !wavefront_ptr_dev ||
        !scratch)
        return LCD_ERR_INVALID_ARGUMENT;
    int64_t need = 0;
    lcd_small_scratch_bytes(n, entries, &need);
    if (scratch_bytes < need) return LCD_ERR_WORKSPACE;
    if (((uintptr_t)scratch & 255) != 0) return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    char *base = static_cast<char *>(scratch);
    double *ell_val = reinterpret_cast<double *>(base);
    base += align256((size_t)n * entries * 8);
    double *bp = reinterpret_cast<double *>(base);
    base += align256((size_t)n * 8);
    double *dinv = reinterpret_cast<double *>(base);
    base += align256((size_t)n * 8);
    double *xp = reinterpret_cast<double *>(base);
    const SmallLayout lay{n, ell_pc, ell_src, row_of, diag_src};
    const int blocks = (n + 255) / 256 < 148 * 8 ? (n + 255) / 256 : 148 * 8;
    small_pack_kernel<<<blocks, 256, 0, st>>>(lay, entries, Ax, b, ell_val, bp, dinv, xp);
    LCD_CUDA_TRY(cudaGetLastError());
    const SmallSolveParams p{lay, wavefront_ptr_dev, n_levels, max_width, has_far, ell_val, bp, dinv, xp, x};
    return csc ? launch_small<true>(p, entries, st) : launch_small<false>(p, entries, st);
}
