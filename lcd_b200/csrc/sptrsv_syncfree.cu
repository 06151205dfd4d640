// Sync-free sparse triangular solves (CSR pull, CSC push, multi-RHS) for sm_100a.
//
// Scheduling.  Rows are handed out in node order through a ticket taken by each
// thread block when it starts running, so a block only ever waits for rows that
// belong to blocks already resident or finished: the waits cannot deadlock.
// A block owns a contiguous chunk of rows; one lane group (1..32 lanes) owns a row.
//
// Hand-off (CSR).  The solution vector is pre-filled with a reserved NaN bit
// pattern.  A consumer polls the operand x[c] itself: an aligned 8-byte store is
// single-copy atomic, so no flag, counter or fence is needed.  Rows of the own
// chunk are mirrored in shared memory, which turns dependences between nearby
// rows (the critical chain of banded / grid matrices) into shared-memory polls.
//
// Every wait is bounded by a wall-clock budget; on expiry the kernel records
// LCD_ERR_TIMEOUT in the status block, all other waiters observe it and drain.
#include "common.cuh"

namespace lcd {

template <int G, int TPB, int MINB>
__global__ void __launch_bounds__(TPB, MINB) csr_syncfree_kernel(const CsrSolveParams p) {
    constexpr int R = TPB / G;
    __shared__ double sx[R];
    __shared__ int s_chunk;
    const int tid = threadIdx.x;
    if (tid == 0) s_chunk = atomicAdd(&p.status[kStatusTicket], 1);
    if (tid < R) reinterpret_cast<unsigned long long *>(sx)[tid] = kPendingBits;
    __syncthreads();
    volatile double *sxv = sx;
    const int row0 = s_chunk * R;  // node id of the chunk's first row
    const int local = tid / G;
    const int lane = tid % G;
    const int task = row0 + local;
    // (no early return: every lane of a warp takes part in the votes below)
    bool done = task >= p.n;
    const bool upper = p.flags & LCD_SOLVE_UPPER;
    const bool exact = p.flags & LCD_SOLVE_EXACT;
    const int r = upper ? p.n - 1 - task : task;
    constexpr unsigned kFull = 0xffffffffu;
    const unsigned gmask =
        G == 32 ? kFull : (((1u << G) - 1u) << ((threadIdx.x & 31) & ~(G - 1)));

    int lo = 0, hi = 0, d = -1;
    bool failed = false;
    if (done) {
        // a group past the last row: nothing to do
    } else if (!csr_row_range(p, r, lo, hi, d)) {
        if (lane == 0)
            raise_error(p.status, (p.flags & LCD_SOLVE_OF_FULL) ? LCD_ERR_MISSING_DIAGONAL
                                                               : LCD_ERR_BAD_POINTERS, r);
        failed = true;
        lo = hi = 0;
        d = -1;
    }
    double acc = 0.0, dv = 1.0, rinv = 1.0;
    if (lane == 0 && !done) {
        acc = __ldg(p.b + r);
        if (d >= 0) dv = __ldg(p.Ax + d);
        if (!exact) rinv = 1.0 / dv;  // off the critical path: computed before any wait
    }
    int j = lo + lane;
    bool have = j < hi;
    int c = 0;
    double a = 0.0;
    if (have) { c = __ldg(p.Ai + j); a = __ldg(p.Ax + j); }
    Deadline dl;
    dl.start(p.budget_ns);
    for (;;) {
        if (have) {
            const int tc = upper ? p.n - 1 - c : c;
            if ((unsigned)tc >= (unsigned)task) {  // not strictly before this row
                raise_error(p.status, LCD_ERR_INDEX_RANGE, r);
                failed = true;
                have = false;
            } else {
                const double xv = (tc >= row0) ? sxv[tc - row0] : ld_relaxed_f64(p.x + c);
                if (!is_pending(xv)) {
                    acc = exact ? __dsub_rn(acc, __dmul_rn(a, xv)) : fma(-a, xv, acc);
                    j += G;
                    have = j < hi;
                    if (have) { c = __ldg(p.Ai + j); a = __ldg(p.Ax + j); }
                } else if (dl.tick(p.status, r)) {
                    failed = true;
                    have = false;
                }
            }
        }
        // Votes are full-warp ballots read through the group's mask, and the reduction runs in
        // a warp-uniform branch: a vote or shuffle with one member mask per group is executed
        // once per group and leaves the groups split (measured: branch_resolving as the top
        // stall of this kernel).
        bool group_done;
        if (G == 1) {
            group_done = !done && !have;
        } else {
            const unsigned idle = __ballot_sync(kFull, done || !have);
            group_done = !done && (idle & gmask) == gmask;
        }
        if (G == 1 ? group_done : __any_sync(kFull, group_done)) {
            double sum = acc;
            if (G > 1) {
#pragma unroll
                for (int off = G / 2; off > 0; off >>= 1) sum += __shfl_xor_sync(kFull, sum, off, G);
                const unsigned bad = __ballot_sync(kFull, failed);
                if (group_done) failed = (bad & gmask) != 0;
            }
            if (group_done) {
                if (lane == 0) {
                    double val = (d < 0) ? sum : (exact ? sum / dv : sum * rinv);
                    if (failed) val = __longlong_as_double(kCanonicalNaN);
                    val = publishable(val);
                    st_relaxed_f64(p.x + r, val);
                    sxv[local] = val;
                }
                done = true;
            }
        }
        if (G == 1 ? done : __all_sync(kFull, done)) break;
    }
}

// Tunables of the thread-per-row kernel (set through lcd_set_tuning).
struct RowTuning {
    int sleep_local_ns;   // pause after a failed poll of the shared-memory mirror
    int sleep_global_ns;  // pause after a failed poll of x in global memory
    int gap_ns;           // pause per row of distance between the awaited row and the
                          // progress of the warp that owns it (0 = off)
    int variant;          // 0: thread-per-row kernel for one lane per row, 1: generic kernel
    int stage_percent;    // staging area for matrix entries, percent of the average chunk
};
static RowTuning g_row_tuning = {0, 200, 0, 0, 120};

// Thread per row.  Leading operands that live before the chunk and are already
// available are consumed first without waiting; everything else goes through a
// single try-advance loop (shared-memory mirror for rows of the own chunk, global
// memory otherwise).  Rows complete roughly in index order inside a warp, so a
// per-warp completion count tells a waiting thread how far the producer's warp is
// from the row it needs; distant waiters pause instead of burning issue slots that
// the threads on the critical chain need.
template <int TPB, int MINB, bool EXACT>
__global__ void __launch_bounds__(TPB, MINB)
csr_syncfree_row_kernel(const CsrSolveParams p, const RowTuning tune, const int cap) {
    constexpr int kWarps = TPB / 32;
    // dynamic shared memory: x mirror of the chunk | staged values | staged operands
    extern __shared__ __align__(16) unsigned char row_smem[];
    double *sx = reinterpret_cast<double *>(row_smem);
    double *sval = sx + TPB;
    int *sidx = reinterpret_cast<int *>(sval + cap);
    __shared__ int s_wdone[kWarps];
    __shared__ int s_chunk;
    const int tid = threadIdx.x;
    if (tid == 0) s_chunk = atomicAdd(&p.status[kStatusTicket], 1);
    reinterpret_cast<unsigned long long *>(sx)[tid] = kPendingBits;
    if (tid < kWarps) s_wdone[tid] = 0;
    __syncthreads();
    volatile double *sxv = sx;
    volatile int *wdone = s_wdone;
    const int row0 = p.task_begin + s_chunk * TPB;
    const int task = row0 + tid;
    const bool upper = p.flags & LCD_SOLVE_UPPER;
    // The rows of a chunk are contiguous in the matrix, so their entries form one
    // segment of Ai / Ax: stage it with coalesced loads before anybody waits, so
    // that no matrix fetch sits on a dependence chain.  Staged operands are stored
    // as node ids relative to the chunk (>= 0: a row of this chunk, mirrored in
    // shared memory; < 0: a row of an earlier chunk, polled in global memory).
    const int task_end = min(row0 + TPB, p.task_end);
    const int first_row = upper ? p.n - task_end : row0;
    const int last_row = upper ? p.n - 1 - row0 : task_end - 1;
    long long seg_begin = 0;
    int count = 0;
    if (task_end > row0) {
        seg_begin = __ldg(p.Ap + first_row);
        const long long seg_end = __ldg(p.Ap + last_row + 1);
        if (seg_begin >= 0 && seg_end >= seg_begin && seg_end <= p.nnz)
            count = (int)min((long long)cap, seg_end - seg_begin);
        else
            seg_begin = 0;
    }
    for (int k = tid; k < count; k += TPB) {
        const int c = __ldg(p.Ai + seg_begin + k);
        // out-of-range columns become "far in the future": caught by the per-row check
        const bool in_range = (unsigned)c < (unsigned)p.n;
        sidx[k] = in_range ? (upper ? p.n - 1 - c : c) - row0 : TPB;
        sval[k] = __ldg(p.Ax + seg_begin + k);
    }
    __syncthreads();
    if (task >= p.task_end) return;
    const int r = upper ? p.n - 1 - task : task;
    int lo = 0, hi = 0, d = -1;
    if (!csr_row_range(p, r, lo, hi, d)) {
        raise_error(p.status, (p.flags & LCD_SOLVE_OF_FULL) ? LCD_ERR_MISSING_DIAGONAL
                                                           : LCD_ERR_BAD_POINTERS, r);
        const double nanv = __longlong_as_double(kCanonicalNaN);
        sxv[tid] = nanv;
        st_relaxed_f64(p.x + r, nanv);
        return;
    }
    const int sbase = (int)seg_begin;  // seg_begin <= nnz < 2^31
    double acc = __ldg(p.b + r);
    double dv = 1.0, rinv = 1.0;
    if (d >= 0) dv = ((unsigned)(d - sbase) < (unsigned)count) ? sval[d - sbase] : __ldg(p.Ax + d);
    if (!EXACT) rinv = 1.0 / dv;  // off the critical path: computed before any wait
    // operand j: cl = node id relative to the chunk, a = matrix value
#define LCD_FETCH(j_, cl_, a_)                                                   \
    do {                                                                         \
        const unsigned pos_ = (unsigned)((j_) - sbase);                          \
        if (pos_ < (unsigned)count) {                                            \
            cl_ = sidx[pos_];                                                    \
            a_ = sval[pos_];                                                     \
        } else {                                                                 \
            const int c_ = __ldg(p.Ai + (j_));                                   \
            a_ = __ldg(p.Ax + (j_));                                             \
            cl_ = ((unsigned)c_ < (unsigned)p.n) ? (upper ? p.n - 1 - c_ : c_) - row0 : TPB; \
        }                                                                        \
    } while (0)
#define LCD_GLOBAL_X(cl_) (p.x + (upper ? p.n - 1 - ((cl_) + row0) : (cl_) + row0))
#define LCD_ACCUMULATE(a_, xv_) \
    acc = EXACT ? __dsub_rn(acc, __dmul_rn((a_), (xv_))) : fma(-(a_), (xv_), acc)
    int j = lo;
    int cl = 0, cl_next = 0;
    double a = 0.0, a_next = 0.0;
    bool failed = false;
    if (j < hi) {
        LCD_FETCH(j, cl, a);
        // fast-forward over operands of earlier chunks that are already there
        while (cl < 0) {
            const double xv = ld_relaxed_f64(LCD_GLOBAL_X(cl));
            if (is_pending(xv)) break;
            LCD_ACCUMULATE(a, xv);
            if (++j == hi) break;
            LCD_FETCH(j, cl, a);
        }
    }
    if (j + 1 < hi) LCD_FETCH(j + 1, cl_next, a_next);
    Deadline dl;
    dl.start(p.budget_ns);
    // One loop, publication inside it: a lane that is done never has to reconverge
    // with lanes of its warp that still wait (they may be waiting for this very row).
    for (;;) {
        if (j < hi && !failed) {
            if (cl >= tid) {  // not strictly before this row (or out of range)
                raise_error(p.status, LCD_ERR_INDEX_RANGE, r);
                failed = true;
            } else {
                const double xv = cl >= 0 ? sxv[cl] : ld_relaxed_f64(LCD_GLOBAL_X(cl));
                if (!is_pending(xv)) {
                    LCD_ACCUMULATE(a, xv);
                    ++j;
                    cl = cl_next;
                    a = a_next;
                    if (j + 1 < hi) LCD_FETCH(j + 1, cl_next, a_next);
                } else if (dl.tick(p.status, r)) {
                    failed = true;
                } else if (cl >= 0) {
                    int pause = tune.sleep_local_ns;
                    if (tune.gap_ns) {
                        const int gap = (cl & 31) - wdone[cl >> 5];  // rows the owner warp owes
                        if (gap > 1) pause += (gap - 1) * tune.gap_ns;
                    }
                    if (pause > 0) __nanosleep(pause);
                } else if (tune.sleep_global_ns > 0) {
                    __nanosleep(tune.sleep_global_ns);
                }
            }
        }
        if (j >= hi || failed) {
            double val = (d < 0) ? acc : (EXACT ? acc / dv : acc * rinv);
            if (failed) val = __longlong_as_double(kCanonicalNaN);
            val = publishable(val);
            sxv[tid] = val;
            st_relaxed_f64(p.x + r, val);
            if (p.need_mask) {  // rows of other GPUs wait for this value in their own memory
                unsigned m = p.need_mask[r];
                while (m) {
                    const int q = __ffs(m) - 1;
                    m &= m - 1;
                    st_relaxed_sys_f64(p.peers[q] + r, val);
                }
            }
            if (tune.gap_ns) atomicAdd(&s_wdone[tid >> 5], 1);
            if (p.trace) p.trace[task] = clock64();
            break;
        }
    }
#undef LCD_FETCH
#undef LCD_GLOBAL_X
#undef LCD_ACCUMULATE
}

// Multi-RHS: the block of right-hand sides is row-major, W consecutive lanes own a
// row, lane l owns the right-hand sides l, l + W, ... (KR of them at most).  A lane
// polls exactly the operand elements it consumes (written by the same lane position of
// the producer row), so lanes never have to agree on anything.  Few lanes per row keep
// many rows in flight, which is what grid-like matrices need.
template <int W, int KR, int TPB>
__global__ void __launch_bounds__(TPB) csr_syncfree_multi_kernel(const CsrSolveParams p) {
    constexpr int R = TPB / W;
    constexpr int NC = W * KR;  // columns of the shared-memory mirror
    extern __shared__ double smem_multi[];  // R x NC
    __shared__ int s_chunk;
    const int tid = threadIdx.x;
    if (tid == 0) s_chunk = atomicAdd(&p.status[kStatusTicket], 1);
    for (int k = tid; k < R * NC; k += TPB)
        reinterpret_cast<unsigned long long *>(smem_multi)[k] = kPendingBits;
    __syncthreads();
    volatile double *sxv = smem_multi;
    const int row0 = s_chunk * R;
    const int local = tid / W;
    const int lane = tid % W;
    const int task = row0 + local;
    if (task >= p.n) return;
    const bool upper = p.flags & LCD_SOLVE_UPPER;
    const int r = upper ? p.n - 1 - task : task;
    int lo = 0, hi = 0, d = -1;
    bool failed = false;
    if (!csr_row_range(p, r, lo, hi, d)) {
        if (lane == 0)
            raise_error(p.status, (p.flags & LCD_SOLVE_OF_FULL) ? LCD_ERR_MISSING_DIAGONAL
                                                               : LCD_ERR_BAD_POINTERS, r);
        failed = true;
        lo = hi = 0;
        d = -1;
    }
    // number of right-hand sides this lane owns: lane, lane + W, ...
    const int nlive = lane < p.nrhs ? min(KR, (p.nrhs - lane + W - 1) / W) : 0;
    if (nlive == 0) return;
    double acc[KR];
#pragma unroll
    for (int k = 0; k < KR; ++k)
        acc[k] = k < nlive ? __ldg(p.b + (long long)r * p.ld + lane + k * W) : 0.0;
    const double rinv = d >= 0 ? 1.0 / __ldg(p.Ax + d) : 1.0;
    int j = lo;
    bool have = j < hi;
    int c = 0;
    double a = 0.0;
    if (have) { c = __ldg(p.Ai + j); a = __ldg(p.Ax + j); }
    Deadline dl;
    dl.start(p.budget_ns);
    for (;;) {
        if (have) {
            const int tc = upper ? p.n - 1 - c : c;
            if ((unsigned)tc >= (unsigned)task) {
                raise_error(p.status, LCD_ERR_INDEX_RANGE, r);
                failed = true;
                have = false;
            } else {
                // all operands of this lane for entry j; they are published together
                double xv[KR];
                bool ready = true;
                if (tc >= row0) {
                    const int base = (tc - row0) * NC + lane;
#pragma unroll
                    for (int k = 0; k < KR; ++k)
                        if (k < nlive) { xv[k] = sxv[base + k * W]; ready = ready && !is_pending(xv[k]); }
                } else {
                    const double *src = p.x + (long long)c * p.ld + lane;
#pragma unroll
                    for (int k = 0; k < KR; ++k)
                        if (k < nlive) { xv[k] = ld_relaxed_f64(src + k * W); ready = ready && !is_pending(xv[k]); }
                }
                if (ready) {
#pragma unroll
                    for (int k = 0; k < KR; ++k)
                        if (k < nlive) acc[k] = fma(-a, xv[k], acc[k]);
                    ++j;
                    have = j < hi;
                    if (have) { c = __ldg(p.Ai + j); a = __ldg(p.Ax + j); }
                } else if (dl.tick(p.status, r)) {
                    failed = true;
                    have = false;
                }
            }
        } else {
            const double nanv = __longlong_as_double(kCanonicalNaN);
#pragma unroll
            for (int k = 0; k < KR; ++k) {
                if (k < nlive) {
                    const double v = publishable(failed ? nanv : acc[k] * rinv);
                    sxv[local * NC + lane + k * W] = v;
                    st_relaxed_f64(p.x + (long long)r * p.ld + lane + k * W, v);
                }
            }
            break;
        }
    }
}

// ---- CSC, push protocol ---------------------------------------------------
struct CscSolveParams {
    int n;
    long long nnz;
    const int *__restrict__ Ap;
    const int *__restrict__ Ai;
    const double *__restrict__ Ax;
    const double *__restrict__ b;
    double *x;
    int *dep;
    int flags;
    int32_t *status;
    unsigned long long budget_ns;
};

template <int G, int TPB>
__global__ void __launch_bounds__(TPB) csc_syncfree_kernel(const CscSolveParams p) {
    constexpr int R = TPB / G;
    __shared__ int s_chunk;
    const int tid = threadIdx.x;
    if (tid == 0) s_chunk = atomicAdd(&p.status[kStatusTicket], 1);
    __syncthreads();
    const int local = tid / G;
    const int lane = tid % G;
    const int task = s_chunk * R + local;
    if (task >= p.n) return;
    const bool upper = p.flags & LCD_SOLVE_UPPER;
    const bool exact = p.flags & LCD_SOLVE_EXACT;
    const int i = upper ? p.n - 1 - task : task;
    const unsigned gmask =
        G == 32 ? 0xffffffffu : (((1u << G) - 1u) << ((threadIdx.x & 31) & ~(G - 1)));
    const int s = __ldg(p.Ap + i), e = __ldg(p.Ap + i + 1);
    int state = 0;  // 0 waiting, 1 go, 2 give up
    if (s < 0 || e <= s || (long long)e > p.nnz) {
        if (lane == 0) raise_error(p.status, LCD_ERR_BAD_POINTERS, i);
        state = 2;
    }
    const int d = upper ? e - 1 : s;
    const int lo = upper ? s : s + 1;
    const int hi = upper ? e - 1 : e;
    double bv = 0.0, dv = 1.0, rinv = 1.0;
    if (lane == 0 && state == 0) {
        bv = __ldg(p.b + i);
        dv = __ldg(p.Ax + d);
        if (!exact) rinv = 1.0 / dv;
    }
    Deadline dl;
    dl.start(p.budget_ns);
    for (;;) {
        if (lane == 0 && state == 0) {
            if (ld_relaxed_s32(p.dep + i) == 0) { acquire_fence(); state = 1; }
            else if (dl.tick(p.status, i)) state = 2;
        }
        if (G > 1) state = __shfl_sync(gmask, state, 0, G);
        if (state == 1) {
            double xi = 0.0;
            if (lane == 0) {
                const double accv = ld_relaxed_f64(p.x + i);
                xi = exact ? __dsub_rn(bv, accv) / dv : (bv - accv) * rinv;
                st_relaxed_f64(p.x + i, xi);
            }
            if (G > 1) xi = __shfl_sync(gmask, xi, 0, G);
            for (int j = lo + lane; j < hi; j += G) {
                const int r = __ldg(p.Ai + j);
                const bool ok = upper ? (r >= 0 && r < i) : (r > i && r < p.n);
                if (!ok) {
                    raise_error(p.status, LCD_ERR_INDEX_RANGE, i);
                    continue;
                }
                red_relaxed_add_f64(p.x + r, __dmul_rn(__ldg(p.Ax + j), xi));
                red_release_add_s32(p.dep + r, -1);
            }
            break;
        }
        if (state == 2) break;
    }
}

__global__ void csc_edge_count_kernel(int n, const int *__restrict__ Ap,
                                      const int *__restrict__ Ai, int upper, int *count) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int s = Ap[i], e = Ap[i + 1];
    const int lo = upper ? s : s + 1, hi = upper ? e - 1 : e;
    for (int j = lo; j < hi; ++j) {
        const int r = Ai[j];
        const bool ok = upper ? (r >= 0 && r < i) : (r > i && r < n);
        if (ok) atomicAdd(count + r, 1);
    }
}

__global__ void fill_u64_kernel(unsigned long long *dst, long long count, unsigned long long v) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < count; k += stride)
        dst[k] = v;
}

__global__ void transpose_f64_kernel(long long rows, long long cols, const double *__restrict__ in,
                                     long long ld_in, double *__restrict__ out, long long ld_out) {
    // in is rows x cols with leading dimension ld_in (element (r,c) at in[r*ld_in + c]);
    // out is cols x rows.  32x32 tiles through padded shared memory.
    __shared__ double tile[32][33];
    const long long c0 = (long long)blockIdx.x * 32, r0 = (long long)blockIdx.y * 32;
    for (int k = threadIdx.y; k < 32; k += blockDim.y) {
        const long long r = r0 + k, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[k][threadIdx.x] = in[r * ld_in + c];
    }
    __syncthreads();
    for (int k = threadIdx.y; k < 32; k += blockDim.y) {
        const long long c = c0 + k, r = r0 + threadIdx.x;
        if (r < rows && c < cols) out[c * ld_out + r] = tile[threadIdx.x][k];
    }
}

static int pick_lanes(long long nnz, int n) {
    const double avg = n > 0 ? (double)nnz / n : 0.0;
    if (avg <= 24) return 1;
    if (avg <= 48) return 2;
    if (avg <= 96) return 4;
    if (avg <= 192) return 8;
    if (avg <= 384) return 16;
    return 32;
}

// Shared memory of the thread-per-row kernel: the x mirror plus room for the
// chunk's matrix entries (12 bytes each).  `stage` scales the staging area
// relative to the average chunk (0 disables staging).
static size_t row_kernel_smem(int tpb, long long nnz, int n, int *cap_out) {
    const size_t limit = 227 * 1024 - 256;
    const double avg = n > 0 ? (double)nnz / n : 0.0;
    long long cap = g_row_tuning.stage_percent > 0
                        ? (long long)(avg * tpb * g_row_tuning.stage_percent / 100.0) + 256 : 0;
    const long long max_cap = ((long long)limit - (long long)tpb * 8) / 12;
    if (cap > max_cap) cap = max_cap;
    cap &= ~1ll;  // keeps the index area 8-byte aligned
    *cap_out = (int)cap;
    return (size_t)tpb * 8 + (size_t)cap * 12;
}

template <int TPB, int MINB, bool EXACT>
static cudaError_t launch_csr_row_t(const CsrSolveParams &p, cudaStream_t st) {
    int cap = 0;
    const size_t smem = row_kernel_smem(TPB, p.nnz, p.n, &cap);
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(csr_syncfree_row_kernel<TPB, MINB, EXACT>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)(227 * 1024 - 256));
        if (e != cudaSuccess) return e;
        configured = true;
    }
    csr_syncfree_row_kernel<TPB, MINB, EXACT>
        <<<(p.task_end - p.task_begin + TPB - 1) / TPB, TPB, smem, st>>>(p, g_row_tuning, cap);
    return cudaGetLastError();
}

static cudaError_t launch_csr_row(const CsrSolveParams &p, int tpb, cudaStream_t st) {
    const bool exact = p.flags & LCD_SOLVE_EXACT;
    if (tpb == 1024)
        return exact ? launch_csr_row_t<1024, 1, true>(p, st) : launch_csr_row_t<1024, 1, false>(p, st);
    if (tpb == 512)
        return exact ? launch_csr_row_t<512, 2, true>(p, st) : launch_csr_row_t<512, 2, false>(p, st);
    return exact ? launch_csr_row_t<256, 4, true>(p, st) : launch_csr_row_t<256, 4, false>(p, st);
}

template <int G>
static cudaError_t launch_csr(const CsrSolveParams &p, int tpb, cudaStream_t st) {
    if (tpb == 1024) {
        constexpr int R = 1024 / G;
        csr_syncfree_kernel<G, 1024, 1><<<(p.n + R - 1) / R, 1024, 0, st>>>(p);
    } else if (tpb == 512) {
        constexpr int R = 512 / G;
        csr_syncfree_kernel<G, 512, 3><<<(p.n + R - 1) / R, 512, 0, st>>>(p);
    } else {
        constexpr int R = 256 / G;
        csr_syncfree_kernel<G, 256, 6><<<(p.n + R - 1) / R, 256, 0, st>>>(p);
    }
    return cudaGetLastError();
}

template <int G>
static cudaError_t launch_csc(const CscSolveParams &p, cudaStream_t st) {
    constexpr int TPB = 256, R = TPB / G;
    csc_syncfree_kernel<G, TPB><<<(p.n + R - 1) / R, TPB, 0, st>>>(p);
    return cudaGetLastError();
}

template <int W, int KR>
static cudaError_t launch_multi(const CsrSolveParams &p, cudaStream_t st) {
    constexpr int TPB = 512, R = TPB / W;
    const size_t smem = (size_t)R * W * KR * sizeof(double);
    if (smem > 48 * 1024) {
        static bool configured = false;
        if (!configured) {
            cudaError_t e = cudaFuncSetAttribute(csr_syncfree_multi_kernel<W, KR, TPB>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem);
            if (e != cudaSuccess) return e;
            configured = true;
        }
    }
    csr_syncfree_multi_kernel<W, KR, TPB><<<(p.n + R - 1) / R, TPB, smem, st>>>(p);
    return cudaGetLastError();
}

}  // namespace lcd

using namespace lcd;

extern "C" int lcd_set_tuning(int key, int value) {
    switch (key) {
        case LCD_TUNE_SLEEP_LOCAL_NS: g_row_tuning.sleep_local_ns = value; break;
        case LCD_TUNE_SLEEP_GLOBAL_NS: g_row_tuning.sleep_global_ns = value; break;
        case LCD_TUNE_GAP_NS: g_row_tuning.gap_ns = value; break;
        case LCD_TUNE_ROW_VARIANT: g_row_tuning.variant = value; break;
        case LCD_TUNE_STAGE_PERCENT: g_row_tuning.stage_percent = value; break;
        case LCD_TUNE_CHAIN_CLUSTER: return set_chain_cluster_limit(value);
        case LCD_TUNE_ORDERED_PAUSE_NS: return set_ordered_pause(value);
        case LCD_TUNE_SMALL_THREADS: return set_small_threads(value);
        case LCD_TUNE_ILU0_LOOKAHEAD: return set_ilu0_lookahead(value);
        case LCD_TUNE_ORDERED_MIN_LANES: return set_ordered_min_lanes(value);
        default: return LCD_ERR_INVALID_ARGUMENT;
    }
    return LCD_OK;
}

extern "C" int lcd_fill_u64(uint64_t *dst, int64_t count, uint64_t value, void *stream) {
    if (count < 0 || (count > 0 && !dst)) return LCD_ERR_INVALID_ARGUMENT;
    if (count == 0) return LCD_OK;
    const int blocks = (int)((count + 1023) / 1024 < 148 * 16 ? (count + 1023) / 1024 : 148 * 16);
    fill_u64_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<unsigned long long *>(dst), count, value);
    LCD_CUDA_TRY(cudaGetLastError());
    return LCD_OK;
}

extern "C" int lcd_transpose_f64(int64_t rows, int64_t cols, const double *in, int64_t ld_in,
                                 double *out, int64_t ld_out, void *stream) {
    if (rows < 0 || cols < 0 || ld_in < cols || ld_out < rows) return LCD_ERR_INVALID_ARGUMENT;
    if (rows == 0 || cols == 0) return LCD_OK;
    const long long gx = (cols + 31) / 32, gy = (rows + 31) / 32;
    if (gy > 65535) {
        // split the row range so that gridDim.y stays legal
        const int64_t step = 65535LL * 32;
        for (int64_t r = 0; r < rows; r += step) {
            const int64_t part = rows - r < step ? rows - r : step;
            dim3 grid((unsigned)gx, (unsigned)((part + 31) / 32));
            transpose_f64_kernel<<<grid, dim3(32, 8), 0, (cudaStream_t)stream>>>(
                part, cols, in + r * ld_in, ld_in, out + r, ld_out);
        }
    } else {
        dim3 grid((unsigned)gx, (unsigned)gy);
        transpose_f64_kernel<<<grid, dim3(32, 8), 0, (cudaStream_t)stream>>>(rows, cols, in, ld_in,
                                                                           out, ld_out);
    }
    LCD_CUDA_TRY(cudaGetLastError());
    return LCD_OK;
}

extern "C" int lcd_sptrsv_csr_syncfree(int32_t n, int64_t nnz, const int32_t *Ap,
                                       const int32_t *Ai, const double *Ax,
                                       const int32_t *diag_pos, const double *b, double *x,
                                       int flags, int lanes_per_row, int threads_per_block,
                                       int32_t *status_dev, int32_t timeout_ms, void *stream,
                                       int *status_host) {
    if (n < 0 || nnz < 0 || !status_dev) return LCD_ERR_INVALID_ARGUMENT;
    if ((flags & LCD_SOLVE_OF_FULL) && !diag_pos) return LCD_ERR_INVALID_ARGUMENT;
    if ((flags & LCD_SOLVE_UNIT_DIAG) && !(flags & LCD_SOLVE_OF_FULL))
        return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && (!Ap || !b || !x || (nnz > 0 && (!Ai || !Ax)))) return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && x == b) return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    int G = lanes_per_row > 0 ? lanes_per_row : pick_lanes(nnz, n);
    if (flags & LCD_SOLVE_EXACT) G = 1;
    int tpb = threads_per_block > 0 ? threads_per_block : 1024;
    if (tpb != 256 && tpb != 512 && tpb != 1024) return LCD_ERR_INVALID_ARGUMENT;
    int rc = reset_status(status_dev, st);
    if (rc) return rc;
    if (n > 0) {
        LCD_CUDA_TRY(cudaMemsetAsync(x, 0xFF, (size_t)n * sizeof(double), st));
        CsrSolveParams p{n, nnz, Ap, Ai, Ax, diag_pos, b, x, flags, 1, 1, status_dev,
                         timeout_ns(timeout_ms), debug_trace(), 0, n, nullptr, {nullptr}};
        cudaError_t e;
        switch (G) {
            case 1:
                e = g_row_tuning.variant == 0 ? launch_csr_row(p, tpb, st) : launch_csr<1>(p, tpb, st);
                break;
            case 2: e = launch_csr<2>(p, tpb, st); break;
            case 4: e = launch_csr<4>(p, tpb, st); break;
            case 8: e = launch_csr<8>(p, tpb, st); break;
            case 16: e = launch_csr<16>(p, tpb, st); break;
            case 32: e = launch_csr<32>(p, tpb, st); break;
            default: return LCD_ERR_INVALID_ARGUMENT;
        }
        LCD_CUDA_TRY(e);
    }
    return finish(status_dev, st, status_host);
}

extern "C" int lcd_sptrsv_csr_syncfree_multi(int32_t n, int64_t nnz, int32_t nrhs,
                                             const int32_t *Ap, const int32_t *Ai,
                                             const double *Ax, const int32_t *diag_pos,
                                             const double *B, double *X, int64_t ld, int flags,
                                             int32_t *status_dev, int32_t timeout_ms,
                                             void *stream, int *status_host) {
    if (n < 0 || nnz < 0 || nrhs < 1 || nrhs > 64 || ld < nrhs || !status_dev)
        return LCD_ERR_INVALID_ARGUMENT;
    if ((flags & LCD_SOLVE_OF_FULL) && !diag_pos) return LCD_ERR_INVALID_ARGUMENT;
    if ((flags & LCD_SOLVE_UNIT_DIAG) && !(flags & LCD_SOLVE_OF_FULL))
        return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && (!Ap || !B || !X || X == B)) return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    int rc = reset_status(status_dev, st);
    if (rc) return rc;
    if (n > 0) {
        // X may be strided (ld > nrhs): fill the whole block, padding included.
        LCD_CUDA_TRY(cudaMemsetAsync(X, 0xFF, (size_t)n * (size_t)ld * sizeof(double), st));
        CsrSolveParams p{n, nnz, Ap, Ai, Ax, diag_pos, B, X, flags, nrhs, ld, status_dev,
                         timeout_ns(timeout_ms), nullptr, 0, n, nullptr, {nullptr}};
        cudaError_t e;
        // few lanes per row keep many rows in flight; a lane owns up to 8 right-hand sides
        if (nrhs <= 1) e = launch_multi<1, 1>(p, st);
        else if (nrhs <= 2) e = launch_multi<2, 1>(p, st);
        else if (nrhs <= 4) e = launch_multi<4, 1>(p, st);
        else if (nrhs <= 8) e = launch_multi<4, 2>(p, st);
        else if (nrhs <= 16) e = launch_multi<4, 4>(p, st);
        else if (nrhs <= 32) e = launch_multi<8, 4>(p, st);
        else e = launch_multi<8, 8>(p, st);
        LCD_CUDA_TRY(e);
    }
    return finish(status_dev, st, status_host);
}

extern "C" int lcd_csc_edge_count(int32_t n, const int32_t *Ap, const int32_t *Ai, int flags,
                                  int32_t *edge_count, void *stream) {
    if (n < 0 || (n > 0 && (!Ap || !edge_count))) return LCD_ERR_INVALID_ARGUMENT;
    if (n == 0) return LCD_OK;
    cudaStream_t st = (cudaStream_t)stream;
    LCD_CUDA_TRY(cudaMemsetAsync(edge_count, 0, (size_t)n * sizeof(int32_t), st));
    csc_edge_count_kernel<<<(n + 255) / 256, 256, 0, st>>>(n, Ap, Ai,
                                                          (flags & LCD_SOLVE_UPPER) ? 1 : 0,
                                                          edge_count);
    LCD_CUDA_TRY(cudaGetLastError());
    return LCD_OK;
}

extern "C" int lcd_sptrsv_csc_syncfree(int32_t n, int64_t nnz, const int32_t *Ap,
                                       const int32_t *Ai, const double *Ax, const double *b,
                                       double *x, int32_t *dep_count, int flags,
                                       int lanes_per_col, int32_t *status_dev,
                                       int32_t timeout_ms, void *stream, int *status_host) {
    if (n < 0 || nnz < 0 || !status_dev) return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && (!Ap || !Ai || !Ax || !b || !x || !dep_count || x == b))
        return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    int G = lanes_per_col > 0 ? lanes_per_col : pick_lanes(nnz, n);
    int rc = reset_status(status_dev, st);
    if (rc) return rc;
    if (n > 0) {
        LCD_CUDA_TRY(cudaMemsetAsync(x, 0, (size_t)n * sizeof(double), st));
        CscSolveParams p{n, nnz, Ap, Ai, Ax, b, x, dep_count, flags, status_dev,
                         timeout_ns(timeout_ms)};
        cudaError_t e;
        switch (G) {
            case 1: e = launch_csc<1>(p, st); break;
            case 2: e = launch_csc<2>(p, st); break;
            case 4: e = launch_csc<4>(p, st); break;
            case 8: e = launch_csc<8>(p, st); break;
            case 16: e = launch_csc<16>(p, st); break;
            case 32: e = launch_csc<32>(p, st); break;
            default: return LCD_ERR_INVALID_ARGUMENT;
        }
        LCD_CUDA_TRY(e);
    }
    return finish(status_dev, st, status_host);
}

// ---- block-row partition across GPUs --------------------------------------------
// need[c] gets bit q set when a row owned by rank q (q != owner of c) stores an
// off-diagonal entry in column c.  bounds[0..parts] are node (task) boundaries.
__global__ void partition_need_kernel(int n, const int *__restrict__ Ap, const int *__restrict__ Ai,
                                      int upper, int of_full_unused, const int *__restrict__ bounds,
                                      int parts, unsigned *need_words) {
    const int task = blockIdx.x * blockDim.x + threadIdx.x;
    if (task >= n) return;
    const int r = upper ? n - 1 - task : task;
    int owner = 0;
    while (owner + 1 < parts && task >= bounds[owner + 1]) ++owner;
    const int s = Ap[r], e = Ap[r + 1];
    const int lo = upper ? s + 1 : s, hi = upper ? e : e - 1;
    for (int j = lo; j < hi; ++j) {
        const int c = Ai[j];
        if ((unsigned)c >= (unsigned)n) continue;
        const int tc = upper ? n - 1 - c : c;
        if (tc < bounds[owner])  // produced on another GPU
            atomicOr(need_words + (c >> 2), (1u << owner) << ((c & 3) * 8));
    }
}

extern "C" int lcd_partition_need_mask(int32_t n, const int32_t *Ap, const int32_t *Ai, int flags,
                                       const int32_t *bounds_dev, int32_t parts,
                                       unsigned char *need_mask, void *stream) {
    if (n < 0 || parts < 1 || parts > 8 || (n > 0 && (!Ap || !Ai || !bounds_dev || !need_mask)))
        return LCD_ERR_INVALID_ARGUMENT;
    if (n == 0) return LCD_OK;
    cudaStream_t st = (cudaStream_t)stream;
    // the mask array must be padded to a multiple of 4 bytes (it is updated word-wise)
    LCD_CUDA_TRY(cudaMemsetAsync(need_mask, 0, ((size_t)n + 3) / 4 * 4, st));
    partition_need_kernel<<<(n + 255) / 256, 256, 0, st>>>(
        n, Ap, Ai, (flags & LCD_SOLVE_UPPER) ? 1 : 0, 0, bounds_dev, parts,
        reinterpret_cast<unsigned *>(need_mask));
    LCD_CUDA_TRY(cudaGetLastError());
    return LCD_OK;
}

extern "C" int lcd_sptrsv_csr_syncfree_part(int32_t n, int64_t nnz, const int32_t *Ap,
                                            const int32_t *Ai, const double *Ax, const double *b,
                                            double *x, int flags, int32_t task_begin,
                                            int32_t task_end, const unsigned char *need_mask,
                                            double *const *peer_x, int32_t n_ranks,
                                            int threads_per_block, int32_t *status_dev,
                                            int32_t timeout_ms, void *stream, int *status_host) {
    if (n < 0 || nnz < 0 || !status_dev || task_begin < 0 || task_end < task_begin || task_end > n ||
        n_ranks < 1 || n_ranks > 8)
        return LCD_ERR_INVALID_ARGUMENT;
    if (flags & (LCD_SOLVE_OF_FULL | LCD_SOLVE_UNIT_DIAG)) return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && (!Ap || !Ai || !Ax || !b || !x || x == b)) return LCD_ERR_INVALID_ARGUMENT;
    if (need_mask && !peer_x) return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    int tpb = threads_per_block > 0 ? threads_per_block : 1024;
    if (tpb != 256 && tpb != 512 && tpb != 1024) return LCD_ERR_INVALID_ARGUMENT;
    int rc = reset_status(status_dev, st);
    if (rc) return rc;
    if (task_end > task_begin) {
        // x is NOT filled here: every rank fills its x with the reserved pattern and all
        // ranks synchronise on the host before the first rank is allowed to publish
        CsrSolveParams p{n, nnz, Ap, Ai, Ax, nullptr, b, x, flags, 1, 1, status_dev,
                         timeout_ns(timeout_ms), nullptr, task_begin, task_end, need_mask, {nullptr}};
        for (int q = 0; q < n_ranks && peer_x; ++q) p.peers[q] = peer_x[q];
        LCD_CUDA_TRY(launch_csr_row(p, tpb, st));
    }
    return finish(status_dev, st, status_host);
}
