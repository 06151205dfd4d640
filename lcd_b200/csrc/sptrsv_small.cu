// Triangular solves small enough for one thread block (sm_100a), for CSR and CSC storage.
//
// A solve with a few hundred levels of a few hundred rows each is bound by the hand-off
// between levels, not by bandwidth: through L2 (polling or a grid barrier) a level costs
// 0.5 - 2 us, whatever the kernel.  Here one block walks the level sets with a
// __syncthreads() per level and keeps the recent part of x in shared memory:
//
//   * positions.  Rows are renumbered by their place t in the level order.  x lives in a
//     ring of kRing doubles indexed by t mod kRing; an operand at most kRing / 2 places
//     back (always the case for grid-like matrices) is a shared-memory read, anything
//     further back comes from the position-ordered copy in global memory.
//   * no pointer chasing, few instructions on the critical path.  The block's time per level
//     is the instruction latency of the warps that own the level's rows, so everything a task
//     needs sits in two records whose addresses follow from t alone: {values of its entries,
//     right-hand side, reciprocal diagonal} (doubles, gathered per solve by a fully parallel
//     pass) and {positions of its operands} (ints, per pattern), fetched with 128-bit loads
//     two turns (several levels) before the task's level comes up.  x is stored by position
//     (coalesced); a last parallel pass puts it back into matrix order.
//   * whole warps per level.  The scoreboard that tracks outstanding loads belongs to the warp,
//     not the lane: if lanes of one warp had their turns in consecutive levels, the lanes of
//     level l + 1 would wait for the prefetches the lanes of level l had just issued into the
//     same registers (measured: an L2 round trip per level).  So every level is padded to a
//     multiple of 32 task slots: a warp's lanes always work in the same level, and the next
//     level belongs to other warps.
//   * CSC (the push loop of compiler/demo/sptrsv.py:37-43) is served by the same pull walk:
//     the per-pattern pass transposes the structure (a column's entry becomes an operand of
//     its row's task, operands sorted by column as the loop accumulates them), so there are no
//     atomics and the result does not depend on timing.
// Nothing spins: the only synchronisation is the block barrier.
#include "common.cuh"

namespace lcd {

constexpr int kRing = 16384;       // doubles of x kept in shared memory
constexpr int kWptrChunk = 4096;   // level offsets staged per refill
constexpr int kSmallMaxEntries = 8;

struct SmallLayout {
    int n;                              // task slots (every level padded to a multiple of 32)
    int entries;                        // E: operand slots per task (2, 4 or 8)
    const int *__restrict__ rec_pc;     // [n * E] position of operand e of task t, -1: padding
    const int *__restrict__ rec_src;    // [n * E] index of its value in Ax, -1: padding
    const int *__restrict__ row_of;     // [n] matrix row (column) of task t, -1: padding slot
    const int *__restrict__ diag_src;   // [n] index of the diagonal in Ax, -1: unit diagonal
};

struct SmallSolveParams {
    SmallLayout lay;
    const int *__restrict__ wptr;
    int n_levels;
    int max_width;
    const double *__restrict__ rec_val;  // [n * (E + 2)]: values, right-hand side, reciprocal diagonal
    double *xp;                          // [n] x by position
    long long *trace;                    // profiling aid (lcd_debug_set_trace): SM cycle counter after
                                         // every level's barrier [n_levels], then, for the tasks of
                                         // thread 0, at the start / after the stores / at the end [3 each]
};

// ---- per pattern -------------------------------------------------------------------
struct SmallOp {
    int op, flags, n;
    long long nnz;
    const int *__restrict__ Ap;
    const int *__restrict__ Ai;
    const int *__restrict__ dpos;
};

__device__ __forceinline__ bool small_is_upper(int op) { return op == LCD_OP_CSR_UPPER || op == LCD_OP_CSC_UPPER; }
__device__ __forceinline__ bool small_is_csc(int op) { return op == LCD_OP_CSC_LOWER || op == LCD_OP_CSC_UPPER; }

// off-diagonal range [lo, hi) and diagonal position of node v's row / column
__device__ __forceinline__ bool small_range(const SmallOp &q, int v, int &i, int &lo, int &hi, int &d) {
    const bool upper = small_is_upper(q.op);
    i = upper ? q.n - 1 - v : v;
    if (!small_is_csc(q.op)) {
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

// pass 1: place of every node in the order, widest level, longest row (CSR)
__global__ void small_measure_kernel(const SmallOp q, const int *__restrict__ order,
                                     const int *__restrict__ level, const int *__restrict__ wptr,
                                     const int *__restrict__ slot_ptr, int n_levels, int *pos,
                                     int *info, int32_t *status) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < n_levels) atomicMax(info + 1, wptr[t + 1] - wptr[t]);
    if (t >= q.n) return;
    const int v = order[t];
    if ((unsigned)v >= (unsigned)q.n) { raise_error(status, LCD_ERR_INDEX_RANGE, t); return; }
    const int l = level[v];
    if ((unsigned)l >= (unsigned)n_levels || t < wptr[l] || t >= wptr[l + 1]) {
        raise_error(status, LCD_ERR_INDEX_RANGE, t);     // order and levels do not belong together
        return;
    }
    pos[v] = slot_ptr[l] + (t - wptr[l]);    // the level's first slot is a multiple of 32
    int i, lo, hi, d;
    if (!small_range(q, v, i, lo, hi, d)) {
        raise_error(status, (q.flags & LCD_SOLVE_OF_FULL) ? LCD_ERR_MISSING_DIAGONAL : LCD_ERR_BAD_POINTERS, i);
        return;
    }
    if (!small_is_csc(q.op)) atomicMax(info + 0, hi - lo);
}

// pass 2 (CSC): operands per task = entries per ROW; cursor[t] counts them
__global__ void small_count_rows_kernel(const SmallOp q, const int *__restrict__ order,
                                        const int *__restrict__ pos, int *cursor, int *info,
                                        int32_t *status) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= q.n) return;
    const bool upper = small_is_upper(q.op);
    const int v = order[t];
    if ((unsigned)v >= (unsigned)q.n) return;
    int i, lo, hi, d;
    if (!small_range(q, v, i, lo, hi, d)) return;
    for (int j = lo; j < hi; ++j) {
        const int r = q.Ai[j];
        const bool side = (unsigned)r < (unsigned)q.n && (upper ? r < i : r > i);
        if (!side) { raise_error(status, LCD_ERR_INDEX_RANGE, i); continue; }
        const int target = pos[upper ? q.n - 1 - r : r];
        if (target < 0) { raise_error(status, LCD_ERR_INDEX_RANGE, i); continue; }
        atomicMax(info + 0, atomicAdd(cursor + target, 1) + 1);
    }
}

__global__ void small_fill_kernel(const SmallOp q, const int *__restrict__ order,
                                  const int *__restrict__ pos, int E, int *rec_pc, int *rec_src,
                                  int *row_of, int *diag_src, int *cursor, int *info, int32_t *status) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= q.n) return;
    const bool upper = small_is_upper(q.op);
    const bool csc = small_is_csc(q.op);
    const int v = order[t];
    int i = 0, lo = 0, hi = 0, d = -1;
    const bool ok = (unsigned)v < (unsigned)q.n && small_range(q, v, i, lo, hi, d) && pos[v] >= 0;
    if (!ok) return;                     // reported by the measuring pass; the slot stays padding
    const int slot = pos[v];             // (all slots were preset to padding by the caller)
    row_of[slot] = i;
    diag_src[slot] = d;
    if (!csc) {
        for (int e = 0; e < E; ++e) {
            int pc = -1, src = -1;
            if (lo + e < hi) {
                const int c = q.Ai[lo + e];
                // an operand lies strictly on the solved side of the diagonal ...
                const bool side = (unsigned)c < (unsigned)q.n && (upper ? c > i : c < i);
                if (!side) {
                    raise_error(status, LCD_ERR_INDEX_RANGE, i);
                } else {
                    const int other = pos[upper ? q.n - 1 - c : c];
                    // ... and stands before the task in the order
                    if (other < 0 || other >= slot) raise_error(status, LCD_ERR_CYCLE, i);
                    else {
                        pc = other;
                        src = lo + e;
                        if (slot - other > kRing / 2) atomicAdd(info + 2, 1);
                    }
                }
            }
            rec_pc[(size_t)slot * E + e] = pc;
            rec_src[(size_t)slot * E + e] = src;
        }
        return;
    }
    // CSC: entry (r, i) of this column is an operand of row r's task (the slots were cleared
    // to -1 by the caller; cursor hands out the slots, a later pass sorts them)
    for (int j = lo; j < hi; ++j) {
        const int r = q.Ai[j];
        const bool side = (unsigned)r < (unsigned)q.n && (upper ? r < i : r > i);
        if (!side) continue;                         // reported by the counting pass
        const int target = pos[upper ? q.n - 1 - r : r];
        if (target <= slot) { raise_error(status, LCD_ERR_CYCLE, i); continue; }
        const int k = atomicAdd(cursor + target, 1);
        if (k >= E) continue;                        // cannot happen: E covers the longest row
        rec_pc[(size_t)target * E + k] = slot;
        rec_src[(size_t)target * E + k] = j;
        if (target - slot > kRing / 2) atomicAdd(info + 2, 1);
    }
}

// CSC: the operands of a task in the order the column loop accumulates them (ascending column
// for a lower, descending for an upper solve), which also makes the result independent of the
// order the slots were handed out in.
__global__ void small_sort_slots_kernel(int n, int E, int upper, const int *__restrict__ row_of,
                                        int *rec_pc, int *rec_src) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n) return;
    int *pc = rec_pc + (size_t)t * E, *src = rec_src + (size_t)t * E;
    for (int a = 1; a < E; ++a) {
        const int p = pc[a], s = src[a];
        if (p < 0) break;
        const int key = upper ? -row_of[p] : row_of[p];
        int b = a - 1;
        while (b >= 0 && (upper ? -row_of[pc[b]] : row_of[pc[b]]) > key) {
            pc[b + 1] = pc[b];
            src[b + 1] = src[b];
            --b;
        }
        pc[b + 1] = p;
        src[b + 1] = s;
    }
}

// ---- per solve ------------------------------------------------------------------------
__global__ void small_pack_kernel(const SmallLayout lay, const double *__restrict__ Ax,
                                  const double *__restrict__ b, double *rec_val) {
    const int E = lay.entries, stride = gridDim.x * blockDim.x;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < lay.n; t += stride) {
        double *rec = rec_val + (size_t)t * (E + 2);
        for (int e = 0; e < E; ++e) {
            const int s = lay.rec_src[(size_t)t * E + e];
            rec[e] = s >= 0 ? Ax[s] : 0.0;
        }
        const int row = lay.row_of[t];
        const int d = lay.diag_src[t];
        rec[E] = row >= 0 ? b[row] : 0.0;            // (padding slots solve to 0 and go nowhere)
        rec[E + 1] = row < 0 ? 0.0 : (d >= 0 ? 1.0 / Ax[d] : 1.0);
    }
}

// The walk stores x by position (coalesced); this pass puts it back into matrix order.
__global__ void small_unpack_kernel(int n, const int *__restrict__ row_of, const double *__restrict__ xp,
                                    double *__restrict__ x) {
    const int stride = gridDim.x * blockDim.x;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < n; t += stride)
        if (row_of[t] >= 0) x[row_of[t]] = xp[t];
}

template <int E>
struct SmallTask {
    double val[E];
    double bb, dinv;
    int pc[E];
};

template <int E>
__device__ __forceinline__ void small_load(SmallTask<E> &q, const SmallSolveParams &p, int t) {
    if (t < p.lay.n) {
        // two records per task, 16-byte aligned (E + 2 and E are even): 128-bit loads
        const double2 *rv = reinterpret_cast<const double2 *>(p.rec_val + (size_t)t * (E + 2));
#pragma unroll
        for (int k = 0; k < E / 2; ++k) {
            const double2 v = __ldg(rv + k);
            q.val[2 * k] = v.x;
            q.val[2 * k + 1] = v.y;
        }
        const double2 tail = __ldg(rv + E / 2);
        q.bb = tail.x;
        q.dinv = tail.y;
        if (E == 2) {
            const int2 c = __ldg(reinterpret_cast<const int2 *>(p.lay.rec_pc + (size_t)t * E));
            q.pc[0] = c.x;
            q.pc[1] = c.y;
        } else {
            const int4 *rc = reinterpret_cast<const int4 *>(p.lay.rec_pc + (size_t)t * E);
#pragma unroll
            for (int k = 0; k < E / 4; ++k) {
                const int4 c = __ldg(rc + k);
                q.pc[4 * k] = c.x; q.pc[4 * k + 1] = c.y; q.pc[4 * k + 2] = c.z; q.pc[4 * k + 3] = c.w;
            }
        }
    }
}

template <int E, int T, int DEPTH>
__global__ void __launch_bounds__(T, 1) sptrsv_small_kernel(const SmallSolveParams p) {
    extern __shared__ __align__(16) double ring[];  // kRing doubles
    __shared__ int s_wptr[kWptrChunk + 1];
    const int tid = threadIdx.x;
    const bool use_ring = p.max_width <= kRing / 2;
    // two register sets used in turn: a set is reloaded right after its task and not touched
    // again until two turns later, so its loads have several levels to arrive
    SmallTask<E> q0, q1;
    int t = tid;
    int phase = 0;
    small_load(q0, p, t);
    if (DEPTH > 1) small_load(q1, p, t + T);
    int traced = 0;
    auto run = [&](SmallTask<E> &c) {
        if (p.trace && tid == 0) p.trace[p.n_levels + 3 * traced] = clock64();
        double acc = c.bb;
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const int pc = c.pc[e];
            if (pc >= 0) {
                const double xv = (use_ring && t - pc <= kRing / 2) ? ring[pc & (kRing - 1)]
                                                                    : *(volatile const double *)(p.xp + pc);
                acc = fma(-c.val[e], xv, acc);
            }
        }
        const double xi = acc * c.dinv;
        ring[t & (kRing - 1)] = xi;
        p.xp[t] = xi;                      // consecutive tasks, consecutive addresses (a plain store:
                                           // the block barrier orders it for the block's own readers)
        if (p.trace && tid == 0) p.trace[p.n_levels + 3 * traced + 1] = clock64();
        small_load(c, p, t + DEPTH * T);
        t += T;
        if (p.trace && tid == 0) p.trace[p.n_levels + 3 * traced++ + 2] = clock64();
    };
    for (int base = 0; base < p.n_levels; base += kWptrChunk) {
        const int count = min(kWptrChunk, p.n_levels - base);
        __syncthreads();  // the previous chunk of offsets is no longer read
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
            if (p.trace && tid == 0) p.trace[base + l] = clock64();
        }
    }
}

template <int E, int T, int DEPTH>
static int launch_small_t(const SmallSolveParams &p, cudaStream_t st) {
    static bool configured = false;
    const int smem = kRing * (int)sizeof(double);
    if (!configured) {
        LCD_CUDA_TRY(cudaFuncSetAttribute(sptrsv_small_kernel<E, T, DEPTH>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        configured = true;
    }
    sptrsv_small_kernel<E, T, DEPTH><<<1, T, smem, st>>>(p);
    LCD_CUDA_TRY(cudaGetLastError());
    return LCD_OK;
}

static int g_small_threads = 0;  // LCD_TUNE_SMALL_THREADS: 0 = by level width

template <int E>
static int launch_small_e(const SmallSolveParams &p, cudaStream_t st) {
    int threads = g_small_threads;
    if (threads == 0) threads = p.max_width <= 512 ? 512 : 1024;
    if (threads == 256) return launch_small_t<E, 256, 2>(p, st);
    if (threads == 512) return launch_small_t<E, 512, 2>(p, st);
    return launch_small_t<E, 1024, (E > 4 ? 1 : 2)>(p, st);
}

int set_small_threads(int threads) {
    if (threads != 0 && threads != 256 && threads != 512 && threads != 1024) return LCD_ERR_INVALID_ARGUMENT;
    g_small_threads = threads;
    return LCD_OK;
}

static inline size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

static bool small_op_ok(int op) {
    return op == LCD_OP_CSR_LOWER || op == LCD_OP_CSR_UPPER || op == LCD_OP_CSC_LOWER || op == LCD_OP_CSC_UPPER;
}

}  // namespace lcd

using namespace lcd;

extern "C" int lcd_small_max_entries(void) { return kSmallMaxEntries; }

extern "C" int lcd_small_plan_measure(int op, int flags, int32_t n, int64_t nnz, const int32_t *Ap,
                                      const int32_t *Ai, const int32_t *diag_pos, const int32_t *order,
                                      const int32_t *level, const int32_t *wavefront_ptr_dev,
                                      const int32_t *slot_ptr_dev, int32_t n_levels, int32_t n_slots,
                                      int32_t *pos, int32_t *cursor, int32_t *info_dev,
                                      int32_t *status_dev, void *stream, int32_t *info_host) {
    if (n < 0 || nnz < 0 || n_levels < 0 || n_slots < n || !info_dev || !status_dev || !info_host ||
        !small_op_ok(op))
        return LCD_ERR_INVALID_ARGUMENT;
    const bool csc = op == LCD_OP_CSC_LOWER || op == LCD_OP_CSC_UPPER;
    if (csc && (flags & (LCD_SOLVE_OF_FULL | LCD_SOLVE_UNIT_DIAG))) return LCD_ERR_INVALID_ARGUMENT;
    if ((flags & LCD_SOLVE_OF_FULL) && !diag_pos) return LCD_ERR_INVALID_ARGUMENT;
    if ((flags & LCD_SOLVE_UNIT_DIAG) && !(flags & LCD_SOLVE_OF_FULL)) return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && (!Ap || !order || !level || !wavefront_ptr_dev || !slot_ptr_dev || !pos ||
                  (csc && (!cursor || !Ai))))
        return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    int rc = reset_status(status_dev, st);
    if (rc) return rc;
    LCD_CUDA_TRY(cudaMemsetAsync(info_dev, 0, 4 * sizeof(int32_t), st));
    if (n > 0) {
        LCD_CUDA_TRY(cudaMemsetAsync(pos, 0xFF, (size_t)n * sizeof(int32_t), st));
        const SmallOp q{op, flags & (LCD_SOLVE_OF_FULL | LCD_SOLVE_UNIT_DIAG), n, nnz, Ap, Ai, diag_pos};
        const int m = n > n_levels ? n : n_levels;
        small_measure_kernel<<<(m + 255) / 256, 256, 0, st>>>(q, order, level, wavefront_ptr_dev, slot_ptr_dev,
                                                              n_levels, pos, info_dev, status_dev);
        if (csc) {
            LCD_CUDA_TRY(cudaMemsetAsync(cursor, 0, (size_t)n_slots * sizeof(int32_t), st));
            small_count_rows_kernel<<<(n + 255) / 256, 256, 0, st>>>(q, order, pos, cursor, info_dev,
                                                                     status_dev);
        }
        LCD_CUDA_TRY(cudaGetLastError());
    }
    LCD_CUDA_TRY(cudaMemcpyAsync(info_host, info_dev, 4 * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    int host = 0;
    return finish(status_dev, st, &host);
}

extern "C" int lcd_small_plan_fill(int op, int flags, int32_t n, int64_t nnz, const int32_t *Ap,
                                   const int32_t *Ai, const int32_t *diag_pos, const int32_t *order,
                                   const int32_t *pos, int32_t n_slots, int32_t entries, int32_t *rec_pc,
                                   int32_t *rec_src, int32_t *row_of, int32_t *diag_src,
                                   int32_t *cursor, int32_t *info_dev, int32_t *status_dev,
                                   void *stream, int32_t *far_host) {
    if (n < 0 || nnz < 0 || n_slots < n || (entries != 2 && entries != 4 && entries != 8) || !info_dev ||
        !status_dev || !far_host || !small_op_ok(op))
        return LCD_ERR_INVALID_ARGUMENT;
    const bool csc = op == LCD_OP_CSC_LOWER || op == LCD_OP_CSC_UPPER;
    if (n > 0 && (!Ap || (nnz > 0 && !Ai) || !order || !pos || !rec_pc || !rec_src || !row_of || !diag_src ||
                  (csc && !cursor)))
        return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    int rc = reset_status(status_dev, st);
    if (rc) return rc;
    LCD_CUDA_TRY(cudaMemsetAsync(info_dev + 2, 0, sizeof(int32_t), st));
    if (n > 0) {
        const SmallOp q{op, flags & (LCD_SOLVE_OF_FULL | LCD_SOLVE_UNIT_DIAG), n, nnz, Ap, Ai, diag_pos};
        // every slot starts as padding (-1 everywhere); the tasks then fill theirs
        LCD_CUDA_TRY(cudaMemsetAsync(rec_pc, 0xFF, (size_t)n_slots * entries * sizeof(int32_t), st));
        LCD_CUDA_TRY(cudaMemsetAsync(rec_src, 0xFF, (size_t)n_slots * entries * sizeof(int32_t), st));
        LCD_CUDA_TRY(cudaMemsetAsync(row_of, 0xFF, (size_t)n_slots * sizeof(int32_t), st));
        LCD_CUDA_TRY(cudaMemsetAsync(diag_src, 0xFF, (size_t)n_slots * sizeof(int32_t), st));
        if (csc) LCD_CUDA_TRY(cudaMemsetAsync(cursor, 0, (size_t)n_slots * sizeof(int32_t), st));
        small_fill_kernel<<<(n + 255) / 256, 256, 0, st>>>(q, order, pos, entries, rec_pc, rec_src, row_of,
                                                           diag_src, cursor, info_dev, status_dev);
        if (csc)
            small_sort_slots_kernel<<<(n_slots + 255) / 256, 256, 0, st>>>(
                n_slots, entries, op == LCD_OP_CSC_UPPER ? 1 : 0, row_of, rec_pc, rec_src);
        LCD_CUDA_TRY(cudaGetLastError());
    }
    LCD_CUDA_TRY(cudaMemcpyAsync(far_host, info_dev + 2, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    int host = 0;
    return finish(status_dev, st, &host);
}

extern "C" int lcd_small_scratch_bytes(int32_t n_slots, int32_t entries, int64_t *bytes) {
    if (n_slots < 0 || (entries != 2 && entries != 4 && entries != 8) || !bytes) return LCD_ERR_INVALID_ARGUMENT;
    const size_t m = (size_t)(n_slots > 0 ? n_slots : 1);
    *bytes = (int64_t)(align256(m * (entries + 2) * 8) + align256(m * 8) + 256);
    return LCD_OK;
}

extern "C" int lcd_sptrsv_small(int32_t n, int32_t n_slots, int32_t entries, const double *Ax,
                                const double *b, double *x, const int32_t *rec_pc, const int32_t *rec_src,
                                const int32_t *row_of, const int32_t *diag_src,
                                const int32_t *slot_ptr_dev, int32_t n_levels, int32_t max_width,
                                void *scratch, int64_t scratch_bytes, void *stream) {
    if (n < 0 || n_slots < n || n_levels < 0 || (entries != 2 && entries != 4 && entries != 8))
        return LCD_ERR_INVALID_ARGUMENT;
    if (n == 0) return LCD_OK;
    if (!Ax || !b || !x || x == b || !rec_pc || !rec_src || !row_of || !diag_src || !slot_ptr_dev || !scratch)
        return LCD_ERR_INVALID_ARGUMENT;
    int64_t need = 0;
    lcd_small_scratch_bytes(n_slots, entries, &need);
    if (scratch_bytes < need) return LCD_ERR_WORKSPACE;
    if (((uintptr_t)scratch & 255) != 0 || ((uintptr_t)rec_pc & 15) != 0) return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    char *base = static_cast<char *>(scratch);
    double *rec_val = reinterpret_cast<double *>(base);
    base += align256((size_t)n_slots * (entries + 2) * 8);
    double *xp = reinterpret_cast<double *>(base);
    const SmallLayout lay{n_slots, entries, rec_pc, rec_src, row_of, diag_src};
    const int blocks = (n_slots + 255) / 256 < 148 * 8 ? (n_slots + 255) / 256 : 148 * 8;
    small_pack_kernel<<<blocks, 256, 0, st>>>(lay, Ax, b, rec_val);
    LCD_CUDA_TRY(cudaGetLastError());
    // (the widest level in slots: rounded up to whole warps)
    const SmallSolveParams p{lay, slot_ptr_dev, n_levels, (max_width + 31) & ~31, rec_val, xp, debug_trace()};
    int rc;
    if (entries == 2) rc = launch_small_e<2>(p, st);
    else if (entries == 4) rc = launch_small_e<4>(p, st);
    else rc = launch_small_e<8>(p, st);
    if (rc) return rc;
    small_unpack_kernel<<<blocks, 256, 0, st>>>(n_slots, row_of, xp, x);
    LCD_CUDA_TRY(cudaGetLastError());
    return LCD_OK;
}
