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
//     reciprocal diagonal} (doubles, gathered by a fully parallel pass whenever the matrix
//     values change) and {positions of its operands} (ints, per pattern), fetched with 128-bit
//     loads two turns (several levels) before the task's level comes up; the right-hand side
//     follows one turn ahead, straight from b.  x is stored by position (coalesced, what the
//     operands read) and into matrix order (a scattered store nobody waits for).
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
    const int *__restrict__ wptr;        // slot table: first slot of (block, level), blocks x (n_levels + 1)
    int n_levels;
    int max_width;                       // widest slice of a level in slots
    int blocks;                          // thread blocks that share the walk (1: the one-block solver)
    int32_t *status;                     // bounded waits for operands of other blocks
    unsigned long long budget_ns;
    const double *__restrict__ rec_val;  // [n * (E + 2)]: coefficients, (unused), reciprocal diagonal
    const double *__restrict__ b;        // right-hand side, matrix order
    double *x;                           // result, matrix order
    double *xp;                          // [n] x by position (what the walk's operands read)
    long long *trace;                    // profiling aid (lcd_debug_set_trace): SM cycle counter after
                                         // every level's barrier [n_levels], then, for the tasks of
                                         // thread 0, at the start / after the stores / at the end [3 each]
    // Shared walk with R = 1 << rshift right-hand sides (row-major n x R blocks with leading
    // dimension ld): the walk runs on R interleaved copies of the pattern.  Copy r of slot s is
    // the task s * R + r; it reads the record of slot s, operand slots pc * R + r, and element r
    // of its row of b and x.  Everything below (ring, x by position, level table) counts tasks.
    int rshift;
    int ld;
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
// Shared walk: block b owns the nodes [n * b / blocks, n * (b + 1) / blocks).  The operands of a
// triangular solve have smaller node numbers, so they belong to the same or an earlier block: the
// dependences between blocks all point one way, and the blocks form a pipeline instead of
// meeting at every level.  Within a level the tasks are sorted by node, so a block's tasks of a
// level are consecutive: cuts[b * n_levels + l] = tasks of level l that belong to blocks < b.
__device__ __forceinline__ int block_of_node(int v, int n, int blocks) {
    return (int)((((long long)v + 1) * blocks - 1) / n);
}

__global__ void small_cuts_kernel(int n, int blocks, int n_levels, const int *__restrict__ order,
                                  const int *__restrict__ wptr, int *cuts) {
    const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (id >= (long long)blocks * n_levels) return;
    const int b = (int)(id / n_levels), l = (int)(id % n_levels);
    const int first = (int)((long long)n * b / blocks);      // the block's first node
    int lo = wptr[l], hi = wptr[l + 1];
    const int start = lo;
    while (lo < hi) {                                         // first task of the level with node >= first
        const int mid = (lo + hi) >> 1;
        if (order[mid] < first) lo = mid + 1; else hi = mid;
    }
    cuts[id] = lo - start;
}

__global__ void small_measure_kernel(const SmallOp q, const int *__restrict__ order,
                                     const int *__restrict__ level, const int *__restrict__ wptr,
                                     const int *__restrict__ slot_ptr, const int *__restrict__ cuts,
                                     int n_levels, int blocks, int *pos, int *info, int32_t *status) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < n_levels && blocks == 1) atomicMax(info + 1, wptr[t + 1] - wptr[t]);   // widest level
    if (t >= q.n) return;
    const int v = order[t];
    if ((unsigned)v >= (unsigned)q.n) { raise_error(status, LCD_ERR_INDEX_RANGE, t); return; }
    const int l = level[v];
    if ((unsigned)l >= (unsigned)n_levels || t < wptr[l] || t >= wptr[l + 1]) {
        raise_error(status, LCD_ERR_INDEX_RANGE, t);     // order and levels do not belong together
        return;
    }
    {   // the first slot of every (block, level) is a multiple of 32
        const int o = t - wptr[l];
        const int b = blocks > 1 ? block_of_node(v, q.n, blocks) : 0;
        const int before = blocks > 1 ? cuts[(size_t)b * n_levels + l] : 0;
        if (o < before) { raise_error(status, LCD_ERR_UNSORTED, t); return; }   // level not sorted by node
        pos[v] = slot_ptr[(size_t)b * (n_levels + 1) + l] + (o - before);
        if (blocks > 1) atomicMax(info + 1, o - before + 1);                     // widest slice
    }
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

// Block that owns slot g: block b's slots are [table[b * stride], table[(b + 1) * stride]) with
// stride = n_levels + 1 (the last block ends at n_slots).
__device__ __forceinline__ int block_of_slot(const int *__restrict__ table, int blocks, int stride, int g) {
    int lo = 0, hi = blocks;          // last block whose first slot is <= g
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (table[(size_t)mid * stride] <= g) lo = mid; else hi = mid;
    }
    return lo;
}

__global__ void small_fill_kernel(const SmallOp q, const int *__restrict__ order,
                                  const int *__restrict__ pos, const int *__restrict__ level,
                                  const int *__restrict__ slot_ptr, int n_levels, int blocks, int E,
                                  int *rec_pc, int *rec_src, int *row_of, int *diag_src, int *cursor,
                                  int *info, int32_t *status) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= q.n) return;
    const int stride = n_levels + 1;
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
                    const int node = upper ? q.n - 1 - c : c;
                    const int other = pos[node];
                    // ... and stands in an earlier level
                    if (other < 0 || level[node] >= level[v]) raise_error(status, LCD_ERR_CYCLE, i);
                    else {
                        pc = other;
                        src = lo + e;
                        // an operand of the own block beyond the shared-memory window is read
                        // from global memory (counted: the caller reports it)
                        if (slot - other > kRing / 2 &&
                            block_of_slot(slot_ptr, blocks, stride, other) ==
                                block_of_slot(slot_ptr, blocks, stride, slot))
                            atomicAdd(info + 2, 1);
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
        const int node = upper ? q.n - 1 - r : r;
        const int target = pos[node];
        if (target < 0 || level[node] <= level[v]) { raise_error(status, LCD_ERR_CYCLE, i); continue; }
        const int k = atomicAdd(cursor + target, 1);
        if (k >= E) continue;                        // cannot happen: E covers the longest row
        rec_pc[(size_t)target * E + k] = slot;
        rec_src[(size_t)target * E + k] = j;
        if (target - slot > kRing / 2 &&
            block_of_slot(slot_ptr, blocks, stride, target) == block_of_slot(slot_ptr, blocks, stride, slot))
            atomicAdd(info + 2, 1);
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

// ---- per value set --------------------------------------------------------------------
// Coefficients and reciprocal diagonals into slot order (fully parallel; repeated only when the
// matrix values change - the right-hand side is read in place by the walk).
// (one block: the right-hand side travels in the record too, b != NULL, and the pass runs per solve)
__global__ void small_pack_kernel(const SmallLayout lay, const double *__restrict__ Ax,
                                  const double *__restrict__ b, double *rec_val) {
    const int E = lay.entries, stride = gridDim.x * blockDim.x;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < lay.n; t += stride) {
        // (records are 16-byte aligned and E is even: pairs of indices in, pairs of doubles out)
        const int2 *src = reinterpret_cast<const int2 *>(lay.rec_src + (size_t)t * E);
        double2 *rec = reinterpret_cast<double2 *>(rec_val + (size_t)t * (E + 2));
        for (int e = 0; e < E / 2; ++e) {
            const int2 s = __ldg(src + e);
            rec[e] = make_double2(s.x >= 0 ? Ax[s.x] : 0.0, s.y >= 0 ? Ax[s.y] : 0.0);
        }
        const int row = lay.row_of[t];
        const int d = lay.diag_src[t];
        rec[E / 2] = make_double2((b && row >= 0) ? b[row] : 0.0,
                                  row < 0 ? 0.0 : (d >= 0 ? 1.0 / Ax[d] : 1.0));   // (padding slots solve to 0)
    }
}

// One block: the walk stores x by position only; this pass puts it into matrix order.
__global__ void small_unpack_kernel(int n, const int *__restrict__ row_of, const double *__restrict__ xp,
                                    double *__restrict__ x) {
    const int stride = gridDim.x * blockDim.x;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < n; t += stride)
        if (row_of[t] >= 0) x[row_of[t]] = xp[t];
}

// ---- per solve ------------------------------------------------------------------------
template <int E, bool SHARED>
struct SmallTask {
    double val[E];
    double bb, dinv;
    int pc[E];                   // slots of the operands (-1: none)
    int row;                     // shared walk: the task's element of b and x (-1: padding slot)
    double rx[SHARED ? E : 1];   // shared walk: operands of other blocks, fetched a turn ahead
                                 // (the pending pattern: not yet there)
};

// Shared walk: the operands of task `t` (slot relative to `base`) that other blocks own are
// requested one turn before the task runs - a load from L2 costs about as much as two levels of
// the walk, and a block that trails its neighbours by a few levels finds them there already.
template <int E>
__device__ __forceinline__ void small_peek(SmallTask<E, true> &q, const SmallSolveParams &p, int base,
                                           int count, int t) {
#pragma unroll
    for (int e = 0; e < E; ++e) {
        q.rx[e] = __longlong_as_double((long long)kPendingBits);
        if (t < count) {
            const int pc = q.pc[e];
            if (pc >= 0 && (unsigned)(pc - base) >= (unsigned)t) q.rx[e] = ld_relaxed_f64(p.xp + pc);
        }
    }
}

// Second stage of a task's prefetch, one turn before it runs: its record (coefficients, operand
// slots, row) was requested a turn earlier; now the right-hand side, straight from b in matrix
// order - no gathering pass per solve.
template <int E, bool SHARED>
__device__ __forceinline__ void small_values(SmallTask<E, SHARED> &q, const SmallSolveParams &p, int count,
                                             int t) {
    q.bb = (t < count && q.row >= 0) ? __ldg(p.b + q.row) : 0.0;
}

// t: slot relative to the block's first slot `base`; count: slots of the block
template <int E, bool SHARED>
__device__ __forceinline__ void small_load(SmallTask<E, SHARED> &q, const SmallSolveParams &p, int base,
                                           int count, int t) {
    if (t < count) {
        t += base;
        const int copy = SHARED ? t & ((1 << p.rshift) - 1) : 0;   // which right-hand side
        const int copies = SHARED ? 1 << p.rshift : 1;
        if (SHARED) t >>= p.rshift;                                // the slot whose record this is
        // two records per task, 16-byte aligned (E + 2 and E are even): 128-bit loads
        const double2 *rv = reinterpret_cast<const double2 *>(p.rec_val + (size_t)t * (E + 2));
#pragma unroll
        for (int k = 0; k < E / 2; ++k) {
            const double2 v = __ldg(rv + k);
            q.val[2 * k] = v.x;
            q.val[2 * k + 1] = v.y;
        }
        const double2 tail = __ldg(rv + E / 2);
        q.dinv = tail.y;
        if (SHARED) {
            const int row = __ldg(p.lay.row_of + t);
            q.row = row >= 0 ? row * p.ld + copy : -1;   // (element of b and x, not the row)
        } else {
            q.bb = tail.x;                // one block: the right-hand side came with the record
        }
        if (E == 2) {
            const int2 c = __ldg(reinterpret_cast<const int2 *>(p.lay.rec_pc + (size_t)t * E));
            q.pc[0] = c.x * copies + copy;   // (-1, no operand, stays negative)
            q.pc[1] = c.y * copies + copy;
        } else {
            const int4 *rc = reinterpret_cast<const int4 *>(p.lay.rec_pc + (size_t)t * E);
#pragma unroll
            for (int k = 0; k < E / 4; ++k) {
                const int4 c = __ldg(rc + k);
                q.pc[4 * k] = c.x * copies + copy;
                q.pc[4 * k + 1] = c.y * copies + copy;
                q.pc[4 * k + 2] = c.z * copies + copy;
                q.pc[4 * k + 3] = c.w * copies + copy;
            }
        }
    } else {
        q.row = -1;
    }
}

// With blocks > 1 (cooperative launch: all blocks are resident) block b walks its slice of every
// level.  Operands of the own block are handed over through the shared-memory ring behind the
// block barrier, as in the one-block form; operands that another block owns are polled in the
// position-ordered x in global memory, which starts out filled with the reserved NaN pattern.
// Rows of a level do not depend on each other, so a thread may spin on such an operand without
// holding up anything but its own block's barrier.  Because operands lie in earlier levels, and
// for a triangular matrix mostly in slices with smaller numbers, the blocks fall into a pipeline:
// block b trails block b - 1 by one hand-off through L2, once - not once per level.
template <int E, int T, int DEPTH, bool SHARED>
__global__ void __launch_bounds__(T, 1) sptrsv_small_kernel(const SmallSolveParams p) {
    extern __shared__ __align__(16) double ring[];  // kRing doubles
    __shared__ int s_wptr[kWptrChunk + 1];
    const int tid = threadIdx.x;
    const bool use_ring = p.max_width <= kRing / 2;   // (max_width counts tasks)
    constexpr bool shared_walk = SHARED;
    const int *table = p.wptr + (size_t)blockIdx.x * (p.n_levels + 1);
    // the block's first slot and how many it has (one block: all of them, known without a look)
    const int rshift = SHARED ? p.rshift : 0;
    const int base = SHARED ? __ldg(table) << rshift : 0;
    const int count = SHARED ? (__ldg(table + p.n_levels) << rshift) - base : p.lay.n;
    double *xp = p.xp + base;
    // two register sets used in turn: a set is reloaded right after its task and not touched
    // again until two turns later, so its loads have several levels to arrive
    SmallTask<E, SHARED> q0, q1;
    int t = tid;
    int phase = 0;
    small_load(q0, p, base, count, t);
    if (DEPTH > 1) small_load(q1, p, base, count, t + T);
    if (SHARED) {
        small_values(q0, p, count, t);
        if (DEPTH > 1) small_values(q1, p, count, t + T);
    }
    if (SHARED) {
#pragma unroll
        for (int e = 0; e < E; ++e) {
            q0.rx[e] = __longlong_as_double((long long)kPendingBits);
            q1.rx[e] = q0.rx[e];
        }
    }
    int traced = 0;
    auto run = [&](SmallTask<E, SHARED> &c, SmallTask<E, SHARED> &next) {
        if (p.trace && tid == 0 && blockIdx.x == 0) p.trace[p.n_levels + 3 * traced] = clock64();
        double acc = c.bb;
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const int pc = c.pc[e];
            if (pc >= 0) {
                const int rel = pc - base;
                double xv;
                if (!SHARED || (unsigned)rel < (unsigned)t) {   // a slot of this block (earlier level)
                    xv = (use_ring && t - rel <= kRing / 2) ? ring[rel & (kRing - 1)]
                                                            : *(volatile const double *)(xp + rel);
                } else if (!SHARED) {
                    xv = __longlong_as_double(kCanonicalNaN);   // (cannot happen: one block owns all)
                } else {                                  // another block's: fetched a turn ago,
                    xv = c.rx[e];                         // else wait for it (bounded)
                    if (is_pending(xv)) {
                        Deadline dl;
                        dl.start(p.budget_ns);
                        for (;;) {
                            xv = ld_relaxed_f64(p.xp + pc);
                            if (!is_pending(xv)) break;
                            if (dl.tick(p.status, pc)) { xv = __longlong_as_double(kCanonicalNaN); break; }
                        }
                    }
                }
                acc = fma(-c.val[e], xv, acc);
            }
        }
        const double xi = acc * c.dinv;
        ring[t & (kRing - 1)] = xi;
        // consecutive tasks, consecutive addresses.  One block: a plain store (the block barrier
        // orders it for the block's own readers); shared walk: other blocks poll it
        if (shared_walk) st_relaxed_f64(xp + t, publishable(xi));
        else xp[t] = xi;
        if (SHARED && c.row >= 0) p.x[c.row] = xi;   // the result in matrix order (nobody reads it here)
        if (p.trace && tid == 0 && blockIdx.x == 0) p.trace[p.n_levels + 3 * traced + 1] = clock64();
        small_load(c, p, base, count, t + DEPTH * T);
        t += T;
        if constexpr (SHARED && DEPTH > 1) {
            small_values(next, p, count, t);         // next turn's task: its record is there by now
            small_peek(next, p, base, count, t);
        } else if constexpr (SHARED) {
            small_values(c, p, count, t);            // (one register set: waits for the record just loaded)
        }
        if (p.trace && tid == 0 && blockIdx.x == 0) p.trace[p.n_levels + 3 * traced++ + 2] = clock64();
    };
    for (int first = 0; first < p.n_levels; first += kWptrChunk) {
        const int levels = min(kWptrChunk, p.n_levels - first);
        __syncthreads();  // the previous chunk of offsets is no longer read
        for (int k = tid; k <= levels; k += T) s_wptr[k] = (__ldg(table + first + k) << rshift) - base;
        __syncthreads();
        for (int l = 0; l < levels; ++l) {
            const int we = s_wptr[l + 1];
            while (t < we) {
                if (DEPTH == 1 || phase == 0) run(q0, q1);
                else run(q1, q0);
                phase ^= 1;
            }
            __syncthreads();
            if (p.trace && tid == 0 && blockIdx.x == 0) p.trace[first + l] = clock64();
            if (SHARED && p.trace && tid == 0) {     // shared walk: timer after every level of the first,
                                                     // the middle and the last block [8..11) x n_levels
                const int which = blockIdx.x == 0 ? 0 : (blockIdx.x == gridDim.x / 2 ? 1 : (blockIdx.x == gridDim.x - 1 ? 2 : -1));
                if (which >= 0) p.trace[(8ll + which) * p.n_levels + first + l] = (long long)global_timer();
            }
        }
    }
}

template <int E, int T, int DEPTH>
static int launch_small_t(const SmallSolveParams &p, cudaStream_t st) {
    static bool configured = false;
    const int smem = kRing * (int)sizeof(double);
    if (!configured) {
        LCD_CUDA_TRY(cudaFuncSetAttribute(sptrsv_small_kernel<E, T, DEPTH, false>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        LCD_CUDA_TRY(cudaFuncSetAttribute(sptrsv_small_kernel<E, T, DEPTH, true>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        configured = true;
    }
    if (p.blocks <= 1) {
        sptrsv_small_kernel<E, T, DEPTH, false><<<1, T, smem, st>>>(p);
    } else {
        // blocks wait for each other: they must all be resident (cooperative launch, one per SM)
        static int per_sm = -1;
        if (per_sm < 0)
            LCD_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                &per_sm, sptrsv_small_kernel<E, T, DEPTH, true>, T, smem));
        if ((long long)per_sm * sm_count() < p.blocks) return LCD_ERR_TOO_LARGE;
        SmallSolveParams q = p;
        void *args[] = {(void *)&q};
        LCD_CUDA_TRY(cudaLaunchCooperativeKernel((void *)sptrsv_small_kernel<E, T, DEPTH, true>, dim3((unsigned)p.blocks),
                                                 dim3(T), args, (size_t)smem, st));
    }
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

extern "C" int lcd_small_level_cuts(int32_t n, int32_t blocks, int32_t n_levels, const int32_t *order,
                                    const int32_t *wavefront_ptr_dev, int32_t *cuts_dev, void *stream) {
    if (n < 0 || blocks < 1 || blocks > 1024 || n_levels < 0) return LCD_ERR_INVALID_ARGUMENT;
    if (n == 0 || n_levels == 0) return LCD_OK;
    if (!order || !wavefront_ptr_dev || !cuts_dev) return LCD_ERR_INVALID_ARGUMENT;
    const long long m = (long long)blocks * n_levels;
    small_cuts_kernel<<<(unsigned)((m + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        n, blocks, n_levels, order, wavefront_ptr_dev, cuts_dev);
    LCD_CUDA_TRY(cudaGetLastError());
    return LCD_OK;
}

extern "C" int lcd_small_plan_measure(int op, int flags, int32_t n, int64_t nnz, const int32_t *Ap,
                                      const int32_t *Ai, const int32_t *diag_pos, const int32_t *order,
                                      const int32_t *level, const int32_t *wavefront_ptr_dev,
                                      const int32_t *slot_ptr_dev, const int32_t *cuts_dev,
                                      int32_t n_levels, int32_t blocks, int32_t n_slots, int32_t *pos,
                                      int32_t *cursor, int32_t *info_dev,
                                      int32_t *status_dev, void *stream, int32_t *info_host) {
    if (n < 0 || nnz < 0 || n_levels < 0 || n_slots < n || !info_dev || !status_dev || !info_host ||
        !small_op_ok(op) || blocks < 1 || blocks > 1024 || (blocks > 1 && !cuts_dev))
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
                                                              cuts_dev, n_levels, blocks, pos, info_dev,
                                                              status_dev);
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
                                   const int32_t *level, const int32_t *slot_ptr_dev, int32_t n_levels,
                                   int32_t blocks, const int32_t *pos, int32_t n_slots, int32_t entries,
                                   int32_t *rec_pc,
                                   int32_t *rec_src, int32_t *row_of, int32_t *diag_src,
                                   int32_t *cursor, int32_t *info_dev, int32_t *status_dev,
                                   void *stream, int32_t *far_host) {
    if (n < 0 || nnz < 0 || n_slots < n || (entries != 2 && entries != 4 && entries != 8) || !info_dev ||
        !status_dev || !far_host || !small_op_ok(op) || blocks < 1 || blocks > 1024 || n_levels < 0)
        return LCD_ERR_INVALID_ARGUMENT;
    const bool csc = op == LCD_OP_CSC_LOWER || op == LCD_OP_CSC_UPPER;
    if (n > 0 && (!Ap || (nnz > 0 && !Ai) || !order || !level || !slot_ptr_dev || !pos || !rec_pc || !rec_src || !row_of || !diag_src ||
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
        small_fill_kernel<<<(n + 255) / 256, 256, 0, st>>>(q, order, pos, level, slot_ptr_dev, n_levels, blocks,
                                                           entries, rec_pc, rec_src, row_of, diag_src, cursor,
                                                           info_dev, status_dev);
        if (csc)
            small_sort_slots_kernel<<<(n_slots + 255) / 256, 256, 0, st>>>(
                n_slots, entries, op == LCD_OP_CSC_UPPER ? 1 : 0, row_of, rec_pc, rec_src);
        LCD_CUDA_TRY(cudaGetLastError());
    }
    LCD_CUDA_TRY(cudaMemcpyAsync(far_host, info_dev + 2, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    int host = 0;
    return finish(status_dev, st, &host);
}

extern "C" int lcd_small_scratch_bytes_multi(int32_t n_slots, int32_t entries, int32_t nrhs, int64_t *bytes) {
    if (n_slots < 0 || (entries != 2 && entries != 4 && entries != 8) || !bytes || nrhs < 1 || nrhs > 16 ||
        (nrhs & (nrhs - 1)) != 0)
        return LCD_ERR_INVALID_ARGUMENT;
    const size_t m = (size_t)(n_slots > 0 ? n_slots : 1);
    *bytes = (int64_t)(align256(m * (entries + 2) * 8) + align256(m * nrhs * 8) + 256);
    return LCD_OK;
}

extern "C" int lcd_small_scratch_bytes(int32_t n_slots, int32_t entries, int64_t *bytes) {
    return lcd_small_scratch_bytes_multi(n_slots, entries, 1, bytes);
}

extern "C" int lcd_sptrsv_small_multi(int32_t n, int32_t n_slots, int32_t entries, const double *Ax,
                                      const double *b, double *x, int32_t nrhs, int64_t ld,
                                      const int32_t *rec_pc, const int32_t *rec_src,
                                      const int32_t *row_of, const int32_t *diag_src,
                                      const int32_t *slot_ptr_dev, int32_t n_levels, int32_t blocks,
                                      int32_t max_width, int32_t gather_values, void *scratch,
                                      int64_t scratch_bytes, int32_t *status_dev, int32_t timeout_ms,
                                      void *stream, int *status_host) {
    if (n < 0 || n_slots < n || n_levels < 0 || (entries != 2 && entries != 4 && entries != 8) ||
        blocks < 1 || blocks > 1024 || !status_dev || nrhs < 1 || nrhs > 16 || (nrhs & (nrhs - 1)) != 0 ||
        ld < nrhs || (nrhs > 1 && blocks == 1))
        return LCD_ERR_INVALID_ARGUMENT;
    // tasks and elements of b and x are counted in 32-bit integers
    if ((long long)n_slots * nrhs > 0x7fffffffll || (long long)n * ld > 0x7fffffffll) return LCD_ERR_TOO_LARGE;
    if (n == 0) {
        const int rc0 = reset_status(status_dev, (cudaStream_t)stream);
        return rc0 ? rc0 : finish(status_dev, (cudaStream_t)stream, status_host);
    }
    if (!Ax || !b || !x || x == b || !rec_pc || !rec_src || !row_of || !diag_src || !slot_ptr_dev || !scratch)
        return LCD_ERR_INVALID_ARGUMENT;
    int64_t need = 0;
    lcd_small_scratch_bytes_multi(n_slots, entries, nrhs, &need);
    if (scratch_bytes < need) return LCD_ERR_WORKSPACE;
    if (((uintptr_t)scratch & 255) != 0 || ((uintptr_t)rec_pc & 15) != 0) return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    char *base = static_cast<char *>(scratch);
    double *rec_val = reinterpret_cast<double *>(base);
    base += align256((size_t)n_slots * (entries + 2) * 8);
    double *xp = reinterpret_cast<double *>(base);
    const SmallLayout lay{n_slots, entries, rec_pc, rec_src, row_of, diag_src};
    int rc = reset_status(status_dev, st);
    if (rc) return rc;
    const int grid = (n_slots + 255) / 256 < sm_count() * 8 ? (n_slots + 255) / 256 : sm_count() * 8;
    if (blocks == 1 || gather_values) {
        // one block: coefficients and right-hand side per solve (small systems: a few microseconds);
        // shared walk: coefficients only, and only when asked - it reads b in place
        small_pack_kernel<<<grid, 256, 0, st>>>(lay, Ax, blocks == 1 ? b : nullptr, rec_val);
        LCD_CUDA_TRY(cudaGetLastError());
    }
    if (blocks > 1) {   // blocks poll each other's results: the value is its own ready flag
        rc = lcd_fill_u64(reinterpret_cast<uint64_t *>(xp), (int64_t)n_slots * nrhs, kPendingBits, st);
        if (rc) return rc;
    }
    int rshift = 0;
    while ((1 << rshift) < nrhs) ++rshift;
    // (the widest slice in tasks: slots rounded up to whole warps, times the right-hand sides)
    const SmallSolveParams p{lay, slot_ptr_dev, n_levels, ((max_width + 31) & ~31) << rshift, blocks, status_dev,
                             timeout_ns(timeout_ms), rec_val, b, x, xp, debug_trace(), rshift, (int)ld};
    if (entries == 2) rc = launch_small_e<2>(p, st);
    else if (entries == 4) rc = launch_small_e<4>(p, st);
    else rc = launch_small_e<8>(p, st);
    if (rc) return rc;
    if (blocks == 1) {
        small_unpack_kernel<<<grid, 256, 0, st>>>(n_slots, row_of, xp, x);
        LCD_CUDA_TRY(cudaGetLastError());
    }
    return finish(status_dev, st, status_host);
}

extern "C" int lcd_sptrsv_small(int32_t n, int32_t n_slots, int32_t entries, const double *Ax,
                                const double *b, double *x, const int32_t *rec_pc, const int32_t *rec_src,
                                const int32_t *row_of, const int32_t *diag_src,
                                const int32_t *slot_ptr_dev, int32_t n_levels, int32_t blocks,
                                int32_t max_width, int32_t gather_values, void *scratch,
                                int64_t scratch_bytes, int32_t *status_dev, int32_t timeout_ms,
                                void *stream, int *status_host) {
    return lcd_sptrsv_small_multi(n, n_slots, entries, Ax, b, x, 1, 1, rec_pc, rec_src, row_of, diag_src,
                                  slot_ptr_dev, n_levels, blocks, max_width, gather_values, scratch,
                                  scratch_bytes, status_dev, timeout_ms, stream, status_host);
}
