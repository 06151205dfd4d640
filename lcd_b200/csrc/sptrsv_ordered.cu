// Sync-free CSR triangular solves that take their rows in a caller-given topological
// order (sm_100a), for one or many right-hand sides.
//
// Why an order.  The index-ordered sync-free kernels hand rows out by ascending index,
// which is a valid topological order of a triangular matrix but a poor one for grid-like
// matrices: the rows resident at one time then form a thin slab whose parallelism is one
// grid line.  The level sets of lcd_dag_build list the rows level by level; handing rows
// out in that order keeps whole levels of independent rows in flight, and - unlike the
// level-synchronous kernels - nothing ever waits for a whole level: a row waits for
// exactly its own operands (point-to-point), so there is no grid barrier and no launch
// per level.
//
// Scheduling.  Persistent warps draw tasks from ticket counters, 32 / W consecutive tasks
// per draw: groups of W lanes (W * KR >= nrhs, lane l of a group owns the right-hand sides
// l, l + W, ...) take one row each, so no row ever queues behind another row of its own
// warp.  A task only waits for tasks with smaller numbers, all of which belong to warps
// that are running or finished: every wait terminates.
//
// No pointer chasing on the dependence chain.  A first pass turns (order, Ap, diag_pos)
// into one 16-byte record per task {row, first entry, entry count, diagonal position}
// (structure only: reusable while the pattern and the order stay).  The solve kernel is a
// software pipeline per warp, staged in shared memory by asynchronous copies (cp.async,
// one commit group per batch): while batch k is solved, the records of batch k + 2 and
// the entries, diagonal and right-hand side of batch k + 1 are in flight, each stage's
// addresses coming from copies that landed a batch earlier.  Staging in shared memory
// instead of registers keeps the kernel at 64 registers (KR <= 2), i.e. 32 warps per SM:
// the solve is bound by memory latency, so resident warps are what fills HBM.  A warp holds
// no more than these three batches: a task queued behind others in one warp waits for them,
// which costs hand-offs when levels are narrow.  What remains on the chain of a row is:
// poll its operands, multiply-add, publish.
//
// Waiting.  All groups of a warp make one non-blocking attempt per trip and the trip ends
// in a warp-wide vote, so no lane spins inside a branch (rows of one warp may depend on
// each other).  Every lane runs every trip, and a group's vote is a full-warp ballot read
// through the group's mask: a vote instruction with one mask per group is executed once per
// group and leaves the groups split behind it (measured: 500 warp instructions per trip
// instead of 50, 3.4 us per hand-off instead of 1.9).  A warp none of whose groups progressed
// sleeps before the next trip, with an exponentially growing pause: rows far behind the
// frontier then stop competing for L2 with the polls that matter.  Every wait is bounded
// (status block, LCD_ERR_TIMEOUT).
//
// Rows per warp.  A warp moves on when its slowest row is done, so few rows per warp are
// better than many: with one right-hand side two lanes per row (16 rows per warp, the second
// lane idle) take half the time of one lane per row.  With many right-hand sides a lane takes
// four of them (KR = 4, three entries of a row per trip, 74 registers, three blocks per SM).
//
// Hand-off.  Two forms: (a) X pre-filled with the reserved NaN pattern, consumers poll
// the operand elements themselves (one L2 round trip per hop; costs one extra write pass
// over X); (b) a per-row flag array: producers store their elements, then one lane
// releases the row's flag; consumers poll the flag, fence, and read (two round trips per
// hop, no pass over X).
#include "common.cuh"

namespace lcd {

constexpr int kOrdThreads = 256;
constexpr int kOrdWarps = kOrdThreads / 32;
constexpr int kStage = 4;          // entries of a row tried per trip
constexpr int kCounterStride = 64;  // ints between two ticket counters
static int g_ordered_pause_ns = 256;  // longest pause between two polls of a waiting warp
static int g_ordered_min_lanes = 2;   // lanes per row at least (1 measured 2x slower than 2)

struct __align__(16) TaskMeta {
    int row;  // matrix row, -1: nothing to do (an error was raised)
    int lo;   // first off-diagonal entry
    int cnt;  // number of off-diagonal entries
    int d;    // position of the diagonal, -1: implicit unit diagonal
};

struct OrderedParams {
    CsrSolveParams m;
    const TaskMeta *__restrict__ meta;
    int *row_flags;  // form (b): n ints, zero on entry; NULL: form (a)
    int n_tasks;
    unsigned max_pause_ns;
    int *counters;   // kOrdWarps ticket counters, kCounterStride ints apart, zero on entry
    long long *trace;  // profiling aid (lcd_debug_set_trace), 3n words: nanosecond timer when a row's
                       // batch came up / when the row was published, and its number of waiting trips
};

int set_ordered_pause(int ns) {
    if (ns < 0 || ns > 100000) return LCD_ERR_INVALID_ARGUMENT;
    g_ordered_pause_ns = ns;
    return LCD_OK;
}
int set_ordered_min_lanes(int lanes) {
    if (lanes < 100 && lanes != 1 && lanes != 2 && lanes != 4 && lanes != 8) return LCD_ERR_INVALID_ARGUMENT;
    g_ordered_min_lanes = lanes;
    return LCD_OK;
}

__global__ void __launch_bounds__(256)
ordered_meta_kernel(const CsrSolveParams p, const int *__restrict__ order, int n_tasks, TaskMeta *meta) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n_tasks) return;
    TaskMeta mt{-1, 0, 0, -1};
    const int node = __ldg(order + t);
    if ((unsigned)node >= (unsigned)p.n) {
        raise_error(p.status, LCD_ERR_INDEX_RANGE, t);
    } else {
        const int r = (p.flags & LCD_SOLVE_UPPER) ? p.n - 1 - node : node;
        int lo = 0, hi = 0, d = -1;
        if (!csr_row_range(p, r, lo, hi, d))
            raise_error(p.status, (p.flags & LCD_SOLVE_OF_FULL) ? LCD_ERR_MISSING_DIAGONAL
                                                               : LCD_ERR_BAD_POINTERS, r);
        else
            mt = TaskMeta{r, lo, hi - lo, d};
    }
    meta[t] = mt;
}

// ---- asynchronous copies into shared memory (cp.async, completion by commit groups) ----
__device__ __forceinline__ unsigned smem_address(const void *p) {
    return (unsigned)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void cp_async_4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_address(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_8(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_address(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_address(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

constexpr int kMetaRing = 4;  // batches whose records are kept in shared memory
constexpr int kDataRing = 2;  // batches whose entries / right-hand sides are kept there
constexpr int kTicketDraws = 1;  // places of its stream a warp takes per draw (more = deeper queue per warp)

struct __align__(16) RowData {   // 64 bytes
    int col[kStage];
    double val[kStage];
    double diag;
    double pad;
};

template <int W, int KR>
struct WarpStage {
    static constexpr int G = 32 / W;
    int4 meta[kMetaRing][G];
    RowData row[kDataRing][G];
    double rhs[kDataRing][KR][32];
};

// SYS: block-row partition across GPUs - operands may arrive from a peer (system-scope polls)
// and a published value is also stored into the x arrays of the ranks that need it.
template <int W, int KR, bool FLAGS, bool SYS = false>
__global__ void __launch_bounds__(kOrdThreads, KR >= 4 ? 3 : 4) csr_ordered_kernel(const OrderedParams q) {
    constexpr int S = KR <= 2 ? kStage : (KR <= 4 ? 3 : 1);   // entries tried per trip (registers)
    extern __shared__ __align__(16) unsigned char ordered_smem[];
    const CsrSolveParams &p = q.m;
    constexpr int G = 32 / W;
    constexpr unsigned kFull = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const int g = lane / W, gl = lane % W;
    const unsigned gmask = W == 32 ? kFull : (((1u << W) - 1u) << (g * W));
    const bool upper = p.flags & LCD_SOLVE_UPPER;
    WarpStage<W, KR> &stage = reinterpret_cast<WarpStage<W, KR> *>(ordered_smem)[threadIdx.x >> 5];

    // Tickets.  One counter for the whole grid would be the bottleneck (atomics on one
    // address serialise), and a ticket that covers consecutive batches would queue rows of one
    // level behind each other in one warp.  So the batches (G tasks each) are dealt round-robin
    // to kOrdWarps streams with a counter each (256 bytes apart), warp w of every block serves
    // stream w, and a draw takes kTicketDraws places of the stream: batches 8 (q + j) + w.
    // Every running block serves every stream, so the earliest unfinished batch always belongs
    // to a warp that is running or will draw it next.
    int *counter = q.counters + (threadIdx.x >> 5) * kCounterStride;
    const int stream = threadIdx.x >> 5;
    int tk_base = 0, tk_pos = kTicketDraws, tk_pending = 0;
    if (lane == 0) tk_pending = atomicAdd(counter, kTicketDraws);
    auto draw = [&]() {
        if (tk_pos == kTicketDraws) {
            // (the following draw is issued now and read kTicketDraws batches later)
            tk_base = __shfl_sync(kFull, tk_pending, 0);
            if (lane == 0) tk_pending = atomicAdd(counter, kTicketDraws);
            tk_pos = 0;
        }
        const long long first = ((long long)(tk_base + tk_pos++) * kOrdWarps + stream) * G;
        return first < q.n_tasks ? (int)first : q.n_tasks;
    };
    // stage 1: the records of batch `seq` (first task t0) on their way to shared memory
    auto fetch_meta = [&](int seq, int t0) {
        if (gl == 0) {
            int4 *dst = &stage.meta[seq & (kMetaRing - 1)][g];
            if (t0 + g < q.n_tasks) cp_async_16(dst, q.meta + t0 + g);
            else *dst = make_int4(-1, 0, 0, -1);
        }
    };
    // stage 2: entries, diagonal and right-hand side of batch `seq`, whose records have arrived
    auto fetch_data = [&](int seq) {
        const int4 mt = stage.meta[seq & (kMetaRing - 1)][g];
        RowData &rd = stage.row[seq & (kDataRing - 1)][g];
        if (mt.x >= 0) {
            for (int k = gl; k < kStage; k += W) {
                if (k < mt.z) {
                    cp_async_4(&rd.col[k], p.Ai + mt.y + k);
                    cp_async_8(&rd.val[k], p.Ax + mt.y + k);
                }
            }
            if (gl == 0) {
                if (mt.w >= 0) cp_async_8(&rd.diag, p.Ax + mt.w);
                else rd.diag = 1.0;
            }
#pragma unroll
            for (int c = 0; c < KR; ++c) {
                const int col = gl + W * c;
                if (col < p.nrhs)
                    cp_async_8(&stage.rhs[seq & (kDataRing - 1)][c][lane], p.b + (long long)mt.x * p.ld + col);
            }
        }
    };

    // prologue: records of the first two batches, then the data of the first
    int tb[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) tb[k] = draw();
    fetch_meta(0, tb[0]);
    fetch_meta(1, tb[1]);
    cp_async_commit();
    cp_async_wait<0>();
    __syncwarp();
    fetch_data(0);
    cp_async_commit();

    for (int seq = 0; tb[0] < q.n_tasks; ++seq) {
        // group seq - 1 = {records of batch seq + 1, data of batch seq} has landed
        cp_async_wait<0>();
        __syncwarp();
        // ---- issue group seq: records of batch seq + 2, data of batch seq + 1 ----
        fetch_meta(seq + 2, tb[2]);
        fetch_data(seq + 1);
        cp_async_commit();

        // ---- solve the group's row of batch seq ----
        // Every lane runs every trip and every vote is a full-warp ballot read through the
        // group's mask: a vote with one mask per group would be executed once per group, and the
        // lanes would stay split behind it (measured with one lane per row: 32 serial copies of
        // the trip, 500 warp instructions per trip instead of 50).
        const int4 mt = stage.meta[seq & (kMetaRing - 1)][g];
        const RowData &rd = stage.row[seq & (kDataRing - 1)][g];
        const int r = mt.x, lo = mt.y, cnt = mt.z;
        int cidx[S];
        double cval[S], acc[KR];
        double rinv = 1.0;
        bool active = r >= 0, failed = false;
        int e = 0, m = 0;
        // entries [e, e + m) are staged in cidx / cval; an entry that is not an earlier row fails the row
        auto check_chunk = [&]() {
#pragma unroll
            for (int i = 0; i < S; ++i) {
                if (i < m) {
                    const int c = cidx[i];
                    if (!((unsigned)c < (unsigned)p.n && (upper ? c > r : c < r))) failed = true;
                }
            }
            if (failed) {
                if (gl == 0) raise_error(p.status, LCD_ERR_INDEX_RANGE, r);
                m = 0;
                e = cnt;
            }
        };
        if (active) {
#pragma unroll
            for (int i = 0; i < S; ++i) { cidx[i] = rd.col[i]; cval[i] = rd.val[i]; }   // (S <= kStage)
#pragma unroll
            for (int c = 0; c < KR; ++c) acc[c] = stage.rhs[seq & (kDataRing - 1)][c][lane];
            rinv = 1.0 / rd.diag;
            m = min(S, cnt);
            check_chunk();
            if (q.trace && gl == 0) q.trace[r] = (long long)global_timer();
        }
        unsigned pause = 0;
        int trips = 0;
        Deadline dl;
        dl.start(p.budget_ns);
        for (;;) {
            // -- poll: one non-blocking attempt at the staged entries --
            double xv[S][KR];
            bool ready = true;
            if (FLAGS) {
#pragma unroll
                for (int i = 0; i < S; ++i)
                    if (active && i < m) ready = ready && ld_relaxed_s32(q.row_flags + cidx[i]) != 0;
            } else {
#pragma unroll
                for (int i = 0; i < S; ++i) {
#pragma unroll
                    for (int c = 0; c < KR; ++c) {
                        const int col = gl + W * c;
                        xv[i][c] = 0.0;
                        if (active && i < m && col < p.nrhs) {
                            const double *src = p.x + (long long)cidx[i] * p.ld + col;
                            xv[i][c] = SYS ? ld_relaxed_sys_f64(src) : ld_relaxed_f64(src);
                            ready = ready && !is_pending(xv[i][c]);
                        }
                    }
                }
            }
            if (W > 1) ready = (__ballot_sync(kFull, ready) & gmask) == gmask;
            if (FLAGS) {
                const bool take = active && ready;
                if (take) acquire_fence();
#pragma unroll
                for (int i = 0; i < S; ++i) {
#pragma unroll
                    for (int c = 0; c < KR; ++c) {
                        const int col = gl + W * c;
                        xv[i][c] = (take && i < m && col < p.nrhs)
                                       ? __ldcg(p.x + (long long)cidx[i] * p.ld + col) : 0.0;
                    }
                }
            }
            // -- consume, then publish in the trip that consumed the last operand --
            const bool progressed = active && (ready || failed);
            bool publish = false;
            if (progressed) {
#pragma unroll
                for (int i = 0; i < S; ++i) {
                    if (i < m) {
#pragma unroll
                        for (int c = 0; c < KR; ++c) acc[c] = fma(-cval[i], xv[i][c], acc[c]);
                    }
                }
                e += m;
                if (e < cnt) {      // rows longer than one staged chunk: fetch the next one
                    m = min(S, cnt - e);
#pragma unroll
                    for (int i = 0; i < S; ++i) {
                        if (i < m) {
                            if (S < kStage && e + i < kStage) {   // still among the staged entries
                                cidx[i] = rd.col[e + i];
                                cval[i] = rd.val[e + i];
                            } else {
                                cidx[i] = __ldg(p.Ai + lo + e + i);
                                cval[i] = __ldg(p.Ax + lo + e + i);
                            }
                        }
                    }
                    check_chunk();
                }
                publish = e >= cnt;
            }
            if (publish) {
                const double nanv = __longlong_as_double(kCanonicalNaN);
#pragma unroll
                for (int c = 0; c < KR; ++c) {
                    const int col = gl + W * c;
                    if (col < p.nrhs) {
                        const double v = failed ? nanv : acc[c] * rinv;
                        if (FLAGS) __stcg(p.x + (long long)r * p.ld + col, v);
                        else st_relaxed_f64(p.x + (long long)r * p.ld + col, publishable(v));
                        if (SYS && p.need_mask) {   // rows of other GPUs wait for it in their own memory
                            unsigned mk = p.need_mask[r];
                            while (mk) {
                                const int peer = __ffs(mk) - 1;
                                mk &= mk - 1;
                                st_relaxed_sys_f64(p.peers[peer] + (long long)r * p.ld + col, publishable(v));
                            }
                        }
                    }
                }
                active = false;
                m = 0;
                if (q.trace && gl == 0) {
                    q.trace[p.n + r] = (long long)global_timer();
                    q.trace[2ll * p.n + r] = trips;
                }
            }
            if (FLAGS) {
                __syncwarp();   // the group's stores are ordered before the release of its flag
                if (publish && gl == 0) st_release_s32(q.row_flags + r, 1);
            }
            ++trips;
            const unsigned still = __ballot_sync(kFull, active);
            if (still == 0) break;
            if (__any_sync(kFull, progressed)) {
                pause = 0;
            } else {
                // nobody moved: bounded wait (a raised error or the deadline fails the waiting rows)
                if (__any_sync(kFull, active && dl.tick(p.status, r))) failed = active;
                pause = pause ? min(pause * 2, q.max_pause_ns) : 32u;
                if (q.max_pause_ns) __nanosleep(pause);
            }
        }
        tb[0] = tb[1];
        tb[1] = tb[2];
        tb[2] = draw();
    }
    cp_async_wait<0>();   // nothing of this warp is in flight when the block leaves
}

template <int W, int KR, bool FLAGS, bool SYS = false>
static int launch_ordered_t(const OrderedParams &q, long long window_rows, cudaStream_t st) {
    static int per_sm = 0;
    const size_t smem = sizeof(WarpStage<W, KR>) * kOrdWarps;
    if (per_sm == 0) {
        if (smem > 48 * 1024)
            LCD_CUDA_TRY(cudaFuncSetAttribute(csr_ordered_kernel<W, KR, FLAGS, SYS>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        int v = 0;
        LCD_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, csr_ordered_kernel<W, KR, FLAGS, SYS>,
                                                                  kOrdThreads, smem));
        if (v < 1) return LCD_ERR_CUDA;
        per_sm = v;
    }
    constexpr int rows_per_block = kOrdWarps * (32 / W);
    long long grid = (long long)per_sm * sm_count();
    const long long useful = ((long long)q.n_tasks + rows_per_block - 1) / rows_per_block;
    if (grid > useful) grid = useful;
    if (window_rows > 0) {
        const long long want = (window_rows + rows_per_block - 1) / rows_per_block;
        if (grid > want) grid = want;
    }
    if (grid < 1) grid = 1;
    csr_ordered_kernel<W, KR, FLAGS, SYS><<<(unsigned)grid, kOrdThreads, smem, st>>>(q);
    LCD_CUDA_TRY(cudaGetLastError());
    return LCD_OK;
}

template <int W, int KR>
static int launch_ordered(const OrderedParams &q, long long window_rows, cudaStream_t st) {
    return q.row_flags ? launch_ordered_t<W, KR, true>(q, window_rows, st)
                       : launch_ordered_t<W, KR, false>(q, window_rows, st);
}

}  // namespace lcd

using namespace lcd;

extern "C" int lcd_sptrsv_csr_ordered(int32_t n, int64_t nnz, int32_t nrhs, const int32_t *Ap,
                                      const int32_t *Ai, const double *Ax, const int32_t *diag_pos,
                                      const double *B, double *X, int64_t ld, int flags,
                                      const int32_t *order, int32_t *task_records, int records_ready,
                                      int32_t *row_flags, int64_t window_rows, int32_t *status_dev,
                                      int32_t timeout_ms, void *stream, int *status_host) {
    if (n < 0 || nnz < 0 || nrhs < 1 || nrhs > 64 || ld < nrhs || !status_dev || window_rows < 0)
        return LCD_ERR_INVALID_ARGUMENT;
    if (flags & LCD_SOLVE_EXACT) return LCD_ERR_INVALID_ARGUMENT;  // operands are taken as they arrive
    if ((flags & LCD_SOLVE_OF_FULL) && !diag_pos) return LCD_ERR_INVALID_ARGUMENT;
    if ((flags & LCD_SOLVE_UNIT_DIAG) && !(flags & LCD_SOLVE_OF_FULL)) return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && (!Ap || !B || !X || X == B || !task_records || (nnz > 0 && (!Ai || !Ax))))
        return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && !records_ready && !order) return LCD_ERR_INVALID_ARGUMENT;
    if (((uintptr_t)task_records & 15) != 0) return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    int rc = reset_status(status_dev, st);
    if (rc) return rc;
    if (n > 0) {
        if (row_flags) LCD_CUDA_TRY(cudaMemsetAsync(row_flags, 0, (size_t)n * sizeof(int32_t), st));
        else LCD_CUDA_TRY(cudaMemsetAsync(X, 0xFF, (size_t)n * (size_t)ld * sizeof(double), st));
        OrderedParams q;
        q.m = CsrSolveParams{n, nnz, Ap, Ai, Ax, diag_pos, B, X, flags, nrhs, ld, status_dev,
                             timeout_ns(timeout_ms), nullptr, 0, n, nullptr, {nullptr}};
        q.meta = reinterpret_cast<const TaskMeta *>(task_records);
        q.row_flags = row_flags;
        q.n_tasks = n;
        q.max_pause_ns = (unsigned)g_ordered_pause_ns;
        q.counters = task_records + 4 * (size_t)n;
        q.trace = debug_trace();
        LCD_CUDA_TRY(cudaMemsetAsync(q.counters, 0, kOrdWarps * kCounterStride * sizeof(int32_t), st));
        if (!records_ready) {
            ordered_meta_kernel<<<(n + 255) / 256, 256, 0, st>>>(
                q.m, order, n, reinterpret_cast<TaskMeta *>(task_records));
            LCD_CUDA_TRY(cudaGetLastError());
        }
        // (lanes per row) x (right-hand sides per lane) >= nrhs.  Measured on a 3-D grid (192^3):
        // with one lane per row (32 rows per warp) a solve takes twice as long as with two, even
        // for one right-hand side (a warp moves on when its slowest row is done); two to eight
        // lanes per row are fastest up to eight right-hand sides; beyond that four right-hand
        // sides per lane (three entries per trip, three blocks per SM) beat two: 1.8 / 2.3 / 3.3 ms
        // for 16 / 32 / 64 right-hand sides against 2.0 / 2.8 / 4.7.
        int W, KR;
        if (g_ordered_min_lanes >= 100) {        // explicit variant (tuning runs): 100 * W + KR
            W = g_ordered_min_lanes / 100;
            KR = g_ordered_min_lanes % 100;
            if (W * KR < nrhs) return LCD_ERR_INVALID_ARGUMENT;
        } else {
            W = nrhs <= 2 ? 2 : (nrhs <= 4 ? 4 : (nrhs <= 32 ? 8 : 16));
            KR = nrhs <= 8 ? 1 : 4;
            if (KR == 1 && g_ordered_min_lanes > W) W = g_ordered_min_lanes;   // 4 or 8 lanes per row
            if (nrhs == 1 && g_ordered_min_lanes == 1) W = 1;
        }
#define LCD_ORDERED_CASE(w, k) if (W == w && KR == k) rc = launch_ordered<w, k>(q, window_rows, st); else
        LCD_ORDERED_CASE(1, 1) LCD_ORDERED_CASE(2, 1) LCD_ORDERED_CASE(4, 1) LCD_ORDERED_CASE(8, 1)
        LCD_ORDERED_CASE(8, 2) LCD_ORDERED_CASE(16, 2) LCD_ORDERED_CASE(32, 2)
        LCD_ORDERED_CASE(8, 4) LCD_ORDERED_CASE(16, 4)
        rc = LCD_ERR_INVALID_ARGUMENT;
#undef LCD_ORDERED_CASE
        if (rc) return rc;
    }
    return finish(status_dev, st, status_host);
}

// Block-row partition of one solve across the GPUs of a node, rows in level order: this rank
// solves the nodes listed in `order_local` (its block of rows, in the order of the global level
// sets) and publishes what other ranks need into their x arrays (plain peer stores).
extern "C" int lcd_sptrsv_csr_ordered_part(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                                           const double *Ax, const double *b, double *x, int flags,
                                           const int32_t *order_local, int32_t n_local,
                                           int32_t *task_records, int records_ready,
                                           const unsigned char *need_mask, double *const *peer_x,
                                           int32_t n_ranks, int64_t window_rows, int32_t *status_dev,
                                           int32_t timeout_ms, void *stream, int *status_host) {
    if (n < 0 || nnz < 0 || n_local < 0 || n_local > n || !status_dev || window_rows < 0 || n_ranks < 1 ||
        n_ranks > 8)
        return LCD_ERR_INVALID_ARGUMENT;
    if (flags & ~LCD_SOLVE_UPPER) return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && (!Ap || !Ai || !Ax || !b || !x || x == b || !task_records)) return LCD_ERR_INVALID_ARGUMENT;
    if (n_local > 0 && !records_ready && !order_local) return LCD_ERR_INVALID_ARGUMENT;
    if (need_mask && !peer_x) return LCD_ERR_INVALID_ARGUMENT;
    if (((uintptr_t)task_records & 15) != 0) return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    int rc = reset_status(status_dev, st);
    if (rc) return rc;
    if (n_local > 0) {
        // x is NOT filled here: every rank fills its x with the reserved pattern and all ranks
        // synchronise on the host before the first rank is allowed to publish
        OrderedParams q;
        q.m = CsrSolveParams{n, nnz, Ap, Ai, Ax, nullptr, b, x, flags, 1, 1, status_dev,
                             timeout_ns(timeout_ms), nullptr, 0, n, need_mask, {nullptr}};
        for (int k = 0; k < n_ranks && peer_x; ++k) q.m.peers[k] = peer_x[k];
        q.meta = reinterpret_cast<const TaskMeta *>(task_records);
        q.row_flags = nullptr;
        q.n_tasks = n_local;
        q.max_pause_ns = (unsigned)g_ordered_pause_ns;
        q.counters = task_records + 4 * (size_t)n_local;
        q.trace = nullptr;
        LCD_CUDA_TRY(cudaMemsetAsync(q.counters, 0, kOrdWarps * kCounterStride * sizeof(int32_t), st));
        if (!records_ready) {
            ordered_meta_kernel<<<(n_local + 255) / 256, 256, 0, st>>>(
                q.m, order_local, n_local, reinterpret_cast<TaskMeta *>(task_records));
            LCD_CUDA_TRY(cudaGetLastError());
        }
        rc = launch_ordered_t<2, 1, false, true>(q, window_rows, st);
        if (rc) return rc;
    }
    return finish(status_dev, st, status_host);
}
