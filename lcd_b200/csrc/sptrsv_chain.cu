// Block-recurrence chain solver: CSR triangular solves whose levels hold only a few rows.
//
// Such a matrix is one long dependence chain: level-by-level substitution pays one
// hand-off (a poll, a barrier, or a dozen dependent instructions of a lone warp) per
// level, and there are hundreds of thousands of levels.  The chain is shortened
// algebraically instead.  Rows are grouped into blocks of 64 consecutive rows; with
// D_B the 64 x 64 diagonal block and L_BC the coupling of block B to block C, the solve
//        D_B x_B = r_B - L_B,B-1 x_B-1 - sum_{C <= B-2} L_BC x_C
// is rewritten, once per value set (lcd_chain_prepare, fully parallel), as
//        x_B = y_B - T_B x_B-1,     T_B = D_B^-1 L_B,B-1,     y_B = M_B ( r_B - sum_{C <= B-2} L_BC x_C ),
//        M_B = D_B^-1
// so that the part of the chain that cannot be overlapped, x_B-1 -> x_B, is one dense
// 64 x 64 mat-vec shared by four warps (no dependent chain inside it), and everything that
// reaches at least two blocks back is taken off that path.  T_B and M_B are kept as 32 x 32
// tiles (T00 T01 / T10 T11 and M11, M21, M22; M12 is zero).
//
// The solve kernel works on chunks of 512 rows.  It runs as thread-block clusters of eight
// where the device hosts them: a cluster takes one ticket and its blocks take eight
// consecutive chunks (a chunk only waits for chunks with smaller numbers, which are running
// or done, so the waits terminate), and the hand-over between consecutive chunks of a
// cluster goes through distributed shared memory instead of L2.
//   tiles: one SM streams only about 32 bytes per clock from L2, less than the four main warps
//     consume, so six of a chunk's eight T tiles (32 KB each) are requested at launch, long
//     before the chunk's turn, into a shared-memory ring by bulk asynchronous copies; the last
//     two follow into freed stages (one lane of the last warp keeps the ring full);
//   phase A (256 threads, two rows each, a warp per 64-row block): at launch the operands that
//     lie in the chunk, two or more blocks back, go into a shared-memory list (one column-major
//     strip per 32 rows, so a warp reads it without bank conflicts and with one trip count);
//     16 chunks before the turn the operands from before the chunk are fetched by polling x in
//     global memory without waiting (a solution vector pre-filled with a reserved NaN is its
//     own ready flag) and y_B = M_B t_B is formed from what is there; 2 chunks before the turn
//     the missing ones are polled once more and each that has arrived adds its value times one
//     column of M_B; complete blocks are published, the others parked;
//   helpers (3 warps, blocks B mod 3): parked blocks - the late operands (all of a warp's
//     blocks polled in turn), the listed ones (polling the chunk's x in shared memory), one
//     column of M_B for each;
//   main warps (4): warp (half, side) multiplies tile T[half][side] with half `side` of x_B-1
//     (read from shared memory as broadcasts); the side-0 warps hand their partial sums over
//     through a named barrier, the side-1 warps add y_B and publish x_B; all four meet at a
//     128-thread barrier per block;
//   every wait is bounded; a failed wait raises an error and poisons the rest of the chunk
//     with NaN so that later chunks do not wait for it.
//
// The result differs from plain substitution only by rounding; the relative residual
// stays at the 1e-16 level for diagonally dominant blocks.  Operands from earlier chunks
// are subtracted in the order they arrive, so two runs can differ in the last bits.
// Callers that need the sequential order, bit for bit, use the LCD_SOLVE_EXACT path of
// lcd_sptrsv_csr_syncfree instead.
#include "common.cuh"

#include <type_traits>

namespace lcd {

constexpr int kChainThreads = 256;                    // four main warps, three helpers, loader warp
constexpr int kChainWorkers = 256;
constexpr int kChainRows = 512;                       // rows per chunk
constexpr int kChainRowsPerThread = kChainRows / kChainWorkers;
constexpr int kChainBlocks = kChainRows / 32;         // 32-row halves (operand strips are per half)
constexpr int kChainPairs = kChainRows / 64;          // 64-row blocks
constexpr int kPairsPerWarp = kChainPairs / 8;        // phase A: blocks per warp
constexpr int kChainMain = 4;                         // main warps
constexpr int kChainHelpers = 3;
constexpr int kChainStages = 6;                       // ring of T tiles (32 KB per stage)
constexpr int kTileDoubles = 1024;
constexpr int kPairDoubles = 7 * kTileDoubles;        // per 64-row block: M11, M21, M22, T00, T01, T10, T11
constexpr int kPairT = 3 * kTileDoubles;              // offset of the four T tiles
constexpr int kStageDoubles = 4 * kTileDoubles;
constexpr int kChainHalo = 64;                        // the block before the chunk
constexpr int kChainGateFar = 16;                     // chunks ahead at which a chunk gathers its operands
constexpr int kChainGate = 2;                         // chunks ahead at which pending operands are polled again
constexpr int kChainCluster = 8;                      // blocks per cluster (portable maximum)
constexpr int kStatusDone = 6;                        // status word: chunks finished
constexpr unsigned kFullMask = 0xffffffffu;

// ---- numeric preparation ------------------------------------------------------------
// One thread block per 64-row block, seven warps.  Each warp walks the rows of one 32-row
// half in order and builds one 32 x 32 tile: row r of every tile satisfies the same recurrence
//        row_r = (rhs_r - sum_{k<r} D[r][k] row_k) / D[r][r]
// (D the half's own diagonal block) with right-hand sides e_r (the inverse of D) or row r of
// the coupling to the half one, two or three halves back; lane c carries column c.  Only the
// stored entries are visited: a row's entries are loaded 32 at a time, the ones that matter
// to the warp are found with a ballot and handed round with shuffles.  The walks do not read
// one another.  Top half (b): M11 = D_b^-1, W1 = M11 L_b,b-1, W2 = M11 L_b,b-2.  Bottom half
// (b+1): M22 = D_b+1^-1, V1 = M22 L_b+1,b, V2 = M22 L_b+1,b-1, V3 = M22 L_b+1,b-2.
// Eliminating x_b from the bottom half's equation then takes three dense products:
//        M21 = -V1 M11,   T11 = V2 - V1 W1,   T10 = V3 - V1 W2       (T00 = W2, T01 = W1).
// Tiles sit in shared memory with column c of row r at r * 32 + (c ^ r): rows and columns are
// both read without bank conflicts.
constexpr int kPrepThreads = 224;
constexpr int kPrepSmemBytes = 7 * kTileDoubles * 8;
__device__ __forceinline__ int swz(int row, int col) { return row * 32 + (col ^ row); }

__global__ void __launch_bounds__(kPrepThreads)
chain_prepare_kernel(const CsrSolveParams p, double *__restrict__ ws, int pair_begin, int pair_end) {
    extern __shared__ __align__(16) double prep_tiles[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int odd = warp >= 3;                   // bottom half
    const int which = odd ? warp - 3 : warp;     // 0: inverse, k: coupling to the half k back
    double *T = prep_tiles + warp * kTileDoubles;
    const int gp = pair_begin + blockIdx.x;
    if (gp >= pair_end) return;
    const bool upper = p.flags & LCD_SOLVE_UPPER;
    const int base = (gp * 2 + odd) * 32;
    // entry kinds: 1, 2, 3 = three, two, one half back, 4 = this half (before row r)
    const int mine = 4 - which;
    int lo = 0, hi = 0;
    double diag = 1.0;  // rows past the end, and rows with bad pointers, act as identity rows
    // (the walk multiplies by the reciprocal: one division per row of the half, not one per
    // row and tile)
    {
        const int task = base + lane;
        if (task < p.n) {
            const int r = upper ? p.n - 1 - task : task;
            int d = -1;
            if (csr_row_range(p, r, lo, hi, d)) {
                if (d >= 0) diag = __ldg(p.Ax + d);
            } else {
                lo = hi = 0;
            }
        }
    }
    diag = 1.0 / diag;
    // the first 32 entries of the next row are requested while the current row is processed
    int nlo = __shfl_sync(kFullMask, lo, 0), nhi = __shfl_sync(kFullMask, hi, 0);
    int pc = -1;
    double pa = 0.0;
    if (nlo + lane < nhi) { pc = __ldg(p.Ai + nlo + lane); pa = __ldg(p.Ax + nlo + lane); }
    for (int r = 0; r < 32; ++r) {
        const int rlo = nlo, rhi = nhi;
        int cc = pc;
        double ca = pa;
        if (r + 1 < 32) {
            nlo = __shfl_sync(kFullMask, lo, r + 1);
            nhi = __shfl_sync(kFullMask, hi, r + 1);
            pc = -1;
            pa = 0.0;
            if (nlo + lane < nhi) { pc = __ldg(p.Ai + nlo + lane); pa = __ldg(p.Ax + nlo + lane); }
        }
        const double d = __shfl_sync(kFullMask, diag, r);
        double acc = (which == 0 && lane == r) ? 1.0 : 0.0;
        for (int j0 = rlo; j0 < rhi; j0 += 32) {
            if (j0 != rlo) {
                cc = -1;
                ca = 0.0;
                if (j0 + lane < rhi) { cc = __ldg(p.Ai + j0 + lane); ca = __ldg(p.Ax + j0 + lane); }
            }
            int where = 0;   // (kind << 5) + column within the half the entry points to
            if ((unsigned)cc < (unsigned)p.n) {
                const int tc = upper ? p.n - 1 - cc : cc;
                const int off = tc - (base - 96);
                if (off >= 0 && tc < base + r) where = off + 32;
            }
            unsigned todo = __ballot_sync(kFullMask, (where >> 5) == 4 || (where >> 5) == mine);
            while (todo) {
                const int src = __ffs(todo) - 1;
                todo &= todo - 1;
                const int w = __shfl_sync(kFullMask, where, src);
                const double av = __shfl_sync(kFullMask, ca, src);
                const int c = w & 31;
                if (w >= 128) acc = fma(-av, T[swz(c, lane)], acc);
                else if (lane == c) acc += av;
            }
        }
        T[swz(r, lane)] = acc * d;
        __syncwarp();
    }
    __syncthreads();
    // Growth of the explicit inverses: (largest entry of any tile) x (largest diagonal entry of
    // the half), about 1 for diagonally dominant blocks and huge for blocks whose inverse
    // grows along the substitution (then multiplying by it loses digits that substitution
    // keeps).  The maximum over all blocks goes to the word behind the tiles; NaN counts as inf.
    double *growth_word = ws + (long long)((p.n + 63) / 64) * kPairDoubles;
    double tile_max = 0.0;
    auto absmax = [](double m, double v) {
        v = fabs(v);
        return (v != v) ? (double)INFINITY : (v > m ? v : m);
    };
    for (int k = 0; k < 32; ++k) tile_max = absmax(tile_max, T[swz(k, lane)]);
    // (diag holds the reciprocal of the row's diagonal entry)
    double diag_max = absmax(0.0, 1.0 / diag);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        tile_max = absmax(tile_max, __shfl_xor_sync(kFullMask, tile_max, off));
        diag_max = absmax(diag_max, __shfl_xor_sync(kFullMask, diag_max, off));
    }
    // Output layouts.  Inverse tiles (M11, M21, M22): element (r, k) at k * 32 + r, so that lane
    // r of a warp applying them loads its row coalesced.  T tiles: elements (r, 2q), (r, 2q + 1)
    // side by side at (q * 32 + r) * 2, so that lane r of a main warp reads its row from shared
    // memory with 16-byte loads that do not conflict.
    const double *tM11 = prep_tiles, *tW1 = tM11 + kTileDoubles, *tW2 = tW1 + kTileDoubles;
    const double *tM22 = tW2 + kTileDoubles, *tV1 = tM22 + kTileDoubles, *tV2 = tV1 + kTileDoubles;
    const double *tV3 = tV2 + kTileDoubles;
    double *out = ws + (long long)gp * kPairDoubles;
    if (warp == 6) {
        double2 *o00 = reinterpret_cast<double2 *>(out + kPairT);
        double2 *o01 = o00 + kTileDoubles / 2;
        for (int k = 0; k < 32; ++k) {
            out[k * 32 + lane] = tM11[swz(lane, k)];
            out[2 * kTileDoubles + k * 32 + lane] = tM22[swz(lane, k)];
        }
        for (int q = 0; q < 16; ++q) {
            o00[q * 32 + lane] = make_double2(tW2[swz(lane, 2 * q)], tW2[swz(lane, 2 * q + 1)]);
            o01[q * 32 + lane] = make_double2(tW1[swz(lane, 2 * q)], tW1[swz(lane, 2 * q + 1)]);
        }
    } else {
        // products: warp pair 0 -> M21, 1 -> T11, 2 -> T10; each warp 16 columns, lane = row
        const int prod = warp >> 1, c0 = (warp & 1) * 16;
        const double *X = prod == 0 ? tM11 : prod == 1 ? tW1 : tW2;
        const double *S = prod == 1 ? tV2 : tV3;
        double acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = prod == 0 ? 0.0 : S[swz(lane, c0 + j)];
        for (int k = 0; k < 32; ++k) {
            const double v = tV1[swz(lane, k)];
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] = fma(-v, X[swz(k, c0 + j)], acc[j]);
        }
        double prod_max = 0.0;
#pragma unroll
        for (int j = 0; j < 16; ++j) prod_max = absmax(prod_max, acc[j]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
            prod_max = absmax(prod_max, __shfl_xor_sync(kFullMask, prod_max, off));
        tile_max = absmax(tile_max, prod_max);
        if (prod == 0) {
#pragma unroll
            for (int j = 0; j < 16; ++j) out[kTileDoubles + (c0 + j) * 32 + lane] = acc[j];
        } else {
            double2 *o = reinterpret_cast<double2 *>(out + kPairT + (prod == 1 ? 3 : 2) * kTileDoubles);
#pragma unroll
            for (int j = 0; j < 16; j += 2) o[((c0 + j) / 2) * 32 + lane] = make_double2(acc[j], acc[j + 1]);
        }
    }
    if (lane == 0) {
        // non-negative doubles order like their bit patterns (inf above every finite value)
        const double growth = tile_max * diag_max;
        atomicMax(reinterpret_cast<unsigned long long *>(growth_word),
                  (unsigned long long)__double_as_longlong(growth != growth ? (double)INFINITY : growth));
    }
}

// ---- asynchronous-copy plumbing --------------------------------------------------------
__device__ __forceinline__ unsigned smem_addr(const void *ptr) {
    return (unsigned)__cvta_generic_to_shared(ptr);
}
__device__ __forceinline__ void mbar_init(unsigned long long *bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long *bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(unsigned long long *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(unsigned long long *bar, unsigned parity) {
    unsigned done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
__device__ __forceinline__ bool mbar_test_wait(unsigned long long *bar, unsigned parity) {
    unsigned done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
__device__ __forceinline__ int ld_acquire_shared(const int *ptr) {
    int v;
    asm volatile("ld.acquire.cta.shared.s32 %0, [%1];" : "=r"(v) : "r"(smem_addr(ptr)) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_shared(int *ptr, int v) {
    asm volatile("st.release.cta.shared.s32 [%0], %1;" ::"r"(smem_addr(ptr)), "r"(v) : "memory");
}
// global -> shared bulk copy (source, destination and size are multiples of 16 bytes);
// completion is signalled on the mbarrier as transferred bytes
__device__ __forceinline__ void bulk_load(void *dst, const void *src, unsigned bytes,
                                          unsigned long long *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}
__device__ __forceinline__ void chain_prefetch_l2(const void *ptr) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr));
}
__device__ __forceinline__ void chain_prefetch_l1(const void *ptr) {
    asm volatile("prefetch.global.L1 [%0];" ::"l"(ptr));
}
// Named barriers of the main warps.  A row half's two warps meet at kBarZ0 + half (64 threads:
// the warp with the partial sum arrives, the finishing warp waits); all four meet at kBarStep
// once per block.  Named barriers have no timeout, so every warp performs them unconditionally.
constexpr int kBarZ0 = 2, kBarStep = 4;
__device__ __forceinline__ void pair_arrive(int id) {
    asm volatile("bar.arrive %0, 64;" ::"r"(id) : "memory");
}
__device__ __forceinline__ void pair_sync(int id) {
    asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory");
}
__device__ __forceinline__ void step_sync() {
    asm volatile("bar.sync %0, %1;" ::"n"(kBarStep), "n"(kChainMain * 32) : "memory");
}
// one arrival per warp, predicated instead of branched so that the warp stays converged
__device__ __forceinline__ void mbar_arrive_lane0(unsigned long long *bar, int lane) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.eq.s32 p, %1, 0;\n\t"
        "@p mbarrier.arrive.shared::cta.b64 _, [%0];\n\t}" ::"r"(smem_addr(bar)),
        "r"(lane)
        : "memory");
}
__device__ __forceinline__ void workers_barrier() {
    asm volatile("bar.sync 1, %0;" ::"n"(kChainWorkers) : "memory");
}

// A wait of a whole warp: every lane polls its own condition, but the loop is left by all
// lanes together (a vote decides).  Lanes that left a polling loop one by one would run the
// code after it as separately scheduled groups, and every warp-wide shuffle there would
// cost a re-synchronisation of the groups (measured: 15,000 cycles for one 32-step mat-vec).
template <class Ready>
__device__ __forceinline__ bool warp_wait(Ready ready, Deadline &dl, volatile int *failed_flag,
                                          int32_t *status, int node) {
    unsigned polls = 0;
    for (;;) {
        if (__all_sync(kFullMask, ready())) return true;
        if ((++polls & 15u) == 0 &&
            __any_sync(kFullMask, *failed_flag != 0 || dl.tick(status, node)))
            return false;
    }
}

// ---- thread-block cluster plumbing ------------------------------------------------------
// Consecutive chunks run on the blocks of one cluster, so that the hand-over between them (the
// two blocks of x before a chunk) is a store into the next block's shared memory instead of a
// round trip through L2.
__device__ __forceinline__ unsigned cluster_ctarank() {
    unsigned r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ unsigned cluster_nctarank() {
    unsigned r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_barrier() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// address of the same shared-memory location in another block of the cluster
__device__ __forceinline__ unsigned cluster_map(const void *ptr, unsigned rank) {
    unsigned out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_addr(ptr)), "r"(rank));
    return out;
}
__device__ __forceinline__ void st_cluster_f64(unsigned addr, double v) {
    asm volatile("st.shared::cluster.f64 [%0], %1;" ::"r"(addr), "d"(v) : "memory");
}
__device__ __forceinline__ int ld_cluster_s32(unsigned addr) {
    int v;
    asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}

// ---- the solve ---------------------------------------------------------------------------
struct ChainParams {
    CsrSolveParams m;
    const double *__restrict__ ws;
    int cap;  // capacity of the in-chunk operand list (entries)
    int chunk_begin;  // this launch solves the chunks [chunk_begin, ...) up to row_end (solve order)
    int row_end;
    int gate_far;  // chunks ahead of its turn at which a chunk gathers its operands
    int gate;      // ... and at which it polls the ones that were missing once more
};

// y += M d for one 64-row block (M11, M21, M22 at m11, element (r, k) at k * 32 + r, m11
// already offset by the lane): shuffle / FMA pairs on independent accumulators
__device__ __noinline__ void apply_inverse(const double *m11, double d0, double d1, double &ytop,
                                           double &ybot) {
    const double *m21 = m11 + kTileDoubles, *m22 = m21 + kTileDoubles;
    double y0 = 0.0, y1 = 0.0, z0 = 0.0, z1 = 0.0, z2 = 0.0, z3 = 0.0;
#pragma unroll
    for (int k = 0; k < 32; k += 2) {
        const double ta = __shfl_sync(kFullMask, d0, k), tb = __shfl_sync(kFullMask, d0, k + 1);
        const double tc = __shfl_sync(kFullMask, d1, k), td = __shfl_sync(kFullMask, d1, k + 1);
        y0 = fma(__ldg(m11 + k * 32), ta, y0);
        y1 = fma(__ldg(m11 + (k + 1) * 32), tb, y1);
        z0 = fma(__ldg(m21 + k * 32), ta, z0);
        z1 = fma(__ldg(m21 + (k + 1) * 32), tb, z1);
        z2 = fma(__ldg(m22 + k * 32), tc, z2);
        z3 = fma(__ldg(m22 + (k + 1) * 32), td, z3);
    }
    ytop += y0 + y1;
    ybot += (z0 + z1) + (z2 + z3);
}

// y += M d where only a few rows of d are nonzero: one column of M per such row, the loads of
// four columns in flight together (many rows: the whole product)
__device__ __forceinline__ void add_columns(const double *m11, const double d0, const double d1,
                                            double &ytop, double &ybot) {
    unsigned top = __ballot_sync(kFullMask, d0 != 0.0), bot = __ballot_sync(kFullMask, d1 != 0.0);
    if (__popc(top) + __popc(bot) > 12) {
        apply_inverse(m11, d0, d1, ytop, ybot);
        return;
    }
    while (top) {
        int c[4];
        double dv[4], a[4], b[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            c[u] = -1;
            if (top) { c[u] = __ffs(top) - 1; top &= top - 1; }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            dv[u] = __shfl_sync(kFullMask, d0, c[u] & 31);
            a[u] = c[u] >= 0 ? __ldg(m11 + c[u] * 32) : 0.0;
            b[u] = c[u] >= 0 ? __ldg(m11 + kTileDoubles + c[u] * 32) : 0.0;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (c[u] >= 0) { ytop = fma(a[u], dv[u], ytop); ybot = fma(b[u], dv[u], ybot); }
    }
    while (bot) {
        int c[4];
        double dv[4], b[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            c[u] = -1;
            if (bot) { c[u] = __ffs(bot) - 1; bot &= bot - 1; }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            dv[u] = __shfl_sync(kFullMask, d1, c[u] & 31);
            b[u] = c[u] >= 0 ? __ldg(m11 + 2 * kTileDoubles + c[u] * 32) : 0.0;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (c[u] >= 0) ybot = fma(b[u], dv[u], ybot);
    }
}

// one 32 x 32 tile times one half of the previous block: lane r's row (16-byte loads that
// do not conflict) against broadcast loads of x
__device__ __forceinline__ double tile_matvec(const double2 *w, const double2 *xa, double a0) {
    double a1 = 0.0, a2 = 0.0, a3 = 0.0;
#pragma unroll
    for (int qd = 0; qd < 16; qd += 2) {
        const double2 u0 = w[qd * 32], u1 = w[(qd + 1) * 32];
        const double2 v0 = xa[qd], v1 = xa[qd + 1];
        a0 = fma(-u0.x, v0.x, a0);
        a1 = fma(-u0.y, v0.y, a1);
        a2 = fma(-u1.x, v1.x, a2);
        a3 = fma(-u1.y, v1.y, a3);
    }
    return (a0 + a1) + (a2 + a3);
}

template <bool TRACE>
__global__ void __launch_bounds__(kChainThreads, 1)
csr_chain_kernel(const ChainParams q) {
    const CsrSolveParams &p = q.m;
    extern __shared__ __align__(128) unsigned char chain_smem[];
    double *ring = reinterpret_cast<double *>(chain_smem);      // kChainStages x (T00, T01, T10, T11)
    double *sxh = ring + kChainStages * kStageDoubles;           // halo, chunk, zero slot
    double *sx = sxh + kChainHalo;                               // x of the chunk (chunk-local index)
    double *sacc = sx + kChainRows + 2;                          // partial sums after phase A
    double *sy = sacc + kChainRows;                              // y_B, from phase A or the helpers
    unsigned long long *spend = reinterpret_cast<unsigned long long *>(sy + kChainRows + 64);  // operands from
                                                                 // before the chunk still pending per row
    double *eval = reinterpret_cast<double *>(spend + kChainRows);  // in-chunk operands: values
    int *ecol = reinterpret_cast<int *>(eval + q.cap);           // ... and chunk-local columns
    __shared__ unsigned long long s_full[kChainStages];
    __shared__ unsigned long long s_empty[kChainStages];
    __shared__ int s_chunk;
    __shared__ int s_failed;
    __shared__ int s_tiles;                                    // ring stages that have landed
    __shared__ int s_width[kChainBlocks];
    __shared__ int s_bptr[kChainBlocks + 1];
    __shared__ double s_z[2][32];
    __shared__ int s_early[kChainPairs];                       // y_B was computed in phase A
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    volatile int *failed_flag = &s_failed;
    // One ticket per cluster: its blocks take consecutive chunks.  (A cluster is resident as a
    // whole, and a chunk still only waits for chunks with smaller numbers.)
    const unsigned crank = cluster_ctarank(), csize = cluster_nctarank();
    if (tid == 0) {
        if (crank == 0) s_chunk = q.chunk_begin + atomicAdd(&p.status[kStatusTicket], 1) * (int)csize;
        s_failed = 0;
        s_tiles = 0;
    }
    if (tid < kChainHalo) reinterpret_cast<unsigned long long *>(sxh)[tid] = kPendingBits;
    if (tid == kChainThreads - 32) {
        for (int s = 0; s < kChainStages; ++s) { mbar_init(&s_full[s], 1); mbar_init(&s_empty[s], 1); }
        mbar_init_fence();
    }
    __syncthreads();
    if (csize > 1) cluster_barrier();   // ticket and halo sentinels are in place everywhere
    const int chunk = (csize > 1 ? ld_cluster_s32(cluster_map(&s_chunk, 0)) : s_chunk) + (int)crank;
    // (the body is a lambda so that every thread, whatever its role, comes back to the closing
    // cluster barrier: no block may leave while a neighbour can still store into it)
    auto body = [&]() {
    const int row0 = chunk * kChainRows;
    const int rows_here = min(kChainRows, q.row_end - row0);
    if (rows_here <= 0) return;
    const bool upper = p.flags & LCD_SOLVE_UPPER;
    const int npair = (rows_here + 63) / 64;
    const double *wsc = q.ws + (long long)(row0 / 64) * kPairDoubles;
    constexpr unsigned kStageBytes = kStageDoubles * sizeof(double);
    Deadline dl;
    dl.start(p.budget_ns);

    // the first stages of the ring are requested right away (nothing to wait for)
    int issued = 0;
    if (tid == kChainThreads - 32)
        for (; issued < min(kChainStages, npair); ++issued) {
            mbar_expect_tx(&s_full[issued], kStageBytes);
            bulk_load(ring + issued * kStageDoubles, wsc + (long long)issued * kPairDoubles + kPairT,
                      kStageBytes, &s_full[issued]);
        }

    // ---- phase A: warp w owns the 64-row blocks w, w + 8, ..., a thread one row of each of
    // their halves (row k of the thread: half k & 1 of block w + 8 (k >> 1)) ----------------
    // A1 (pattern only, nothing to wait for): operands in the chunk that lie before the
    // previous 64-row block are counted, the per-half strips are laid out and filled.
    auto half_of = [&](int k) { return 2 * (warp + 8 * (k >> 1)) + (k & 1); };
    int lo_[kChainRowsPerThread], hi_[kChainRowsPerThread], cnt_[kChainRowsPerThread];
    bool failed = false;
#pragma unroll
    for (int k = 0; k < kChainRowsPerThread; ++k) {
        const int local = half_of(k) * 32 + lane;
        lo_[k] = hi_[k] = cnt_[k] = 0;
        sx[local] = __longlong_as_double((long long)kPendingBits);
        sy[local] = __longlong_as_double((long long)kPendingBits);
        if (local < rows_here) {
            const int task = row0 + local;
            const int r = upper ? p.n - 1 - task : task;
            const int near0 = (local & ~63) - 64;  // chunk-local start of the block before
            int lo = 0, hi = 0, d = -1;
            if (!csr_row_range(p, r, lo, hi, d)) {
                raise_error(p.status, (p.flags & LCD_SOLVE_OF_FULL) ? LCD_ERR_MISSING_DIAGONAL
                                                                   : LCD_ERR_BAD_POINTERS, r);
                failed = true;
            } else {
                lo_[k] = lo;
                hi_[k] = hi;
                int listed = 0;
                for (int j = lo; j < hi; ++j) {
                    const int c = __ldg(p.Ai + j);
                    const int tc = ((unsigned)c < (unsigned)p.n) ? (upper ? p.n - 1 - c : c) : task;
                    if (tc >= task) {  // not strictly before this row (or out of range)
                        raise_error(p.status, LCD_ERR_INDEX_RANGE, r);
                        failed = true;
                        hi_[k] = lo;   // the row is not touched again
                        break;
                    }
                    const int cl = tc - row0;
                    if (cl >= 0 && cl < near0) ++listed;
                }
                cnt_[k] = failed ? 0 : listed;
            }
        }
        const int width = (__reduce_max_sync(kFullMask, cnt_[k]) + 1) & ~1;
        if (lane == 0) s_width[half_of(k)] = width;
    }
    if (tid == 0) sx[kChainRows] = 0.0;  // padding entries of the strips point here
    workers_barrier();
    if (warp == 0) {
        int incl = lane < kChainBlocks ? s_width[lane] * 32 : 0;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int t = __shfl_up_sync(kFullMask, incl, off);
            if (lane >= off) incl += t;
        }
        if (lane < kChainBlocks) s_bptr[lane + 1] = incl;
        if (lane == 0) s_bptr[0] = 0;
    }
    workers_barrier();
    const bool overflow = s_bptr[kChainBlocks] > q.cap;  // block-uniform
    if (!overflow) {
#pragma unroll
        for (int k = 0; k < kChainRowsPerThread; ++k) {
            const int blk = half_of(k);
            const int local = blk * 32 + lane;
            const int width = s_width[blk];
            if (width == 0) continue;
            const int near0 = (local & ~63) - 64;
            int pos = s_bptr[blk] + lane;
            const int pos_end = pos + width * 32;
            if (local < rows_here && cnt_[k] > 0)
                for (int j = lo_[k]; j < hi_[k]; ++j) {
                    const int c = __ldg(p.Ai + j);
                    const int cl = (upper ? p.n - 1 - c : c) - row0;
                    if (cl >= 0 && cl < near0) {
                        ecol[pos] = cl;
                        eval[pos] = __ldg(p.Ax + j);
                        pos += 32;
                    }
                }
            for (; pos < pos_end; pos += 32) { ecol[pos] = kChainRows; eval[pos] = 0.0; }
        }
    }
    // Hundreds of resident chunks spinning on operands that are many chunks away would only
    // congest L2 for the few chunks whose turn it is, and would find most of them missing: the
    // chunk sleeps until its turn is kChainGateFar chunks away.
    auto sleep_until = [&](const int ahead) {
        if (tid == 0) {
            while (ld_relaxed_s32(&p.status[kStatusDone]) < chunk - ahead) {
                __nanosleep(200);
                if (dl.tick(p.status, row0)) break;
            }
        }
        workers_barrier();
    };
    sleep_until(q.gate_far);
    // A2: contributions of rows before the chunk that are not covered by the T tiles (they
    // belong to earlier tickets, so a bounded spin is safe).  Every operand that is already
    // there is consumed without waiting; operands still pending are remembered in a bit mask.
    double acc_[kChainRowsPerThread];
    unsigned long long pend_[kChainRowsPerThread];
#pragma unroll
    for (int k = 0; k < kChainRowsPerThread; ++k) {
        const int local = half_of(k) * 32 + lane;
        acc_[k] = 0.0;
        pend_[k] = 0ull;
        if (local >= rows_here || failed) continue;
        const int r = upper ? p.n - 1 - (row0 + local) : row0 + local;
        // tasks before far_end are fetched here, the rest is covered by the strips and tiles
        const int far_end = min(row0, row0 + (local & ~63) - 64);
        double acc = __ldg(p.b + r);
        // (four entries at a time: their loads are in flight together)
        for (int j = lo_[k]; j < hi_[k] && !failed; j += 4) {
            int c[4];
            double a[4], xv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const bool in = j + u < hi_[k];
                c[u] = in ? __ldg(p.Ai + j + u) : -1;
                a[u] = in ? __ldg(p.Ax + j + u) : 0.0;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (c[u] >= 0 && (upper ? p.n - 1 - c[u] : c[u]) >= far_end) c[u] = -1;
                xv[u] = c[u] >= 0 ? ld_relaxed_f64(p.x + c[u]) : 0.0;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (c[u] < 0 || failed) continue;
                if (is_pending(xv[u])) {
                    const int bit = j + u - lo_[k];
                    if (bit < 64) { pend_[k] |= 1ull << bit; continue; }
                    while (is_pending(xv[u] = ld_relaxed_f64(p.x + c[u])))   // very long rows: wait here
                        if (dl.tick(p.status, r)) { failed = true; break; }
                    if (failed) continue;
                }
                acc = fma(-a[u], xv[u], acc);
            }
        }
        acc_[k] = acc;
    }
    {
        // the chunk's tiles are pulled towards L2 now, before its turn (all resident chunks
        // doing so at launch would only evict one another's tiles)
        const char *src = reinterpret_cast<const char *>(wsc);
        const long long bytes = (long long)npair * kPairDoubles * 8;
        for (long long off = (long long)tid * 128; off < bytes; off += (long long)kChainThreads * 128)
            chain_prefetch_l2(src + off);
    }
    // Every block gets y_B = M t_B right here, from the warp that holds its rows:
    // y_top = M11 t_top, y_bottom = M21 t_top + M22 t_bottom, formed without the operands that
    // are still missing.  The product is linear: a late operand delta_i of row i adds delta_i
    // times column i of M, which costs one load per lane instead of 96.
    double ytop_[kPairsPerWarp], ybot_[kPairsPerWarp];
    bool formed_[kPairsPerWarp];
#pragma unroll
    for (int kk = 0; kk < kPairsPerWarp; ++kk) {
        const int pr = warp + 8 * kk;
        const int base = pr * 64;
        ytop_[kk] = ybot_[kk] = 0.0;
        formed_[kk] = pr < npair && !overflow && __all_sync(kFullMask, !failed);
        if (!formed_[kk]) continue;
        // (operands through shared memory, not shuffles: the lanes may run as separate groups
        // after the per-lane loops above)
        sacc[base + lane] = base + lane < rows_here ? acc_[2 * kk] : 0.0;
        sacc[base + 32 + lane] = base + 32 + lane < rows_here ? acc_[2 * kk + 1] : 0.0;
        __syncwarp();
        const double *m11 = wsc + (long long)pr * kPairDoubles + lane;
        const double *m21 = m11 + kTileDoubles, *m22 = m21 + kTileDoubles;
        const double2 *tt = reinterpret_cast<const double2 *>(sacc + base);
        const double2 *tb = tt + 16;
        double y0 = 0.0, y1 = 0.0, z0 = 0.0, z1 = 0.0, z2 = 0.0, z3 = 0.0;
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
            const double2 ta = tt[c / 2], tc = tb[c / 2];
            y0 = fma(__ldg(m11 + (c + 0) * 32), ta.x, y0);
            y1 = fma(__ldg(m11 + (c + 1) * 32), ta.y, y1);
            z0 = fma(__ldg(m21 + (c + 0) * 32), ta.x, z0);
            z1 = fma(__ldg(m21 + (c + 1) * 32), ta.y, z1);
            z2 = fma(__ldg(m22 + (c + 0) * 32), tc.x, z2);
            z3 = fma(__ldg(m22 + (c + 1) * 32), tc.y, z3);
        }
        ytop_[kk] = y0 + y1;
        ybot_[kk] = (z0 + z1) + (z2 + z3);
    }
    // Shortly before the chunk's turn: one sweep over what was pending (four loads in flight
    // per thread), the columns of M for what has arrived since, and y_B is published - or
    // parked (state 2) for the helper warps where operands are missing even now or lie inside
    // the chunk.  The helper warps then have (almost) nothing to do while the main warps run.
    sleep_until(q.gate);
    double dlt_[kChainRowsPerThread];
    auto sweep = [&]() {   // one pass over what is still pending; true when something is left
        bool any = false;
#pragma unroll
        for (int k = kChainRowsPerThread - 1; k >= 0; --k) {
            dlt_[k] = 0.0;
            unsigned long long mask = pend_[k];
            if (!mask) continue;
            double acc = 0.0;
            unsigned long long left = mask;
            while (left) {
                int jq[4];
                double xq[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    jq[u] = -1;
                    if (left) { jq[u] = lo_[k] + __ffsll((long long)left) - 1; left &= left - 1; }
                }
                int cq[4];
                double aq[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    cq[u] = jq[u] >= 0 ? __ldg(p.Ai + jq[u]) : 0;
                    aq[u] = jq[u] >= 0 ? __ldg(p.Ax + jq[u]) : 0.0;
                }
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    xq[u] = jq[u] >= 0 ? ld_relaxed_f64(p.x + cq[u]) : 0.0;
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (jq[u] >= 0 && !is_pending(xq[u])) {
                        acc = fma(-aq[u], xq[u], acc);
                        mask &= ~(1ull << (jq[u] - lo_[k]));
                    }
            }
            dlt_[k] = acc;
            acc_[k] += acc;   // (blocks without a parked product start from the plain sums)
            pend_[k] = mask;
            any |= mask != 0;
        }
        return any;
    };
    bool left_over = !failed && sweep();
    if (failed) { for (int k = 0; k < kChainRowsPerThread; ++k) dlt_[k] = 0.0; }
    int state_[kPairsPerWarp];
#pragma unroll
    for (int kk = 0; kk < kPairsPerWarp; ++kk) {
        const int pr = warp + 8 * kk;
        const int base = pr * 64;
        int state = 0;
        if (formed_[kk] && __all_sync(kFullMask, !failed)) {
            add_columns(wsc + (long long)pr * kPairDoubles + lane, dlt_[2 * kk], dlt_[2 * kk + 1],
                        ytop_[kk], ybot_[kk]);
            const bool late = __any_sync(kFullMask, (pend_[2 * kk] | pend_[2 * kk + 1]) != 0);
            if (late || (s_width[2 * pr] | s_width[2 * pr + 1]) != 0) {
                sacc[base + lane] = ytop_[kk];
                sacc[base + 32 + lane] = ybot_[kk];
                state = 2;
            } else {
                sy[base + lane] = publishable(ytop_[kk]);
                sy[base + 32 + lane] = publishable(ybot_[kk]);
                state = 1;
            }
        }
        state_[kk] = state;
        if (lane == 0 && pr < kChainPairs) s_early[pr] = state;
    }
    // What is still pending now (operands in the chunks just before this one) is left to the
    // helper warp of the row's block: waiting for it here would hold back the main warps, whose
    // first blocks rarely depend on it.
    (void)left_over;
#pragma unroll
    for (int k = 0; k < kChainRowsPerThread; ++k) {
        const int local = half_of(k) * 32 + lane;
        if (local < rows_here && state_[k >> 1] == 0) sacc[local] = acc_[k];
        spend[local] = local < rows_here ? pend_[k] : 0ull;
    }
    if (failed) *failed_flag = 1;
    workers_barrier();
    volatile double *sxv = sx;
    volatile double *syv = sy;

    if (warp == kChainThreads / 32 - 1) {
        // ---- loader warp (one lane): keeps the ring of T tiles full and announces, in order,
        // the stages that have landed (the consumers then read one counter instead of waiting
        // on a barrier per stage, which costs them about 150 cycles per block)
        if (lane != 0) return;
        int retired = 0;
        unsigned idle = 0;
        bool stop = false;
        const unsigned long long give_up = global_timer() + p.budget_ns;
        while (retired < issued || (issued < npair && !stop)) {
            bool progressed = false;
            if (!stop && issued < npair) {
                const int s = issued % kChainStages;
                if (issued < kChainStages ||
                    mbar_test_wait(&s_empty[s], ((issued / kChainStages) - 1) & 1)) {
                    mbar_expect_tx(&s_full[s], kStageBytes);
                    bulk_load(ring + s * kStageDoubles, wsc + (long long)issued * kPairDoubles + kPairT,
                              kStageBytes, &s_full[s]);
                    ++issued;
                    progressed = true;
                }
            }
            if (retired < issued &&
                mbar_test_wait(&s_full[retired % kChainStages], (retired / kChainStages) & 1)) {
                ++retired;
                st_release_shared(&s_tiles, retired);
                progressed = true;
            }
            if (progressed) {
                idle = 0;
            } else if ((++idle & 255u) == 0) {
                // after an error nothing more is requested, but no copy may still be in flight
                // when the block's shared memory is released: what was requested is awaited
                if (*failed_flag || aborted(p.status)) stop = true;
                if (global_timer() > give_up) break;
            }
        }
        return;
    }

    if (warp < kChainMain) {
        // ---- main warps: x_B = y_B - T_B x_B-1, four warps to a 64 x 64 block -------------
        // Warp (half, side): rows half * 32 + lane of the block against columns side * 32 ..
        // of the previous block.  The side-0 warp hands its partial sums to the side-1 warp of
        // the same rows, which adds y, publishes x_B (shared memory, the next chunk's halo,
        // global memory) and then all four meet before the next block.  The loops always run
        // to the end and always perform their barrier operations; after a failed wait they
        // only publish NaN.
        // Trace layout (64-bit words, C = number of chunks): [0, n) cycle counter at each row's
        // publication; [2n, 2n + C) cycle counter at the main warps' start; 2n + C + 4 chunk + k:
        // timer (ns) at main start, halo complete, first and last publication; 2n + 5C +
        // 8 chunk + k: cycles waited for y of blocks with and without operands inside the chunk, their sum, bit mask of the blocks that waited,
        // cycles at the partial-sum barrier, in the mat-vec, at the step barrier, from the
        // partial-sum barrier to the publication; 2n + 13C + 16 chunk + B: cycle counter when a
        // helper published y_B.
        const int half = warp & 1, side = warp >> 1;
        const double nanv = __longlong_as_double(kCanonicalNaN);
        const double2 *w = reinterpret_cast<const double2 *>(ring) + (half * 2 + side) * (kTileDoubles / 2) + lane;
        const double2 *xa = reinterpret_cast<const double2 *>(sxh + side * 32);
        bool dead = *failed_flag != 0;
        if (side == 0) {
            int tiles = 0;   // stages known to have landed
            // These warps also make sure, while they wait for the other two to publish, that the
            // next block's tiles have landed: the barrier hands that knowledge on, and the
            // finishing warps (whose every instruction is on the critical path) never look.
            auto await_stage = [&](const int B) {
                if (!dead && tiles <= B && B < npair)
                    dead = !warp_wait([&] { return (tiles = ld_acquire_shared(&s_tiles)) > B; }, dl,
                                      failed_flag, p.status, row0 + B * 64);
            };
            await_stage(0);
            step_sync();                                   // the halo is there
            for (int B = 0; B < npair; ++B) {
                const int s = B % kChainStages;
                const double part = tile_matvec(w + s * (kStageDoubles / 2), xa, 0.0);
                s_z[half][lane] = dead ? nanv : part;      // a failure travels as NaN
                __syncwarp();
                pair_arrive(kBarZ0 + half);
                xa += 32;
                await_stage(B + 1);
                step_sync();                               // x_B is there, the stage is free
                if (half == 0) mbar_arrive_lane0(&s_empty[s], lane);
            }
            if (dead && lane == 0) *failed_flag = 1;
            return;
        }
        const bool tracer = TRACE && half == 0 && lane == 0;
        const long long n_chunks = (p.n + kChainRows - 1) / kChainRows;
        long long *chunk_times = TRACE ? p.trace + 2ll * p.n + n_chunks + 4ll * chunk : nullptr;
        if (tracer) { p.trace[2ll * p.n + chunk] = clock64(); chunk_times[0] = (long long)global_timer(); }
        {
            // this warp's half of the block before the chunk
            const int t = row0 - kChainHalo + half * 32 + lane;
            double v = 0.0;
            if (row0 > 0 && !dead) {   // (a chunk after the first has a whole block before it)
                const int r = upper ? p.n - 1 - t : t;
                if (crank > 0) {       // the previous chunk's block stores it into this halo
                    volatile double *mine = sxh + half * 32 + lane;
                    dead = !warp_wait([&] { return !is_pending(v = *mine); }, dl, failed_flag, p.status, r);
                } else {
                    dead = !warp_wait([&] { return !is_pending(v = ld_relaxed_f64(p.x + r)); }, dl,
                                      failed_flag, p.status, r);
                }
            }
            sxh[half * 32 + lane] = v;
        }
        step_sync();
        if (tracer) chunk_times[1] = (long long)global_timer();
        // Every instruction of this loop is on the critical path of the whole solve (a lone
        // warp issues one about every four cycles), so it carries nothing it can do without.
        int local = half * 32 + lane;
        double ynext = dead ? nanv : syv[local];
        bool ylate = __any_sync(kFullMask, is_pending(ynext));
        const int step = upper ? -64 : 64;
        double *xout = p.x + (upper ? p.n - 1 - (row0 + local) : row0 + local);
        const bool push = crank + 1 < csize && row0 + kChainRows < q.row_end;   // (then the chunk is full)
        const unsigned next_halo = push ? cluster_map(sxh, crank + 1) + (half * 32 + lane) * 8 : 0u;
        long long y_wait_ = 0, y_listed_ = 0, y_far_ = 0, z_wait_ = 0, mv_ = 0, ss_ = 0, pub_ = 0; int y_waits_ = 0;
        auto step_block = [&](const int B, auto pushing) {
            constexpr bool kPush = decltype(pushing)::value;
            const int s = B % kChainStages;
            double y = ynext;
            if (!dead && ylate) {
                long long c0_ = TRACE ? clock64() : 0;
                dead = !warp_wait([&] { return !is_pending(y = syv[local]); }, dl, failed_flag,
                                  p.status, row0 + local);
                if (TRACE) { const long long w_ = clock64() - c0_; y_wait_ += w_; y_waits_ |= 1 << B; if ((s_width[2 * B] | s_width[2 * B + 1]) != 0) y_listed_ += w_; else y_far_ += w_; }
                if (dead) y = nanv;
            }
            ynext = syv[local + 64];   // (one block of slack behind sy keeps this in bounds)
            long long m0_ = 0, m1_ = 0;
            if (TRACE) asm volatile("mov.u64 %0, %%clock64;" : "=l"(m0_) : "d"(y) : "memory");
            const double sum = tile_matvec(w + s * (kStageDoubles / 2), xa, y);
            if (TRACE) { asm volatile("mov.u64 %0, %%clock64;" : "=l"(m1_) : "d"(sum) : "memory"); mv_ += m1_ - m0_; }
            long long z0_ = TRACE ? clock64() : 0;
            pair_sync(kBarZ0 + half);                      // the other 32 columns' partial sums
            if (TRACE) z_wait_ += clock64() - z0_;
            // (a sum is never the reserved all-ones pattern: arithmetic returns the canonical NaN)
            const double val = sum + s_z[half][lane];
            sxv[local] = val;       // (rows past the end: their T rows and y are zero, so is val)
            if (kPush) st_cluster_f64(next_halo, val);     // the next chunk's halo
            ylate = __any_sync(kFullMask, is_pending(ynext));   // (decided here, where the warp waits anyway)
            if (local < rows_here) {
                st_relaxed_f64(xout, val);
                if (TRACE) { p.trace[row0 + local] = clock64(); if (tracer && (B == 0 || B == npair - 1)) chunk_times[B == 0 ? 2 : 3] = (long long)global_timer(); }
            }
            long long s0_ = TRACE ? clock64() : 0;
            if (TRACE) pub_ += s0_ - z0_;
            step_sync();                                   // "x_B is there"
            if (TRACE) ss_ += clock64() - s0_;
            xout += step;
            xa += 32;
            local += 64;
        };
        const int plain = push ? npair - 1 : npair;   // the last block also feeds the neighbour
        for (int B = 0; B < plain; ++B) step_block(B, std::false_type());
        if (push) step_block(npair - 1, std::true_type());
        if (tracer) {
            long long *o = p.trace + 2ll * p.n + 5 * n_chunks + 8ll * chunk;
            o[0] = y_listed_; o[1] = y_far_; o[2] = y_wait_; o[3] = y_waits_; o[4] = z_wait_; o[5] = mv_; o[6] = ss_; o[7] = pub_;
        }
        if (dead && lane == 0) *failed_flag = 1;
        if (half == 0 && lane == 0) atomicAdd(&p.status[kStatusDone], 1);
        return;
    }

    // ---- helper warps: y_B for the blocks B = warp - 4, warp - 4 + 3, ... that phase A left --
    // Parked products (state 2): y_B was formed in phase A without a few operands.  A late
    // operand delta_i of row i adds delta_i times column i of M.
    auto finish_parked = [&](const int pr, const double d0, const double d1) {
        const double *m11 = wsc + (long long)pr * kPairDoubles + lane;
        double ytop = sacc[pr * 64 + lane], ybot = sacc[pr * 64 + 32 + lane];
        add_columns(m11, d0, d1, ytop, ybot);
        syv[pr * 64 + lane] = publishable(ytop);
        syv[pr * 64 + 32 + lane] = publishable(ybot);
        if (TRACE && lane == 0) p.trace[2ll * p.n + 13ll * ((p.n + kChainRows - 1) / kChainRows) + 16ll * chunk + pr] = clock64();
    };
    // the columns of M that row `lane` of half h will need, towards L1
    auto prefetch_columns = [&](const int pr, const int h) {
        const double *col = wsc + (long long)pr * kPairDoubles + (h ? 2 * kTileDoubles : 0) + lane * 32;
        chain_prefetch_l1(col);
        chain_prefetch_l1(col + 16);
        if (!h) { chain_prefetch_l1(col + kTileDoubles); chain_prefetch_l1(col + kTileDoubles + 16); }
    };
    {
        // Operands from the chunks just before: all of this warp's parked blocks are polled in
        // turn, one load per row and pass, all loads of a pass in flight together, so that an
        // operand is picked up about one round trip after the chunk before publishes it.
        // Blocks without operands inside the chunk are finished as soon as they are complete;
        // the others follow in order, each once its operands inside the chunk are there.
        constexpr int kMine = (kChainPairs + kChainHelpers - 1) / kChainHelpers;
        const int first = warp - kChainMain;
        unsigned long long mask[kMine][2];
        double delta[kMine][2];
        int lo[kMine][2];
        unsigned remaining = 0, listed = 0;
#pragma unroll
        for (int i = 0; i < kMine; ++i) {
            const int pr = first + i * kChainHelpers;
            const bool parked = pr < npair && s_early[pr] == 2;
            if (parked) remaining |= 1u << i;
            if (parked && (s_width[2 * pr] | s_width[2 * pr + 1]) != 0) listed |= 1u << i;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                mask[i][h] = 0ull;
                delta[i][h] = 0.0;
                lo[i][h] = 0;
                if (!parked) continue;
                const int local = pr * 64 + h * 32 + lane;
                mask[i][h] = spend[local];
                // (rows with an operand inside the chunk have their list's first entry filled)
                const bool in_chunk = s_width[2 * pr + h] != 0 && ecol[s_bptr[2 * pr + h] + lane] != kChainRows;
                if (mask[i][h]) {
                    const int r = upper ? p.n - 1 - (row0 + local) : row0 + local;
                    int hi = 0, d = -1;
                    csr_row_range(p, r, lo[i][h], hi, d);
                }
                if (mask[i][h] || in_chunk) prefetch_columns(pr, h);
            }
        }
        // Blocks that only wait for operands from the chunks before: where at most two rows per
        // half do, their columns of M are loaded now, so that the last operand's arrival is
        // followed by shuffles and multiply-adds only.
        int wt[kMine][2], wb[kMine][2];
        double wa[kMine][2], wc[kMine][2], wd[kMine][2];
        unsigned quick = 0;
#pragma unroll
        for (int i = 0; i < kMine; ++i) {
            const int pr = first + i * kChainHelpers;
            unsigned top = __ballot_sync(kFullMask, mask[i][0] != 0), bot = __ballot_sync(kFullMask, mask[i][1] != 0);
            const bool few = (remaining >> i & 1u) && !(listed >> i & 1u) && __popc(top) <= 2 && __popc(bot) <= 2;
            if (few) quick |= 1u << i;
            const double *m11 = wsc + (long long)pr * kPairDoubles + lane;
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                wt[i][u] = wb[i][u] = -1;
                wa[i][u] = wc[i][u] = wd[i][u] = 0.0;
                if (few && top) { wt[i][u] = __ffs(top) - 1; top &= top - 1; }
                if (few && bot) { wb[i][u] = __ffs(bot) - 1; bot &= bot - 1; }
                if (wt[i][u] >= 0) { wa[i][u] = __ldg(m11 + wt[i][u] * 32); wc[i][u] = __ldg(m11 + kTileDoubles + wt[i][u] * 32); }
                if (wb[i][u] >= 0) wd[i][u] = __ldg(m11 + 2 * kTileDoubles + wb[i][u] * 32);
            }
        }
        // (column and coefficient of the operand a row is waiting for stay in registers: a
        // pass then costs one round trip to L2, not two)
        int col[kMine][2];
        double coef[kMine][2];
        auto next_operand = [&](const int i, const int h) {
            col[i][h] = -1;
            coef[i][h] = 0.0;
            if (mask[i][h]) {
                const int at = lo[i][h] + __ffsll((long long)mask[i][h]) - 1;
                col[i][h] = __ldg(p.Ai + at);
                coef[i][h] = __ldg(p.Ax + at);
            }
        };
#pragma unroll
        for (int i = 0; i < kMine; ++i) { next_operand(i, 0); next_operand(i, 1); }
        unsigned polls = 0;
        while (remaining) {
            double xv[kMine][2];
#pragma unroll
            for (int i = 0; i < kMine; ++i)
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    xv[i][h] = col[i][h] >= 0 ? ld_relaxed_f64(p.x + col[i][h])
                                              : __longlong_as_double((long long)kPendingBits);
#pragma unroll
            for (int i = 0; i < kMine; ++i) {
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    if (!is_pending(xv[i][h])) {
                        delta[i][h] = fma(-coef[i][h], xv[i][h], delta[i][h]);
                        mask[i][h] &= mask[i][h] - 1;
                        next_operand(i, h);
                    }
                if (!(remaining >> i & 1u)) continue;
                if (!__all_sync(kFullMask, (mask[i][0] | mask[i][1]) == 0)) continue;
                if (quick >> i & 1u) {
                    const int pr = first + i * kChainHelpers;
                    double ytop = sacc[pr * 64 + lane], ybot = sacc[pr * 64 + 32 + lane];
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        if (wt[i][u] >= 0) {             // (warp-uniform)
                            const double dt = __shfl_sync(kFullMask, delta[i][0], wt[i][u]);
                            ytop = fma(wa[i][u], dt, ytop);
                            ybot = fma(wc[i][u], dt, ybot);
                        }
                        if (wb[i][u] >= 0)
                            ybot = fma(wd[i][u], __shfl_sync(kFullMask, delta[i][1], wb[i][u]), ybot);
                    }
                    syv[pr * 64 + lane] = publishable(ytop);
                    syv[pr * 64 + 32 + lane] = publishable(ybot);
                    if (TRACE && lane == 0) p.trace[2ll * p.n + 13ll * ((p.n + kChainRows - 1) / kChainRows) + 16ll * chunk + pr] = clock64();
                } else if (!(listed >> i & 1u)) {
                    finish_parked(first + i * kChainHelpers, delta[i][0], delta[i][1]);
                }
                remaining &= ~(1u << i);
            }
            if (remaining && (++polls & 15u) == 0 &&
                __any_sync(kFullMask, *failed_flag != 0 || dl.tick(p.status, row0))) {
                if (lane == 0) *failed_flag = 1;
                return;
            }
        }
#pragma unroll
        for (int i = 0; i < kMine; ++i) {
            if (!(listed >> i & 1u)) continue;
            const int pr = first + i * kChainHelpers;
            bool bad = false;
            // Which rows can end up with a correction is known before the operands are: rows
            // with an entry in the list, and rows that already have one from the chunks before.
            // Their columns of M are loaded now, while the warp waits, so that what follows the
            // arrival of the last operand is shuffles and multiply-adds only (the block two
            // blocks ahead of an operand has one step of the main warps to get its y out).
            const double *m11 = wsc + (long long)pr * kPairDoubles + lane;
            unsigned top = __ballot_sync(kFullMask, delta[i][0] != 0.0 ||
                (s_width[2 * pr] != 0 && ecol[s_bptr[2 * pr] + lane] != kChainRows));
            unsigned bot = __ballot_sync(kFullMask, delta[i][1] != 0.0 ||
                (s_width[2 * pr + 1] != 0 && ecol[s_bptr[2 * pr + 1] + lane] != kChainRows));
            const bool few = __popc(top) <= 4 && __popc(bot) <= 4;
            int ct[4], cb[4];
            double at[4], bt[4], bb[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                ct[u] = cb[u] = -1;
                at[u] = bt[u] = bb[u] = 0.0;
                if (few && top) { ct[u] = __ffs(top) - 1; top &= top - 1; }
                if (few && bot) { cb[u] = __ffs(bot) - 1; bot &= bot - 1; }
                if (ct[u] >= 0) { at[u] = __ldg(m11 + ct[u] * 32); bt[u] = __ldg(m11 + kTileDoubles + ct[u] * 32); }
                if (cb[u] >= 0) bb[u] = __ldg(m11 + 2 * kTileDoubles + cb[u] * 32);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int blk = 2 * pr + h;
                const int width = s_width[blk];
                int pos = s_bptr[blk] + lane;
                double t0 = delta[i][h], t1 = 0.0;
                for (int j = 0; j < width && !bad; j += 2, pos += 64) {
                    const int c0 = ecol[pos], c1 = ecol[pos + 32];
                    const double e0 = eval[pos], e1 = eval[pos + 32];
                    double x0 = 0.0, x1 = 0.0;
                    bad = !warp_wait([&] {
                        x0 = sxv[c0];
                        x1 = sxv[c1];
                        return !is_pending(x0) && !is_pending(x1);
                    }, dl, failed_flag, p.status, row0 + pr * 64);
                    t0 = fma(-e0, x0, t0);
                    t1 = fma(-e1, x1, t1);
                }
                delta[i][h] = t0 + t1;
            }
            if (bad) {
                if (lane == 0) *failed_flag = 1;
                return;
            }
            if (!few) {
                finish_parked(pr, delta[i][0], delta[i][1]);
                continue;
            }
            double ytop = sacc[pr * 64 + lane], ybot = sacc[pr * 64 + 32 + lane];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (ct[u] >= 0) {                // (warp-uniform)
                    const double dt = __shfl_sync(kFullMask, delta[i][0], ct[u]);
                    ytop = fma(at[u], dt, ytop);
                    ybot = fma(bt[u], dt, ybot);
                }
                if (cb[u] >= 0) ybot = fma(bb[u], __shfl_sync(kFullMask, delta[i][1], cb[u]), ybot);
            }
            syv[pr * 64 + lane] = publishable(ytop);
            syv[pr * 64 + 32 + lane] = publishable(ybot);
            if (TRACE && lane == 0) p.trace[2ll * p.n + 13ll * ((p.n + kChainRows - 1) / kChainRows) + 16ll * chunk + pr] = clock64();
        }
    }
    // Then the blocks without a parked product (their operand list did not fit), in order.
    for (int pr = warp - kChainMain; pr < npair; pr += kChainHelpers) {
        if (s_early[pr]) continue;
        bool bad = __any_sync(kFullMask, *failed_flag != 0);   // (kept warp-uniform throughout)
        const double *m11 = wsc + (long long)pr * kPairDoubles + lane;
        double t[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int blk = 2 * pr + h;
            const int local = blk * 32 + lane;
            const bool active = local < rows_here;
            const int r = upper ? p.n - 1 - (row0 + local) : row0 + local;
            double t0 = active ? sacc[local] : 0.0, t1 = 0.0;
            unsigned long long mask = spend[local];
            if (!bad && __any_sync(kFullMask, mask != 0)) {
                // operands from before the chunk that had not been produced when phase A looked
                int lo = 0, hi = 0, d = -1;
                if (mask) csr_row_range(p, r, lo, hi, d);
                bad = !warp_wait([&] {
                    unsigned long long left = mask;
                    for (int u = 0; u < 4 && left; ++u) {
                        const int bit = __ffsll((long long)left) - 1;
                        left &= left - 1;
                        const double xv = ld_relaxed_f64(p.x + __ldg(p.Ai + lo + bit));
                        if (!is_pending(xv)) {
                            t0 = fma(-__ldg(p.Ax + lo + bit), xv, t0);
                            mask &= ~(1ull << bit);
                        }
                    }
                    return mask == 0;
                }, dl, failed_flag, p.status, r);
            }
            if (!overflow) {
                const int width = s_width[blk];
                int pos = s_bptr[blk] + lane;
                for (int j = 0; j < width && !bad; j += 2, pos += 64) {
                    const int c0 = ecol[pos], c1 = ecol[pos + 32];
                    const double e0 = eval[pos], e1 = eval[pos + 32];
                    double x0 = 0.0, x1 = 0.0;
                    bad = !warp_wait([&] {
                        x0 = sxv[c0];
                        x1 = sxv[c1];
                        return !is_pending(x0) && !is_pending(x1);
                    }, dl, failed_flag, p.status, row0 + pr * 64);
                    t0 = fma(-e0, x0, t0);
                    t1 = fma(-e1, x1, t1);
                }
            } else if (active) {
                // the strips did not fit: read the operands from the matrix again
                int lo = 0, hi = 0, d = -1;
                csr_row_range(p, r, lo, hi, d);
                for (int j = lo; j < hi && !bad; ++j) {
                    const int c = __ldg(p.Ai + j);
                    if ((unsigned)c >= (unsigned)p.n) continue;
                    const int cl = (upper ? p.n - 1 - c : c) - row0;
                    if (cl < 0 || cl >= pr * 64 - 64) continue;
                    double xv = 0.0;
                    while (is_pending(xv = sxv[cl]))
                        if (*failed_flag || dl.tick(p.status, r)) { bad = true; break; }
                    t0 = fma(-__ldg(p.Ax + j), xv, t0);
                }
            }
            bad = __any_sync(kFullMask, bad);
            t[h] = t0 + t1;
        }
        if (bad) {
            if (lane == 0) *failed_flag = 1;
            return;
        }
        double ytop = 0.0, ybot = 0.0;
        apply_inverse(m11, t[0], t[1], ytop, ybot);
        syv[pr * 64 + lane] = publishable(ytop);
        syv[pr * 64 + 32 + lane] = publishable(ybot);
    }
    };
    body();
    if (csize > 1) cluster_barrier();
}

static size_t chain_smem_bytes(int *cap_out) {
    const size_t limit = 227 * 1024 - 2048;  // static shared memory takes about 1.2 KB
    const size_t fixed = (size_t)kChainStages * kStageDoubles * 8 +
                         ((size_t)kChainHalo + kChainRows + 2 + 3 * kChainRows + 64) * 8;
    const size_t cap = ((limit - fixed) / 12) & ~(size_t)1;
    *cap_out = (int)cap;
    return fixed + cap * 12;
}

}  // namespace lcd

using namespace lcd;

static int g_last_cluster = 0;
static int g_cluster_limit = 0;   // 0: as many as the device hosts

namespace lcd {
int set_chain_cluster_limit(int blocks) {
    if (blocks != 0 && blocks != 1 && blocks != 2 && blocks != 4 && blocks != 8)
        return LCD_ERR_INVALID_ARGUMENT;
    g_cluster_limit = blocks;
    return LCD_OK;
}
}  // namespace lcd

extern "C" int lcd_chain_cluster_size(void) { return g_last_cluster; }

extern "C" int lcd_chain_workspace_bytes(int32_t n, int64_t *bytes) {
    if (n < 0 || !bytes) return LCD_ERR_INVALID_ARGUMENT;
    *bytes = ((int64_t)n + 63) / 64 * kPairDoubles * 8 + 256;
    return LCD_OK;
}

static int chain_check(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                       const double *Ax, const int32_t *diag_pos, int flags, const void *workspace,
                       int64_t workspace_bytes) {
    if (n < 0 || nnz < 0 || (n > 0 && (!Ap || !Ai || !Ax || !workspace)))
        return LCD_ERR_INVALID_ARGUMENT;
    if ((flags & LCD_SOLVE_OF_FULL) && !diag_pos) return LCD_ERR_INVALID_ARGUMENT;
    if ((flags & LCD_SOLVE_UNIT_DIAG) && !(flags & LCD_SOLVE_OF_FULL)) return LCD_ERR_INVALID_ARGUMENT;
    int64_t need = 0;
    lcd_chain_workspace_bytes(n, &need);
    if (workspace_bytes < need) return LCD_ERR_WORKSPACE;
    // the tiles are fetched with bulk copies, which need 16-byte aligned addresses
    if (reinterpret_cast<uintptr_t>(workspace) & 15) return LCD_ERR_INVALID_ARGUMENT;
    return LCD_OK;
}

static bool chain_range_ok(int32_t n, int32_t row_begin, int32_t row_end, int granule) {
    return row_begin >= 0 && row_begin <= row_end && row_end <= n && row_begin % granule == 0 &&
           (row_end % granule == 0 || row_end == n);
}

extern "C" int lcd_chain_prepare_rows(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                                      const double *Ax, const int32_t *diag_pos, int flags,
                                      void *workspace, int64_t workspace_bytes, int32_t row_begin,
                                      int32_t row_end, void *stream) {
    int rc = chain_check(n, nnz, Ap, Ai, Ax, diag_pos, flags, workspace, workspace_bytes);
    if (rc) return rc;
    if (!chain_range_ok(n, row_begin, row_end, 64)) return LCD_ERR_INVALID_ARGUMENT;
    if (row_begin == row_end) return LCD_OK;
    const int pair_begin = row_begin / 64, pair_end = (row_end + 63) / 64;
    CsrSolveParams p{n, nnz, Ap, Ai, Ax, diag_pos, nullptr, nullptr, flags, 1, 1, nullptr,
                     0, nullptr, 0, n, nullptr, {nullptr}};
    // the attribute belongs to the current device's copy of the function
    LCD_CUDA_TRY(cudaFuncSetAttribute(chain_prepare_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      kPrepSmemBytes));
    if (row_begin == 0)   // the growth word behind the tiles restarts with the first range
        LCD_CUDA_TRY(cudaMemsetAsync(static_cast<double *>(workspace) + ((int64_t)n + 63) / 64 * kPairDoubles,
                                     0, sizeof(double), (cudaStream_t)stream));
    chain_prepare_kernel<<<pair_end - pair_begin, kPrepThreads, kPrepSmemBytes, (cudaStream_t)stream>>>(
        p, static_cast<double *>(workspace), pair_begin, pair_end);
    LCD_CUDA_TRY(cudaGetLastError());
    return LCD_OK;
}

extern "C" int lcd_chain_growth(int32_t n, const void *workspace, int64_t workspace_bytes, void *stream,
                                double *growth_host) {
    if (n < 0 || !workspace || !growth_host) return LCD_ERR_INVALID_ARGUMENT;
    int64_t need = 0;
    lcd_chain_workspace_bytes(n, &need);
    if (workspace_bytes < need) return LCD_ERR_WORKSPACE;
    LCD_CUDA_TRY(cudaMemcpyAsync(growth_host,
                                 static_cast<const double *>(workspace) + ((int64_t)n + 63) / 64 * kPairDoubles,
                                 sizeof(double), cudaMemcpyDeviceToHost, (cudaStream_t)stream));
    LCD_CUDA_TRY(cudaStreamSynchronize((cudaStream_t)stream));
    return LCD_OK;
}

extern "C" int lcd_chain_prepare(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                                 const double *Ax, const int32_t *diag_pos, int flags,
                                 void *workspace, int64_t workspace_bytes, void *stream) {
    return lcd_chain_prepare_rows(n, nnz, Ap, Ai, Ax, diag_pos, flags, workspace, workspace_bytes, 0, n,
                                  stream);
}

extern "C" int lcd_sptrsv_csr_chain_rows(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                                         const double *Ax, const int32_t *diag_pos, const double *b,
                                         double *x, int flags, const void *workspace,
                                         int64_t workspace_bytes, int32_t row_begin, int32_t row_end,
                                         int32_t *status_dev, int32_t timeout_ms, void *stream,
                                         int *status_host) {
    if (!status_dev) return LCD_ERR_INVALID_ARGUMENT;
    int rc = chain_check(n, nnz, Ap, Ai, Ax, diag_pos, flags, workspace, workspace_bytes);
    if (rc) return rc;
    if (n > 0 && (!b || !x || x == b)) return LCD_ERR_INVALID_ARGUMENT;
    if (!chain_range_ok(n, row_begin, row_end, kChainRows)) return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    if (row_begin == 0) {
        // the first range of a solve: error state, ticket and chunk counters start from zero and
        // the whole of x becomes "not produced yet"
        rc = reset_status(status_dev, st);
        if (rc) return rc;
        if (n > 0) LCD_CUDA_TRY(cudaMemsetAsync(x, 0xFF, (size_t)n * sizeof(double), st));
    } else {
        // a later range: the tickets restart, the count of finished chunks and a raised error stay
        LCD_CUDA_TRY(cudaMemsetAsync(status_dev + kStatusTicket, 0, sizeof(int32_t), st));
    }
    if (row_end > row_begin) {
        ChainParams q;
        q.m = CsrSolveParams{n, nnz, Ap, Ai, Ax, diag_pos, b, x, flags & ~LCD_SOLVE_EXACT, 1, 1,
                             status_dev, timeout_ns(timeout_ms), debug_trace(), 0, n, nullptr, {nullptr}};
        q.ws = static_cast<const double *>(workspace);
        q.chunk_begin = row_begin / kChainRows;
        q.row_end = row_end;
        q.gate_far = kChainGateFar;
        q.gate = kChainGate;
        const size_t smem = chain_smem_bytes(&q.cap);
        // the attribute belongs to the current device's copy of the function
        auto kernel = q.m.trace ? csr_chain_kernel<true> : csr_chain_kernel<false>;
        LCD_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        const int chunks = (row_end - row_begin + kChainRows - 1) / kChainRows;
        // clusters of up to eight blocks (consecutive chunks hand over through shared memory);
        // where the device cannot host such a cluster the same kernel runs as plain blocks
        int cluster = 1;
        const int wanted = g_cluster_limit ? g_cluster_limit : kChainCluster;
        for (int size = wanted; size > 1 && chunks > 1 && cluster == 1; size >>= 1) {
            cudaLaunchConfig_t probe = {};
            probe.gridDim = dim3(size);
            probe.blockDim = dim3(kChainThreads);
            probe.dynamicSmemBytes = smem;
            cudaLaunchAttribute attr;
            attr.id = cudaLaunchAttributeClusterDimension;
            attr.val.clusterDim.x = size;
            attr.val.clusterDim.y = attr.val.clusterDim.z = 1;
            probe.attrs = &attr;
            probe.numAttrs = 1;
            int fit = 0;
            if (cudaOccupancyMaxActiveClusters(&fit, kernel, &probe) == cudaSuccess && fit > 0)
                cluster = size;
            else
                cudaGetLastError();
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((chunks + cluster - 1) / cluster * cluster);
        cfg.blockDim = dim3(kChainThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = cluster;
        attr.val.clusterDim.y = attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        g_last_cluster = cluster;
        LCD_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, q));
        LCD_CUDA_TRY(cudaGetLastError());
    }
    if (row_end < n) return LCD_OK;       // more ranges follow: nothing is awaited
    return finish(status_dev, st, status_host);
}

extern "C" int lcd_sptrsv_csr_chain(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                                    const double *Ax, const int32_t *diag_pos, const double *b,
                                    double *x, int flags, const void *workspace,
                                    int64_t workspace_bytes, int32_t *status_dev,
                                    int32_t timeout_ms, void *stream, int *status_host) {
    return lcd_sptrsv_csr_chain_rows(n, nnz, Ap, Ai, Ax, diag_pos, b, x, flags, workspace,
                                     workspace_bytes, 0, n, status_dev, timeout_ms, stream, status_host);
}
