// Block-inverse chain solver: CSR triangular solves whose levels hold only a few rows.
//
// Such a matrix is one long dependence chain: level-by-level substitution pays one
// hand-off (a poll, a barrier, or a dozen dependent instructions of a lone warp) per
// level, and there are hundreds of thousands of levels.  The chain is shortened
// algebraically instead: rows are grouped into blocks of 32 consecutive rows, the
// 32 x 32 lower-triangular diagonal block D_b of every group is inverted once per
// matrix (lcd_chain_prepare, fully parallel, one warp per block), and the solve
// becomes a block forward substitution
//        x_b = D_b^{-1} ( b_b - sum_{c < b} L_bc x_c )
// in which the 5-6 levels inside a block collapse into one dense 32 x 32 mat-vec done
// with warp shuffles (no dependent chain: 32 independent shuffle/FMA pairs).
//
//   phase A (all threads of a block, several rows each): subtract the contributions of
//     rows before the chunk (polling x in global memory, rows of earlier tickets), copy
//     the operands that come from earlier 32-row blocks of the chunk into a compact
//     shared-memory list, leave partial sums in shared memory;
//   phase B (warp 0): walks the chunk block by block; lanes subtract their compact
//     operands (values of earlier blocks are final in shared memory, nothing to wait for),
//     then apply the inverse block from registers (loaded one block ahead) and publish.
//
// The result differs from plain substitution only by rounding (the inverse is applied
// instead of substituting inside the block); the relative residual stays at the 1e-16
// level for diagonally dominant blocks.  Callers that need the sequential order use the
// LCD_SOLVE_EXACT path of lcd_sptrsv_csr_syncfree instead.
#include "common.cuh"

namespace lcd {

constexpr int kChainThreads = 256;
constexpr int kChainRows = 1024;                       // rows per chunk
constexpr int kChainRowsPerThread = kChainRows / kChainThreads;
constexpr int kChainBlocks = kChainRows / 32;

// ---- numeric preparation: invert the 32 x 32 diagonal blocks ----------------------
constexpr int kInvWarps = 2;

__global__ void __launch_bounds__(kInvWarps * 32)
chain_block_inverse_kernel(const CsrSolveParams p, double *__restrict__ minv, int n_blocks) {
    __shared__ double D[kInvWarps][32][33];
    __shared__ double M[kInvWarps][32][33];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int blk = blockIdx.x * kInvWarps + warp;
    if (blk >= n_blocks) return;
    const bool upper = p.flags & LCD_SOLVE_UPPER;
    const int base = blk * 32;
    const int task = base + lane;
    for (int k = 0; k < 32; ++k) { D[warp][lane][k] = 0.0; M[warp][lane][k] = 0.0; }
    double diag = 1.0;  // rows past the end form an identity block
    if (task < p.n) {
        const int r = upper ? p.n - 1 - task : task;
        int lo = 0, hi = 0, d = -1;
        if (csr_row_range(p, r, lo, hi, d)) {
            if (d >= 0) diag = __ldg(p.Ax + d);
            for (int j = lo; j < hi; ++j) {
                const int c = __ldg(p.Ai + j);
                if ((unsigned)c >= (unsigned)p.n) continue;
                const int tc = upper ? p.n - 1 - c : c;
                if (tc >= base && tc < task) D[warp][lane][tc - base] += __ldg(p.Ax + j);
            }
        }
    }
    D[warp][lane][lane] = diag;
    __syncwarp();
    // lane c solves D m = e_c by forward substitution: column c of the inverse
    const int c = lane;
    for (int r = c; r < 32; ++r) {
        double s = (r == c) ? 1.0 : 0.0;
        for (int k = c; k < r; ++k) s = fma(-D[warp][r][k], M[warp][k][c], s);
        M[warp][r][c] = s / D[warp][r][r];
    }
    __syncwarp();
    // element (r, k) at k * 32 + r: the solver's lane r reads column after column coalesced
    double *out = minv + (long long)blk * 1024;
    for (int k = 0; k < 32; ++k) out[k * 32 + lane] = M[warp][lane][k];
}

// ---- the solve -------------------------------------------------------------------
struct ChainParams {
    CsrSolveParams m;
    const double *__restrict__ minv;
    int cap;  // capacity of the compact operand list (entries)
};

__device__ __forceinline__ int before_fill(const int *eptr, int local) { return eptr[local]; }

__device__ __forceinline__ void chain_prefetch_l2(const void *ptr) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr));
}

__global__ void __launch_bounds__(kChainThreads, 1)
csr_chain_kernel(const ChainParams q) {
    const CsrSolveParams &p = q.m;
    extern __shared__ __align__(16) unsigned char chain_smem[];
    double *sx = reinterpret_cast<double *>(chain_smem);      // x of the chunk
    double *sacc = sx + kChainRows + 2;                        // partial sums after phase A (sx has a zero slot)
    double *eval = sacc + kChainRows;                          // compact operands: values
    int *ecol = reinterpret_cast<int *>(eval + q.cap);         // ... and chunk-local columns
    int *eptr = ecol + q.cap;                                  // kChainRows + 1 offsets
    __shared__ int s_chunk;
    __shared__ int s_failed;
    __shared__ int s_warp_sums[kChainThreads / 32 + 1];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) { s_chunk = atomicAdd(&p.status[kStatusTicket], 1); s_failed = 0; }
    __syncthreads();
    const int row0 = s_chunk * kChainRows;
    const int rows_here = min(kChainRows, p.n - row0);
    if (rows_here <= 0) return;
    const bool upper = p.flags & LCD_SOLVE_UPPER;
    // pull this chunk's inverse blocks towards L2 while phase A waits on earlier chunks
    {
        const char *src = reinterpret_cast<const char *>(q.minv + (long long)(row0 / 32) * 1024);
        const long long bytes = (long long)((rows_here + 31) / 32) * 1024 * 8;
        for (long long off = (long long)tid * 128; off < bytes; off += (long long)kChainThreads * 128)
            chain_prefetch_l2(src + off);
    }

    // ---- phase A: thread t owns rows t, t + 256, t + 512, t + 768 of the chunk ---------
    // A1 (pattern only, nothing to wait for): count the operands that come from earlier
    // 32-row blocks of the chunk, lay the compact list out (every row padded to a multiple
    // of four entries that point at a zero slot) and fill it.
    int lo_[kChainRowsPerThread], hi_[kChainRowsPerThread], cnt_[kChainRowsPerThread];
    bool failed = false;
#pragma unroll
    for (int k = 0; k < kChainRowsPerThread; ++k) {
        const int local = tid + k * kChainThreads;
        lo_[k] = hi_[k] = cnt_[k] = 0;
        if (local >= rows_here) continue;
        const int task = row0 + local;
        const int r = upper ? p.n - 1 - task : task;
        const int base = local & ~31;  // first row of this row's 32-block, chunk-local
        int lo = 0, hi = 0, d = -1;
        if (!csr_row_range(p, r, lo, hi, d)) {
            raise_error(p.status, (p.flags & LCD_SOLVE_OF_FULL) ? LCD_ERR_MISSING_DIAGONAL
                                                               : LCD_ERR_BAD_POINTERS, r);
            failed = true;
            continue;
        }
        lo_[k] = lo;
        hi_[k] = hi;
        int externals = 0;
        for (int j = lo; j < hi; ++j) {
            const int c = __ldg(p.Ai + j);
            const int tc = ((unsigned)c < (unsigned)p.n) ? (upper ? p.n - 1 - c : c) : task;
            if (tc >= task) {  // not strictly before this row (or out of range)
                raise_error(p.status, LCD_ERR_INDEX_RANGE, r);
                failed = true;
                break;
            }
            const int cl = tc - row0;
            if (cl >= 0 && cl < base) ++externals;
        }
        cnt_[k] = (externals + 3) & ~3;
    }
    // exclusive scan of the padded counts in row order (rows are interleaved over threads,
    // so the four row groups are scanned one after another)
    int running = 0;
#pragma unroll
    for (int k = 0; k < kChainRowsPerThread; ++k) {
        int incl = cnt_[k];
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += t;
        }
        __syncthreads();
        if (lane == 31) s_warp_sums[warp] = incl;
        __syncthreads();
        int before = running;
        for (int w = 0; w < warp; ++w) before += s_warp_sums[w];
        int total = 0;
        for (int w = 0; w < kChainThreads / 32; ++w) total += s_warp_sums[w];
        eptr[tid + k * kChainThreads] = before + incl - cnt_[k];
        running += total;
    }
    if (tid == 0) { eptr[kChainRows] = running; sx[kChainRows] = 0.0; }  // zero slot for padding
    const bool overflow = running > q.cap;  // block-uniform
    if (!overflow) {
#pragma unroll
        for (int k = 0; k < kChainRowsPerThread; ++k) {
            const int local = tid + k * kChainThreads;
            if (local >= rows_here || cnt_[k] == 0) continue;
            const int task = row0 + local, base = local & ~31;
            int pos = before_fill(eptr, local);
            const int pos_end = pos + cnt_[k];
            for (int j = lo_[k]; j < hi_[k]; ++j) {
                const int c = __ldg(p.Ai + j);
                if ((unsigned)c >= (unsigned)p.n) continue;
                const int cl = (upper ? p.n - 1 - c : c) - row0;
                if (cl >= 0 && cl < base && cl + row0 < task) {
                    ecol[pos] = cl;
                    eval[pos] = __ldg(p.Ax + j);
                    ++pos;
                }
            }
            for (; pos < pos_end; ++pos) { ecol[pos] = kChainRows; eval[pos] = 0.0; }
        }
    }
    // A2: contributions of rows before the chunk (they belong to earlier tickets, so a
    // bounded spin is safe).  First every operand that is already there is consumed without
    // waiting; operands still pending are remembered in a bit mask and revisited afterwards,
    // so that when the previous chunk finishes only those few remain to be fetched.
    Deadline dl;
    dl.start(p.budget_ns);
    double acc_[kChainRowsPerThread];
    unsigned long long pend_[kChainRowsPerThread];
#pragma unroll
    for (int k = 0; k < kChainRowsPerThread; ++k) {
        const int local = tid + k * kChainThreads;
        acc_[k] = 0.0;
        pend_[k] = 0ull;
        if (local >= rows_here || failed) continue;
        const int r = upper ? p.n - 1 - (row0 + local) : row0 + local;
        double acc = __ldg(p.b + r);
        for (int j = lo_[k]; j < hi_[k] && !failed; ++j) {
            const int c = __ldg(p.Ai + j);
            const int tc = upper ? p.n - 1 - c : c;
            if (tc >= row0) continue;  // this chunk: compact list or inverse block
            double xv = ld_relaxed_f64(p.x + c);
            if (is_pending(xv)) {
                if (j - lo_[k] < 64) { pend_[k] |= 1ull << (j - lo_[k]); continue; }
                while (is_pending(xv = ld_relaxed_f64(p.x + c)))   // very long rows: wait here
                    if (dl.tick(p.status, r)) { failed = true; break; }
                if (failed) break;
            }
            acc = fma(-__ldg(p.Ax + j), xv, acc);
        }
        acc_[k] = acc;
    }
#pragma unroll
    for (int k = kChainRowsPerThread - 1; k >= 0; --k) {
        const int local = tid + k * kChainThreads;
        if (local >= rows_here) continue;
        const int r = upper ? p.n - 1 - (row0 + local) : row0 + local;
        double acc = acc_[k];
        unsigned long long mask = pend_[k];
        while (mask && !failed) {
            const int j = lo_[k] + __ffsll((long long)mask) - 1;
            mask &= mask - 1;
            const int c = __ldg(p.Ai + j);
            double xv;
            while (is_pending(xv = ld_relaxed_f64(p.x + c)))
                if (dl.tick(p.status, r)) { failed = true; break; }
            if (!failed) acc = fma(-__ldg(p.Ax + j), xv, acc);
        }
        sacc[local] = acc;
    }
    if (failed) s_failed = 1;
    __syncthreads();
    if (tid >= 32) return;

    // ---- phase B: warp 0 walks the chunk, one 32-row block per step ----------------------
    if (p.trace && lane == 0) p.trace[(long long)p.n + row0] = clock64();
    volatile double *sxv = sx;
    const bool chunk_failed = s_failed != 0;
    const double nanv = __longlong_as_double(kCanonicalNaN);
    const int n_blocks_here = (rows_here + 31) / 32;
    const double *mbase = q.minv + (long long)(row0 / 32) * 1024 + lane;
    double m[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) m[k] = __ldg(mbase + k * 32);
    for (int blk = 0; blk < n_blocks_here; ++blk) {
        const int base = blk * 32;
        const int local = base + lane;
        const bool active = local < rows_here;
        const int r = upper ? p.n - 1 - (row0 + local) : row0 + local;
        // the next block's inverse is requested now and consumed one step later
        double mnext[32];
        const bool more = blk + 1 < n_blocks_here;
#pragma unroll
        for (int k = 0; k < 32; ++k) mnext[k] = more ? __ldg(mbase + (long long)(blk + 1) * 1024 + k * 32) : 0.0;
        double acc = active ? sacc[local] : 0.0;
        if (chunk_failed) {
            if (active) { sxv[local] = nanv; st_relaxed_f64(p.x + r, nanv); }
            __syncwarp();
            continue;
        }
        if (active) {
            if (!overflow) {
                // every row's list is a multiple of four entries (padding reads a zero slot)
                int e = eptr[local];
                const int e_end = eptr[local + 1];
                double acc1 = 0.0, acc2 = 0.0, acc3 = 0.0;
                for (; e < e_end; e += 4) {
                    const int c0 = ecol[e], c1 = ecol[e + 1], c2 = ecol[e + 2], c3 = ecol[e + 3];
                    const double a0 = eval[e], a1 = eval[e + 1], a2 = eval[e + 2], a3 = eval[e + 3];
                    acc = fma(-a0, sxv[c0], acc);
                    acc1 = fma(-a1, sxv[c1], acc1);
                    acc2 = fma(-a2, sxv[c2], acc2);
                    acc3 = fma(-a3, sxv[c3], acc3);
                }
                acc += (acc1 + acc2) + acc3;
            } else {
                // the compact list did not fit: read the operands from the matrix again
                int lo = 0, hi = 0, d = -1;
                csr_row_range(p, r, lo, hi, d);
                for (int j = lo; j < hi; ++j) {
                    const int c = __ldg(p.Ai + j);
                    if ((unsigned)c >= (unsigned)p.n) continue;
                    const int cl = (upper ? p.n - 1 - c : c) - row0;
                    if (cl >= 0 && cl < base) acc = fma(-__ldg(p.Ax + j), sxv[cl], acc);
                }
            }
        }
        // x_block = inverse block * acc_block: 32 independent shuffle / FMA pairs
        double x0 = 0.0, x1 = 0.0, x2 = 0.0, x3 = 0.0;
#pragma unroll
        for (int k = 0; k < 32; k += 4) {
            x0 = fma(m[k + 0], __shfl_sync(0xffffffffu, acc, k + 0), x0);
            x1 = fma(m[k + 1], __shfl_sync(0xffffffffu, acc, k + 1), x1);
            x2 = fma(m[k + 2], __shfl_sync(0xffffffffu, acc, k + 2), x2);
            x3 = fma(m[k + 3], __shfl_sync(0xffffffffu, acc, k + 3), x3);
        }
        if (active) {
            const double val = publishable((x0 + x1) + (x2 + x3));
            sxv[local] = val;
            st_relaxed_f64(p.x + r, val);
            if (p.trace) p.trace[row0 + local] = clock64();
        }
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 32; ++k) m[k] = mnext[k];
    }
}

static size_t chain_smem_bytes(long long nnz, int n, int *cap_out) {
    const size_t limit = 227 * 1024 - 512;
    const size_t fixed = ((size_t)kChainRows * 2 + 2) * 8 + ((size_t)kChainRows + 2) * 4;
    const double avg = n > 0 ? (double)nnz / n : 0.0;
    long long cap = (long long)(avg * kChainRows * 0.75) + 4 * kChainRows;  // incl. padding
    const long long max_cap = ((long long)limit - (long long)fixed) / 12;
    if (cap > max_cap) cap = max_cap;
    cap &= ~1ll;
    *cap_out = (int)cap;
    return fixed + (size_t)cap * 12;
}

}  // namespace lcd

using namespace lcd;

extern "C" int lcd_chain_workspace_bytes(int32_t n, int64_t *bytes) {
    if (n < 0 || !bytes) return LCD_ERR_INVALID_ARGUMENT;
    *bytes = ((int64_t)n + 31) / 32 * 1024 * 8 + 256;
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
    if (reinterpret_cast<uintptr_t>(workspace) & 7) return LCD_ERR_INVALID_ARGUMENT;
    return LCD_OK;
}

extern "C" int lcd_chain_prepare(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                                 const double *Ax, const int32_t *diag_pos, int flags,
                                 void *workspace, int64_t workspace_bytes, void *stream) {
    int rc = chain_check(n, nnz, Ap, Ai, Ax, diag_pos, flags, workspace, workspace_bytes);
    if (rc || n == 0) return rc;
    const int n_blocks = (n + 31) / 32;
    CsrSolveParams p{n, nnz, Ap, Ai, Ax, diag_pos, nullptr, nullptr, flags, 1, 1, nullptr,
                     0, nullptr, 0, n, nullptr, {nullptr}};
    chain_block_inverse_kernel<<<(n_blocks + kInvWarps - 1) / kInvWarps, kInvWarps * 32, 0,
                                 (cudaStream_t)stream>>>(p, static_cast<double *>(workspace), n_blocks);
    LCD_CUDA_TRY(cudaGetLastError());
    return LCD_OK;
}

extern "C" int lcd_sptrsv_csr_chain(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                                    const double *Ax, const int32_t *diag_pos, const double *b,
                                    double *x, int flags, const void *workspace,
                                    int64_t workspace_bytes, int32_t *status_dev,
                                    int32_t timeout_ms, void *stream, int *status_host) {
    if (!status_dev) return LCD_ERR_INVALID_ARGUMENT;
    int rc = chain_check(n, nnz, Ap, Ai, Ax, diag_pos, flags, workspace, workspace_bytes);
    if (rc) return rc;
    if (n > 0 && (!b || !x || x == b)) return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    rc = reset_status(status_dev, st);
    if (rc) return rc;
    if (n > 0) {
        LCD_CUDA_TRY(cudaMemsetAsync(x, 0xFF, (size_t)n * sizeof(double), st));
        ChainParams q;
        q.m = CsrSolveParams{n, nnz, Ap, Ai, Ax, diag_pos, b, x, flags & ~LCD_SOLVE_EXACT, 1, 1,
                             status_dev, timeout_ns(timeout_ms), debug_trace(), 0, n, nullptr, {nullptr}};
        q.minv = static_cast<const double *>(workspace);
        const size_t smem = chain_smem_bytes(nnz, n, &q.cap);
        static bool configured = false;
        if (!configured) {
            LCD_CUDA_TRY(cudaFuncSetAttribute(csr_chain_kernel,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)(227 * 1024 - 512)));
            configured = true;
        }
        csr_chain_kernel<<<(n + kChainRows - 1) / kChainRows, kChainThreads, smem, st>>>(q);
        LCD_CUDA_TRY(cudaGetLastError());
    }
    return finish(status_dev, st, status_host);
}
