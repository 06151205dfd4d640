// On-device construction of the dependence DAG and its level sets (sm_100a).
//
// Output arrays are element-wise identical to what the reference's generated
// inspector plus dag_preprocessing produce:
//   1. every node counts and then emits the edge instances of its segment in
//      the order the inspector visits them                    (count / scan / emit)
//   2. edges are brought into (source, destination) order by stable LSD radix
//      passes over 8-bit digits                               (sort)
//   3. repeated edges are dropped, successors compacted       (flag / scan / compact)
//   4. the distinct edges are regrouped by destination        (sort) and levels are
//      propagated with a pull scheme that polls the predecessor's level word
//      itself (-1 = not known yet), own-chunk levels mirrored in shared memory
//   5. nodes are ordered by (level, id) with stable radix passes on the level.
// All primitives (scan, radix pass) are written here; nothing is allocated.
#include "common.cuh"

namespace lcd {

// ---------------------------------------------------------------- scan ----
constexpr int kScanThreads = 512;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;

__device__ __forceinline__ int block_exclusive_scan(int value, int *warp_sums, int &block_total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = value;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += t;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    const int nwarps = blockDim.x >> 5;
    if (warp == 0) {
        int w = lane < nwarps ? warp_sums[lane] : 0;
        int wi = w;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, wi, off);
            if (lane >= off) wi += t;
        }
        if (lane < nwarps) warp_sums[lane] = wi - w;  // exclusive
        if (lane == 31) warp_sums[32] = wi;           // block total
    }
    __syncthreads();
    block_total = warp_sums[32];
    const int result = warp_sums[warp] + incl - value;
    __syncthreads();
    return result;
}

__global__ void __launch_bounds__(kScanThreads)
scan_reduce_kernel(const int *__restrict__ in, long long n, int *__restrict__ block_sums) {
    __shared__ int warp_sums[33];
    const long long base = (long long)blockIdx.x * kScanTile + (long long)threadIdx.x * kScanItems;
    int s = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k)
        if (base + k < n) s += in[base + k];
    int total;
    block_exclusive_scan(s, warp_sums, total);
    if (threadIdx.x == 0) block_sums[blockIdx.x] = total;
}

// One block: exclusive scan of block_sums in place; total (64-bit) to *total_out.
__global__ void __launch_bounds__(kScanThreads)
scan_sums_kernel(int *block_sums, int nb, long long *total_out) {
    __shared__ int warp_sums[33];
    long long carry = 0;
    for (int base = 0; base < nb; base += kScanThreads) {
        const int k = base + threadIdx.x;
        const int v = k < nb ? block_sums[k] : 0;
        int total;
        const int ex = block_exclusive_scan(v, warp_sums, total);
        if (k < nb) block_sums[k] = (int)(carry + ex);
        carry += total;
    }
    if (threadIdx.x == 0) *total_out = carry;
}

__global__ void __launch_bounds__(kScanThreads)
scan_apply_kernel(const int *in, long long n, const int *__restrict__ block_offsets,
                  const long long *__restrict__ total, int *out) {
    __shared__ int warp_sums[33];
    const long long base = (long long)blockIdx.x * kScanTile + (long long)threadIdx.x * kScanItems;
    int v[kScanItems];
    int s = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        v[k] = base + k < n ? in[base + k] : 0;
        s += v[k];
    }
    int block_total;
    int run = block_exclusive_scan(s, warp_sums, block_total) + block_offsets[blockIdx.x];
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        if (base + k < n) out[base + k] = run;
        run += v[k];
    }
    // entry n receives the grand total (out has n+1 entries)
    if (blockIdx.x == 0 && threadIdx.x == 0) out[n] = (int)*total;
}

static inline int scan_blocks(long long n) { return (int)((n + kScanTile - 1) / kScanTile); }

// out[0..n] = exclusive prefix sums of in[0..n) (out[n] = total).  `block_sums`
// needs scan_blocks(n)+1 ints, `total_dev` one 64-bit word.  In-place is allowed.
static cudaError_t exclusive_scan(const int *in, long long n, int *out, int *block_sums,
                                  long long *total_dev, cudaStream_t st) {
    const int nb = n > 0 ? scan_blocks(n) : 1;
    scan_reduce_kernel<<<nb, kScanThreads, 0, st>>>(in, n, block_sums);
    scan_sums_kernel<<<1, kScanThreads, 0, st>>>(block_sums, nb, total_dev);
    scan_apply_kernel<<<nb, kScanThreads, 0, st>>>(in, n, block_sums, total_dev, out);
    return cudaGetLastError();
}

// ---------------------------------------------------------- radix pass ----
constexpr int kSortThreads = 256;
constexpr int kSortRounds = 16;
constexpr int kSortTile = kSortThreads * kSortRounds;

__global__ void __launch_bounds__(kSortThreads)
radix_hist_kernel(const unsigned *__restrict__ keys, long long m, int shift, int nb,
                  int *__restrict__ hist) {
    __shared__ int h[256];
    h[threadIdx.x] = 0;
    __syncthreads();
    const long long base = (long long)blockIdx.x * kSortTile;
    for (int r = 0; r < kSortRounds; ++r) {
        const long long k = base + (long long)r * kSortThreads + threadIdx.x;
        if (k < m) atomicAdd(&h[(keys[k] >> shift) & 255u], 1);
    }
    __syncthreads();
    hist[(long long)threadIdx.x * nb + blockIdx.x] = h[threadIdx.x];  // digit-major
}

__global__ void __launch_bounds__(kSortThreads)
radix_scatter_kernel(const unsigned *__restrict__ keys_in, const unsigned *__restrict__ vals_in,
                     long long m, int shift, int nb, const int *__restrict__ offsets,
                     unsigned *__restrict__ keys_out, unsigned *__restrict__ vals_out) {
    constexpr int kWarps = kSortThreads / 32;
    __shared__ int running[256];
    __shared__ int warp_cnt[kWarps][256];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    running[threadIdx.x] = offsets[(long long)threadIdx.x * nb + blockIdx.x];
#pragma unroll
    for (int w = 0; w < kWarps; ++w) warp_cnt[w][threadIdx.x] = 0;
    __syncthreads();
    const long long base = (long long)blockIdx.x * kSortTile;
    const unsigned lt_mask = (1u << lane) - 1u;
    for (int r = 0; r < kSortRounds; ++r) {
        const long long k = base + (long long)r * kSortThreads + threadIdx.x;
        const bool valid = k < m;
        unsigned key = 0, val = 0;
        if (valid) { key = keys_in[k]; val = vals_in[k]; }
        const int dg = valid ? (int)((key >> shift) & 255u) : 256;
        const unsigned peers = __match_any_sync(0xffffffffu, dg);
        const int rank = __popc(peers & lt_mask);
        const int cnt = __popc(peers);
        if (valid && rank == 0) warp_cnt[warp][dg] = cnt;
        __syncthreads();
        if (valid) {
            int off = running[dg] + rank;
            for (int w = 0; w < warp; ++w) off += warp_cnt[w][dg];
            keys_out[off] = key;
            vals_out[off] = val;
        }
        __syncthreads();
        if (valid && rank == 0) {
            atomicAdd(&running[dg], cnt);
            warp_cnt[warp][dg] = 0;
        }
        __syncthreads();
    }
}

static inline int sort_blocks(long long m) { return (int)((m + kSortTile - 1) / kSortTile); }
static inline int bits_for(long long max_value) {
    int b = 1;
    while (b < 32 && (1ll << b) <= max_value) ++b;
    return b;
}

struct SortScratch {
    int *hist;          // 256 * sort_blocks(m) + 1
    int *block_sums;    // scan_blocks(256 * sort_blocks) + 1
    long long *total;
};

// Stable sort of (keys, vals) on the low `bits` bits of keys.  Ping-pongs between
// (k0,v0) and (k1,v1); *result_in_first tells where the sorted data ended up.
static cudaError_t radix_sort_pairs(unsigned *k0, unsigned *v0, unsigned *k1, unsigned *v1,
                                    long long m, int bits, const SortScratch &s,
                                    cudaStream_t st, bool *result_in_first) {
    bool first = true;
    if (m > 0) {
        const int nb = sort_blocks(m);
        for (int shift = 0; shift < bits; shift += 8) {
            unsigned *ki = first ? k0 : k1, *vi = first ? v0 : v1;
            unsigned *ko = first ? k1 : k0, *vo = first ? v1 : v0;
            radix_hist_kernel<<<nb, kSortThreads, 0, st>>>(ki, m, shift, nb, s.hist);
            cudaError_t e = exclusive_scan(s.hist, 256ll * nb, s.hist, s.block_sums, s.total, st);
            if (e != cudaSuccess) return e;
            radix_scatter_kernel<<<nb, kSortThreads, 0, st>>>(ki, vi, m, shift, nb, s.hist, ko, vo);
            first = !first;
        }
    }
    *result_in_first = first;
    return cudaGetLastError();
}

// ----------------------------------------------------------- edge rule ----
struct EdgeRule {
    int op;
    int n;
    long long nnz;
    const int *__restrict__ ptr;
    const int *__restrict__ idx;
};

__device__ __forceinline__ bool src_major(int op) {
    return op == LCD_OP_CSC_LOWER || op == LCD_OP_CSC_UPPER;
}

// Visits the edge instances of node v in inspector order; f(src, dst) per edge.
// Returns an LCD_* code for malformed input.
template <typename F>
__device__ __forceinline__ int visit_edges(const EdgeRule &q, int v, F f) {
    const bool upper = q.op == LCD_OP_CSR_UPPER || q.op == LCD_OP_CSC_UPPER ||
                       q.op == LCD_OP_CSR_UPPER_ROWS;
    const int i = upper ? q.n - 1 - v : v;
    const int s = q.ptr[i], e = q.ptr[i + 1];
    if (s < 0 || e < s || (long long)e > q.nnz) return LCD_ERR_BAD_POINTERS;
    int lo = s, hi = e;
    if (q.op == LCD_OP_CSR_LOWER || q.op == LCD_OP_CSC_UPPER) hi = e - 1;
    if (q.op == LCD_OP_CSC_LOWER || q.op == LCD_OP_CSR_UPPER) lo = s + 1;
    int rc = LCD_OK;
    for (int j = lo; j < hi; ++j) {
        const int c = q.idx[j];
        if (c < 0 || c >= q.n) { rc = LCD_ERR_INDEX_RANGE; continue; }
        switch (q.op) {
            case LCD_OP_CSR_LOWER:
            case LCD_OP_CSR_LOWER_ROWS: if (i > c) f(c, i); break;
            case LCD_OP_CSC_LOWER: if (c > i) f(i, c); break;
            case LCD_OP_ILU0_CSR:
                if (c >= i) return rc;
                f(c, i);
                break;
            case LCD_OP_CSR_UPPER:
            case LCD_OP_CSR_UPPER_ROWS: if (c > i) f(q.n - 1 - c, v); break;
            default: if (c < i) f(v, q.n - 1 - c); break;  // LCD_OP_CSC_UPPER
        }
    }
    return rc;
}

__global__ void count_edges_kernel(const EdgeRule q, int *__restrict__ cnt, int32_t *status) {
    const int v = blockIdx.x * blockDim.x + threadIdx.x;
    if (v >= q.n) return;
    int c = 0;
    const int rc = visit_edges(q, v, [&](int, int) { ++c; });
    if (rc) raise_error(status, rc, v);
    cnt[v] = c;
}

__global__ void emit_edges_kernel(const EdgeRule q, const int *__restrict__ offs,
                                  unsigned *__restrict__ src_out, unsigned *__restrict__ dst_out,
                                  int *edge_count) {
    const int v = blockIdx.x * blockDim.x + threadIdx.x;
    if (v >= q.n) return;
    int pos = offs[v];
    const bool by_src = src_major(q.op);
    visit_edges(q, v, [&](int src, int dst) {
        src_out[pos] = (unsigned)src;
        dst_out[pos] = (unsigned)dst;
        ++pos;
        if (by_src) atomicAdd(edge_count + dst, 1);
    });
}

// head[p] = 1 for the first instance of each distinct (src, dst) pair.
__global__ void flag_heads_kernel(const unsigned *__restrict__ src, const unsigned *__restrict__ dst,
                                  long long m, int *__restrict__ head) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x; p < m; p += stride)
        head[p] = (p == 0 || src[p] != src[p - 1] || dst[p] != dst[p - 1]) ? 1 : 0;
}

__global__ void compact_edges_kernel(const unsigned *__restrict__ src, const unsigned *__restrict__ dst,
                                     long long m, const int *__restrict__ pos,
                                     int *__restrict__ dag_index, unsigned *__restrict__ usrc,
                                     unsigned *__restrict__ udst, int *out_degree, int *dep_count) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x; p < m; p += stride) {
        if (pos[p + 1] == pos[p]) continue;  // not a head
        const int o = pos[p];
        dag_index[o] = (int)dst[p];
        usrc[o] = src[p];
        udst[o] = dst[p];
        atomicAdd(out_degree + src[p], 1);
        atomicAdd(dep_count + dst[p], 1);
    }
}

// ------------------------------------------------------- level kernel ----
constexpr int kLevelThreads = 512;

__global__ void __launch_bounds__(kLevelThreads)
level_kernel(int n, const int *__restrict__ pred_ptr, const unsigned *__restrict__ pred,
             int *level, int *max_level, int32_t *status, unsigned long long budget_ns, int cap) {
    __shared__ int sl[kLevelThreads];
    __shared__ int s_chunk;
    __shared__ int s_max;
    const int tid = threadIdx.x;
    if (tid == 0) { s_chunk = atomicAdd(&status[kStatusTicket], 1); s_max = -1; }
    sl[tid] = -1;
    __syncthreads();
    volatile int *slv = sl;
    const int row0 = s_chunk * kLevelThreads;
    const int v = row0 + tid;
    if (v < n) {
        int p = pred_ptr[v];
        const int pe = pred_ptr[v + 1];
        int lvl = 0;
        bool have = p < pe;
        int u = have ? (int)pred[p] : 0;
        Deadline dl;
        dl.start(budget_ns);
        for (;;) {
            if (have) {
                if ((unsigned)u >= (unsigned)v) {  // an edge must come from an earlier node
                    raise_error(status, LCD_ERR_CYCLE, v);
                    have = false;
                } else {
                    const int lu = (u >= row0) ? slv[u - row0] : ld_relaxed_s32(level + u);
                    if (lu >= 0) {
                        lvl = max(lvl, lu + 1);
                        ++p;
                        have = p < pe;
                        if (have) u = (int)pred[p];
                    } else if (dl.tick(status, v)) {
                        have = false;
                    }
                }
            } else {
                // a caller that only asks "are there at least `cap` levels?" gets its answer
                // here: the status word stops every other waiter within a few polls
                if (cap > 0 && lvl >= cap) raise_error(status, LCD_ERR_LEVEL_CAP, v);
                asm volatile("st.relaxed.gpu.global.s32 [%0], %1;" ::"l"(level + v), "r"(lvl) : "memory");
                slv[tid] = lvl;
                atomicMax(&s_max, lvl);
                break;
            }
        }
    }
    __syncthreads();
    if (tid == 0 && s_max >= 0) atomicMax(max_level, s_max);
}

__global__ void level_hist_kernel(int n, const int *__restrict__ level, int *hist) {
    const int v = blockIdx.x * blockDim.x + threadIdx.x;
    if (v < n) atomicAdd(hist + level[v], 1);
}

__global__ void iota_levels_kernel(int n, const int *__restrict__ level, unsigned *keys,
                                   unsigned *vals) {
    const int v = blockIdx.x * blockDim.x + threadIdx.x;
    if (v < n) { keys[v] = (unsigned)level[v]; vals[v] = (unsigned)v; }
}

__global__ void copy_u32_to_i32_kernel(long long m, const unsigned *__restrict__ in, int *out) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x; p < m; p += stride)
        out[p] = (int)in[p];
}

__global__ void adjacent_diff_kernel(int n, const int *__restrict__ offs, int *out) {
    const int v = blockIdx.x * blockDim.x + threadIdx.x;
    if (v < n) out[v] = offs[v + 1] - offs[v];
}

// ---------------------------------------------------- diagonal table ----
__global__ void diag_positions_kernel(int n, const int *__restrict__ ptr,
                                      const int *__restrict__ idx, long long nnz, int *pos,
                                      int32_t *status) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n) return;
    const long long start = ptr[s], end = ptr[s + 1];
    if (start < 0 || end < start || end > nnz) {
        raise_error(status, LCD_ERR_BAD_POINTERS, s);
        pos[s] = -1;
        return;
    }
    for (long long p = start + 1; p < end; ++p)
        if (idx[p] < idx[p - 1]) { raise_error(status, LCD_ERR_UNSORTED, s); break; }
    long long lo = start, hi = end;  // leftmost entry >= s
    while (lo < hi) {
        const long long mid = (lo + hi) >> 1;
        if (idx[mid] < s) lo = mid + 1; else hi = mid;
    }
    pos[s] = (lo < end && idx[lo] == s) ? (int)lo : -1;
}

// ------------------------------------------------------ workspace plan ----
struct Bump {
    char *base;
    size_t used;
    template <typename T> T *take(size_t count) {
        used = (used + 255) & ~(size_t)255;
        T *p = base ? reinterpret_cast<T *>(base + used) : nullptr;
        used += count * sizeof(T);
        return p;
    }
};

struct DagScratch {
    unsigned *k0, *v0, *k1, *v1;  // cap entries each
    int *flags;                   // cap + 1
    int *cnt;                     // n + 1
    int *pred_ptr;                // n + 1
    int *out_degree;              // n + 1
    int *max_level;               // 1 (+ padding)
    SortScratch sort;
    int *scan_sums;
    long long *scan_total;
};

static DagScratch plan_scratch(Bump &b, int n, long long cap) {
    DagScratch s;
    const long long big = cap > n ? cap : n;
    s.k0 = b.take<unsigned>(big + 1);
    s.v0 = b.take<unsigned>(big + 1);
    s.k1 = b.take<unsigned>(big + 1);
    s.v1 = b.take<unsigned>(big + 1);
    s.flags = b.take<int>(big + 2);
    s.cnt = b.take<int>((size_t)n + 2);
    s.pred_ptr = b.take<int>((size_t)n + 2);
    s.out_degree = b.take<int>((size_t)n + 2);
    s.max_level = b.take<int>(64);
    const long long hist_len = 256ll * sort_blocks(big + 1) + 1;
    s.sort.hist = b.take<int>(hist_len + 1);
    s.sort.block_sums = b.take<int>(scan_blocks(hist_len) + 2);
    s.sort.total = b.take<long long>(8);
    s.scan_sums = b.take<int>(scan_blocks(big + 2) + 2);
    s.scan_total = b.take<long long>(8);
    return s;
}

// ---- Gauss-Seidel rows -> diagonal-last rows ------------------------------------------
// One thread per row.  count: operands (entries left of the diagonal) + 1 diagonal slot.
__global__ void gs_count_kernel(int n, long long nnz, const int *__restrict__ Ap,
                                const int *__restrict__ Ai, int mode, int *__restrict__ len,
                                int32_t *status) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int s = Ap[i], e = Ap[i + 1];
    if (s < 0 || e < s || (long long)e > nnz) {
        raise_error(status, LCD_ERR_BAD_POINTERS, i);
        len[i] = 1;
        return;
    }
    int operands = 0;
    for (int j = s; j < e; ++j) {
        const int c = Ai[j];
        if (c < 0 || c > i || (c == i && mode == 0)) raise_error(status, LCD_ERR_INDEX_RANGE, i);
        else if (c < i) ++operands;
    }
    len[i] = operands + 1;
}

__global__ void gs_fill_kernel(int n, const int *__restrict__ Ap, const int *__restrict__ Ai,
                               const int *__restrict__ Ap_out, int *__restrict__ Ai_out,
                               int *__restrict__ perm, const int32_t *status) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n || status[kStatusCode] != 0) return;
    int pos = Ap_out[i];
    const int slot = Ap_out[i + 1] - 1;
    int last = -1;
    for (int j = Ap[i]; j < Ap[i + 1]; ++j) {
        const int c = Ai[j];
        if (c < i) {
            Ai_out[pos] = c;
            perm[j] = pos++;
        } else {
            perm[j] = -1;
            last = j;   // the reference's loop keeps the last entry equal to the row index
        }
    }
    Ai_out[slot] = i;
    if (last >= 0) perm[last] = slot;
}

__global__ void gs_diag_kernel(int n, const int *__restrict__ Ap_out, const double *__restrict__ D,
                               double *__restrict__ Ax_out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) Ax_out[Ap_out[i + 1] - 1] = D ? D[i] : 1.0;
}

__global__ void gs_scatter_kernel(long long nnz, const int *__restrict__ perm,
                                  const double *__restrict__ Ax, double *__restrict__ Ax_out) {
    const long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (j < nnz && perm[j] >= 0) Ax_out[perm[j]] = Ax[j];
}

// ---- band chains ---------------------------------------------------------------------
// Tasks of the reference's warp executor with band_width > 1: inside every band of band_width
// consecutive levels the nodes that are connected by DAG edges form one task (a chain solved
// by one lane group), tasks ordered by their first node in level order, nodes inside a task
// in level order.  Connected components by lock-free union-find over positions in the level
// order (the smaller position becomes the root, so a component's label is the position of
// its first node), then one stable sort by label.
__device__ __forceinline__ int chain_find(int *parent, int v) {
    int p = parent[v];
    while (p != v) {            // path halving
        const int gp = parent[p];
        if (gp != p) parent[v] = gp;
        v = p;
        p = gp;
    }
    return v;
}

__global__ void chain_init_kernel(int n, const int *__restrict__ wavefronts, int *pos, int *parent,
                                  int32_t *status) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n) return;
    parent[t] = t;
    const int v = wavefronts[t];
    if ((unsigned)v >= (unsigned)n) raise_error(status, LCD_ERR_INDEX_RANGE, t);
    else pos[v] = t;
}

__global__ void chain_union_kernel(int n, const int *__restrict__ dag_ptr, const int *__restrict__ dag_index,
                                   const int *__restrict__ level, const int *__restrict__ pos,
                                   int band_width, int *parent) {
    const int u = blockIdx.x * blockDim.x + threadIdx.x;
    if (u >= n) return;
    const int band = level[u] / band_width;
    for (int e = dag_ptr[u]; e < dag_ptr[u + 1]; ++e) {
        const int w = dag_index[e];
        if ((unsigned)w >= (unsigned)n || level[w] / band_width != band) continue;
        int a = pos[u], b = pos[w];
        for (;;) {              // hook the larger root under the smaller one
            a = chain_find(parent, a);
            b = chain_find(parent, b);
            if (a == b) break;
            if (a < b) { const int t = a; a = b; b = t; }
            if (atomicCAS(parent + a, a, b) == a) break;
        }
    }
}

__global__ void chain_label_kernel(int n, const int *__restrict__ wavefronts, int *parent,
                                   unsigned *keys, unsigned *vals) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n) return;
    int r = t;
    while (parent[r] != r) r = parent[r];
    keys[t] = (unsigned)r;
    vals[t] = (unsigned)wavefronts[t];
}

__global__ void chain_heads_kernel(int n, const unsigned *__restrict__ keys, int *head) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < n) head[t] = (t == 0 || keys[t] != keys[t - 1]) ? 1 : 0;
}

__global__ void chain_emit_kernel(int n, const unsigned *__restrict__ vals, const int *__restrict__ headscan,
                                  const int *__restrict__ wavefront_ptr, int n_levels, int band_width,
                                  int *task_nodes, int *task_ptr, int *band_ptr) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    const int n_bands = (n_levels + band_width - 1) / band_width;
    if (t <= n_bands) {
        const int first_level = t * band_width < n_levels ? t * band_width : n_levels;
        band_ptr[t] = headscan[wavefront_ptr[first_level]];   // tasks that start before the band
    }
    if (t >= n) return;
    task_nodes[t] = (int)vals[t];
    if (headscan[t + 1] != headscan[t]) task_ptr[headscan[t]] = t;
    if (t == n - 1) task_ptr[headscan[n]] = n;
}

static inline int grid_for(long long m, int threads) {
    long long g = (m + threads - 1) / threads;
    const long long cap = 148ll * 32;
    return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace lcd

using namespace lcd;

extern "C" int lcd_dag_workspace_bytes(int op, int32_t n, int64_t nnz, int64_t *bytes) {
    if (op < 0 || op > LCD_OP_CSR_UPPER_ROWS || n < 0 || nnz < 0 || !bytes)
        return LCD_ERR_INVALID_ARGUMENT;
    Bump b{nullptr, 0};
    b.take<int32_t>(LCD_STATUS_WORDS);
    plan_scratch(b, n, nnz);
    *bytes = (int64_t)b.used + 256;
    return LCD_OK;
}

extern "C" int lcd_dag_build(int op, int32_t n, const int32_t *ptr, const int32_t *idx,
                             int64_t nnz, int32_t *dep_count, int32_t *edge_count,
                             int32_t *dag_ptr, int32_t *dag_index, int64_t *n_edges_host,
                             int32_t *level, int32_t *wavefronts, int32_t *wavefront_ptr,
                             int32_t *n_levels_host, void *workspace, int64_t workspace_bytes,
                             int32_t timeout_ms, void *stream) {
    return lcd_dag_build_capped(op, n, ptr, idx, nnz, dep_count, edge_count, dag_ptr, dag_index,
                                n_edges_host, level, wavefronts, wavefront_ptr, n_levels_host, 0,
                                workspace, workspace_bytes, timeout_ms, stream);
}

extern "C" int lcd_dag_build_capped(int op, int32_t n, const int32_t *ptr, const int32_t *idx,
                                    int64_t nnz, int32_t *dep_count, int32_t *edge_count,
                                    int32_t *dag_ptr, int32_t *dag_index, int64_t *n_edges_host,
                                    int32_t *level, int32_t *wavefronts, int32_t *wavefront_ptr,
                                    int32_t *n_levels_host, int32_t level_cap, void *workspace,
                                    int64_t workspace_bytes, int32_t timeout_ms, void *stream) {
    if (op < 0 || op > LCD_OP_CSR_UPPER_ROWS || n < 0 || nnz < 0 || !n_edges_host || !n_levels_host ||
        level_cap < 0)
        return LCD_ERR_INVALID_ARGUMENT;
    *n_edges_host = 0;
    *n_levels_host = 0;
    if (n == 0) return LCD_OK;
    if (!ptr || (nnz > 0 && !idx) || !dep_count || !edge_count || !dag_ptr || !dag_index ||
        !level || !wavefronts || !wavefront_ptr || !workspace)
        return LCD_ERR_INVALID_ARGUMENT;
    if (nnz > 0x7fffffffll - 4096) return LCD_ERR_TOO_LARGE;
    int64_t need = 0;
    lcd_dag_workspace_bytes(op, n, nnz, &need);
    if (workspace_bytes < need) return LCD_ERR_WORKSPACE;
    cudaStream_t st = (cudaStream_t)stream;
    Bump bump{reinterpret_cast<char *>(workspace), 0};
    int32_t *status = bump.take<int32_t>(LCD_STATUS_WORDS);
    DagScratch s = plan_scratch(bump, n, nnz);
    int rc = reset_status(status, st);
    if (rc) return rc;
    const EdgeRule q{op, n, nnz, ptr, idx};
    const int nblk = (n + 255) / 256;
    const bool by_src = (op == LCD_OP_CSC_LOWER || op == LCD_OP_CSC_UPPER);

    // 1. count, scan, emit
    count_edges_kernel<<<nblk, 256, 0, st>>>(q, s.cnt, status);
    LCD_CUDA_TRY(exclusive_scan(s.cnt, n, s.cnt, s.scan_sums, s.scan_total, st));
    long long n_inst = 0;
    LCD_CUDA_TRY(cudaMemcpyAsync(&n_inst, s.scan_total, sizeof n_inst, cudaMemcpyDeviceToHost, st));
    LCD_CUDA_TRY(cudaMemsetAsync(edge_count, 0, (size_t)n * sizeof(int32_t), st));
    LCD_CUDA_TRY(cudaStreamSynchronize(st));
    rc = lcd_read_status(status, st, nullptr);
    if (rc) return rc;
    if (n_inst > nnz) return LCD_ERR_TOO_LARGE;  // cannot happen: one edge per stored entry at most
    emit_edges_kernel<<<nblk, 256, 0, st>>>(q, s.cnt, s.k0, s.v0, edge_count);
    // destination-major rules: the per-node instance count is the edge multiplicity
    if (!by_src) adjacent_diff_kernel<<<nblk, 256, 0, st>>>(n, s.cnt, edge_count);
    LCD_CUDA_TRY(cudaGetLastError());

    // 2. (src, dst) order.  keys = src in k*, vals = dst in v*.
    const int node_bits = bits_for(n > 1 ? n - 1 : 1);
    unsigned *src = s.k0, *dst = s.v0, *src_alt = s.k1, *dst_alt = s.v1;
    bool in_first = true;
    if (by_src) {
        // emission is source-major but destinations inside a segment may be unsorted:
        // sort by destination first (dst as key), then by source.
        LCD_CUDA_TRY(radix_sort_pairs(dst, src, dst_alt, src_alt, n_inst, node_bits, s.sort, st,
                                      &in_first));
        if (!in_first) { unsigned *t = src; src = src_alt; src_alt = t; t = dst; dst = dst_alt; dst_alt = t; }
    }
    LCD_CUDA_TRY(radix_sort_pairs(src, dst, src_alt, dst_alt, n_inst, node_bits, s.sort, st,
                                  &in_first));
    if (!in_first) { unsigned *t = src; src = src_alt; src_alt = t; t = dst; dst = dst_alt; dst_alt = t; }

    // 3. distinct edges
    LCD_CUDA_TRY(cudaMemsetAsync(dep_count, 0, (size_t)n * sizeof(int32_t), st));
    LCD_CUDA_TRY(cudaMemsetAsync(s.out_degree, 0, ((size_t)n + 1) * sizeof(int), st));
    long long n_uniq = 0;
    if (n_inst > 0) {
        flag_heads_kernel<<<grid_for(n_inst, 256), 256, 0, st>>>(src, dst, n_inst, s.flags);
        LCD_CUDA_TRY(exclusive_scan(s.flags, n_inst, s.flags, s.scan_sums, s.scan_total, st));
        compact_edges_kernel<<<grid_for(n_inst, 256), 256, 0, st>>>(
            src, dst, n_inst, s.flags, dag_index, src_alt, dst_alt, s.out_degree, dep_count);
        LCD_CUDA_TRY(cudaMemcpyAsync(&n_uniq, s.scan_total, sizeof n_uniq, cudaMemcpyDeviceToHost, st));
    }
    LCD_CUDA_TRY(exclusive_scan(s.out_degree, n, dag_ptr, s.scan_sums, s.scan_total, st));
    LCD_CUDA_TRY(exclusive_scan(dep_count, n, s.pred_ptr, s.scan_sums, s.scan_total, st));
    LCD_CUDA_TRY(cudaStreamSynchronize(st));
    *n_edges_host = n_uniq;

    // 4. predecessor lists (distinct edges regrouped by destination), levels
    //    distinct edges live in (src_alt, dst_alt); (src, dst) is free now.
    LCD_CUDA_TRY(radix_sort_pairs(dst_alt, src_alt, dst, src, n_uniq, node_bits, s.sort, st, &in_first));
    const unsigned *pred = in_first ? src_alt : src;
    LCD_CUDA_TRY(cudaMemsetAsync(level, 0xFF, (size_t)n * sizeof(int32_t), st));
    LCD_CUDA_TRY(cudaMemsetAsync(s.max_level, 0xFF, sizeof(int), st));
    rc = reset_status(status, st);
    if (rc) return rc;
    level_kernel<<<(n + kLevelThreads - 1) / kLevelThreads, kLevelThreads, 0, st>>>(
        n, s.pred_ptr, pred, level, s.max_level, status, timeout_ns(timeout_ms), level_cap);
    LCD_CUDA_TRY(cudaGetLastError());
    int max_level = -1;
    LCD_CUDA_TRY(cudaMemcpyAsync(&max_level, s.max_level, sizeof max_level, cudaMemcpyDeviceToHost, st));
    LCD_CUDA_TRY(cudaStreamSynchronize(st));
    rc = lcd_read_status(status, st, nullptr);
    if (rc == LCD_ERR_LEVEL_CAP) {
        // at least level_cap + 1 levels: the level arrays stay unfinished, everything else is built
        *n_levels_host = -level_cap;
        return LCD_OK;
    }
    if (rc) return rc;
    const int n_levels = max_level + 1;
    *n_levels_host = n_levels;

    // 5. nodes by (level, id); level offsets
    LCD_CUDA_TRY(cudaMemsetAsync(s.cnt, 0, ((size_t)n + 1) * sizeof(int), st));
    level_hist_kernel<<<nblk, 256, 0, st>>>(n, level, s.cnt);
    LCD_CUDA_TRY(exclusive_scan(s.cnt, n_levels, wavefront_ptr, s.scan_sums, s.scan_total, st));
    iota_levels_kernel<<<nblk, 256, 0, st>>>(n, level, s.k0, s.v0);
    LCD_CUDA_TRY(radix_sort_pairs(s.k0, s.v0, s.k1, s.v1, n, bits_for(n_levels > 1 ? n_levels - 1 : 1),
                                  s.sort, st, &in_first));
    copy_u32_to_i32_kernel<<<grid_for(n, 256), 256, 0, st>>>(n, in_first ? s.v0 : s.v1, wavefronts);
    LCD_CUDA_TRY(cudaGetLastError());
    LCD_CUDA_TRY(cudaStreamSynchronize(st));
    return LCD_OK;
}

extern "C" int lcd_diag_positions(int32_t n, const int32_t *ptr, const int32_t *idx, int64_t nnz,
                                  int32_t *pos, int32_t *status_dev, void *stream,
                                  int *status_host) {
    if (n < 0 || nnz < 0 || !status_dev || (n > 0 && (!ptr || !pos)))
        return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    int rc = reset_status(status_dev, st);
    if (rc) return rc;
    if (n > 0) {
        diag_positions_kernel<<<(n + 255) / 256, 256, 0, st>>>(n, ptr, idx, nnz, pos, status_dev);
        LCD_CUDA_TRY(cudaGetLastError());
    }
    return finish(status_dev, st, status_host);
}

extern "C" int lcd_gs_layout_workspace_bytes(int32_t n, int64_t *bytes) {
    if (n < 0 || !bytes) return LCD_ERR_INVALID_ARGUMENT;
    Bump b{nullptr, 0};
    b.take<long long>(8);
    b.take<int>(n);
    b.take<int>(scan_blocks(n) + 2);
    *bytes = (int64_t)b.used + 256;
    return LCD_OK;
}

extern "C" int lcd_gs_layout(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai, int mode,
                             int32_t *Ap_out, int32_t *Ai_out, int32_t *perm,
                             int64_t *nnz_out_host, void *workspace, int64_t workspace_bytes,
                             int32_t *status_dev, void *stream, int *status_host) {
    if (n < 0 || nnz < 0 || (mode != 0 && mode != 1) || !status_dev || !nnz_out_host)
        return LCD_ERR_INVALID_ARGUMENT;
    *nnz_out_host = 0;
    if (n > 0 && (!Ap || (nnz > 0 && (!Ai || !perm)) || !Ap_out || !Ai_out || !workspace))
        return LCD_ERR_INVALID_ARGUMENT;
    int64_t need = 0;
    lcd_gs_layout_workspace_bytes(n, &need);
    if (n > 0 && workspace_bytes < need) return LCD_ERR_WORKSPACE;
    cudaStream_t st = (cudaStream_t)stream;
    int rc = reset_status(status_dev, st);
    if (rc) return rc;
    if (n > 0) {
        Bump b{static_cast<char *>(workspace), 0};
        long long *total = b.take<long long>(8);
        int *len = b.take<int>(n);
        int *sums = b.take<int>(scan_blocks(n) + 2);
        gs_count_kernel<<<(n + 255) / 256, 256, 0, st>>>(n, nnz, Ap, Ai, mode, len, status_dev);
        LCD_CUDA_TRY(cudaGetLastError());
        LCD_CUDA_TRY(exclusive_scan(len, n, Ap_out, sums, total, st));
        long long total_host = 0;
        LCD_CUDA_TRY(cudaMemcpyAsync(&total_host, total, sizeof total_host, cudaMemcpyDeviceToHost, st));
        LCD_CUDA_TRY(cudaStreamSynchronize(st));
        const int32_t last = (int32_t)total_host;
        LCD_CUDA_TRY(cudaMemcpyAsync(Ap_out + n, &last, sizeof last, cudaMemcpyHostToDevice, st));
        gs_fill_kernel<<<(n + 255) / 256, 256, 0, st>>>(n, Ap, Ai, Ap_out, Ai_out, perm, status_dev);
        LCD_CUDA_TRY(cudaGetLastError());
        LCD_CUDA_TRY(cudaStreamSynchronize(st));   // `last` is read by the copy above
        *nnz_out_host = total_host;
    }
    return finish(status_dev, st, status_host);
}

extern "C" int lcd_gs_values(int32_t n, int64_t nnz, const int32_t *Ap_out, const int32_t *perm,
                             const double *Ax, const double *D, double *Ax_out, void *stream) {
    if (n < 0 || nnz < 0) return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && (!Ap_out || !Ax_out || (nnz > 0 && (!perm || !Ax)))) return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    if (n > 0) {
        gs_diag_kernel<<<(n + 255) / 256, 256, 0, st>>>(n, Ap_out, D, Ax_out);
        LCD_CUDA_TRY(cudaGetLastError());
    }
    if (nnz > 0) {
        gs_scatter_kernel<<<(unsigned)((nnz + 255) / 256), 256, 0, st>>>(nnz, perm, Ax, Ax_out);
        LCD_CUDA_TRY(cudaGetLastError());
    }
    return LCD_OK;
}

extern "C" int lcd_band_chains_workspace_bytes(int32_t n, int64_t *bytes) {
    if (n < 0 || !bytes) return LCD_ERR_INVALID_ARGUMENT;
    Bump b{nullptr, 0};
    b.take<int32_t>(LCD_STATUS_WORDS);
    plan_scratch(b, n, n);
    *bytes = (int64_t)b.used + 256;
    return LCD_OK;
}

extern "C" int lcd_band_chains(int32_t n, const int32_t *dag_ptr, const int32_t *dag_index,
                               const int32_t *level, const int32_t *wavefronts,
                               const int32_t *wavefront_ptr_dev, int32_t n_levels, int32_t band_width,
                               int32_t *task_nodes, int32_t *task_ptr, int32_t *band_ptr,
                               int32_t *n_tasks_host, void *workspace, int64_t workspace_bytes,
                               void *stream) {
    if (n < 0 || n_levels < 0 || band_width < 1 || !n_tasks_host) return LCD_ERR_INVALID_ARGUMENT;
    *n_tasks_host = 0;
    if (!task_ptr || !band_ptr || !workspace) return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && (!dag_ptr || !dag_index || !level || !wavefronts || !wavefront_ptr_dev || !task_nodes))
        return LCD_ERR_INVALID_ARGUMENT;
    int64_t need = 0;
    lcd_band_chains_workspace_bytes(n, &need);
    if (workspace_bytes < need) return LCD_ERR_WORKSPACE;
    cudaStream_t st = (cudaStream_t)stream;
    if (n == 0) {
        LCD_CUDA_TRY(cudaMemsetAsync(task_ptr, 0, sizeof(int32_t), st));
        LCD_CUDA_TRY(cudaMemsetAsync(band_ptr, 0, sizeof(int32_t), st));
        LCD_CUDA_TRY(cudaStreamSynchronize(st));
        return LCD_OK;
    }
    Bump bump{reinterpret_cast<char *>(workspace), 0};
    int32_t *status = bump.take<int32_t>(LCD_STATUS_WORDS);
    DagScratch s = plan_scratch(bump, n, n);
    int rc = reset_status(status, st);
    if (rc) return rc;
    const int nblk = (n + 255) / 256;
    int *pos = s.cnt, *parent = s.pred_ptr;
    chain_init_kernel<<<nblk, 256, 0, st>>>(n, wavefronts, pos, parent, status);
    chain_union_kernel<<<nblk, 256, 0, st>>>(n, dag_ptr, dag_index, level, pos, band_width, parent);
    chain_label_kernel<<<nblk, 256, 0, st>>>(n, wavefronts, parent, s.k0, s.v0);
    LCD_CUDA_TRY(cudaGetLastError());
    bool in_first = true;
    LCD_CUDA_TRY(radix_sort_pairs(s.k0, s.v0, s.k1, s.v1, n, bits_for(n > 1 ? n - 1 : 1), s.sort, st,
                                  &in_first));
    const unsigned *keys = in_first ? s.k0 : s.k1, *vals = in_first ? s.v0 : s.v1;
    chain_heads_kernel<<<nblk, 256, 0, st>>>(n, keys, s.flags);
    LCD_CUDA_TRY(exclusive_scan(s.flags, n, s.flags, s.scan_sums, s.scan_total, st));
    const int n_bands = (n_levels + band_width - 1) / band_width;
    const int m = n > n_bands + 1 ? n : n_bands + 1;
    chain_emit_kernel<<<(m + 255) / 256, 256, 0, st>>>(n, vals, s.flags, wavefront_ptr_dev, n_levels,
                                                       band_width, task_nodes, task_ptr, band_ptr);
    LCD_CUDA_TRY(cudaGetLastError());
    long long total = 0;
    LCD_CUDA_TRY(cudaMemcpyAsync(&total, s.scan_total, sizeof total, cudaMemcpyDeviceToHost, st));
    LCD_CUDA_TRY(cudaStreamSynchronize(st));
    rc = lcd_read_status(status, st, nullptr);
    if (rc) return rc;
    *n_tasks_host = (int32_t)total;
    return LCD_OK;
}

// ---- CSC -> supernodal layout ------------------------------------------------------------
// Counterpart of convert_csc_to_supernodal (utils/symbolic_cholesky_csc.py:883-1021 of the
// reference, a triple Python loop over sets): column j + 1 joins column j's supernode when the
// symmetric difference of their row patterns has at most relaxation + 1 elements; the row
// structure of a supernode is the sorted union of its columns' patterns; every column stores one
// value per row of that union.  Here: a two-pointer comparison per column pair, a scan for the
// supernode numbers, a stable radix sort of (supernode, row) pairs + flag / scan / compact for
// the unions, a 64-bit scan for the panel offsets, and a binary search per stored entry for the
// values.  Columns must be sorted (what the reference's set logic does not need, SciPy delivers).
namespace lcd {

__device__ __forceinline__ int column_of_entry(const int *__restrict__ Cp, int n, long long k) {
    int lo = 0, hi = n;          // last column whose pointer is <= k
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if ((long long)Cp[mid] <= k) lo = mid; else hi = mid;
    }
    return lo;
}

__global__ void sn_merge_kernel(int n, long long nnz, const int *__restrict__ Cp,
                                const int *__restrict__ Ci, int relaxation, int *begin,
                                int32_t *status) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    const int s = Cp[j], e = Cp[j + 1];
    if (s < 0 || e < s || (long long)e > nnz || (j == 0 && s != 0)) {
        raise_error(status, LCD_ERR_BAD_POINTERS, j);
        begin[j] = 1;
        return;
    }
    for (int k = s; k < e; ++k) {
        const int r = Ci[k];
        if ((unsigned)r >= (unsigned)n) { raise_error(status, LCD_ERR_INDEX_RANGE, j); break; }
        if (k > s && r <= Ci[k - 1]) { raise_error(status, LCD_ERR_UNSORTED, j); break; }
    }
    if (j == 0) { begin[0] = 1; return; }
    const int ps = Cp[j - 1];
    if (ps < 0 || ps > s) { begin[j] = 1; return; }   // (reported by the thread of column j - 1)
    // symmetric difference of columns j - 1 and j, given up once it exceeds the allowance
    int a = ps, b = s, differ = 0;
    const int limit = relaxation + 1;
    while (differ <= limit && (a < s || b < e)) {
        if (a < s && b < e) {
            const int ra = Ci[a], rb = Ci[b];
            if (ra == rb) { ++a; ++b; }
            else if (ra < rb) { ++a; ++differ; }
            else { ++b; ++differ; }
        } else {
            differ += (s - a) + (e - b);
            break;
        }
    }
    begin[j] = differ > limit ? 1 : 0;
}

__global__ void sn_number_kernel(int n, const int *__restrict__ begin, const int *__restrict__ scan,
                                 int *col_to_super, int *super_begin) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j > n) return;
    if (j == n) { super_begin[scan[n]] = n; return; }
    col_to_super[j] = scan[j + 1] - 1;
    if (begin[j]) super_begin[scan[j]] = j;
}

__global__ void sn_pairs_kernel(int n, long long nnz, const int *__restrict__ Cp,
                                const int *__restrict__ Ci, const int *__restrict__ col_to_super,
                                unsigned *rows, unsigned *supers) {
    for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < nnz;
         k += (long long)gridDim.x * blockDim.x) {
        rows[k] = (unsigned)Ci[k];
        supers[k] = (unsigned)col_to_super[column_of_entry(Cp, n, k)];
    }
}

// (supers, rows) sorted by supernode, then row: heads of runs are the union's elements
__global__ void sn_heads_kernel(long long m, const unsigned *__restrict__ supers,
                                const unsigned *__restrict__ rows, int *head, int *count) {
    for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < m;
         t += (long long)gridDim.x * blockDim.x) {
        const bool first = t == 0 || supers[t] != supers[t - 1] || rows[t] != rows[t - 1];
        head[t] = first ? 1 : 0;
        if (first) atomicAdd(count + supers[t], 1);
    }
}

__global__ void sn_rows_kernel(long long m, const unsigned *__restrict__ rows,
                               const int *__restrict__ head, const int *__restrict__ headscan,
                               int *Li) {
    for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < m;
         t += (long long)gridDim.x * blockDim.x)
        if (head[t]) Li[headscan[t]] = (int)rows[t];
}

// One block: 64-bit exclusive scan of width * length per supernode (panel offsets), widest
// supernode, and the summary the host reads.
__global__ void __launch_bounds__(1024)
sn_panels_kernel(int n, const int *__restrict__ nsuper_dev, const int *__restrict__ super_begin,
                 const int *__restrict__ Lip, long long *base, long long *summary) {
    __shared__ long long part[1024];
    __shared__ long long carry;
    __shared__ int widest;
    const int n_super = *nsuper_dev;
    if (threadIdx.x == 0) { carry = 0; widest = 0; }
    __syncthreads();
    for (int s0 = 0; s0 < n_super; s0 += 1024) {
        const int s = s0 + threadIdx.x;
        long long size = 0;
        if (s < n_super) {
            const int width = super_begin[s + 1] - super_begin[s];
            size = (long long)width * (Lip[s + 1] - Lip[s]);
            atomicMax(&widest, width);
        }
        part[threadIdx.x] = size;
        __syncthreads();
        for (int off = 1; off < 1024; off <<= 1) {       // inclusive scan of the tile
            const long long add = threadIdx.x >= off ? part[threadIdx.x - off] : 0;
            __syncthreads();
            part[threadIdx.x] += add;
            __syncthreads();
        }
        if (s < n_super) base[s] = carry + part[threadIdx.x] - size;
        __syncthreads();
        if (threadIdx.x == 1023) carry += part[1023];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        base[n_super] = carry;
        summary[0] = n_super;
        summary[1] = Lip[n_super];
        summary[2] = widest;
        summary[3] = carry;
    }
}

__global__ void sn_colptr_kernel(int n, const int *__restrict__ nsuper_dev,
                                 const int *__restrict__ col_to_super, const int *__restrict__ super_begin,
                                 const int *__restrict__ Lip, const long long *__restrict__ base,
                                 long long *Lp) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j > n) return;
    if (j == n) { Lp[n] = base[*nsuper_dev]; return; }
    const int s = col_to_super[j];
    Lp[j] = base[s] + (long long)(j - super_begin[s]) * (Lip[s + 1] - Lip[s]);
}

__global__ void sn_fill_kernel(int n, long long nnz, const int *__restrict__ Cp,
                               const int *__restrict__ Ci, const double *__restrict__ Cx,
                               const int *__restrict__ col_to_super, const int *__restrict__ Lip,
                               const int *__restrict__ Li, const long long *__restrict__ Lp,
                               double *Lx, int32_t *status) {
    for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < nnz;
         k += (long long)gridDim.x * blockDim.x) {
        const int j = column_of_entry(Cp, n, k);
        const int s = col_to_super[j], row = Ci[k];
        int lo = Lip[s], hi = Lip[s + 1];
        const int end = hi;
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (Li[mid] < row) lo = mid + 1; else hi = mid;
        }
        if (lo < end && Li[lo] == row) Lx[Lp[j] + (lo - Lip[s])] = Cx[k];
        else raise_error(status, LCD_ERR_INDEX_RANGE, j);   // the layout belongs to another pattern
    }
}

}  // namespace lcd

extern "C" int lcd_supernodal_layout_workspace_bytes(int32_t n, int64_t nnz, int64_t *bytes) {
    if (n < 0 || nnz < 0 || !bytes) return LCD_ERR_INVALID_ARGUMENT;
    Bump b{nullptr, 0};
    b.take<int32_t>(LCD_STATUS_WORDS);
    plan_scratch(b, n, nnz);
    b.take<long long>((size_t)n + 2);
    b.take<long long>(8);
    *bytes = (int64_t)b.used + 256;
    return LCD_OK;
}

extern "C" int lcd_supernodal_layout(int32_t n, int64_t nnz, const int32_t *Cp, const int32_t *Ci,
                                     int32_t relaxation, int32_t *col_to_super, int32_t *super_begin,
                                     int32_t *Lip, int32_t *Li, int64_t *Lp, int64_t *summary_host,
                                     void *workspace, int64_t workspace_bytes, void *stream) {
    if (n < 0 || nnz < 0 || relaxation < 0 || !summary_host || !workspace) return LCD_ERR_INVALID_ARGUMENT;
    if (!super_begin || !Lip || !Lp) return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && (!Cp || !col_to_super || (nnz > 0 && (!Ci || !Li)))) return LCD_ERR_INVALID_ARGUMENT;
    int64_t need = 0;
    lcd_supernodal_layout_workspace_bytes(n, nnz, &need);
    if (workspace_bytes < need) return LCD_ERR_WORKSPACE;
    cudaStream_t st = (cudaStream_t)stream;
    for (int k = 0; k < 4; ++k) summary_host[k] = 0;
    if (n == 0) {
        LCD_CUDA_TRY(cudaMemsetAsync(super_begin, 0, sizeof(int32_t), st));
        LCD_CUDA_TRY(cudaMemsetAsync(Lip, 0, sizeof(int32_t), st));
        LCD_CUDA_TRY(cudaMemsetAsync(Lp, 0, sizeof(int64_t), st));
        LCD_CUDA_TRY(cudaStreamSynchronize(st));
        return LCD_OK;
    }
    Bump bump{reinterpret_cast<char *>(workspace), 0};
    int32_t *status = bump.take<int32_t>(LCD_STATUS_WORDS);
    DagScratch s = plan_scratch(bump, n, nnz);
    long long *base = bump.take<long long>((size_t)n + 2);
    long long *summary = bump.take<long long>(8);
    int rc = reset_status(status, st);
    if (rc) return rc;
    const int nblk = (n + 1 + 255) / 256;
    int *begin = s.cnt, *scan = s.pred_ptr, *count = s.out_degree;
    sn_merge_kernel<<<nblk, 256, 0, st>>>(n, nnz, Cp, Ci, relaxation, begin, status);
    LCD_CUDA_TRY(exclusive_scan(begin, n, scan, s.scan_sums, s.scan_total, st));
    sn_number_kernel<<<nblk, 256, 0, st>>>(n, begin, scan, col_to_super, super_begin);
    LCD_CUDA_TRY(cudaGetLastError());
    rc = lcd_read_status(status, st, nullptr);    // malformed columns: nothing below may index with them
    if (rc) return rc;
    LCD_CUDA_TRY(cudaMemsetAsync(count, 0, ((size_t)n + 1) * sizeof(int), st));
    if (nnz > 0) {
        sn_pairs_kernel<<<grid_for(nnz, 256), 256, 0, st>>>(n, nnz, Cp, Ci, col_to_super, s.k0, s.v0);
        // by row, then (stable) by supernode
        bool in_first = true;
        LCD_CUDA_TRY(radix_sort_pairs(s.k0, s.v0, s.k1, s.v1, nnz, bits_for(n > 1 ? n - 1 : 1), s.sort,
                                      st, &in_first));
        unsigned *rows = in_first ? s.k0 : s.k1, *supers = in_first ? s.v0 : s.v1;
        unsigned *rows_alt = in_first ? s.k1 : s.k0, *supers_alt = in_first ? s.v1 : s.v0;
        LCD_CUDA_TRY(radix_sort_pairs(supers, rows, supers_alt, rows_alt, nnz,
                                      bits_for(n > 1 ? n - 1 : 1), s.sort, st, &in_first));
        const unsigned *sup = in_first ? supers : supers_alt, *row = in_first ? rows : rows_alt;
        // (the heads go to the key buffer the sort left free, their scan to the flag array)
        int *heads = reinterpret_cast<int *>(in_first ? supers_alt : supers);
        sn_heads_kernel<<<grid_for(nnz, 256), 256, 0, st>>>(nnz, sup, row, heads, count);
        LCD_CUDA_TRY(exclusive_scan(heads, nnz, s.flags, s.scan_sums, s.scan_total, st));
        sn_rows_kernel<<<grid_for(nnz, 256), 256, 0, st>>>(nnz, row, heads, s.flags, Li);
    }
    // Lip = exclusive scan of the union sizes (entries past the last supernode repeat the total)
    LCD_CUDA_TRY(exclusive_scan(count, n, Lip, s.scan_sums, s.scan_total, st));
    sn_panels_kernel<<<1, 1024, 0, st>>>(n, scan + n, super_begin, Lip, base, summary);
    sn_colptr_kernel<<<nblk, 256, 0, st>>>(n, scan + n, col_to_super, super_begin, Lip, base,
                                           reinterpret_cast<long long *>(Lp));
    LCD_CUDA_TRY(cudaGetLastError());
    long long host[4] = {0, 0, 0, 0};
    LCD_CUDA_TRY(cudaMemcpyAsync(host, summary, sizeof host, cudaMemcpyDeviceToHost, st));
    LCD_CUDA_TRY(cudaStreamSynchronize(st));
    rc = lcd_read_status(status, st, nullptr);
    if (rc) return rc;
    for (int k = 0; k < 4; ++k) summary_host[k] = host[k];
    return LCD_OK;
}

extern "C" int lcd_supernodal_fill(int32_t n, int64_t nnz, const int32_t *Cp, const int32_t *Ci,
                                   const double *Cx, const int32_t *col_to_super, const int32_t *Lip,
                                   const int32_t *Li, const int64_t *Lp, double *Lx,
                                   int64_t panel_values, int32_t *status_dev, void *stream,
                                   int *status_host) {
    if (n < 0 || nnz < 0 || panel_values < 0 || !status_dev) return LCD_ERR_INVALID_ARGUMENT;
    if (nnz > 0 && (!Cp || !Ci || !Cx || !col_to_super || !Lip || !Li || !Lp || !Lx))
        return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    int rc = reset_status(status_dev, st);
    if (rc) return rc;
    if (panel_values > 0) LCD_CUDA_TRY(cudaMemsetAsync(Lx, 0, (size_t)panel_values * sizeof(double), st));
    if (nnz > 0) {
        sn_fill_kernel<<<grid_for(nnz, 256), 256, 0, st>>>(n, nnz, Cp, Ci, Cx, col_to_super, Lip, Li,
                                                          reinterpret_cast<const long long *>(Lp), Lx,
                                                          status_dev);
        LCD_CUDA_TRY(cudaGetLastError());
    }
    return finish(status_dev, st, status_host);
}
