/*
 * CPU oracle for the dependence-DAG hot path.  TEST INFRASTRUCTURE ONLY: this
 * file is a sequential restatement of the reference's algorithms used to check
 * the CUDA kernels and as the timed CPU baseline.  Nothing in the product
 * package may call it.
 *
 * Parity status: pinned.  Every function here is checked against outputs of
 * the reference's own Python pipeline (committed as fixtures under
 * tests/golden/, produced by tests/golden/make_golden.py) and against the
 * golden vectors held by the reference's unit tests.
 *
 * Build with -ffp-contract=off so that a*b-c is rounded twice like the Python
 * originals.
 *
 * Reference locations followed (paths inside the reference project):
 *   edge rules ............ generated inspector, compiler/dag_codegen.py:1164-1196,1293-1389
 *   dep/edge counts ....... compiler/dag_codegen.py:1391-1402,1421-1482
 *   successor CSR ......... compiler/dag_preprocessing.py:115-143
 *   Kahn levels ........... compiler/dag_preprocessing.py:146-163
 *   flattening ............ compiler/dag_preprocessing.py:166-204
 *   diagonal table ........ compiler/structural_lookups.py:279-333
 *   SpTRSV CSR / CSC ...... compiler/demo/sptrsv.py:26-43
 *   ILU0 CSR .............. compiler/demo/spilu0.py:21-47
 *   supernodal solve ...... benchmark/sptrsv_supernodal.py:12-28,
 *                           utils/dense_blas.py:19-33,228-242
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { ORC_CSR_LOWER = 0, ORC_CSC_LOWER = 1, ORC_ILU0_CSR = 2,
       ORC_CSR_UPPER = 3, ORC_CSC_UPPER = 4, ORC_CSR_LOWER_ROWS = 5,
       ORC_CSR_UPPER_ROWS = 6 };

/* ---- edge enumeration ------------------------------------------------- */
/* Calls emit(src,dst) for every edge instance of the operator's rule, in the
 * order the generated inspector visits them.  Upper-triangular operators are
 * defined on reversed node ids v = n-1-i ("upper = lower on the index-reversed
 * matrix"), which is what the reference produces for a reversed-index loop. */
typedef struct { int64_t count; uint64_t *keys; int32_t *edge_count; } emit_t;

static inline void emit(emit_t *e, int32_t src, int32_t dst) {
    if (e->keys) e->keys[e->count] = ((uint64_t)(uint32_t)src << 32) | (uint32_t)dst;
    if (e->edge_count) e->edge_count[dst] += 1;
    e->count++;
}

static void enumerate_edges(int kind, int32_t n, const int32_t *ptr,
                            const int32_t *idx, emit_t *e) {
    for (int32_t v = 0; v < n; ++v) {
        if (kind == ORC_CSR_LOWER) {
            int32_t i = v;
            for (int32_t j = ptr[i]; j < ptr[i + 1] - 1; ++j)
                if (i > idx[j]) emit(e, idx[j], i);
        } else if (kind == ORC_CSR_LOWER_ROWS) {
            /* Gauss-Seidel rows (compiler/demo/gauss_seidel.py:18-41): the whole row is
             * visited, an entry left of the diagonal is a flow dependence */
            int32_t i = v;
            for (int32_t j = ptr[i]; j < ptr[i + 1]; ++j)
                if (i > idx[j]) emit(e, idx[j], i);
        } else if (kind == ORC_CSC_LOWER) {
            int32_t i = v;
            for (int32_t j = ptr[i] + 1; j < ptr[i + 1]; ++j)
                if (idx[j] > i) emit(e, i, idx[j]);
        } else if (kind == ORC_ILU0_CSR) {
            int32_t i = v;
            for (int32_t j = ptr[i]; j < ptr[i + 1]; ++j) {
                if (idx[j] >= i) break;
                emit(e, idx[j], i);
            }
        } else if (kind == ORC_CSR_UPPER_ROWS) {
            /* full rows visited last to first (the reversed-index loop over the U part of a
             * factor kept in place): an entry right of the diagonal is a flow dependence.  No
             * loop nest of the reference states this rule; it is "ORC_CSR_UPPER on the upper
             * triangle of the matrix" and is checked against exactly that. */
            int32_t i = n - 1 - v;
            for (int32_t j = ptr[i]; j < ptr[i + 1]; ++j)
                if (idx[j] > i) emit(e, n - 1 - idx[j], v);
        } else if (kind == ORC_CSR_UPPER) {
            int32_t i = n - 1 - v;          /* row, diagonal first */
            for (int32_t j = ptr[i] + 1; j < ptr[i + 1]; ++j)
                if (idx[j] > i) emit(e, n - 1 - idx[j], v);
        } else {                            /* ORC_CSC_UPPER: column, diagonal last */
            int32_t i = n - 1 - v;
            for (int32_t j = ptr[i]; j < ptr[i + 1] - 1; ++j)
                if (idx[j] < i) emit(e, v, n - 1 - idx[j]);
        }
    }
}

int64_t orc_dag_count_edges(int kind, int32_t n, const int32_t *ptr,
                            const int32_t *idx) {
    emit_t e = {0, NULL, NULL};
    enumerate_edges(kind, n, ptr, idx, &e);
    return e.count;
}

static void radix_sort_u64(uint64_t *a, uint64_t *tmp, int64_t m) {
    for (int pass = 0; pass < 8; ++pass) {
        int64_t hist[257];
        memset(hist, 0, sizeof hist);
        int shift = pass * 8;
        for (int64_t k = 0; k < m; ++k) hist[((a[k] >> shift) & 255) + 1]++;
        if (hist[1] == m) continue;          /* digit is all zero */
        for (int d = 0; d < 256; ++d) hist[d + 1] += hist[d];
        for (int64_t k = 0; k < m; ++k) tmp[hist[(a[k] >> shift) & 255]++] = a[k];
        memcpy(a, tmp, (size_t)m * sizeof *a);
    }
}

/*
 * Builds every array the reference's preprocessing produces.
 *   dep_count[n]      unique in-degree
 *   edge_count[n]     in-degree counting repeated edges (push protocol)
 *   dag_ptr[n+1], dag_index[*n_edges]   successors, ascending and distinct
 *   level[n]          Kahn level
 *   wavefronts[n], wavefront_ptr[*n_levels+1]
 * dag_index must have room for orc_dag_count_edges() entries.
 * Returns 0, or 1 when the graph has a cycle (nodes never scheduled).
 */
int orc_dag_build(int kind, int32_t n, const int32_t *ptr, const int32_t *idx,
                  int32_t *dep_count, int32_t *edge_count, int32_t *dag_ptr,
                  int32_t *dag_index, int64_t *n_edges, int32_t *level,
                  int32_t *wavefronts, int32_t *wavefront_ptr, int32_t *n_levels) {
    int64_t cap = orc_dag_count_edges(kind, n, ptr, idx);
    uint64_t *keys = (uint64_t *)malloc((size_t)(cap + 1) * sizeof *keys);
    uint64_t *tmp = (uint64_t *)malloc((size_t)(cap + 1) * sizeof *tmp);
    memset(edge_count, 0, (size_t)n * sizeof *edge_count);
    emit_t e = {0, keys, edge_count};
    enumerate_edges(kind, n, ptr, idx, &e);
    radix_sort_u64(keys, tmp, cap);
    free(tmp);
    /* distinct (src,dst) pairs, ascending by src then dst */
    memset(dep_count, 0, (size_t)n * sizeof *dep_count);
    memset(dag_ptr, 0, (size_t)(n + 1) * sizeof *dag_ptr);
    int64_t m = 0;
    for (int64_t k = 0; k < cap; ++k) {
        if (k && keys[k] == keys[k - 1]) continue;
        int32_t src = (int32_t)(keys[k] >> 32), dst = (int32_t)(keys[k] & 0xffffffffu);
        dag_index[m++] = dst;
        dag_ptr[src + 1] += 1;
        dep_count[dst] += 1;
    }
    free(keys);
    for (int32_t v = 0; v < n; ++v) dag_ptr[v + 1] += dag_ptr[v];
    *n_edges = m;
    /* Kahn: a node enters the level after the last of its predecessors. */
    int32_t *remaining = (int32_t *)malloc((size_t)(n + 1) * sizeof *remaining);
    int32_t *queue = (int32_t *)malloc((size_t)(n + 1) * sizeof *queue);
    memcpy(remaining, dep_count, (size_t)n * sizeof *remaining);
    int64_t head = 0, tail = 0;
    int32_t max_level = -1;
    for (int32_t v = 0; v < n; ++v) {
        level[v] = -1;
        if (remaining[v] == 0) { level[v] = 0; queue[tail++] = v; }
    }
    while (head < tail) {
        int32_t u = queue[head++];
        if (level[u] > max_level) max_level = level[u];
        for (int32_t p = dag_ptr[u]; p < dag_ptr[u + 1]; ++p) {
            int32_t w = dag_index[p];
            if (--remaining[w] == 0) { level[w] = level[u] + 1; queue[tail++] = w; }
        }
    }
    free(remaining);
    free(queue);
    int cyclic = tail != n;
    /* nodes ordered by (level, index): counting sort, stable in the index */
    int32_t nl = max_level + 1;
    *n_levels = nl;
    memset(wavefront_ptr, 0, (size_t)(nl + 1) * sizeof *wavefront_ptr);
    for (int32_t v = 0; v < n; ++v)
        if (level[v] >= 0) wavefront_ptr[level[v] + 1] += 1;
    for (int32_t l = 0; l < nl; ++l) wavefront_ptr[l + 1] += wavefront_ptr[l];
    int32_t *cursor = (int32_t *)malloc((size_t)(nl + 1) * sizeof *cursor);
    memcpy(cursor, wavefront_ptr, (size_t)(nl + 1) * sizeof *cursor);
    for (int32_t v = 0; v < n; ++v)
        if (level[v] >= 0) wavefronts[cursor[level[v]]++] = v;
    free(cursor);
    return cyclic;
}

/* Position of the entry equal to the segment id in each sorted segment, -1 if
 * absent.  Returns 0, 1 for a non-monotone pointer array, 2 for an unsorted
 * segment (the reference raises StructuralLookupError for both). */
int orc_diag_positions(int32_t n, const int32_t *ptr, const int32_t *idx,
                       int64_t nnz, int32_t *pos) {
    int64_t previous = ptr[0];
    if (previous < 0 || previous > nnz) return 1;
    for (int32_t s = 0; s < n; ++s) {
        int64_t start = ptr[s], end = ptr[s + 1];
        if (start < previous || end < start || end > nnz) return 1;
        for (int64_t p = start + 1; p < end; ++p)
            if (idx[p] < idx[p - 1]) return 2;
        int64_t lo = start, hi = end;        /* searchsorted(side="left") */
        while (lo < hi) {
            int64_t mid = (lo + hi) / 2;
            if (idx[mid] < s) lo = mid + 1; else hi = mid;
        }
        pos[s] = (lo < end && idx[lo] == s) ? (int32_t)lo : -1;
        previous = end;
    }
    return 0;
}

/* Lower CSR, diagonal last:  x[i] = (b[i] - sum Ax[j] x[Ai[j]]) / Ax[last]. */
void orc_sptrsv_csr_lower(int32_t n, const int32_t *Ap, const int32_t *Ai,
                          const double *Ax, const double *b, double *x) {
    for (int32_t i = 0; i < n; ++i) {
        double s = b[i];
        for (int32_t j = Ap[i]; j < Ap[i + 1] - 1; ++j) s -= Ax[j] * x[Ai[j]];
        x[i] = s / Ax[Ap[i + 1] - 1];
    }
}

/* Gauss-Seidel sweeps, strictly lower rows and a separate diagonal
 * (compiler/demo/gauss_seidel.py:18-26, same loop in
 * compiler/e2e_tests/test_gauss_seidel_e2e.py:19-28); x is updated in place. */
void orc_gauss_seidel_simple_csr(int32_t n, const int32_t *Ap, const int32_t *Ai,
                                 const double *Ax, const double *D, const double *b,
                                 double *x, int32_t max_iter) {
    for (int32_t sweep = 0; sweep < max_iter; ++sweep)
        for (int32_t i = 0; i < n; ++i) {
            x[i] = b[i];
            for (int32_t j = Ap[i]; j < Ap[i + 1]; ++j) x[i] -= Ax[j] * x[Ai[j]];
            x[i] /= D[i];
        }
}

/* Gauss-Seidel sweeps, the diagonal is the last stored entry equal to the row index,
 * 1.0 when absent (compiler/demo/gauss_seidel.py:29-41,
 * compiler/e2e_tests/test_gauss_seidel_e2e.py:31-43). */
void orc_gauss_seidel_full_csr(int32_t n, const int32_t *Ap, const int32_t *Ai,
                               const double *Ax, const double *b, double *x,
                               int32_t max_iter) {
    for (int32_t sweep = 0; sweep < max_iter; ++sweep)
        for (int32_t i = 0; i < n; ++i) {
            double sigma = 0.0, diag = 1.0;
            for (int32_t j = Ap[i]; j < Ap[i + 1]; ++j) {
                if (Ai[j] == i) diag = Ax[j];
                else sigma += Ax[j] * x[Ai[j]];
            }
            x[i] = (b[i] - sigma) / diag;
        }
}

/* Upper CSR, diagonal first, rows visited from the last to the first. */
void orc_sptrsv_csr_upper(int32_t n, const int32_t *Ap, const int32_t *Ai,
                          const double *Ax, const double *b, double *x) {
    for (int32_t i = n - 1; i >= 0; --i) {
        double s = b[i];
        for (int32_t j = Ap[i] + 1; j < Ap[i + 1]; ++j) s -= Ax[j] * x[Ai[j]];
        x[i] = s / Ax[Ap[i]];
    }
}

/* Lower CSC, diagonal first; x doubles as the accumulator and starts at 0. */
void orc_sptrsv_csc_lower(int32_t n, const int32_t *Ap, const int32_t *Ai,
                          const double *Ax, const double *b, double *x) {
    memset(x, 0, (size_t)n * sizeof *x);
    for (int32_t i = 0; i < n; ++i) {
        x[i] = (b[i] - x[i]) / Ax[Ap[i]];
        for (int32_t j = Ap[i] + 1; j < Ap[i + 1]; ++j) x[Ai[j]] += Ax[j] * x[i];
    }
}

/* Upper CSC, diagonal last, columns visited from the last to the first. */
void orc_sptrsv_csc_upper(int32_t n, const int32_t *Ap, const int32_t *Ai,
                          const double *Ax, const double *b, double *x) {
    memset(x, 0, (size_t)n * sizeof *x);
    for (int32_t i = n - 1; i >= 0; --i) {
        x[i] = (b[i] - x[i]) / Ax[Ap[i + 1] - 1];
        for (int32_t j = Ap[i]; j < Ap[i + 1] - 1; ++j) x[Ai[j]] += Ax[j] * x[i];
    }
}

/* Triangular solves with the factors ILU0 leaves in one CSR array: the unit
 * lower factor is the part of each row before the diagonal, the upper factor
 * the part from the diagonal on.  dpos is the diagonal table. */
void orc_sptrsv_csr_unit_lower_of_full(int32_t n, const int32_t *Ap,
                                       const int32_t *Ai, const double *Ax,
                                       const int32_t *dpos, const double *b,
                                       double *x) {
    for (int32_t i = 0; i < n; ++i) {
        double s = b[i];
        for (int32_t j = Ap[i]; j < dpos[i]; ++j) s -= Ax[j] * x[Ai[j]];
        x[i] = s;
    }
}

void orc_sptrsv_csr_upper_of_full(int32_t n, const int32_t *Ap,
                                  const int32_t *Ai, const double *Ax,
                                  const int32_t *dpos, const double *b,
                                  double *x) {
    for (int32_t i = n - 1; i >= 0; --i) {
        double s = b[i];
        for (int32_t j = dpos[i] + 1; j < Ap[i + 1]; ++j) s -= Ax[j] * x[Ai[j]];
        x[i] = s / Ax[dpos[i]];
    }
}

/* In-place ILU0 on CSR with the linear searches of the original loop nest. */
void orc_ilu0_csr(int32_t n, const int32_t *Ap, const int32_t *Ai, double *Ax) {
    for (int32_t i = 0; i < n; ++i) {
        int32_t row_start = Ap[i], row_end = Ap[i + 1];
        for (int32_t kp = row_start; kp < row_end; ++kp) {
            int32_t k = Ai[kp];
            if (k >= i) break;
            double diag = 0.0;
            for (int32_t d = Ap[k]; d < Ap[k + 1]; ++d)
                if (Ai[d] == k) { diag = Ax[d]; break; }
            if (diag != 0.0) {
                Ax[kp] = Ax[kp] / diag;
                double lik = Ax[kp];
                for (int32_t jp = kp + 1; jp < row_end; ++jp) {
                    int32_t j = Ai[jp];
                    for (int32_t q = Ap[k]; q < Ap[k + 1]; ++q)
                        if (Ai[q] == j) { Ax[jp] = Ax[jp] - lik * Ax[q]; break; }
                }
            }
        }
    }
}

/* Same factorisation with a binary search in the (sorted) pivot row: identical
 * arithmetic, usable at sizes where the linear searches take too long. */
void orc_ilu0_csr_fast(int32_t n, const int32_t *Ap, const int32_t *Ai,
                       double *Ax, const int32_t *dpos) {
    for (int32_t i = 0; i < n; ++i) {
        int32_t row_end = Ap[i + 1];
        for (int32_t kp = Ap[i]; kp < row_end; ++kp) {
            int32_t k = Ai[kp];
            if (k >= i) break;
            double diag = dpos[k] >= 0 ? Ax[dpos[k]] : 0.0;
            if (diag == 0.0) continue;
            Ax[kp] = Ax[kp] / diag;
            double lik = Ax[kp];
            for (int32_t jp = kp + 1; jp < row_end; ++jp) {
                int32_t j = Ai[jp], lo = Ap[k], hi = Ap[k + 1];
                while (lo < hi) {
                    int32_t mid = lo + (hi - lo) / 2;
                    if (Ai[mid] < j) lo = mid + 1; else hi = mid;
                }
                if (lo < Ap[k + 1] && Ai[lo] == j) Ax[jp] = Ax[jp] - lik * Ax[lo];
            }
        }
    }
}

/* In-place ILU0 on CSC storage, the right-looking loop nest of compiler/demo/spilu0.py:50-82:
 * column k is divided by its diagonal, then every later column j that has a nonzero in row k
 * gets l_ik * u_kj taken off its entry in row i.  The original finds those columns by scanning
 * all j > k; here row k's entries come from a row index built once (`rowptr`, `rowpos`: for each
 * row the positions of its entries, by ascending column), which visits the same (i, j) pairs -
 * each entry receives at most one update per pivot, so their order within a pivot is
 * immaterial.  Duplicate entries are not supported (the original would use the first match).
 * work: n + 1 + nnz int32 words. */
void orc_ilu0_csc(int32_t n, const int32_t *Ap, const int32_t *Ai, double *Ax, int32_t *work) {
    int32_t *rowptr = work, *rowpos = work + n + 1;
    int32_t nnz = Ap[n];
    for (int32_t i = 0; i <= n; ++i) rowptr[i] = 0;
    for (int32_t p = 0; p < nnz; ++p) rowptr[Ai[p] + 1]++;
    for (int32_t i = 0; i < n; ++i) rowptr[i + 1] += rowptr[i];
    for (int32_t j = 0; j < n; ++j)               /* columns ascending: rows come out sorted */
        for (int32_t p = Ap[j]; p < Ap[j + 1]; ++p) rowpos[rowptr[Ai[p]]++] = p;
    for (int32_t i = n; i > 0; --i) rowptr[i] = rowptr[i - 1];
    rowptr[0] = 0;
    /* column of a stored position, needed to walk row k */
    for (int32_t k = 0; k < n; ++k) {
        double diag = 0.0;
        for (int32_t d = Ap[k]; d < Ap[k + 1]; ++d)
            if (Ai[d] == k) { diag = Ax[d]; break; }
        for (int32_t ip = Ap[k]; ip < Ap[k + 1]; ++ip) {
            int32_t i = Ai[ip];
            if (i <= k) continue;
            if (diag != 0.0) {
                Ax[ip] = Ax[ip] / diag;
                double lik = Ax[ip];
                for (int32_t q = rowptr[k]; q < rowptr[k + 1]; ++q) {
                    int32_t kj = rowpos[q];
                    /* the column j of position kj: the one whose range holds it */
                    int32_t lo = 0, hi = n;
                    while (hi - lo > 1) {
                        int32_t mid = lo + (hi - lo) / 2;
                        if (Ap[mid] <= kj) lo = mid; else hi = mid;
                    }
                    int32_t j = lo;
                    if (j <= k) continue;
                    double ukj = Ax[kj];
                    if (ukj != 0.0)
                        for (int32_t t = Ap[j]; t < Ap[j + 1]; ++t)
                            if (Ai[t] == i) { Ax[t] = Ax[t] - lik * ukj; break; }
                }
            }
        }
    }
}

/* Supernodal lower solve, in place on x (x holds b on entry).  Panels are
 * column-major len x width with leading dimension len; Lp is 64-bit. */
void orc_sptrsv_supernodal(int32_t n_super, const int32_t *sn,
                           const int32_t *Lip, const int32_t *Li,
                           const int64_t *Lp, const double *Lx, double *x,
                           double *work /* max panel length */) {
    for (int32_t s = 0; s < n_super; ++s) {
        int32_t c0 = sn[s], w = sn[s + 1] - sn[s];
        int32_t len = Lip[s + 1] - Lip[s];
        const double *M = Lx + Lp[c0];
        double *xs = x + c0;
        for (int32_t i = 0; i < w; ++i) {
            xs[i] /= M[(int64_t)i * len + i];
            for (int32_t j = i + 1; j < w; ++j) {
                double t = M[(int64_t)i * len + j] * xs[i];
                xs[j] -= t;
            }
        }
        int32_t rows = len - w;
        const double *P = M + w;
        for (int32_t j = 0; j < rows; ++j) work[j] = 0.0;
        for (int32_t i = 0; i < w; ++i)
            for (int32_t j = 0; j < rows; ++j)
                work[j] += P[(int64_t)i * len + j] * xs[i];
        const int32_t *r = Li + Lip[s] + w;
        for (int32_t j = 0; j < rows; ++j) x[r[j]] -= work[j];
    }
}

/* Residual helpers so large checks do not need SciPy on the timing path. */
double orc_residual_csr(int32_t n, const int32_t *Ap, const int32_t *Ai,
                        const double *Ax, const double *x, const double *b,
                        double *bnorm2) {
    double r2 = 0.0, b2 = 0.0;
    for (int32_t i = 0; i < n; ++i) {
        double s = 0.0;
        for (int32_t j = Ap[i]; j < Ap[i + 1]; ++j) s += Ax[j] * x[Ai[j]];
        r2 += (s - b[i]) * (s - b[i]);
        b2 += b[i] * b[i];
    }
    *bnorm2 = b2;
    return r2;
}
