// In-place ILU(0) of a CSR matrix with sorted rows (sm_100a).
//
// Arithmetic follows the sequential loop nest exactly: for each row the pivots
// k < i are applied in ascending order, l_ik = a_ik / a_kk, then
// a_ij <- a_ij - l_ik * a_kj for the stored j > k of row i that row k also
// stores, with the product and the difference rounded separately.  The result
// is therefore bit-identical to the sequential factorisation.
//
// Sync-free mode: rows are handed out by ticket in index order; a lane group
// owns a row and keeps a fixed owner lane per stored entry, a finished row is
// announced with a release store to done[row]; a row polls done[k] of its next
// pivot without blocking (one poll per loop trip), so groups that share a warp
// never wait on each other inside a convergence region.
// Wavefront mode: one launch per level over the same row code.
// Ordered mode: the sync-free kernel with rows handed out in the order of the level sets
// instead of by index: one launch, no barrier between levels, and the rows of a level -
// independent of each other - are resident together.  lcd_spilu0_csr_ordered goes one step
// further and drops the flags: the factor is written to a second array whose entries are
// their own ready flags (ilu0_valueflag_kernel below).
#include "common.cuh"

namespace lcd {

struct Ilu0Params {
    int n;
    long long nnz;
    const int *__restrict__ Ap;
    const int *__restrict__ Ai;
    double *Ax;
    const int *__restrict__ dpos;
    int *done;
    const int *__restrict__ wavefronts;
    int32_t *status;
    unsigned long long budget_ns;
    // column-loop semantics (compiler/demo/spilu0.py:69-75): an explicitly stored zero of the
    // pivot row is treated like a missing entry - no update, so a non-finite multiplier does not
    // turn the target into NaN and its sign of zero is kept
    int skip_stored_zeros;
};

// Applies pivot row k (position kp in row i) with the lanes of one group.
// owner(jp) = (jp - row_start) % G keeps every entry of row i with one lane.
template <int G>
__device__ __forceinline__ void apply_pivot(const Ilu0Params &p, int i, int row_start, int row_end,
                                            int kp, int k, int lane, unsigned gmask) {
    const int dk = __ldg(p.dpos + k);
    const int ks = __ldg(p.Ap + k), ke = __ldg(p.Ap + k + 1);
    // group-uniform checks: the pivot row's segment is searched below and its diagonal read
    if (ks < 0 || ke < ks || (long long)ke > p.nnz || (long long)dk >= p.nnz) {
        if (lane == 0) raise_error(p.status, LCD_ERR_BAD_POINTERS, k);
        return;
    }
    double diag = 0.0;
    if (dk >= 0) diag = ld_relaxed_f64(p.Ax + dk);
    if (diag == 0.0) return;  // group-uniform: every lane read the same value
    const int owner = (kp - row_start) % G;
    double lik = 0.0;
    if (lane == owner) {
        lik = p.Ax[kp] / diag;
        p.Ax[kp] = lik;
    }
    if (G > 1) lik = __shfl_sync(gmask, lik, owner, G);
    // first own position after kp
    int jp = kp + 1 + ((lane - (kp + 1 - row_start)) % G + G) % G;
    for (; jp < row_end; jp += G) {
        const int j = __ldg(p.Ai + jp);
        int lo = ks, hi = ke;  // leftmost entry of row k that is >= j
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (__ldg(p.Ai + mid) < j) lo = mid + 1; else hi = mid;
        }
        if (lo < ke && __ldg(p.Ai + lo) == j) {
            const double ukj = ld_relaxed_f64(p.Ax + lo);
            if (!(p.skip_stored_zeros && ukj == 0.0)) p.Ax[jp] = __dsub_rn(p.Ax[jp], __dmul_rn(lik, ukj));
        }
    }
}

template <int G, int TPB>
__global__ void __launch_bounds__(TPB) ilu0_syncfree_kernel(const Ilu0Params p) {
    constexpr int R = TPB / G;
    __shared__ int s_chunk;
    if (threadIdx.x == 0) s_chunk = atomicAdd(&p.status[kStatusTicket], 1);
    __syncthreads();
    const int local = threadIdx.x / G, lane = threadIdx.x % G;
    const int task = s_chunk * R + local;
    if (task >= p.n) return;
    // rows in index order, or in the order of the level sets (any topological order): a row
    // then waits for rows of earlier tickets only, and rows of one level run side by side
    int i = task;
    if (p.wavefronts) {
        i = __ldg(p.wavefronts + task);
        if ((unsigned)i >= (unsigned)p.n) {
            if (lane == 0) raise_error(p.status, LCD_ERR_INDEX_RANGE, task);
            return;
        }
    }
    const unsigned gmask =
        G == 32 ? 0xffffffffu : (((1u << G) - 1u) << ((threadIdx.x & 31) & ~(G - 1)));
    const int s = __ldg(p.Ap + i), e = __ldg(p.Ap + i + 1);
    bool bad = s < 0 || e < s || (long long)e > p.nnz;
    if (bad && lane == 0) raise_error(p.status, LCD_ERR_BAD_POINTERS, i);
    int kp = s;
    unsigned pause = 0;
    Deadline dl;
    dl.start(p.budget_ns);
    for (;;) {
        int k = -1;
        if (!bad && kp < e) {
            k = __ldg(p.Ai + kp);
            if (k < 0 || k >= p.n) {
                if (lane == 0) raise_error(p.status, LCD_ERR_INDEX_RANGE, i);
                bad = true;
                k = -1;
            } else if (k >= i) {
                k = -1;  // reached the diagonal / upper part: the row is complete
            }
        }
        if (k >= 0) {
            int ready = 0;  // 0 not yet, 1 go, 2 give up
            if (lane == 0) {
                if (ld_relaxed_s32(p.done + k) != 0) { acquire_fence(); ready = 1; }
                else if (dl.tick(p.status, i)) ready = 2;
            }
            if (G > 1) ready = __shfl_sync(gmask, ready, 0, G);
            if (ready == 1) {
                apply_pivot<G>(p, i, s, e, kp, k, lane, gmask);
                ++kp;
                pause = 0;
            } else if (ready == 2) {
                bad = true;
            } else {
                // rows far behind the frontier stop competing for L2 with the polls that matter
                pause = pause ? min(pause * 2, 1024u) : 32u;
                __nanosleep(pause);
            }
        } else {
            // all stores of the group happen before the flag becomes visible
            if (G > 1) __syncwarp(gmask);
            if (lane == 0) {
                __threadfence();
                st_release_s32(p.done + i, 1);
            }
            break;
        }
    }
}

// ---- the same factorisation with the structure work taken off the dependence chain ----
// What a row has to wait for are VALUES of its pivot rows; WHERE those values sit (the pivot
// row's pointers, its diagonal position, the entry of the pivot row under each entry of this
// row) follows from the pattern alone.  The kernel above searches while it holds the pivot;
// this one looks everything up for the next four pivots before it polls their flags, keeps
// the row's own entries in registers (two per lane; longer rows keep the rest in memory), polls
// the four flags together and fetches the values of all pivots that are ready with one round
// of independent loads.  Per row the chain shrinks from about eight dependent loads per
// pivot to two round trips per group of pivots.  Operations on every entry are the same and
// in the same order (pivots ascending, unfused multiply / subtract), so the result is still
// bit-identical to the sequential loop.
constexpr int kIluOwn = 2;     // entries of the row a lane keeps in registers
constexpr int kIluPivots = 4;  // pivots looked up and polled together

template <int G, int TPB>
__global__ void __launch_bounds__(TPB) ilu0_lookahead_kernel(const Ilu0Params p) {
    constexpr int R = TPB / G;
    __shared__ int s_chunk;
    if (threadIdx.x == 0) s_chunk = atomicAdd(&p.status[kStatusTicket], 1);
    __syncthreads();
    const int local = threadIdx.x / G, lane = threadIdx.x % G;
    const int task = s_chunk * R + local;
    if (task >= p.n) return;
    int i = task;
    if (p.wavefronts) {
        i = __ldg(p.wavefronts + task);
        if ((unsigned)i >= (unsigned)p.n) {
            if (lane == 0) raise_error(p.status, LCD_ERR_INDEX_RANGE, task);
            return;
        }
    }
    const unsigned gmask =
        G == 32 ? 0xffffffffu : (((1u << G) - 1u) << ((threadIdx.x & 31) & ~(G - 1)));
    const int s = __ldg(p.Ap + i), e = __ldg(p.Ap + i + 1);
    bool bad = s < 0 || e < s || (long long)e > p.nnz;
    if (bad && lane == 0) raise_error(p.status, LCD_ERR_BAD_POINTERS, i);
    // the lane's own entries of row i: positions s + lane + o * G
    int col[kIluOwn];
    double val[kIluOwn];
#pragma unroll
    for (int o = 0; o < kIluOwn; ++o) {
        const int jp = s + lane + o * G;
        col[o] = -1;
        val[o] = 0.0;
        if (!bad && jp < e) { col[o] = __ldg(p.Ai + jp); val[o] = p.Ax[jp]; }
    }
    const int spill = s + kIluOwn * G;   // entries from here on stay in memory (long rows)
    int kp = s;
    unsigned pause = 0;
    Deadline dl;
    dl.start(p.budget_ns);
    while (!bad) {
        // ---- look up the next pivots (pattern only, nothing to wait for) ----
        int pk[kIluPivots], pks[kIluPivots], pke[kIluPivots], pd[kIluPivots];
        int match[kIluPivots][kIluOwn];
        int npiv = 0;
#pragma unroll
        for (int q = 0; q < kIluPivots; ++q) {
            pk[q] = -1; pks[q] = 0; pke[q] = 0; pd[q] = -1;
            if (npiv == q && kp + q < e) {
                const int k = __ldg(p.Ai + kp + q);
                if (k < 0 || k >= p.n) {
                    if (lane == 0) raise_error(p.status, LCD_ERR_INDEX_RANGE, i);
                    bad = true;
                } else if (k < i) {
                    pk[q] = k;
                    npiv = q + 1;
                }
            }
        }
        if (bad || npiv == 0) break;
#pragma unroll
        for (int q = 0; q < kIluPivots; ++q) {
            if (q < npiv) {
                pks[q] = __ldg(p.Ap + pk[q]);
                pke[q] = __ldg(p.Ap + pk[q] + 1);
                pd[q] = __ldg(p.dpos + pk[q]);
            }
        }
#pragma unroll
        for (int q = 0; q < kIluPivots; ++q) {
            if (q < npiv && (pks[q] < 0 || pke[q] < pks[q] || (long long)pke[q] > p.nnz ||
                             (long long)pd[q] >= p.nnz)) {
                if (lane == 0) raise_error(p.status, LCD_ERR_BAD_POINTERS, pk[q]);
                bad = true;
            }
        }
        if (bad) break;
#pragma unroll
        for (int q = 0; q < kIluPivots; ++q) {
#pragma unroll
            for (int o = 0; o < kIluOwn; ++o) {
                match[q][o] = -1;
                const int jp = s + lane + o * G;
                if (q < npiv && jp < e && jp > kp + q) {
                    int lo = pks[q], hi = pke[q];   // leftmost entry of the pivot row that is >= col
                    while (lo < hi) {
                        const int mid = (lo + hi) >> 1;
                        if (__ldg(p.Ai + mid) < col[o]) lo = mid + 1; else hi = mid;
                    }
                    if (lo < pke[q] && __ldg(p.Ai + lo) == col[o]) match[q][o] = lo;
                }
            }
        }
        // ---- wait for the pivots in order, as many at a time as are ready ----
        int applied = 0;
        unsigned ready_mask = 0;
        while (applied < npiv && !bad) {
            int verdict = 0;   // 2 = give up
            if (lane == 0) {
                unsigned fresh = 0;
#pragma unroll
                for (int q = 0; q < kIluPivots; ++q)
                    if (q >= applied && q < npiv && !(ready_mask >> q & 1u) &&
                        ld_relaxed_s32(p.done + pk[q]) != 0)
                        fresh |= 1u << q;
                if (fresh) { acquire_fence(); ready_mask |= fresh; }
                if (!(ready_mask >> applied & 1u) && dl.tick(p.status, i)) verdict = 2;
            }
            if (G > 1) {
                ready_mask = __shfl_sync(gmask, ready_mask, 0, G);
                verdict = __shfl_sync(gmask, verdict, 0, G);
            }
            if (verdict == 2) { bad = true; break; }
            int upto = applied;
            while (upto < npiv && (ready_mask >> upto & 1u)) ++upto;
            if (upto == applied) {
                // rows far behind the frontier stop competing for L2 with the polls that matter
                pause = pause ? min(pause * 2, 1024u) : 32u;
                __nanosleep(pause);
                continue;
            }
            pause = 0;
            // one round of independent loads: diagonals and matched entries of the ready pivots
            double dg[kIluPivots], u[kIluPivots][kIluOwn];
#pragma unroll
            for (int q = 0; q < kIluPivots; ++q) {
                dg[q] = 0.0;
                const bool on = q >= applied && q < upto;
                if (on && pd[q] >= 0) dg[q] = ld_relaxed_f64(p.Ax + pd[q]);
#pragma unroll
                for (int o = 0; o < kIluOwn; ++o)
                    u[q][o] = (on && match[q][o] >= 0) ? ld_relaxed_f64(p.Ax + match[q][o]) : 0.0;
            }
#pragma unroll
            for (int q = 0; q < kIluPivots; ++q) {
                if (q < applied || q >= upto || dg[q] == 0.0) continue;   // (group-uniform)
                const int rel = kp + q - s, owner = rel % G, slot = rel / G;
                double lik = 0.0;
                if (lane == owner) {
                    if (slot == 0) { lik = val[0] / dg[q]; val[0] = lik; }
                    else if (slot == 1) { lik = val[1] / dg[q]; val[1] = lik; }
                    else { lik = p.Ax[kp + q] / dg[q]; p.Ax[kp + q] = lik; }
                }
                if (G > 1) lik = __shfl_sync(gmask, lik, owner, G);
#pragma unroll
                for (int o = 0; o < kIluOwn; ++o)
                    if (match[q][o] >= 0 && !(p.skip_stored_zeros && u[q][o] == 0.0))
                        val[o] = __dsub_rn(val[o], __dmul_rn(lik, u[q][o]));
                // entries of a long row that live in memory: searched while the pivot is held
                for (int jp = spill + lane; jp < e; jp += G) {
                    if (jp <= kp + q) continue;
                    const int j = __ldg(p.Ai + jp);
                    int lo = pks[q], hi = pke[q];
                    while (lo < hi) {
                        const int mid = (lo + hi) >> 1;
                        if (__ldg(p.Ai + mid) < j) lo = mid + 1; else hi = mid;
                    }
                    if (lo < pke[q] && __ldg(p.Ai + lo) == j) {
                        const double ukj = ld_relaxed_f64(p.Ax + lo);
                        if (!(p.skip_stored_zeros && ukj == 0.0))
                            p.Ax[jp] = __dsub_rn(p.Ax[jp], __dmul_rn(lik, ukj));
                    }
                }
            }
            applied = upto;
        }
        kp += npiv;
        if (npiv < kIluPivots) break;   // the next entry is the diagonal or right of it
    }
    // the row's entries go back to memory, then the flag: all stores of the group happen
    // before the flag becomes visible (also after an error, so that nobody waits for this row)
#pragma unroll
    for (int o = 0; o < kIluOwn; ++o) {
        const int jp = s + lane + o * G;
        if (col[o] >= 0 && jp < e) p.Ax[jp] = val[o];
    }
    // (the release store is cumulative over what the group's lanes wrote before the barrier)
    __syncwarp(gmask);
    if (lane == 0) st_release_s32(p.done + i, 1);
}

// ---- rows in level order, values as their own ready flags --------------------------------
// The kernels above announce a finished row with a release store to done[row] and a consumer
// follows its poll with an acquire fence: two fences and two round trips through L2 per hop.
// Here the factor is written to a second array `out` that starts out filled with the reserved
// NaN pattern (the trick of the triangular solves): a row reads its own entries from A, which
// nobody modifies, polls exactly the entries of its pivot rows that it needs - the diagonal
// u_kk and the matched u_kj - in `out`, and publishes its finished entries there with relaxed
// stores.  No flags, no fences; one round trip per hop.  Arithmetic and its order are those of
// the sequential loop (pivots ascending, unfused multiply / subtract): bit-identical.
// All lanes of a warp run every trip and every vote is a full-warp ballot read through the
// group's mask, as in the ordered triangular solve.  Rows longer than kIluOwn * G entries do
// not fit the lanes' registers: the kernel reports LCD_ERR_TOO_LARGE before it touches anything
// (the caller then uses the flag-based kernel; A is still intact).
// P pivots are looked up and polled together: three measured faster than four (fewer loads and
// votes per trip; 1.17 against 1.32 ms on the 128^3 grid) and than two; three blocks of 256
// threads per SM (77 registers) faster than four with spills and than two.
constexpr int kIluTripPivots = 3;
template <int G, int P, int BPS>
__global__ void __launch_bounds__(256, BPS) ilu0_valueflag_kernel(const Ilu0Params p, double *out) {
    constexpr int R = 256 / G;
    constexpr unsigned kFull = 0xffffffffu;
    __shared__ int s_chunk;
    if (threadIdx.x == 0) s_chunk = atomicAdd(&p.status[kStatusTicket], 1);
    __syncthreads();
    const int local = threadIdx.x / G, gl = threadIdx.x % G;
    const int lane32 = threadIdx.x & 31, gbase = lane32 & ~(G - 1);
    const unsigned gmask = G == 32 ? kFull : (((1u << G) - 1u) << gbase);
    const int task = s_chunk * R + local;
    bool active = task < p.n;
    int i = task;
    if (active && p.wavefronts) {
        i = __ldg(p.wavefronts + task);
        if ((unsigned)i >= (unsigned)p.n) {
            if (gl == 0) raise_error(p.status, LCD_ERR_INDEX_RANGE, task);
            active = false;
        }
    }
    int s = 0, e = 0;
    if (active) {
        s = __ldg(p.Ap + i);
        e = __ldg(p.Ap + i + 1);
        if (s < 0 || e < s || (long long)e > p.nnz) {
            if (gl == 0) raise_error(p.status, LCD_ERR_BAD_POINTERS, i);
            active = false;
        } else if (e - s > kIluOwn * G) {
            if (gl == 0) raise_error(p.status, LCD_ERR_TOO_LARGE, i);
            active = false;
        }
    }
    // the lane's own entries of row i: positions s + gl + o * G
    int col[kIluOwn];
    double val[kIluOwn];
#pragma unroll
    for (int o = 0; o < kIluOwn; ++o) {
        const int jp = s + gl + o * G;
        col[o] = -1;
        val[o] = 0.0;
        if (active && jp < e) { col[o] = __ldg(p.Ai + jp); val[o] = p.Ax[jp]; }
    }
    int kp = s;                 // position of the next pivot in row i
    bool lookup = active;       // the next pivots have to be looked up
    bool failed = false;
    int pd[P], match[P][kIluOwn];
    int npiv = 0, applied = 0;
    bool more = false;
    unsigned pause = 0;
    Deadline dl;
    dl.start(p.budget_ns);
    for (;;) {
        // ---- pattern only: the next pivots, their diagonals, the matches of the own entries ----
        if (lookup) {
            lookup = false;
            npiv = 0;
            applied = 0;
            int pk[P], pks[P], pke[P];
#pragma unroll
            for (int q = 0; q < P; ++q) {
                pk[q] = -1; pks[q] = 0; pke[q] = 0; pd[q] = -1;
                if (npiv == q && kp + q < e && !failed) {
                    const int k = __ldg(p.Ai + kp + q);
                    if (k < 0 || k >= p.n) {
                        if (gl == 0) raise_error(p.status, LCD_ERR_INDEX_RANGE, i);
                        failed = true;
                    } else if (k < i) {
                        pk[q] = k;
                        npiv = q + 1;
                    }
                }
            }
#pragma unroll
            for (int q = 0; q < P; ++q) {
                if (q < npiv) {
                    pks[q] = __ldg(p.Ap + pk[q]);
                    pke[q] = __ldg(p.Ap + pk[q] + 1);
                    pd[q] = __ldg(p.dpos + pk[q]);
                    if (pks[q] < 0 || pke[q] < pks[q] || (long long)pke[q] > p.nnz ||
                        (long long)pd[q] >= p.nnz) {
                        if (gl == 0) raise_error(p.status, LCD_ERR_BAD_POINTERS, pk[q]);
                        failed = true;
                    }
                }
            }
            if (failed) npiv = 0;
            // a full chunk: is the entry behind it another pivot?
            more = false;
            if (npiv == P && kp + P < e) {
                const int k = __ldg(p.Ai + kp + P);
                more = k >= 0 && k < i;
            }
#pragma unroll
            for (int q = 0; q < P; ++q) {
#pragma unroll
                for (int o = 0; o < kIluOwn; ++o) {
                    match[q][o] = -1;
                    const int jp = s + gl + o * G;
                    if (q < npiv && jp < e && jp > kp + q) {
                        int lo = pks[q], hi = pke[q];   // leftmost entry of the pivot row that is >= col
                        while (lo < hi) {
                            const int mid = (lo + hi) >> 1;
                            if (__ldg(p.Ai + mid) < col[o]) lo = mid + 1; else hi = mid;
                        }
                        if (lo < pke[q] && __ldg(p.Ai + lo) == col[o]) match[q][o] = lo;
                    }
                }
            }
        }
        // ---- one non-blocking look at everything the outstanding pivots need ----
        double dg[P], u[P][kIluOwn];
        unsigned mine = 0;     // bit q: this lane has all it needs of pivot q
#pragma unroll
        for (int q = 0; q < P; ++q) {
            dg[q] = 0.0;
            const bool on = active && q >= applied && q < npiv;
            bool ok = true;
            if (on && pd[q] >= 0) {
                dg[q] = ld_relaxed_f64(out + pd[q]);
                ok = !is_pending(dg[q]);
            }
#pragma unroll
            for (int o = 0; o < kIluOwn; ++o) {
                u[q][o] = 0.0;
                if (on && match[q][o] >= 0) {
                    u[q][o] = ld_relaxed_f64(out + match[q][o]);
                    ok = ok && !is_pending(u[q][o]);
                }
            }
            if (ok) mine |= 1u << q;
        }
        // pivots are applied in order: the ready prefix, the same for all lanes of the group
        int upto = applied;
#pragma unroll
        for (int q = 0; q < P; ++q) {
            const bool all = G == 1 ? (mine >> q & 1u) != 0
                                    : (__ballot_sync(kFull, (mine >> q & 1u) != 0) & gmask) == gmask;
            if (q == upto && q < npiv && all) ++upto;
        }
        const bool progressed = active && (upto > applied || npiv == 0 || failed);
#pragma unroll
        for (int q = 0; q < P; ++q) {
            const bool on = active && q >= applied && q < upto && dg[q] != 0.0;   // (group-uniform)
            const int rel = kp + q - s, owner = rel % G, slot = rel / G;
            double lik = 0.0;
            if (on && gl == owner) {
                if (slot == 0) { lik = val[0] / dg[q]; val[0] = lik; }
                else { lik = val[1] / dg[q]; val[1] = lik; }
            }
            if (G > 1) lik = __shfl_sync(kFull, lik, gbase + owner);
            if (on) {
#pragma unroll
                for (int o = 0; o < kIluOwn; ++o)
                    if (match[q][o] >= 0 && !(p.skip_stored_zeros && u[q][o] == 0.0))
                        val[o] = __dsub_rn(val[o], __dmul_rn(lik, u[q][o]));
            }
        }
        if (progressed) {
            applied = upto;
            if (failed || applied == npiv) {
                if (more && !failed) {   // more pivots in the row
                    kp += npiv;
                    lookup = true;
                } else {
                    // the row is finished: its entries become visible one by one, each its own flag
                    const double nanv = __longlong_as_double(kCanonicalNaN);
#pragma unroll
                    for (int o = 0; o < kIluOwn; ++o) {
                        const int jp = s + gl + o * G;
                        if (jp < e) st_relaxed_f64(out + jp, failed ? nanv : publishable(val[o]));
                    }
                    active = false;
                }
            }
        }
        if (__ballot_sync(kFull, active) == 0) break;
        if (__any_sync(kFull, progressed)) {
            pause = 0;
        } else {
            if (__any_sync(kFull, active && dl.tick(p.status, i))) failed = active;
            pause = pause ? min(pause * 2, 256u) : 32u;
            __nanosleep(pause);
        }
    }
}

// Copies the finished factor over A unless the factorisation reported an error.
__global__ void __launch_bounds__(256) ilu0_commit_kernel(const int32_t *status, const double *__restrict__ out,
                                                          double *Ax, long long nnz) {
    if (status[kStatusCode] != 0) return;
    for (long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x; j < nnz;
         j += (long long)gridDim.x * blockDim.x)
        Ax[j] = out[j];
}

template <int G>
__global__ void __launch_bounds__(256) ilu0_level_kernel(const Ilu0Params p, int wave_start,
                                                        int wave_end) {
    const int gtid = blockIdx.x * blockDim.x + threadIdx.x;
    const int t = wave_start + gtid / G, lane = gtid % G;
    if (t >= wave_end) return;
    const int i = __ldg(p.wavefronts + t);
    if ((unsigned)i >= (unsigned)p.n) {
        if (lane == 0) raise_error(p.status, LCD_ERR_INDEX_RANGE, t);
        return;
    }
    const unsigned gmask =
        G == 32 ? 0xffffffffu : (((1u << G) - 1u) << ((threadIdx.x & 31) & ~(G - 1)));
    const int s = __ldg(p.Ap + i), e = __ldg(p.Ap + i + 1);
    if (s < 0 || e < s || (long long)e > p.nnz) {
        if (lane == 0) raise_error(p.status, LCD_ERR_BAD_POINTERS, i);
        return;
    }
    for (int kp = s; kp < e; ++kp) {
        const int k = __ldg(p.Ai + kp);
        if (k >= i) break;
        if (k < 0) { if (lane == 0) raise_error(p.status, LCD_ERR_INDEX_RANGE, i); break; }
        apply_pivot<G>(p, i, s, e, kp, k, lane, gmask);
    }
}

static int g_ilu0_lookahead = 1;   // LCD_TUNE_ILU0_LOOKAHEAD
int set_ilu0_lookahead(int on) {
    g_ilu0_lookahead = on ? 1 : 0;
    return LCD_OK;
}

template <int G>
static cudaError_t launch_ilu0(const Ilu0Params &p, int mode, const int32_t *wptr_host,
                               int n_levels, cudaStream_t st) {
    if (mode == 0 || mode == 2) {
        constexpr int TPB = 256, R = TPB / G;
        if (g_ilu0_lookahead)
            ilu0_lookahead_kernel<G, TPB><<<(p.n + R - 1) / R, TPB, 0, st>>>(p);
        else
            ilu0_syncfree_kernel<G, TPB><<<(p.n + R - 1) / R, TPB, 0, st>>>(p);
    } else {
        for (int l = 0; l < n_levels; ++l) {
            const int ws = wptr_host[l], we = wptr_host[l + 1];
            if (we <= ws) continue;
            const long long threads = (long long)(we - ws) * G;
            ilu0_level_kernel<G><<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(p, ws, we);
        }
    }
    return cudaGetLastError();
}

}  // namespace lcd

using namespace lcd;

extern "C" int lcd_spilu0_csr(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                              double *Ax, const int32_t *diag_pos, int mode, int32_t *done,
                              const int32_t *wavefronts, const int32_t *wavefront_ptr_host,
                              int32_t n_levels, int lanes_per_row, int32_t *status_dev,
                              int32_t timeout_ms, void *stream, int *status_host) {
    const int skip_stored_zeros = (mode & LCD_ILU0_SKIP_STORED_ZEROS) ? 1 : 0;
    mode &= ~LCD_ILU0_SKIP_STORED_ZEROS;
    if (n < 0 || nnz < 0 || !status_dev || mode < 0 || mode > 2) return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && (!Ap || !Ai || !Ax || !diag_pos)) return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && mode != 1 && !done) return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && mode == 1 && (!wavefronts || !wavefront_ptr_host || n_levels < 0))
        return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && mode == 2 && !wavefronts) return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    int G = lanes_per_row;
    if (G <= 0) {
        const double avg = n > 0 ? (double)nnz / n : 0.0;
        G = avg <= 12 ? 4 : (avg <= 40 ? 8 : (avg <= 96 ? 16 : 32));
    }
    int rc = reset_status(status_dev, st);
    if (rc) return rc;
    if (n > 0) {
        if (mode != 1) LCD_CUDA_TRY(cudaMemsetAsync(done, 0, (size_t)n * sizeof(int32_t), st));
        Ilu0Params p{n, nnz, Ap, Ai, Ax, diag_pos, done, mode == 0 ? nullptr : wavefronts, status_dev,
                     timeout_ns(timeout_ms), skip_stored_zeros};
        cudaError_t e;
        switch (G) {
            case 1: e = launch_ilu0<1>(p, mode, wavefront_ptr_host, n_levels, st); break;
            case 2: e = launch_ilu0<2>(p, mode, wavefront_ptr_host, n_levels, st); break;
            case 4: e = launch_ilu0<4>(p, mode, wavefront_ptr_host, n_levels, st); break;
            case 8: e = launch_ilu0<8>(p, mode, wavefront_ptr_host, n_levels, st); break;
            case 16: e = launch_ilu0<16>(p, mode, wavefront_ptr_host, n_levels, st); break;
            case 32: e = launch_ilu0<32>(p, mode, wavefront_ptr_host, n_levels, st); break;
            default: return LCD_ERR_INVALID_ARGUMENT;
        }
        LCD_CUDA_TRY(e);
    }
    return finish(status_dev, st, status_host);
}

extern "C" int lcd_spilu0_csr_ordered(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                                      double *Ax, const int32_t *diag_pos, const int32_t *order,
                                      double *factor_scratch, int flags, int lanes_per_row,
                                      int32_t *status_dev, int32_t timeout_ms, void *stream,
                                      int *status_host) {
    if (n < 0 || nnz < 0 || !status_dev || (flags & ~LCD_ILU0_SKIP_STORED_ZEROS))
        return LCD_ERR_INVALID_ARGUMENT;
    if (n > 0 && (!Ap || !Ai || !diag_pos || (nnz > 0 && (!Ax || !factor_scratch || factor_scratch == Ax))))
        return LCD_ERR_INVALID_ARGUMENT;
    cudaStream_t st = (cudaStream_t)stream;
    int G = lanes_per_row;
    if (G <= 0) {
        const double avg = n > 0 ? (double)nnz / n : 0.0;
        G = avg <= 7 ? 4 : (avg <= 15 ? 8 : (avg <= 31 ? 16 : 32));
    }
    int rc = reset_status(status_dev, st);
    if (rc) return rc;
    if (n > 0 && nnz > 0) {
        rc = lcd_fill_u64(reinterpret_cast<uint64_t *>(factor_scratch), nnz, kPendingBits, st);
        if (rc) return rc;
        Ilu0Params p{n, nnz, Ap, Ai, Ax, diag_pos, nullptr, order, status_dev, timeout_ns(timeout_ms),
                     (flags & LCD_ILU0_SKIP_STORED_ZEROS) ? 1 : 0};
        switch (G) {
            case 4: ilu0_valueflag_kernel<4, kIluTripPivots, 3><<<(n + 63) / 64, 256, 0, st>>>(p, factor_scratch); break;
            case 8: ilu0_valueflag_kernel<8, kIluTripPivots, 3><<<(n + 31) / 32, 256, 0, st>>>(p, factor_scratch); break;
            case 16: ilu0_valueflag_kernel<16, kIluTripPivots, 3><<<(n + 15) / 16, 256, 0, st>>>(p, factor_scratch); break;
            case 32: ilu0_valueflag_kernel<32, kIluTripPivots, 3><<<(n + 7) / 8, 256, 0, st>>>(p, factor_scratch); break;
            default: return LCD_ERR_INVALID_ARGUMENT;
        }
        LCD_CUDA_TRY(cudaGetLastError());
        // A is replaced only when the factor is complete: after an error (a row too long for the
        // lanes' registers, bad pointers, a wait that ran out) the caller still holds A
        ilu0_commit_kernel<<<sm_count() * 8, 256, 0, st>>>(status_dev, factor_scratch, Ax, nnz);
        LCD_CUDA_TRY(cudaGetLastError());
    }
    return finish(status_dev, st, status_host);
}

// ---- variant that allocates nothing -------------------------------------------
// Some callers cannot obtain device memory at the moment they need a factorisation:
// code running inside a memory pool that must not grow, a solver callback invoked
// while another library holds the allocator, or a latency-critical loop in which a
// cudaMalloc (which may synchronise the whole device) is not acceptable.  For them
// the per-row completion flags and the status block of the sync-free ILU(0) live in
// the fixed array below instead of caller-provided scratch.  Every GPU that loads the
// library carries the array (4 MiB + 256 B) until the process exits.

constexpr int kStaticStatusWords = 64;  // status block, padded to keep the flags aligned
static __device__ __align__(256) int32_t g_ilu0_static_scratch[kStaticStatusWords +
                                                              LCD_ILU0_STATIC_MAX_ROWS];

// In host code the array's name is only a handle: the device address has to be asked
// for, once per device, with that device current.
static int32_t *ilu0_static_scratch_for_current_device(int *rc) {
    constexpr int kMaxDevices = 64;
    static int32_t *address[kMaxDevices] = {nullptr};
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        if (e != cudaSuccess) set_cuda_error(e, "cudaGetDevice");
        *rc = e != cudaSuccess ? LCD_ERR_CUDA : LCD_ERR_TOO_LARGE;
        return nullptr;
    }
    if (!address[dev]) {
        void *ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_ilu0_static_scratch);
        if (e != cudaSuccess || !ptr) {
            set_cuda_error(e, "cudaGetSymbolAddress(g_ilu0_static_scratch)");
            *rc = LCD_ERR_CUDA;
            return nullptr;
        }
        address[dev] = static_cast<int32_t *>(ptr);
    }
    *rc = LCD_OK;
    return address[dev];
}

extern "C" int lcd_spilu0_csr_static(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                                     double *Ax, const int32_t *diag_pos, int lanes_per_row,
                                     int32_t timeout_ms, void *stream, int *status_host) {
    if (n < 0 || nnz < 0 || !status_host) return LCD_ERR_INVALID_ARGUMENT;
    if (n > LCD_ILU0_STATIC_MAX_ROWS) return LCD_ERR_TOO_LARGE;  // the fixed scratch holds 2^20 rows
    if (n > 0 && (!Ap || !Ai || !Ax || !diag_pos)) return LCD_ERR_INVALID_ARGUMENT;
    int rc = LCD_OK;
    int32_t *scratch = ilu0_static_scratch_for_current_device(&rc);
    if (!scratch) return rc;
    int32_t *status_dev = scratch;
    int32_t *done = scratch + kStaticStatusWords;
    cudaStream_t st = (cudaStream_t)stream;
    int G = lanes_per_row;
    if (G <= 0) {
        const double avg = n > 0 ? (double)nnz / n : 0.0;
        G = avg <= 12 ? 4 : (avg <= 40 ? 8 : (avg <= 96 ? 16 : 32));
    }
    // the array keeps the previous call's contents: clear what has to start at zero
    rc = reset_status(status_dev, st);
    if (rc) return rc;
    if (n > 0) {
        LCD_CUDA_TRY(cudaMemsetAsync(done, 0, (size_t)n * sizeof(int32_t), st));
        Ilu0Params p{n, nnz, Ap, Ai, Ax, diag_pos, done, nullptr, status_dev,
                     timeout_ns(timeout_ms), 0};
        cudaError_t e;
        switch (G) {
            case 1: e = launch_ilu0<1>(p, 0, nullptr, 0, st); break;
            case 2: e = launch_ilu0<2>(p, 0, nullptr, 0, st); break;
            case 4: e = launch_ilu0<4>(p, 0, nullptr, 0, st); break;
            case 8: e = launch_ilu0<8>(p, 0, nullptr, 0, st); break;
            case 16: e = launch_ilu0<16>(p, 0, nullptr, 0, st); break;
            case 32: e = launch_ilu0<32>(p, 0, nullptr, 0, st); break;
            default: return LCD_ERR_INVALID_ARGUMENT;
        }
        LCD_CUDA_TRY(e);
    }
    return finish(status_dev, st, status_host);
}

// ---- CSC storage -----------------------------------------------------------------------
// ILU0 of a matrix stored by columns (compiler/demo/spilu0.py:50-82) applies the same updates to
// the same entries in the same order as the row form does (every entry (i, j) is updated once
// per pivot k < min(i, j), pivots ascending; l_ik is divided once its updates are in).  So the
// column form is served by the row kernels on the row-ordered view of the values: gather them
// through the position map (row order -> column order), factor, scatter back.
namespace lcd {
__global__ void __launch_bounds__(256)
permute_f64_kernel(long long count, const int32_t *__restrict__ position, const double *__restrict__ in,
                   double *__restrict__ out, int scatter) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < count; k += stride) {
        const int32_t q = __ldg(position + k);
        if (scatter) out[q] = in[k];
        else out[k] = __ldg(in + q);
    }
}
}  // namespace lcd

extern "C" int lcd_permute_f64(int64_t count, const int32_t *position, const double *in, double *out,
                               int scatter, void *stream) {
    if (count < 0 || (count > 0 && (!position || !in || !out || in == out))) return LCD_ERR_INVALID_ARGUMENT;
    if (count == 0) return LCD_OK;
    const long long want = (count + 255) / 256;
    const int blocks = (int)(want < (long long)sm_count() * 16 ? want : (long long)sm_count() * 16);
    permute_f64_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(count, position, in, out, scatter);
    LCD_CUDA_TRY(cudaGetLastError());
    return LCD_OK;
}
