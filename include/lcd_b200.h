/*
 * lcd_b200 -- C ABI of the B200 (sm_100a) dependence-DAG kernels.
 *
 * Every entry point is extern "C", takes raw device pointers, sizes and a CUDA
 * stream handle (cudaStream_t passed as void*), allocates no device memory and
 * returns an LCD_* code (0 = success).  Index arrays are int32, values are
 * float64.  Functions whose last parameter is `int *status_host` enqueue their
 * work on `stream`; when `status_host` is non-NULL they also synchronise the
 * stream and report the device-side status there (and as the return value),
 * when it is NULL they return right after enqueueing and the caller reads the
 * status later with lcd_read_status().
 *
 * Each declaration names the part of the reference (SwiftWare-Lab/lcd, paths
 * inside that project) whose work it replaces.
 */
#ifndef LCD_B200_H
#define LCD_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- return / status codes -------------------------------------------- */
enum {
    LCD_OK = 0,
    LCD_ERR_INVALID_ARGUMENT = 1,
    LCD_ERR_CUDA = 2,             /* a CUDA runtime call failed (see lcd_last_cuda_error) */
    LCD_ERR_WORKSPACE = 3,        /* caller-provided workspace too small */
    LCD_ERR_TIMEOUT = 4,          /* a bounded device wait expired: dependency never satisfied */
    LCD_ERR_UNSORTED = 5,         /* a segment violates the sorted-segment property */
    LCD_ERR_BAD_POINTERS = 6,     /* pointer array not monotone / out of range */
    LCD_ERR_INDEX_RANGE = 7,      /* an index lies outside [0, n) or on the wrong side of the diagonal */
    LCD_ERR_CYCLE = 8,            /* the dependence graph is not acyclic */
    LCD_ERR_MISSING_DIAGONAL = 9, /* a row needs a diagonal entry that is not stored */
    LCD_ERR_TOO_LARGE = 10,       /* a size exceeds a documented limit */
    LCD_ERR_LEVEL_CAP = 11        /* internal to lcd_dag_build_capped: the level propagation reached the
                                     requested cap (reported as a negative level count, not returned) */
};

/* Operators: which edge rule the inspector applies.  The numbering is shared by
 * the DAG build and the solvers.  Upper-triangular operators use reversed node
 * ids v = n-1-i, i.e. "upper = lower on the index-reversed matrix". */
enum {
    LCD_OP_CSR_LOWER = 0, /* rows, diagonal last   (compiler/demo/sptrsv.py:26-34)  */
    LCD_OP_CSC_LOWER = 1, /* cols, diagonal first  (compiler/demo/sptrsv.py:37-43)  */
    LCD_OP_ILU0_CSR = 2,  /* full rows, sorted     (compiler/demo/spilu0.py:21-47)  */
    LCD_OP_CSR_UPPER = 3, /* rows, diagonal first, visited last to first            */
    LCD_OP_CSC_UPPER = 4, /* cols, diagonal last,  visited last to first            */
    LCD_OP_CSR_LOWER_ROWS = 5, /* rows, every stored entry left of the diagonal is an operand,
                                 the diagonal is stored anywhere or kept apart
                                 (compiler/demo/gauss_seidel.py:18-41); DAG build only */
    LCD_OP_CSR_UPPER_ROWS = 6  /* full rows visited last to first, every stored entry right of
                                 the diagonal is an operand: the backward solve on the U part of
                                 an ILU0 factor kept in place (benchmark/spilu0_benchmark.py:
                                 166-190 splits it off instead); DAG build only */
};

/* Flags of the CSR solvers. */
enum {
    LCD_SOLVE_UPPER = 1,      /* backward substitution (rows n-1 .. 0) */
    LCD_SOLVE_UNIT_DIAG = 2,  /* implicit unit diagonal, no division (needs OF_FULL) */
    LCD_SOLVE_OF_FULL = 4,    /* the triangle is the part of a full sorted CSR row before
                                 (lower) / after (upper) diag_pos[row]; used on ILU0 factors */
    LCD_SOLVE_EXACT = 8       /* one lane per row, unfused multiply/subtract in storage order
                                 and a true division: bit-identical to the sequential loop */
};

/* Device-side status block every solver uses: 8 int32 words in device memory,
 * owned by the caller, zeroed by the entry point before the launch.
 * word 0: LCD_* code (also read as "abort" by all waiting threads),
 * word 1: node / row at which the error was detected, word 2: ticket counter. */
#define LCD_STATUS_WORDS 8

const char *lcd_error_string(int code);
const char *lcd_last_cuda_error(void);
int lcd_version(void);

/* Reads status word 0 after synchronising `stream`; *node gets word 1. */
int lcd_read_status(const int32_t *status_dev, void *stream, int32_t *node);

/* ---- DAG build ---------------------------------------------------------- */
/*
 * Replaces the generated Python inspector `extract_dag` (compiler/dag_codegen.py:
 * 1164-1196 edge rule, :1391-1402 edge multiplicity, :1421-1482 dep_count) and
 * compiler/dag_preprocessing.py:115-143 (compact_successors), :146-163
 * (wavefronts_from_dag) and :166-204 (preprocess_wavefront).  All outputs are
 * element-wise identical to those functions' outputs.
 *
 *   dep_count[n]      distinct predecessors of each node
 *   edge_count[n]     predecessors counted with repetition (push protocol)
 *   dag_ptr[n+1], dag_index[>= edge capacity]  successors, ascending and distinct
 *   level[n]          level(v) = 0 without predecessors, else 1 + max over predecessors
 *   wavefronts[n]     nodes ordered by (level, node id)
 *   wavefront_ptr[n+1]   first n_levels+1 entries are valid
 *
 * lcd_dag_workspace_bytes gives the scratch size for a matrix with `nnz` stored
 * entries.  The call synchronises `stream` (sizes are read back between phases).
 * `timeout_ms` bounds the level propagation's device-side waits (0 = default).
 */
int lcd_dag_workspace_bytes(int op, int32_t n, int64_t nnz, int64_t *bytes);
/*
 * The same build with a bound on the level propagation.  The propagation is the one sequential
 * part of the inspector (one hand-off per level); a caller that only has to know whether the DAG
 * is deep - the launcher of the sync-free CSR solve chooses the block-recurrence chain solver
 * from that alone and never reads the level sets - passes level_cap > 0: as soon as a node reaches
 * level `level_cap` the propagation stops, *n_levels_host receives -level_cap, and level,
 * wavefronts and wavefront_ptr are left unfinished (dep_count, edge_count, dag_ptr and dag_index
 * are complete).  A DAG with at most level_cap levels is built in full, as by lcd_dag_build
 * (= level_cap 0).
 */
int lcd_dag_build_capped(int op, int32_t n, const int32_t *ptr, const int32_t *idx, int64_t nnz,
                         int32_t *dep_count, int32_t *edge_count, int32_t *dag_ptr,
                         int32_t *dag_index, int64_t *n_edges_host, int32_t *level,
                         int32_t *wavefronts, int32_t *wavefront_ptr, int32_t *n_levels_host,
                         int32_t level_cap, void *workspace, int64_t workspace_bytes,
                         int32_t timeout_ms, void *stream);
int lcd_dag_build(int op, int32_t n, const int32_t *ptr, const int32_t *idx, int64_t nnz,
                  int32_t *dep_count, int32_t *edge_count, int32_t *dag_ptr,
                  int32_t *dag_index, int64_t *n_edges_host, int32_t *level,
                  int32_t *wavefronts, int32_t *wavefront_ptr, int32_t *n_levels_host,
                  void *workspace, int64_t workspace_bytes, int32_t timeout_ms,
                  void *stream);

/*
 * Band chains: the tasks of the reference's warp executor with band_width > 1
 * (compiler/dag_preprocessing.py:258-298, _band_chains).  Inside every band of band_width
 * consecutive levels, nodes connected by DAG edges form one task; tasks are listed by their
 * first node in level order, nodes inside a task in level order - element-wise what the
 * reference's union-find over Python lists returns.  Inputs are device arrays of lcd_dag_build.
 *   task_nodes[n], task_ptr[n + 1] (first *n_tasks_host + 1 entries valid),
 *   band_ptr[ceil(n_levels / band_width) + 1]  - all device arrays.
 * The call synchronises `stream`.
 */
int lcd_band_chains_workspace_bytes(int32_t n, int64_t *bytes);
int lcd_band_chains(int32_t n, const int32_t *dag_ptr, const int32_t *dag_index, const int32_t *level,
                    const int32_t *wavefronts, const int32_t *wavefront_ptr_dev, int32_t n_levels,
                    int32_t band_width, int32_t *task_nodes, int32_t *task_ptr, int32_t *band_ptr,
                    int32_t *n_tasks_host, void *workspace, int64_t workspace_bytes, void *stream);

/*
 * Rows of a Gauss-Seidel sweep over a lower-triangular matrix -> the diagonal-last rows the
 * CSR solvers read.  Replaces what the reference's generated kernels do per row
 * (compiler/demo/gauss_seidel.py:18-26: strictly lower rows, diagonal in a separate
 * array; :29-41: the diagonal is the last stored entry equal to the row index, 1.0
 * when absent).  One sweep is then one lower-triangular solve on the converted arrays.
 *   lcd_gs_layout  (structure only, once per matrix)
 *     mode 0: diagonal kept apart; mode 1: diagonal searched in the row.
 *     Ap_out: n+1 ints, Ai_out: nnz+n ints (capacity), perm: nnz ints - the slot of
 *     every stored entry in the converted arrays, -1 for an entry that is dropped (a
 *     diagonal entry superseded by a later one).  *nnz_out_host receives Ap_out[n].
 *     workspace: lcd_gs_layout_workspace_bytes(n) bytes.  Errors (status block):
 *     LCD_ERR_INDEX_RANGE for an entry right of the diagonal (only lower-triangular
 *     inputs are served) or, in mode 0, on it; LCD_ERR_BAD_POINTERS.
 *   lcd_gs_values  (every call: the values may have changed)
 *     Ax_out[perm[j]] = Ax[j]; diagonal slots (last of each row) = D[i] in mode 0,
 *     else the row's diagonal entry or 1.0.
 */
int lcd_gs_layout_workspace_bytes(int32_t n, int64_t *bytes);
int lcd_gs_layout(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai, int mode,
                  int32_t *Ap_out, int32_t *Ai_out, int32_t *perm, int64_t *nnz_out_host,
                  void *workspace, int64_t workspace_bytes, int32_t *status_dev, void *stream,
                  int *status_host);
int lcd_gs_values(int32_t n, int64_t nnz, const int32_t *Ap_out, const int32_t *perm,
                  const double *Ax, const double *D, double *Ax_out, void *stream);

/*
 * Diagonal-position table: pos[s] = first p in [ptr[s], ptr[s+1]) with idx[p] == s,
 * else -1.  Replaces compiler/structural_lookups.py:279-333 (_materialize_lookup)
 * including its validation: returns LCD_ERR_BAD_POINTERS / LCD_ERR_UNSORTED where
 * that function raises StructuralLookupError.  `status_dev`: LCD_STATUS_WORDS ints.
 */
int lcd_diag_positions(int32_t n, const int32_t *ptr, const int32_t *idx, int64_t nnz,
                       int32_t *pos, int32_t *status_dev, void *stream, int *status_host);

/* ---- sync-free SpTRSV ----------------------------------------------------- */
/*
 * CSR triangular solve with one dependency hand-off per operand and no counters:
 * x is pre-filled with a reserved NaN pattern, a consumer polls the operand
 * itself.  Replaces the generated sync-free kernels and launchers of
 * compiler/cuda_lowering.py (:519-541 plain, :1343-1410 warp/counter, :1362-1370
 * pull; launchers :673-735, :1070-1119) for the SpTRSV-CSR loop nest.
 *
 *   flags            LCD_SOLVE_* bits
 *   diag_pos         needed with LCD_SOLVE_OF_FULL, else NULL
 *   lanes_per_row    1,2,4,8,16,32 (0 = choose from nnz/n)
 *   threads_per_block  256, 512 or 1024 (0 = 1024); a block owns threads/lanes rows
 *   nnz              number of stored entries (bounds the pointer checks)
 *   x                n doubles, overwritten (must not alias b)
 *   timeout_ms       bound of every device wait (0 = default 4000)
 */
int lcd_sptrsv_csr_syncfree(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai, const double *Ax,
                            const int32_t *diag_pos, const double *b, double *x, int flags,
                            int lanes_per_row, int threads_per_block, int32_t *status_dev,
                            int32_t timeout_ms, void *stream, int *status_host);

/*
 * Block-recurrence chain solver for CSR systems whose levels hold only a few rows (long
 * dependence chains).  No counterpart in the reference, which substitutes level by level;
 * it serves the same loop nest (compiler/demo/sptrsv.py:26-34) and returns the same x up
 * to rounding.  Rows are taken in blocks of 64; lcd_chain_prepare (numeric: repeat it
 * whenever Ax changes; fully parallel) stores per block the inverse of the diagonal
 * block and its product with the coupling to the block before; lcd_sptrsv_csr_chain
 * then advances one dense 64 x 64 mat-vec (four warps) per block instead of about a dozen
 * dependent levels.
 *   workspace: lcd_chain_workspace_bytes(n) bytes (56 KiB per 64 rows), 16-byte aligned.
 *   flags: LCD_SOLVE_UPPER / OF_FULL / UNIT_DIAG as for lcd_sptrsv_csr_syncfree.
 * Explicit inverses are safe for well-conditioned diagonal blocks only: multiplying by an
 * inverse loses about log10(cond) digits that substitution keeps.  The preparation therefore
 * records a growth figure - the largest |entry| of any tile times the largest |diagonal
 * entry| of its rows, maximised over all blocks: about 1 for diagonally dominant matrices,
 * astronomically large for blocks whose inverse grows along the substitution (inf for
 * non-finite tiles).  lcd_chain_growth reads it back (it synchronises the stream); callers
 * compare it with LCD_CHAIN_MAX_GROWTH and solve with lcd_sptrsv_csr_syncfree when it is
 * larger (the decorator's launcher does).  The word lives behind the tiles in the workspace.
 */
#define LCD_CHAIN_MAX_GROWTH 100.0
int lcd_chain_growth(int32_t n, const void *workspace, int64_t workspace_bytes, void *stream,
                     double *growth_host);
int lcd_chain_workspace_bytes(int32_t n, int64_t *bytes);
/* Diagnostic: blocks per thread-block cluster of the last lcd_sptrsv_csr_chain launch of this
 * process (8 where the device hosts such clusters, else 1; 0 before the first launch). */
int lcd_chain_cluster_size(void);
int lcd_chain_prepare(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                      const double *Ax, const int32_t *diag_pos, int flags, void *workspace,
                      int64_t workspace_bytes, void *stream);
int lcd_sptrsv_csr_chain(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                         const double *Ax, const int32_t *diag_pos, const double *b, double *x,
                         int flags, const void *workspace, int64_t workspace_bytes,
                         int32_t *status_dev, int32_t timeout_ms, void *stream, int *status_host);
/*
 * The same two steps on a range [row_begin, row_end) of rows in solve order (for an upper
 * solve, position k is row n - 1 - k).  lcd_chain_prepare_rows: row_begin a multiple of 64,
 * row_end too unless it is n; reads only the matrix entries of those rows.
 * lcd_sptrsv_csr_chain_rows: row_begin a multiple of 512, row_end too unless it is n; the
 * ranges of one solve are issued in order on one stream with the same x and status_dev,
 * the first starting at 0 (it resets the status block and marks all of x as not produced),
 * the last ending at n (it reads the status back when status_host is given; the others
 * return without waiting).  A range needs the tiles, the matrix entries and the
 * right-hand side of its own rows only: a solve can run while later rows are still being
 * uploaded and prepared on other streams.
 */
int lcd_chain_prepare_rows(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                           const double *Ax, const int32_t *diag_pos, int flags, void *workspace,
                           int64_t workspace_bytes, int32_t row_begin, int32_t row_end, void *stream);
int lcd_sptrsv_csr_chain_rows(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                              const double *Ax, const int32_t *diag_pos, const double *b, double *x,
                              int flags, const void *workspace, int64_t workspace_bytes,
                              int32_t row_begin, int32_t row_end, int32_t *status_dev,
                              int32_t timeout_ms, void *stream, int *status_host);

/*
 * Multi-RHS variant: B and X are row-major n x nrhs blocks (leading dimension
 * ld >= nrhs, in doubles); lanes run over right-hand sides.
 * lcd_transpose_f64 converts between column-major and row-major blocks.
 */
int lcd_sptrsv_csr_syncfree_multi(int32_t n, int64_t nnz, int32_t nrhs, const int32_t *Ap, const int32_t *Ai,
                                  const double *Ax, const int32_t *diag_pos, const double *B,
                                  double *X, int64_t ld, int flags, int32_t *status_dev,
                                  int32_t timeout_ms, void *stream, int *status_host);
int lcd_transpose_f64(int64_t rows, int64_t cols, const double *in, int64_t ld_in, double *out,
                      int64_t ld_out, void *stream);

/*
 * CSC triangular solve, push protocol: a column waits until its counter of
 * pending contributions reaches zero, then scatters.  `dep_count` must hold the
 * edge multiplicities (edge_count of lcd_dag_build, or lcd_csc_edge_count) and
 * is consumed by the solve.  x doubles as the accumulator and is zeroed by the
 * call.  Replaces the push-protocol kernel of compiler/cuda_lowering.py:2031-2059.
 * flags: LCD_SOLVE_UPPER only.
 */
int lcd_sptrsv_csc_syncfree(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai, const double *Ax,
                            const double *b, double *x, int32_t *dep_count, int flags,
                            int lanes_per_col, int32_t *status_dev, int32_t timeout_ms,
                            void *stream, int *status_host);
int lcd_csc_edge_count(int32_t n, const int32_t *Ap, const int32_t *Ai, int flags,
                       int32_t *edge_count, void *stream);

/* ---- wavefront SpTRSV ------------------------------------------------------- */
/*
 * Level-by-level solve over `wavefronts` / `wavefront_ptr` (device arrays as built
 * by lcd_dag_build).  mode 0: one launch per level on `stream`; mode 1: a single
 * cooperative launch with a grid-wide barrier between levels, runs of levels that
 * fit one thread block being handled by one block with block-level barriers.
 * Replaces the generated wavefront kernels and launchers of
 * compiler/cuda_lowering.py:1233-1291, :855-1016 (CSR and CSC loop nests).
 * op: LCD_OP_CSR_LOWER / CSR_UPPER / CSC_LOWER / CSC_UPPER.  For CSC x is zeroed
 * by the call and accumulates with atomics.
 */
enum { LCD_WAVEFRONT_PER_LEVEL = 0, LCD_WAVEFRONT_COOPERATIVE = 1 };
int lcd_sptrsv_wavefront(int op, int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                         const double *Ax, const int32_t *diag_pos, const double *b, double *x,
                         int flags, const int32_t *wavefronts, const int32_t *wavefront_ptr_dev,
                         const int32_t *wavefront_ptr_host, int32_t n_levels, int mode,
                         int lanes_per_row, int32_t *status_dev, int32_t timeout_ms, void *stream,
                         int *status_host);

/*
 * The same solve over band chains, the reference's warp tasks with band_width > 1
 * (compiler/dag_preprocessing.py:207-298, per-band launcher compiler/cuda_lowering.py:1022-1068):
 * task t is the chain of nodes task_nodes[task_ptr[t] .. task_ptr[t+1]) (connected inside a
 * band of consecutive levels, in level order) and is solved by one lane group, node after
 * node; band k holds the tasks band_ptr[k] .. band_ptr[k+1]) and bands are separated like
 * levels above.  task_ptr has n_tasks+1 entries, band_ptr n_bands+1 (device and host copy).
 */
int lcd_sptrsv_wavefront_tasks(int op, int32_t n, int64_t nnz, const int32_t *Ap,
                               const int32_t *Ai, const double *Ax, const int32_t *diag_pos,
                               const double *b, double *x, int flags, const int32_t *task_nodes,
                               const int32_t *task_ptr_dev, const int32_t *band_ptr_dev,
                               const int32_t *band_ptr_host, int32_t n_bands, int mode,
                               int lanes_per_row, int32_t *status_dev, int32_t timeout_ms,
                               void *stream, int *status_host);

/* Multi-RHS level-synchronous CSR solve on row-major n x nrhs blocks (nrhs <= 64): a warp
 * per row, lanes over right-hand sides, one cooperative launch.  The choice between this
 * and lcd_sptrsv_csr_syncfree_multi follows the level width (wide levels: this one). */
int lcd_sptrsv_wavefront_multi(int32_t n, int64_t nnz, int32_t nrhs, const int32_t *Ap,
                               const int32_t *Ai, const double *Ax, const int32_t *diag_pos,
                               const double *B, double *X, int64_t ld, int flags,
                               const int32_t *wavefronts, const int32_t *wavefront_ptr_dev,
                               int32_t n_levels, int32_t *status_dev, int32_t timeout_ms,
                               void *stream, int *status_host);

/*
 * Sync-free CSR solve that hands its rows out in a caller-given topological order, for one or
 * many right-hand sides (row-major n x nrhs blocks, nrhs <= 64, leading dimension ld >= nrhs in
 * doubles; nrhs = 1 with ld = 1 is the plain vector solve).  `order` lists node ids (for an upper
 * solve v = n - 1 - row) so that every operand of a row stands before the row: the level
 * sets `wavefronts` of lcd_dag_build are such an order, and so is 0..n-1.  Level order keeps
 * thousands of independent rows in flight on grid-like matrices where index order leaves one
 * grid line; unlike the level-synchronous kernels below nothing waits for a whole level - a
 * row waits for its own operands only - so there is neither a grid barrier nor a launch per
 * level.  Serves the SpTRSV-CSR loop nest (compiler/demo/sptrsv.py:26-34) and, on ILU0
 * factors (LCD_SOLVE_OF_FULL), the forward / backward solves of
 * benchmark/spilu0_benchmark.py:166-190; the reference's closest counterpart is the
 * persistent warp-task launcher, compiler/cuda_lowering.py:1070-1119, which also walks
 * `task_nodes` in level order.
 *   task_records  16 n + 2048 bytes of scratch, 16-byte aligned (the tail holds the ticket
 *               counters, cleared by every call): one record per task {row, first entry,
 *               entry count, diagonal position}, written by a first pass over (order, Ap,
 *               diag_pos) unless records_ready != 0, which reuses what an earlier call with the
 *               same Ap, diag_pos, flags and order left there (order may then be NULL).
 *   row_flags   NULL: X is pre-filled with a reserved NaN pattern and consumers poll the
 *               operands themselves (one extra write pass over X);
 *               n ints of scratch: producers release a flag per row instead (no pass over X,
 *               two L2 round trips per hand-off instead of one).  Zeroed by the call.
 *   window_rows upper bound on the rows in flight (0: as many as the device holds).  Rows far
 *               ahead of the frontier only poll; about four average levels is a good window.
 *   flags       LCD_SOLVE_UPPER / OF_FULL / UNIT_DIAG (not EXACT: operands are consumed in
 *               chunks of four as they arrive).
 * An `order` that lacks a node ends in LCD_ERR_TIMEOUT (bounded waits), never in a hang.
 */
int lcd_sptrsv_csr_ordered(int32_t n, int64_t nnz, int32_t nrhs, const int32_t *Ap,
                           const int32_t *Ai, const double *Ax, const int32_t *diag_pos,
                           const double *B, double *X, int64_t ld, int flags,
                           const int32_t *order, int32_t *task_records, int records_ready,
                           int32_t *row_flags, int64_t window_rows, int32_t *status_dev,
                           int32_t timeout_ms, void *stream, int *status_host);

/*
 * Level walks with the hand-off in shared memory: CSR and CSC (compiler/demo/sptrsv.py:26-43)
 * triangular solves whose cost is the hand-off between levels, not bandwidth.
 *   blocks = 1: solves small enough for one thread block (a few hundred thousand rows at most).
 *       One block walks the level sets with a block barrier per level and keeps the recent part
 *       of x in shared memory; nothing spins.
 *   blocks > 1 (at most one per SM; cooperative launch): block b owns the nodes
 *       [n b / blocks, n (b + 1) / blocks) and walks its tasks of every level.  Operands of the
 *       own block come from shared memory behind the block barrier; operands another block owns
 *       are requested a turn ahead and, if still missing, polled in the position-ordered x in
 *       global memory (pre-filled with the reserved NaN pattern; bounded waits, LCD_ERR_TIMEOUT).
 *       The operands of a triangular solve have smaller node numbers, i.e. they belong to the
 *       same or an earlier block: the blocks form a pipeline that pays one hand-off through L2
 *       per block, not per level.
 * Replaces the generated wavefront launchers (compiler/cuda_lowering.py:855-1016: a launch plus a
 * device synchronisation per level) and the sync-free kernels (:1343-1410, push :2031-2059).  The
 * CSC loop (push) is served by the same pull walk on the transposed structure - no atomics,
 * results do not depend on timing.
 *   Task slots: every slice of a level is padded to a multiple of 32 slots, so that the lanes of
 *       a warp always work in the same level (the scoreboard of outstanding loads belongs to the
 *       warp).  Slots are numbered block by block.  Within a level the tasks are sorted by node,
 *       so a block's tasks of a level are consecutive: lcd_small_level_cuts writes
 *       cuts[b * n_levels + l] = tasks of level l that belong to blocks < b (blocks x n_levels
 *       ints).  From them the caller computes slot_ptr[b * (n_levels + 1) + l] = first slot of
 *       block b's tasks of level l (running sum, block by block, of the slice sizes rounded up to
 *       32; entry n_levels of block b = first slot of block b + 1; n_slots = the last entry).
 *       One block: cuts may be NULL, slot_ptr has n_levels + 1 entries.
 *   lcd_small_plan_measure / lcd_small_plan_fill   once per pattern: `pos` (n ints) receives the
 *       slot of every node (order, level, wavefront_ptr: wavefronts, level and wavefront_ptr of
 *       lcd_dag_build for the same op); info_host[0] = most operands of one task (longest row
 *       without its diagonal), [1] = widest slice.  The fill writes one record per slot with
 *       `entries` = 2, 4 or 8 >= info_host[0] operand slots (more operands than
 *       lcd_small_max_entries(): not served): rec_pc / rec_src [n_slots * entries] = slot of the
 *       operand and index of its value in Ax, -1 for padding; row_of[n_slots] (-1: padding
 *       slot), diag_src[n_slots].  *far_host = operands of the own block more than half the
 *       shared-memory ring back (read from global memory).  cursor: n_slots ints of scratch (CSC
 *       ops only).  Errors through status_dev: LCD_ERR_INDEX_RANGE, LCD_ERR_BAD_POINTERS,
 *       LCD_ERR_CYCLE (an operand that is not in an earlier level).  info_dev: 4 ints of scratch.
 *   lcd_sptrsv_small   every solve: walks the levels.  With gather_values != 0 the call first
 *       gathers the coefficients and reciprocal diagonals into slot order in `scratch` (a
 *       parallel pass: needed on the first call and whenever Ax has changed; with 0 the values of
 *       the previous call stay - the usual case of one matrix and many right-hand sides).  A
 *       task's record is fetched two turns before the task runs, its right-hand side one turn
 *       before, straight from b; x is written by position into `scratch` (what the operands
 *       read) and in matrix order into x.  scratch: lcd_small_scratch_bytes(n_slots, entries)
 *       bytes, 256-byte aligned; rec_pc 16-byte aligned.  Asynchronous on `stream` unless
 *       status_host is given.
 *       LCD_ERR_TOO_LARGE: more blocks than the device can keep resident.
 *   lcd_sptrsv_small_multi   the same walk for nrhs = 1, 2, 4, 8 or 16 right-hand sides (no
 *       reference counterpart; the reference's launchers take one): b and x are row-major
 *       n x nrhs blocks with leading dimension ld (doubles), blocks > 1 for nrhs > 1.  The walk
 *       runs on nrhs interleaved copies of the pattern - task s * nrhs + r is slot s for
 *       right-hand side r and reads slot s's record - so a level's hand-off is still one block
 *       barrier plus the polls of operands that other blocks own.  scratch:
 *       lcd_small_scratch_bytes_multi bytes.  LCD_ERR_TOO_LARGE also when n_slots * nrhs or
 *       n * ld does not fit 31 bits.
 *   op: LCD_OP_CSR_LOWER / CSR_UPPER / CSC_LOWER / CSC_UPPER; flags: LCD_SOLVE_OF_FULL /
 *   UNIT_DIAG for the CSR ops.
 */
int lcd_small_max_entries(void);
int lcd_small_level_cuts(int32_t n, int32_t blocks, int32_t n_levels, const int32_t *order,
                         const int32_t *wavefront_ptr_dev, int32_t *cuts_dev, void *stream);
int lcd_small_plan_measure(int op, int flags, int32_t n, int64_t nnz, const int32_t *Ap,
                           const int32_t *Ai, const int32_t *diag_pos, const int32_t *order,
                           const int32_t *level, const int32_t *wavefront_ptr_dev,
                           const int32_t *slot_ptr_dev, const int32_t *cuts_dev, int32_t n_levels,
                           int32_t blocks, int32_t n_slots, int32_t *pos, int32_t *cursor,
                           int32_t *info_dev, int32_t *status_dev, void *stream, int32_t *info_host);
int lcd_small_plan_fill(int op, int flags, int32_t n, int64_t nnz, const int32_t *Ap,
                        const int32_t *Ai, const int32_t *diag_pos, const int32_t *order,
                        const int32_t *level, const int32_t *slot_ptr_dev, int32_t n_levels,
                        int32_t blocks, const int32_t *pos, int32_t n_slots, int32_t entries,
                        int32_t *rec_pc, int32_t *rec_src, int32_t *row_of, int32_t *diag_src,
                        int32_t *cursor, int32_t *info_dev, int32_t *status_dev, void *stream,
                        int32_t *far_host);
int lcd_small_scratch_bytes(int32_t n_slots, int32_t entries, int64_t *bytes);
int lcd_sptrsv_small(int32_t n, int32_t n_slots, int32_t entries, const double *Ax, const double *b,
                     double *x, const int32_t *rec_pc, const int32_t *rec_src, const int32_t *row_of,
                     const int32_t *diag_src, const int32_t *slot_ptr_dev, int32_t n_levels,
                     int32_t blocks, int32_t max_width, int32_t gather_values, void *scratch,
                     int64_t scratch_bytes, int32_t *status_dev, int32_t timeout_ms, void *stream,
                     int *status_host);
int lcd_small_scratch_bytes_multi(int32_t n_slots, int32_t entries, int32_t nrhs, int64_t *bytes);
int lcd_sptrsv_small_multi(int32_t n, int32_t n_slots, int32_t entries, const double *Ax,
                           const double *b, double *x, int32_t nrhs, int64_t ld,
                           const int32_t *rec_pc, const int32_t *rec_src, const int32_t *row_of,
                           const int32_t *diag_src, const int32_t *slot_ptr_dev, int32_t n_levels,
                           int32_t blocks, int32_t max_width, int32_t gather_values, void *scratch,
                           int64_t scratch_bytes, int32_t *status_dev, int32_t timeout_ms,
                           void *stream, int *status_host);

/* ---- CSC -> supernodal layout ------------------------------------------------------ */
/*
 * Supernodal layout of a lower-triangular matrix stored by columns (sorted rows): replaces
 * detect_supernodes + convert_csc_to_supernodal (utils/symbolic_cholesky_csc.py:883-921,
 * 950-1021).  Column j + 1 joins column j's supernode when the symmetric difference of their row
 * patterns has at most relaxation + 1 elements; the row structure of a supernode (Li[Lip[s] ..
 * Lip[s+1])) is the sorted union of its columns' patterns; column j holds one value per row of
 * that union at Lx[Lp[j] ..] (zero where it stores none).  Two calls because the sizes of Li and
 * Lx depend on the pattern:
 *   lcd_supernodal_layout - structure: col_to_super (n), super_begin (n + 1 ints, the first
 *     n_super + 1 meaningful), Lip (n + 1 ints, likewise), Li (nnz ints, the first Lip[n_super]
 *     meaningful), Lp (n + 1 64-bit offsets).  summary_host[4] = {n_super, Lip[n_super], widest
 *     supernode, Lp[n]}.  Synchronises the stream.
 *   lcd_supernodal_fill - values: zeroes Lx[0 .. panel_values) and scatters Cx into it; repeat
 *     when the values change.
 * The arrays feed lcd_sptrsv_supernodal unchanged (sn = super_begin).
 */
int lcd_supernodal_layout_workspace_bytes(int32_t n, int64_t nnz, int64_t *bytes);
int lcd_supernodal_layout(int32_t n, int64_t nnz, const int32_t *Cp, const int32_t *Ci,
                          int32_t relaxation, int32_t *col_to_super, int32_t *super_begin,
                          int32_t *Lip, int32_t *Li, int64_t *Lp, int64_t *summary_host,
                          void *workspace, int64_t workspace_bytes, void *stream);
int lcd_supernodal_fill(int32_t n, int64_t nnz, const int32_t *Cp, const int32_t *Ci,
                        const double *Cx, const int32_t *col_to_super, const int32_t *Lip,
                        const int32_t *Li, const int64_t *Lp, double *Lx, int64_t panel_values,
                        int32_t *status_dev, void *stream, int *status_host);

/* ---- SpILU0 (CSR, in place) -------------------------------------------------- */
/*
 * In-place ILU(0) of a CSR matrix with sorted rows; arithmetic identical to the
 * sequential loop nest of compiler/demo/spilu0.py:21-47 (pivots in ascending
 * order, unfused multiply/subtract).  Replaces the nested-thread-map kernel of
 * compiler/cuda_lowering.py:1572-1989.  mode: 0 = sync-free (per-row done flags in
 * `done`, n ints, zeroed by the call), 1 = per-level launches over wavefronts,
 * 2 = sync-free with the rows handed out in the order of `wavefronts` (needs `done` and
 * `wavefronts`; one launch, rows of a level run side by side, no barrier between levels).
 * LCD_ILU0_SKIP_STORED_ZEROS may be added to the mode: an explicitly stored zero of a pivot row
 * then causes no update, which is what the column loop does (compiler/demo/spilu0.py:69-75:
 * `if u_kj != 0.0`); the row loop (:36-44) updates with l_ik * 0.  The two differ only for
 * non-finite multipliers and in the sign of zero.
 */
#define LCD_ILU0_SKIP_STORED_ZEROS 8
int lcd_spilu0_csr(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai, double *Ax,
                   const int32_t *diag_pos, int mode, int32_t *done,
                   const int32_t *wavefronts, const int32_t *wavefront_ptr_host,
                   int32_t n_levels, int lanes_per_row, int32_t *status_dev, int32_t timeout_ms,
                   void *stream, int *status_host);

/*
 * The same factorisation in one launch with rows handed out in `order` (the level sets of
 * lcd_dag_build with LCD_OP_ILU0_CSR; NULL = by index) and the factor's entries as their own
 * ready flags: the factor is built in `factor_scratch` (nnz doubles, pre-filled by the call with a
 * reserved NaN pattern), a row polls exactly the entries of its pivot rows that it needs there
 * and publishes its own with plain stores - no flags, no fences, one L2 round trip per
 * dependence.  A is only read until the factor is complete and replaced by it at the end; after
 * an error it is unchanged.  Bit-identical to lcd_spilu0_csr.  Rows must fit the lanes'
 * registers (2 entries per lane, lanes_per_row = 4 / 8 / 16 / 32, 0 = from nnz / n): a longer row
 * gives LCD_ERR_TOO_LARGE - use lcd_spilu0_csr (mode 2) then.  flags: 0 or
 * LCD_ILU0_SKIP_STORED_ZEROS.  Replaces the same reference kernel (compiler/cuda_lowering.py:1572-1989).
 */
int lcd_spilu0_csr_ordered(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai, double *Ax,
                           const int32_t *diag_pos, const int32_t *order, double *factor_scratch,
                           int flags, int lanes_per_row, int32_t *status_dev, int32_t timeout_ms,
                           void *stream, int *status_host);

/*
 * ILU(0) for callers that cannot allocate.  No counterpart in the reference: it exists
 * for users of this library that call it where device memory cannot be requested (inside
 * a fixed memory pool, in a callback that runs while the allocator is held elsewhere, or
 * in a loop where a device-wide synchronising cudaMalloc is not acceptable).
 * Same factorisation and same result as lcd_spilu0_csr in sync-free mode, but the
 * completion flags and the status block live in a fixed array inside the library
 * (4 MiB per GPU, held until the process exits) instead of caller scratch; the call
 * performs no cudaMalloc / cudaFree and calls no allocating routine.
 *   - n is limited to LCD_ILU0_STATIC_MAX_ROWS (1,048,576); larger n returns
 *     LCD_ERR_TOO_LARGE.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress); make that first call outside any stream capture.
 *   - All calls on one device share the array: calls that overlap on the GPU (two
 *     streams, two host threads) race.  Issue them one after the other.
 *   - status_host is required; the call synchronises `stream` and reports there.
 */
#define LCD_ILU0_STATIC_MAX_ROWS (1 << 20)
int lcd_spilu0_csr_static(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                          double *Ax, const int32_t *diag_pos, int lanes_per_row,
                          int32_t timeout_ms, void *stream, int *status_host);
/*
 * ILU0 on CSC storage (compiler/demo/spilu0.py:50-82, the right-looking column loop) is served by
 * the row kernels (mode + LCD_ILU0_SKIP_STORED_ZEROS): the column form updates the same entries in the same order, so the values are
 * gathered into row order through a position map (position[k] = place in the column-ordered
 * array of the k-th entry in row order; the host side builds it with the row pointers, column
 * indices and diagonal positions of the row-ordered view), factored with lcd_spilu0_csr and
 * scattered back.  lcd_permute_f64: scatter = 0: out[k] = in[position[k]]; scatter = 1:
 * out[position[k]] = in[k]; in and out must not alias; positions are not range-checked.
 */
int lcd_permute_f64(int64_t count, const int32_t *position, const double *in, double *out, int scatter,
                    void *stream);

/* ---- supernodal SpTRSV ------------------------------------------------------- */
/*
 * Lower-triangular solve on the supernodal layout of
 * utils/symbolic_cholesky_csc.py:950-1021 (column-major panels, own columns
 * first in each row list), in place on x (x holds b on entry).  Replaces
 * benchmark/sptrsv_supernodal.py:12-28 / :55-94 and the dense helpers
 * utils/dense_blas.py:19-33, :228-242.  Lp is 64-bit.
 *   pending[n_super]  number of panel-row updates each supernode still waits for
 *                     (lcd_supernodal_pending computes it; consumed by the solve)
 */
int lcd_supernodal_pending(int32_t n_super, const int32_t *sn, const int32_t *Lip,
                           const int32_t *Li, const int32_t *col_to_super, int32_t *pending,
                           void *stream);
/*
 * Tasks: the solve is cut into tasks listed in supernode order; task t works on
 * supernode task_super[t]; task_strip[t] == 0 solves the diagonal block and then,
 * like every other strip, multiplies lcd_supernodal_strip_rows() rows of the
 * off-diagonal panel starting at row task_strip[t] * strip_rows.  Every supernode
 * needs its strip-0 task even when it has no off-diagonal rows.
 *   solved[n]         scratch (doubles): x as published for the waiting strips
 *   supernode widths are limited to 1024 columns (LCD_ERR_TOO_LARGE)
 */
int lcd_supernodal_strip_rows(void);
int lcd_sptrsv_supernodal(int32_t n, int32_t n_super, int32_t n_tasks,
                          const int32_t *task_super, const int32_t *task_strip,
                          const int32_t *sn, const int32_t *Lip, const int32_t *Li,
                          const int64_t *Lp, const double *Lx, const int32_t *col_to_super,
                          int32_t *pending, double *solved, double *x, const int64_t *inv_ptr,
                          const double *inv, int32_t *status_dev, int32_t timeout_ms, void *stream,
                          int *status_host);
/*
 * Optional numeric preparation (repeat when Lx changes): the inverse of every supernode's
 * w x w diagonal block, column-major with leading dimension w, is written to
 * inv[inv_ptr[s] ..); inv_ptr[s] = sum of w_t^2 over t < s (n_super + 1 entries, device).
 * With them the solve multiplies by the inverse - independent loads and multiply-adds -
 * instead of substituting through w dependent steps; with inv_ptr == NULL it substitutes.
 * growth_dev (optional, one double in device memory): receives the largest value over all
 * supernodes of (largest |entry| of the inverse) x (largest |diagonal entry| of the block);
 * about 1 for diagonally dominant blocks.  Multiplying by an explicit inverse loses about
 * log10 of that figure in digits, which substitution keeps: above LCD_CHAIN_MAX_GROWTH solve
 * with inv_ptr == NULL instead (lcd_b200.supernodal.analyse does).
 */
int lcd_supernodal_prepare(int32_t n_super, const int32_t *sn, const int32_t *Lip,
                           const int64_t *Lp, const double *Lx, const int64_t *inv_ptr,
                           double *inv, double *growth_dev, void *stream);

/* ---- block-row partition of one solve across the GPUs of a node ---------------- */
/*
 * No counterpart in the reference (it is single-GPU).  One process per GPU; rank q owns
 * the nodes [bounds[q], bounds[q+1]) and holds a full-length x array in its own memory.
 * A rank that produces a value some other rank needs stores it straight into that rank's
 * x array through a peer mapping (NVLink); consumers only ever poll their own memory.
 *   lcd_peer_alloc / lcd_peer_open / lcd_peer_close / lcd_peer_free
 *       allocate an x array that other processes of the node can map (CUDA IPC handle,
 *       64 bytes) -- the only entry points of the library that allocate device memory.
 *   lcd_partition_need_mask
 *       need_mask[c] (one byte per row, array padded to a multiple of 4 bytes) gets bit q
 *       when a row owned by rank q uses column c produced by another rank.
 *   lcd_sptrsv_csr_syncfree_part
 *       solves the nodes [task_begin, task_end) of a CSR triangular system.  x must have
 *       been filled with the reserved pattern (lcd_fill_u64(x, n, ~0)) on EVERY rank, and
 *       all ranks must have synchronised, before any rank makes this call.  peer_x is a
 *       host array of n_ranks device pointers (rank q's x as mapped in this process).
 */
int lcd_peer_alloc(int64_t bytes, void **ptr, unsigned char *handle64);
int lcd_peer_open(const unsigned char *handle64, void **ptr);
int lcd_peer_close(void *ptr);
int lcd_peer_free(void *ptr);
int lcd_partition_need_mask(int32_t n, const int32_t *Ap, const int32_t *Ai, int flags,
                            const int32_t *bounds_dev, int32_t parts, unsigned char *need_mask,
                            void *stream);
int lcd_sptrsv_csr_syncfree_part(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                                 const double *Ax, const double *b, double *x, int flags,
                                 int32_t task_begin, int32_t task_end,
                                 const unsigned char *need_mask, double *const *peer_x,
                                 int32_t n_ranks, int threads_per_block, int32_t *status_dev,
                                 int32_t timeout_ms, void *stream, int *status_host);

/* The same partition with each rank's rows handed out in the order of the global level sets
 * (lcd_sptrsv_csr_ordered's kernel): order_local lists this rank's n_local nodes in that order;
 * task_records: 16 n_local + 2048 bytes of scratch (records_ready as for lcd_sptrsv_csr_ordered).
 * Operands that may come from a peer are polled with system-scope loads.  x must have been
 * filled and all ranks synchronised as for lcd_sptrsv_csr_syncfree_part.  flags: LCD_SOLVE_UPPER. */
int lcd_sptrsv_csr_ordered_part(int32_t n, int64_t nnz, const int32_t *Ap, const int32_t *Ai,
                                const double *Ax, const double *b, double *x, int flags,
                                const int32_t *order_local, int32_t n_local, int32_t *task_records,
                                int records_ready, const unsigned char *need_mask,
                                double *const *peer_x, int32_t n_ranks, int64_t window_rows,
                                int32_t *status_dev, int32_t timeout_ms, void *stream,
                                int *status_host);

/* Scheduling knobs of the one-lane-per-row sync-free kernel (process-wide).  They
 * change waiting behaviour only, never results.  The reference's counterpart is the
 * schedule search of compiler/scheduler.py:172-303 (block size / unroll / protocol). */
enum {
    LCD_TUNE_SLEEP_LOCAL_NS = 0,  /* pause after a failed poll inside the own chunk */
    LCD_TUNE_SLEEP_GLOBAL_NS = 1, /* pause after a failed poll of another chunk's row */
    LCD_TUNE_GAP_NS = 2,          /* extra pause per row the producer's warp still owes */
    LCD_TUNE_ROW_VARIANT = 3,     /* 0: thread-per-row kernel, 1: generic lane-group kernel */
    LCD_TUNE_STAGE_PERCENT = 4,   /* shared-memory staging of a chunk's matrix entries, in percent
                                     of the average chunk size (0 = read entries from global) */
    LCD_TUNE_CHAIN_CLUSTER = 5,   /* blocks per cluster of the chain solver: 0 = as many as the device
                                     hosts (up to 8), 1 = plain blocks, 2 / 4 / 8 = at most that */
    LCD_TUNE_ORDERED_PAUSE_NS = 6, /* lcd_sptrsv_csr_ordered: longest pause of a warp between two
                                     unsuccessful polls (0 = never pause; default 256) */
    LCD_TUNE_SMALL_THREADS = 7,   /* lcd_sptrsv_small: threads of the one block, 256 / 512 / 1024
                                     (0 = 512 while no level is wider than that, else 1024) */
    LCD_TUNE_ILU0_LOOKAHEAD = 8,  /* lcd_spilu0_csr sync-free modes: 1 (default) = pattern look-ups
                                     for the next pivots before their flags are polled, own entries
                                     in registers; 0 = search while the pivot is held.  Same result. */
    LCD_TUNE_ORDERED_MIN_LANES = 9 /* lcd_sptrsv_csr_ordered: lanes per row at least: 1, 2 (default), 4
                                     or 8 (with 2 a warp holds 16 rows, which measured twice as fast
                                     as 32 rows per warp even with one right-hand side); a value
                                     100 * W + KR picks the kernel variant outright (tuning runs) */
};
int lcd_set_tuning(int key, int value);
/* Profiling aid (no reference counterpart): with a non-NULL device array of 64-bit words,
 * the one-lane-per-row solver (n words) and the chain solver (2 n + 29 C words, C the number
 * of 512-row chunks: row stamps, per-chunk start times, wait counters and the helpers'
 * publication stamps) record SM cycle counters and timer values; the ordered solve (3 n words:
 * timer when a row's batch came up, when the row was published, its waiting trips) and the level
 * walk (12 n_levels + 4096 words: cycle counter after every level and around the first thread's
 * tasks; shared walk: timer after every level of the first, middle and last block) likewise.
 * Pass NULL to switch it off again. */
int lcd_debug_set_trace(long long *trace_dev);

/*
 * Machine constants for the scheduler's cost model, measured on the current device: replaces the
 * micro-benchmarks of compiler/scheduler.py:714-775 (empty launches and an atomic kernel timed
 * through Numba).  out_host receives LCD_CALIBRATION_VALUES doubles (LCD_CAL_* indices; a value that
 * could not be measured stays 0).  workspace: at least 64 MiB of device memory, 256-byte aligned
 * (the larger, the closer the copy figure is to the HBM rate).  Synchronises the stream; takes a
 * few milliseconds.
 */
enum {
    LCD_CAL_LAUNCH_S = 0,         /* one kernel launch in a back-to-back sequence */
    LCD_CAL_L2_HANDOFF_S = 1,     /* one hand-off between two thread blocks through global memory */
    LCD_CAL_SMEM_HANDOFF_S = 2,   /* one hand-off between two warps of a block through shared memory */
    LCD_CAL_BLOCK_BARRIER_S = 3,  /* one __syncthreads() of 512 threads */
    LCD_CAL_ATOMIC_S = 4,         /* one atomicAdd on an address every thread of the grid adds to */
    LCD_CAL_GRID_BARRIER_S = 5,   /* one grid-wide barrier, one block of 512 threads per SM */
    LCD_CAL_COPY_BYTES_PER_S = 6, /* device-to-device copy, read + write bytes */
    LCD_CAL_L2_LOAD_S = 7,        /* one dependent ld.relaxed.gpu that hits L2 (mean of 4096 over 32 MB;
                                     SM clock taken at its nominal rate) */
    LCD_CAL_L2_LOAD_P10_S = 8,    /* ... its 10th percentile (lines homed near the SM) */
    LCD_CAL_L2_LOAD_P90_S = 9,    /* ... its 90th percentile (lines homed on the other die) */
    LCD_CALIBRATION_VALUES = 10
};
int lcd_calibrate(void *workspace, int64_t workspace_bytes, void *stream, double *out_host);

/* ---- small device utilities used by the host layer ---------------------------- */
int lcd_fill_u64(uint64_t *dst, int64_t count, uint64_t value, void *stream);
/* 128-bit order-sensitive checksum of an int32 device array, used as the plan-cache
 * key in place of the host-side content hash of compiler/scheduler.py:678-711.
 * out_dev: two 64-bit words of device scratch; out_host (optional): the result,
 * read back after synchronising the stream. */
int lcd_checksum_i32(const int32_t *data, int64_t count, uint64_t *out_dev, uint64_t *out_host,
                     void *stream);
int lcd_device_sm_count(int *sm_count);

#ifdef __cplusplus
}
#endif
#endif /* LCD_B200_H */
