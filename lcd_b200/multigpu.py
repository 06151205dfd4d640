"""Multi-GPU execution of the triangular solves (one process per GPU).

The reference is single-GPU (no collective, no peer access anywhere in it); what
is built here follows the ways the path shards naturally:

* **multi-RHS**: the matrix is replicated, the right-hand-side columns are split
  into contiguous shards, every rank solves its shard with the multi-RHS kernel and
  no data crosses GPUs during the solve; a final ``all_gather`` (NCCL) assembles X
  when asked for.
* **replicas**: ILU0 and the supernodal solve run as independent replicas.

Plumbing only uses ``torch.distributed``; the local solve is the C-ABI kernel and
raises without a GPU (tests on CPU inject their own local solver to exercise the
sharding and gathering logic with the gloo backend).
"""

from __future__ import annotations

import numpy as np

MAX_RHS_PER_LAUNCH = 64


def column_shard(nrhs, world, rank):
    """Contiguous, balanced column range of one rank: the first ``nrhs % world``
    ranks get one extra column."""
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    base, extra = divmod(int(nrhs), int(world))
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


# Levels at least this wide (on average) are solved with the level-ordered sync-free kernel:
# rows of a level run side by side and every gather is a coalesced row of the right-hand-side
# block.  Narrower level structures are dependence chains and go to the index-ordered kernel,
# whose chunks hand values over through shared memory.
ORDERED_MIN_AVERAGE_WIDTH = 256
# Measured on B200 (192^3 grid, 64 right-hand sides on one GPU): point-to-point kernel 4.7 ms,
# level-synchronous kernel (a grid barrier per level) 5.0 ms; with fewer right-hand sides per
# GPU the barrier per level dominates (8 columns: 1.9 ms against 4.5 ms).  The barrier kernel
# is kept for blocks wider than this many columns, i.e. for none at the current limit of 64.
BARRIER_FROM_RHS = 64
_level_sets = {}


def _levels_for(matrix, upper):
    """(level sets, ordered plan) of a device matrix, built once per matrix object."""
    from . import ops
    Ap, Ai, _ = matrix
    key = (Ap.data_ptr(), Ai.data_ptr(), Ap.numel(), Ai.numel(), bool(upper))
    entry = _level_sets.get(key)
    if entry is None:
        if len(_level_sets) >= 8:
            _level_sets.pop(next(iter(_level_sets)))
        dag = ops.dag_build("csr_upper" if upper else "csr_lower", Ap, Ai)
        entry = _level_sets[key] = (dag, ops.OrderedPlan(dag.wavefronts, dag.n_levels))
    return entry


def _solve_rows(matrix, rows_major, upper, out=None):
    """Solve for a row-major n x k block (k <= 64) with the kernel the level width asks for."""
    from . import ops
    Ap, Ai, Ax = matrix
    n = rows_major.shape[0]
    dag, plan = _levels_for(matrix, upper)
    if dag.n_levels > 0 and n / dag.n_levels >= ORDERED_MIN_AVERAGE_WIDTH:
        if rows_major.shape[1] > BARRIER_FROM_RHS:
            return ops.sptrsv_wavefront_multi(Ap, Ai, Ax, rows_major, dag.wavefronts,
                                              dag.wavefront_ptr, out, upper=upper)
        return ops.sptrsv_csr_ordered(Ap, Ai, Ax, rows_major, plan, out, upper=upper)
    return ops.sptrsv_csr_syncfree_multi(Ap, Ai, Ax, rows_major, out, upper=upper)


def _native_local_solve(matrix, block, upper=False, layout="columns"):
    """Solve for this rank's shard on the GPU.  ``layout="columns"``: the shard is column-major
    (k columns of length n, a device tensor of shape (k, n)) and is transposed into the
    row-major blocks the kernels read, 64 columns at a time, and back; ``layout="rows"``: the
    shard already is a row-major n x k block (k <= 64) and goes to the kernel as it is."""
    import torch
    from . import ops
    if layout == "rows":
        n, k = block.shape
        if k > MAX_RHS_PER_LAUNCH:
            raise ValueError(f"a row-major shard holds at most {MAX_RHS_PER_LAUNCH} columns")
        return _solve_rows(matrix, block, upper)
    k, n = block.shape
    out = torch.empty_like(block)
    for first in range(0, k, MAX_RHS_PER_LAUNCH):
        last = min(first + MAX_RHS_PER_LAUNCH, k)
        cols = last - first
        rows_major = ops.transpose(block[first:last].contiguous(), cols, n).view(n, cols)
        solved = _solve_rows(matrix, rows_major, upper)
        ops.transpose(solved, n, cols, out=out[first:last])
    return out


def agree_on_status(dist, group, code, device):
    """MAX of the ranks' status codes (0 = fine): every rank learns that some rank failed
    before anybody raises, so no rank is left alone in a later collective."""
    import torch
    word = torch.tensor([int(code)], dtype=torch.int32, device=device)
    dist.all_reduce(word, op=dist.ReduceOp.MAX, group=group)
    return int(word.item())


class RemoteRankError(RuntimeError):
    """Another rank of the process group reported an error in the step all ranks just did."""

    def __init__(self, code, where):
        self.code = int(code)
        super().__init__(f"{where}: a rank of the process group failed with status {code}")


def _local_status(error):
    """Status code of an exception raised by a local solver (native codes are positive)."""
    code = getattr(error, "code", None)
    return int(code) if isinstance(code, int) and code > 0 else 255


class ShardedMultiRHS:
    """Triangular solve with many right-hand sides sharded by column over the ranks
    of a process group (default: the world group)."""

    def __init__(self, Ap, Ai, Ax, upper=False, group=None, device=None, local_solver=None):
        import torch
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.upper = upper
        self.local_solver = local_solver or _native_local_solve
        if local_solver is None:
            device = torch.device(device if device is not None else
                                  f"cuda:{torch.cuda.current_device()}")
            up = lambda a, dt: (a if isinstance(a, torch.Tensor) else
                                torch.from_numpy(np.ascontiguousarray(a, dtype=dt))).to(device)
            self.matrix = (up(Ap, np.int32), up(Ai, np.int32), up(Ax, np.float64))
            self.device = device
        else:
            self.matrix = (Ap, Ai, Ax)
            self.device = torch.device("cpu" if device is None else device)
        self.n = len(Ap) - 1

    def shard(self, nrhs):
        return column_shard(nrhs, self.world, self.rank)

    def solve(self, B, gather=False, layout="columns", agree=None):
        """``B``: the full column-major ``n x nrhs`` block (host array, every rank
        passes the same) or this rank's shard as a device tensor: ``(k, n)``
        (``layout="columns"``) or a row-major ``(n, k)`` block with k <= 64
        (``layout="rows"``, no transposition).  Returns the local shard in the layout it
        came in; with ``gather=True`` the full ``(nrhs, n)`` block on every rank (row q =
        solution for right-hand side q).

        ``agree`` (default: whenever a collective follows, i.e. with ``gather``): the ranks
        exchange their status before anybody raises, so that an error on one rank raises on
        all of them instead of leaving the others alone in the gather."""
        import torch
        if isinstance(B, np.ndarray):
            if B.ndim != 2 or B.shape[0] != self.n:
                raise ValueError("B must be n x nrhs")
            nrhs = B.shape[1]
            start, stop = self.shard(nrhs)
            local = torch.from_numpy(np.ascontiguousarray(B[:, start:stop].T)).to(self.device)
            layout = "columns"
        else:
            local, nrhs = B, None
        if gather and nrhs is None:
            raise ValueError("gather=True needs the full block to know every shard size")
        agree = (gather and self.world > 1) if agree is None else (agree and self.world > 1)
        failure, solved = None, None
        try:
            if layout == "columns":
                solved = self.local_solver(self.matrix, local, self.upper)
            else:
                solved = self.local_solver(self.matrix, local, self.upper, layout)
        except Exception as error:      # keep the code: the other ranks have to hear of it
            if not agree:
                raise
            failure = error
        if agree:
            status = agree_on_status(self.dist, self.group,
                                     _local_status(failure) if failure is not None else 0,
                                     self.device)
            if failure is not None:
                raise failure
            if status:
                raise RemoteRankError(status, "ShardedMultiRHS.solve")
        if not gather or self.world == 1:
            return solved
        # shards may differ by one column: pad to the widest so that every rank
        # contributes a tensor of the same shape, then drop the padding
        sizes = [column_shard(nrhs, self.world, r) for r in range(self.world)]
        widest = max(e - s for s, e in sizes)
        padded = torch.zeros((widest, self.n), dtype=solved.dtype, device=solved.device)
        padded[:solved.shape[0]] = solved
        parts = [torch.empty_like(padded) for _ in range(self.world)]
        self.dist.all_gather(parts, padded, group=self.group)
        return torch.cat([part[:e - s] for part, (s, e) in zip(parts, sizes)], dim=0)


def row_partition(n, world):
    """Node boundaries of a balanced contiguous block-row partition (world + 1 ints)."""
    return np.asarray([(n * q) // world for q in range(world + 1)], dtype=np.int32)


class _PeerBuffer:
    """A device array other processes of the node can map (CUDA IPC)."""

    def __init__(self, nbytes):
        import ctypes
        from . import _native as nat
        self.nbytes = int(nbytes)
        self._lib = nat.load()
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        nat.check(self._lib.lcd_peer_alloc(self.nbytes, ctypes.byref(ptr), handle), "lcd_peer_alloc")
        self.ptr = ptr.value
        self.handle = handle.raw
        self.mapped = []

    def open_peer(self, handle):
        import ctypes
        from . import _native as nat
        ptr = ctypes.c_void_p()
        nat.check(self._lib.lcd_peer_open(handle, ctypes.byref(ptr)), "lcd_peer_open")
        self.mapped.append(ptr.value)
        return ptr.value

    @property
    def __cuda_array_interface__(self):
        return {"shape": (self.nbytes // 8,), "typestr": "<f8", "data": (self.ptr, False),
                "version": 3, "strides": None}

    def release(self):
        import ctypes
        for ptr in self.mapped:
            self._lib.lcd_peer_close(ctypes.c_void_p(ptr))
        self.mapped = []
        if self.ptr:
            self._lib.lcd_peer_free(ctypes.c_void_p(self.ptr))
            self.ptr = None


class PartitionedSolve:
    """One triangular solve (CSR, lower or upper) split into contiguous block rows,
    one per GPU.  Cross-partition operands travel as plain 8-byte peer stores into the
    consumer's own x array; there is no collective on the data path (the optional
    final gather uses NCCL).

    ``local_solver(rank, bounds, b) -> (status, block)`` replaces the GPU part (tests of the
    partition / agreement / gather logic on CPU ranks); no device memory is touched then."""

    def __init__(self, Ap, Ai, Ax, upper=False, group=None, threads=0, ordered=None,
                 local_solver=None, device=None):
        import torch
        import torch.distributed as dist
        if not dist.is_initialized():
            raise RuntimeError("PartitionedSolve needs an initialised process group")
        self.dist, self.group = dist, group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        if self.world > 8:
            raise ValueError("at most 8 ranks (one node)")
        self.upper, self.threads = upper, threads
        self.n = len(Ap) - 1
        self.bounds = row_partition(self.n, self.world)
        self.local_solver = local_solver
        self.buffer = self.order_local = self.records = None
        if local_solver is not None:
            self.device = torch.device("cpu" if device is None else device)
            return
        import ctypes
        from . import _native as nat, ops
        from .ops import _stream, new_status
        dev = torch.device("cuda", torch.cuda.current_device())
        up = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a, dtype=dt)).to(dev)
        self.Ap, self.Ai, self.Ax = up(Ap, np.int32), up(Ai, np.int32), up(Ax, np.float64)
        self.status = new_status(dev)
        self.device = dev
        lib = nat.load()
        self._lib = lib
        # which ranks need each value
        self.need = torch.zeros((self.n + 3) // 4 * 4, dtype=torch.uint8, device=dev)
        bounds_dev = up(self.bounds, np.int32)
        nat.check(lib.lcd_partition_need_mask(self.n, nat.ptr(self.Ap), nat.ptr(self.Ai),
                                              nat.SOLVE_UPPER if upper else 0, nat.ptr(bounds_dev),
                                              self.world, nat.ptr(self.need), _stream()),
                  "lcd_partition_need_mask")
        # peer-visible x arrays
        self.buffer = _PeerBuffer(max(self.n, 1) * 8)
        handles = [None] * self.world
        dist.all_gather_object(handles, self.buffer.handle, group=group)
        self.peer_ptrs = (ctypes.c_void_p * self.world)()
        for q, handle in enumerate(handles):
            self.peer_ptrs[q] = self.buffer.ptr if q == self.rank else self.buffer.open_peer(handle)
        self.x = torch.as_tensor(self.buffer, device=dev)
        # rows of this rank in the order of the global level sets (wide levels: rows of a level
        # run side by side; the index-ordered kernel keeps one grid line in flight)
        dag = ops.dag_build("csr_upper" if upper else "csr_lower", self.Ap, self.Ai)
        self.levels = dag.n_levels
        wide = dag.n_levels > 0 and self.n / dag.n_levels >= ORDERED_MIN_AVERAGE_WIDTH
        if wide if ordered is None else ordered:
            t0, t1 = int(self.bounds[self.rank]), int(self.bounds[self.rank + 1])
            nodes = dag.wavefronts
            self.order_local = nodes[(nodes >= t0) & (nodes < t1)].contiguous()
            self.records = torch.empty(self.order_local.numel() * 4 + 512, dtype=torch.int32, device=dev)
            self.records_ready = False
            self.window = max(4 * self.n // max(dag.n_levels, 1) // self.world, 148 * 8 * 32)
        del dag
        torch.cuda.synchronize()
        dist.barrier(group=group)

    def _solve_on_gpu(self, b, timeout_ms):
        """(status, this rank's block of x); the status is returned, not raised."""
        import ctypes
        import torch
        from . import _native as nat, ops
        from .ops import _stream
        b_dev = b if isinstance(b, torch.Tensor) else torch.from_numpy(
            np.ascontiguousarray(b, dtype=np.float64)).to(self.device)
        ops.fill_u64(self.x, 0xFFFFFFFFFFFFFFFF)
        torch.cuda.synchronize()
        self.dist.barrier(group=self.group)       # nobody publishes into an unfilled array
        host = ctypes.c_int(0)
        t0, t1 = int(self.bounds[self.rank]), int(self.bounds[self.rank + 1])
        flags = nat.SOLVE_UPPER if self.upper else 0
        need = nat.ptr(self.need) if self.world > 1 else None
        if self.order_local is not None:
            rc = self._lib.lcd_sptrsv_csr_ordered_part(
                self.n, self.Ai.numel(), nat.ptr(self.Ap), nat.ptr(self.Ai), nat.ptr(self.Ax),
                nat.ptr(b_dev), nat.ptr(self.x), flags, nat.ptr(self.order_local),
                self.order_local.numel(), nat.ptr(self.records), 1 if self.records_ready else 0,
                need, self.peer_ptrs, self.world, int(self.window), nat.ptr(self.status),
                int(timeout_ms), _stream(), ctypes.byref(host))
            self.records_ready = rc == 0
        else:
            rc = self._lib.lcd_sptrsv_csr_syncfree_part(
                self.n, self.Ai.numel(), nat.ptr(self.Ap), nat.ptr(self.Ai), nat.ptr(self.Ax),
                nat.ptr(b_dev), nat.ptr(self.x), flags, t0, t1, need, self.peer_ptrs, self.world,
                int(self.threads), nat.ptr(self.status), int(timeout_ms), _stream(),
                ctypes.byref(host))
        lo, hi = (self.n - t1, self.n - t0) if self.upper else (t0, t1)
        return rc, self.x[lo:hi].clone()

    def solve(self, b, gather=True, timeout_ms=0):
        """``b``: full right-hand side (host array or device tensor, same on every
        rank).  Returns x: the full vector on every rank (``gather=True``) or this
        rank's block.

        The closing barrier runs whatever the local outcome was, and the ranks agree on the
        status before anybody raises: an error is per rank (a bad row in one block), and a
        rank that raised early would leave the others alone in the barrier and the gather."""
        import torch
        if self.local_solver is not None:
            rc, mine = self.local_solver(self.rank, self.bounds, b)
        else:
            rc, mine = self._solve_on_gpu(b, timeout_ms)
        self.dist.barrier(group=self.group)       # peers may still be reading / writing x
        status = agree_on_status(self.dist, self.group, rc, self.device) if self.world > 1 else rc
        if rc:
            from ._native import check
            check(rc, "PartitionedSolve.solve")
        if status:
            raise RemoteRankError(status, "PartitionedSolve.solve")
        if not gather or self.world == 1:
            return mine
        widest = int(np.max(np.diff(self.bounds)))
        padded = torch.zeros(widest, dtype=torch.float64, device=self.device)
        padded[:mine.numel()] = mine
        parts = [torch.empty_like(padded) for _ in range(self.world)]
        self.dist.all_gather(parts, padded, group=self.group)
        blocks = [parts[q][:int(self.bounds[q + 1] - self.bounds[q])] for q in range(self.world)]
        if self.upper:
            blocks = blocks[::-1]
        return torch.cat(blocks)

    def close(self):
        if self.buffer is None:
            return
        import torch
        torch.cuda.synchronize()
        self.dist.barrier(group=self.group)
        self.x = None
        self.buffer.release()
        self.buffer = None
