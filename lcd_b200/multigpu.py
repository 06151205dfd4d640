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


# Levels at least this wide (on average) are solved level by level: every gather is a
# coalesced row of the right-hand-side block and nothing waits inside a level.  Narrower
# level structures are dependence chains and go to the sync-free kernel.
WAVEFRONT_MIN_AVERAGE_WIDTH = 256
_level_sets = {}


def _levels_for(matrix, upper):
    """Level sets of a device matrix, built once per matrix object."""
    from . import ops
    Ap, Ai, _ = matrix
    key = (Ap.data_ptr(), Ai.data_ptr(), Ap.numel(), Ai.numel(), bool(upper))
    dag = _level_sets.get(key)
    if dag is None:
        if len(_level_sets) >= 8:
            _level_sets.pop(next(iter(_level_sets)))
        dag = _level_sets[key] = ops.dag_build("csr_upper" if upper else "csr_lower", Ap, Ai)
    return dag


def _native_local_solve(matrix, block, upper=False):
    """Solve for a column-major shard (k columns of length n, device tensor of shape
    (k, n)) with a multi-RHS kernel chosen from the level width; same layout out."""
    import torch
    from . import ops
    Ap, Ai, Ax = matrix
    k, n = block.shape
    out = torch.empty_like(block)
    dag = _levels_for(matrix, upper)
    wide = dag.n_levels > 0 and n / dag.n_levels >= WAVEFRONT_MIN_AVERAGE_WIDTH
    for first in range(0, k, MAX_RHS_PER_LAUNCH):
        last = min(first + MAX_RHS_PER_LAUNCH, k)
        cols = last - first
        rows_major = ops.transpose(block[first:last].contiguous(), cols, n).view(n, cols)
        if wide:
            solved = ops.sptrsv_wavefront_multi(Ap, Ai, Ax, rows_major, dag.wavefronts,
                                                dag.wavefront_ptr, upper=upper)
        else:
            solved = ops.sptrsv_csr_syncfree_multi(Ap, Ai, Ax, rows_major, upper=upper)
        ops.transpose(solved, n, cols, out=out[first:last])
    return out


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

    def solve(self, B, gather=False):
        """``B``: the full column-major ``n x nrhs`` block (host array, every rank
        passes the same) or this rank's shard as a ``(k, n)`` tensor.  Returns the
        local shard ``(k, n)``; with ``gather=True`` the full ``(nrhs, n)`` block on
        every rank (row q = solution for right-hand side q)."""
        import torch
        if isinstance(B, np.ndarray):
            if B.ndim != 2 or B.shape[0] != self.n:
                raise ValueError("B must be n x nrhs")
            nrhs = B.shape[1]
            start, stop = self.shard(nrhs)
            local = torch.from_numpy(np.ascontiguousarray(B[:, start:stop].T)).to(self.device)
        else:
            local, nrhs = B, None
        solved = self.local_solver(self.matrix, local, self.upper)
        if not gather:
            return solved
        if nrhs is None:
            raise ValueError("gather=True needs the full block to know every shard size")
        if self.world == 1:
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
    final gather uses NCCL)."""

    def __init__(self, Ap, Ai, Ax, upper=False, group=None, threads=0):
        import ctypes
        import torch
        import torch.distributed as dist
        from . import _native as nat
        from .ops import _stream, new_status
        if not dist.is_initialized():
            raise RuntimeError("PartitionedSolve needs an initialised process group")
        self.dist, self.group = dist, group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        if self.world > 8:
            raise ValueError("at most 8 ranks (one node)")
        self.upper, self.threads = upper, threads
        dev = torch.device("cuda", torch.cuda.current_device())
        up = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a, dtype=dt)).to(dev)
        self.Ap, self.Ai, self.Ax = up(Ap, np.int32), up(Ai, np.int32), up(Ax, np.float64)
        self.n = len(Ap) - 1
        self.bounds = row_partition(self.n, self.world)
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
        torch.cuda.synchronize()
        dist.barrier(group=group)

    def solve(self, b, gather=True, timeout_ms=0):
        """``b``: full right-hand side (host array or device tensor, same on every
        rank).  Returns x: the full vector on every rank (``gather=True``) or this
        rank's block."""
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
        rc = self._lib.lcd_sptrsv_csr_syncfree_part(
            self.n, self.Ai.numel(), nat.ptr(self.Ap), nat.ptr(self.Ai), nat.ptr(self.Ax),
            nat.ptr(b_dev), nat.ptr(self.x), nat.SOLVE_UPPER if self.upper else 0, t0, t1,
            nat.ptr(self.need) if self.world > 1 else None, self.peer_ptrs, self.world,
            int(self.threads), nat.ptr(self.status), int(timeout_ms), _stream(),
            ctypes.byref(host))
        nat.check(rc, "lcd_sptrsv_csr_syncfree_part")
        lo, hi = (self.n - t1, self.n - t0) if self.upper else (t0, t1)
        mine = self.x[lo:hi].clone()
        self.dist.barrier(group=self.group)       # peers may still be reading / writing x
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
        import torch
        torch.cuda.synchronize()
        self.dist.barrier(group=self.group)
        self.x = None
        self.buffer.release()
