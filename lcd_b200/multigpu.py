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


def _native_local_solve(matrix, block, upper=False):
    """Solve for a column-major shard (k columns of length n, device tensor of shape
    (k, n)) with the multi-RHS kernel; returns the same layout."""
    import torch
    from . import ops
    Ap, Ai, Ax = matrix
    k, n = block.shape
    out = torch.empty_like(block)
    for first in range(0, k, MAX_RHS_PER_LAUNCH):
        last = min(first + MAX_RHS_PER_LAUNCH, k)
        cols = last - first
        rows_major = ops.transpose(block[first:last].contiguous(), cols, n)      # n x cols
        solved = ops.sptrsv_csr_syncfree_multi(Ap, Ai, Ax, rows_major.view(n, cols), upper=upper)
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
