"""Sharding and gathering logic of the multi-GPU layer on CPU: two gloo ranks, the
local solve replaced by the CPU oracle (the native local solve needs a GPU)."""
import os
import sys

import numpy as np
import pytest

from conftest import ROOT


def test_column_shards_are_contiguous_and_balanced():
    from lcd_b200.multigpu import column_shard
    for nrhs, world in ((64, 8), (5, 2), (3, 4), (64, 1), (7, 3)):
        bounds = [column_shard(nrhs, world, r) for r in range(world)]
        assert bounds[0][0] == 0 and bounds[-1][1] == nrhs
        assert all(a[1] == b[0] for a, b in zip(bounds, bounds[1:]))
        sizes = [e - s for s, e in bounds]
        assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        column_shard(4, 2, 2)


def _worker(rank, world, port, result_dir):
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from lcd_b200 import generators as gen
    from lcd_b200.multigpu import ShardedMultiRHS
    from oracle import oracle as cpu

    def oracle_solver(matrix, block, upper):
        Ap, Ai, Ax = matrix
        rows = [cpu.sptrsv_csr_lower(Ap, Ai, Ax, block[q].numpy()) for q in range(block.shape[0])]
        return torch.from_numpy(np.stack(rows)) if rows else block.clone()

    tri = gen.laplacian3d_tril(6, seed=1, nrhs=5)           # 5 columns over 2 ranks: 3 + 2
    Ap, Ai, Ax = tri.csr_arrays()
    solver = ShardedMultiRHS(Ap, Ai, Ax, local_solver=oracle_solver)
    local = solver.solve(np.asarray(tri.b))
    start, stop = solver.shard(5)
    assert local.shape == (stop - start, tri.n)
    full = solver.solve(np.asarray(tri.b), gather=True)
    np.save(os.path.join(result_dir, f"x{rank}.npy"), full.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_multi_rhs_two_ranks_gloo(tmp_path, oracle):
    import torch.multiprocessing as mp
    from lcd_b200 import generators as gen
    port = 29500 + os.getpid() % 2000
    mp.spawn(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    tri = gen.laplacian3d_tril(6, seed=1, nrhs=5)
    Ap, Ai, Ax = tri.csr_arrays()
    want = np.stack([oracle.sptrsv_csr_lower(Ap, Ai, Ax, np.ascontiguousarray(tri.b[:, q])) for q in range(5)])
    for rank in range(2):
        got = np.load(tmp_path / f"x{rank}.npy")
        np.testing.assert_array_equal(got, want)


def _failure_worker(rank, world, port, result_dir):
    """Rank 1's local step fails (a host-made failure); both ranks must raise, nobody may be
    left alone in the gather, and the group must stay usable afterwards."""
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from lcd_b200 import _native as nat, generators as gen
    from lcd_b200.multigpu import PartitionedSolve, RemoteRankError, ShardedMultiRHS
    from oracle import oracle as cpu
    tri = gen.laplacian3d_tril(5, seed=1, nrhs=4)
    Ap, Ai, Ax = tri.csr_arrays()
    outcome = {}

    def failing_columns(matrix, block, upper):
        if dist.get_rank() == 1:
            raise nat.NativeError(nat.ERR_TIMEOUT, "injected", "a wait expired")
        return block.clone()

    try:
        ShardedMultiRHS(Ap, Ai, Ax, local_solver=failing_columns).solve(np.asarray(tri.b), gather=True)
        outcome["columns"] = "returned"
    except nat.NativeError as error:
        outcome["columns"] = ("local", error.code)
    except RemoteRankError as error:
        outcome["columns"] = ("remote", error.code)

    # block rows: each rank solves its rows of the full system with the oracle
    x_full = cpu.sptrsv_csr_lower(Ap, Ai, Ax, np.ascontiguousarray(tri.b[:, 0]))

    def rows_solver(fail_on):
        def solve(rank_, bounds, b):
            block = torch.from_numpy(x_full[bounds[rank_]:bounds[rank_ + 1]].copy())
            return (nat.ERR_INDEX_RANGE if rank_ == fail_on else 0), block
        return solve

    solver = PartitionedSolve(Ap, Ai, Ax, local_solver=rows_solver(fail_on=0))
    try:
        solver.solve(tri.b[:, 0])
        outcome["rows"] = "returned"
    except nat.NativeError as error:
        outcome["rows"] = ("local", error.code)
    except RemoteRankError as error:
        outcome["rows"] = ("remote", error.code)
    # the group is still in step: a clean solve gathers the whole vector on both ranks
    good = PartitionedSolve(Ap, Ai, Ax, local_solver=rows_solver(fail_on=-1)).solve(tri.b[:, 0])
    outcome["gathered_ok"] = bool(np.array_equal(good.numpy(), x_full))
    up = PartitionedSolve(Ap, Ai, Ax, upper=True, local_solver=lambda r, bounds, b: (
        0, torch.from_numpy(x_full[len(x_full) - bounds[r + 1]:len(x_full) - bounds[r]].copy())))
    outcome["upper_ok"] = bool(np.array_equal(up.solve(tri.b[:, 0]).numpy(), x_full))
    import json
    with open(os.path.join(result_dir, f"outcome{rank}.json"), "w") as handle:
        json.dump(outcome, handle)
    dist.barrier()
    dist.destroy_process_group()


def test_one_failing_rank_raises_on_every_rank_gloo(tmp_path):
    import json
    import torch.multiprocessing as mp
    from lcd_b200 import _native as nat
    port = 31500 + os.getpid() % 2000
    mp.spawn(_failure_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    r0 = json.load(open(tmp_path / "outcome0.json"))
    r1 = json.load(open(tmp_path / "outcome1.json"))
    assert r0["columns"] == ["remote", nat.ERR_TIMEOUT] and r1["columns"] == ["local", nat.ERR_TIMEOUT]
    assert r0["rows"] == ["local", nat.ERR_INDEX_RANGE] and r1["rows"] == ["remote", nat.ERR_INDEX_RANGE]
    assert r0["gathered_ok"] and r1["gathered_ok"] and r0["upper_ok"] and r1["upper_ok"]


def test_row_partition_covers_all_rows():
    from lcd_b200.multigpu import row_partition
    for n, world in ((10, 3), (16_777_216, 8), (5, 8), (0, 2)):
        bounds = row_partition(n, world)
        assert bounds[0] == 0 and bounds[-1] == n and len(bounds) == world + 1
        assert np.all(np.diff(bounds) >= 0) and np.max(np.diff(bounds)) - np.min(np.diff(bounds)) <= 1
