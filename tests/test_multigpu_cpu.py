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
