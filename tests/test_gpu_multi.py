"""Multi-GPU paths on real GPUs: child processes, one per GPU (needs >= 2 GPUs;
NVLS is switched off for NCCL, the kernels use plain peer stores)."""
import os
import sys

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _partition_worker(rank, world, port, out_dir):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    from lcd_b200 import generators as gen
    from lcd_b200.multigpu import PartitionedSolve, ShardedMultiRHS
    results = {}
    for name, tri in (("lap3d", gen.laplacian3d_tril(40, seed=0)),
                      ("band", gen.random_band_lower(100_000, seed=3, mean_degree=12.0, band=64))):
        Ap, Ai, Ax = tri.csr_arrays()
        for ordered in (True, False):            # rows in level order / in index order
            solver = PartitionedSolve(Ap, Ai, Ax, ordered=ordered)
            for _ in range(2):                   # the peer buffers and task records are reusable
                x = solver.solve(tri.b, gather=True)
            results[name + ("" if ordered else "_by_index")] = x.cpu().numpy()
            solver.close()
        up = gen.upper_from_lower(tri)
        Up, Ui, Ux = up.csr_arrays()
        solver = PartitionedSolve(Up, Ui, Ux, upper=True)
        results[name + "_upper"] = solver.solve(up.b, gather=True).cpu().numpy()
        solver.close()
    tri = gen.laplacian3d_tril(24, seed=1, nrhs=13)
    Ap, Ai, Ax = tri.csr_arrays()
    sharded = ShardedMultiRHS(Ap, Ai, Ax)
    results["multirhs"] = sharded.solve(np.asarray(tri.b), gather=True).cpu().numpy()
    start, stop = sharded.shard(13)              # the same shard as a row-major block, no transposes
    rows_major = torch.from_numpy(np.ascontiguousarray(np.asarray(tri.b)[:, start:stop])).cuda()
    results["multirhs_rows"] = sharded.solve(rows_major, layout="rows").cpu().numpy()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **results)
    dist.barrier()
    dist.destroy_process_group()


def test_partitioned_and_sharded_solves_on_two_gpus(cuda, oracle, tmp_path):
    import torch
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs at least 2 GPUs on the box")
    import torch.multiprocessing as mp
    from lcd_b200 import generators as gen
    mp.spawn(_partition_worker, args=(world, 29600 + os.getpid() % 2000, str(tmp_path)),
             nprocs=world, join=True)
    want = {}
    for name, tri in (("lap3d", gen.laplacian3d_tril(40, seed=0)),
                      ("band", gen.random_band_lower(100_000, seed=3, mean_degree=12.0, band=64))):
        Ap, Ai, Ax = tri.csr_arrays()
        want[name] = want[name + "_by_index"] = oracle.sptrsv_csr_lower(Ap, Ai, Ax, tri.b)
        up = gen.upper_from_lower(tri)
        Up, Ui, Ux = up.csr_arrays()
        want[name + "_upper"] = oracle.sptrsv_csr_upper(Up, Ui, Ux, up.b)
    tri = gen.laplacian3d_tril(24, seed=1, nrhs=13)
    Ap, Ai, Ax = tri.csr_arrays()
    want["multirhs"] = np.stack([oracle.sptrsv_csr_lower(Ap, Ai, Ax, np.ascontiguousarray(tri.b[:, q]))
                                 for q in range(13)])
    from lcd_b200.multigpu import column_shard
    for rank in range(world):
        got = np.load(tmp_path / f"rank{rank}.npz")
        for name, ref in want.items():
            np.testing.assert_allclose(got[name], ref, rtol=1e-10, atol=1e-12, err_msg=f"{name} rank {rank}")
        start, stop = column_shard(13, world, rank)
        np.testing.assert_allclose(got["multirhs_rows"], want["multirhs"][start:stop].T, rtol=1e-10, atol=1e-12)
