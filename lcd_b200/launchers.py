"""Native launchers behind the reference's launcher contract.

The reference generates a Python launcher per lowering
(``compiler/cuda_lowering.py:673-735`` single sync-free launch, ``:855-1016``
per-level wavefront launches with a device synchronisation after each,
``:1022-1068`` per-band, ``:1070-1119`` persistent warps).  Here a launcher is a
closure that receives the same positional arguments (original parameters, lifted
locals, lookup tables, executor arrays) and forwards the device pointers to one
C-ABI entry point; level loops and barriers live inside the library.

Gauss-Seidel sweeps (``compiler/demo/gauss_seidel.py``) keep their host sweep loop inside the
launcher, as the reference's generated launcher does; a sweep is a triangular solve on the
diagonal-last form of the rows.

A sync-free CSR triangular solve whose levels are narrow (the inspector's row and level
counts arrive as hints from the decorator) goes to the block-recurrence chain solver
instead of the polling kernel.

Executor arrays the native kernels do not need (successor lists, task tables and
ticket counters of the row-form solver, which polls operands instead of counting)
are accepted and ignored, so call sites written for the reference keep working.
"""

from __future__ import annotations

import ast

import numpy as np

from . import ops
from .cuda_lowering import CUDALoweringError, PUSH_DEPENDENCE
from .cuda_runtime import as_tensor
from .scheduler import (chain_solver_preferred, ordered_solver_preferred,
                        small_solver_preferred)

# Launch policy of the wavefront entry point: the cooperative single-launch walk
# unless the level count is small enough for per-level launches to be cheaper.
PER_LEVEL_MAX_LEVELS = 8


def _lanes_from_schedule(lowering, average_work):
    """Lane-group width for one row.  ``n_warp``/``threads_per_block`` describe the
    reference's mapping (a warp or a block per node); natively the group is sized
    to the row length, capped by what the schedule asked for."""
    if lowering.thread_loop_iterator is None:
        return 1
    cap = 32 * max(1, lowering.n_warp or 1)
    lanes = 1
    while lanes < 32 and lanes * 24 < average_work and lanes * 2 <= cap:
        lanes *= 2
    return lanes


def bind(lowering):
    """(kernel, launcher) callables for a lowering of a recognised operator."""
    names = list(lowering.launcher_arguments)
    roles = lowering.roles
    import torch

    def split(args):
        if len(args) != len(names):
            raise TypeError(f"{lowering.launcher_name} expects {len(names)} arguments "
                            f"({', '.join(names)}), received {len(args)}")
        return dict(zip(names, args))

    def matrix(values):
        Ap = as_tensor(values[roles["ptr"]], torch.int32)
        Ai = as_tensor(values[roles["idx"]], torch.int32)
        Ax = as_tensor(values[roles["val"]], torch.float64)
        return Ap, Ai, Ax

    def average_row(Ap, Ai):
        return Ai.numel() / max(1, Ap.numel() - 1)

    def wavefront_arrays(values, serves_tasks=False):
        tasks = None
        if "wavefronts" in values:
            nodes, ptr_host = values["wavefronts"], values["wavefront_ptr"]
        else:
            nodes, ptr_host = values["task_nodes"], values["band_ptr"]
            task_ptr = values["task_ptr"]
            if len(task_ptr) - 1 != len(nodes):    # band chains (band_width > 1)
                if not serves_tasks:
                    raise CUDALoweringError("band_width > 1 task chains are not served natively "
                                            "for this operator")
                tasks = as_tensor(task_ptr, torch.int32)
        nodes = as_tensor(nodes, torch.int32)
        ptr_host = np.ascontiguousarray(
            ptr_host.copy_to_host() if hasattr(ptr_host, "copy_to_host") else
            (ptr_host.cpu().numpy() if hasattr(ptr_host, "cpu") else ptr_host), dtype=np.int32)
        ptr_dev = torch.from_numpy(ptr_host).to(nodes.device)
        if serves_tasks:
            return nodes, ptr_dev, ptr_host, tasks
        return nodes, ptr_dev, ptr_host

    def small_plan_for(op_name, Ap, Ai, hints):
        """The one-block solver's plan for this pattern (kept with the schedule plan), or None
        when the matrix is not small, has rows it does not serve, or is better off elsewhere."""
        dag, cache = hints.get("dag"), hints.setdefault("cache", {})
        if dag is None or dag.capped or "small_plan" in cache:    # (capped: deep, level sets not built)
            return cache.get("small_plan")
        plan = None
        n, nnz = Ap.numel() - 1, Ai.numel()
        if ops.SmallPlan.serves(n, nnz) and small_solver_preferred(n, nnz, dag.n_levels):
            try:
                plan = ops.SmallPlan(op_name, Ap, Ai, dag)
            except ops.NativeError as error:
                if error.code != ops.nat.ERR_TOO_LARGE:
                    raise
        cache["small_plan"] = plan
        return plan

    def walk_plan_for(op_name, Ap, Ai, hints):
        """Plan of the level walk shared by many blocks (wide levels, short rows), or None."""
        dag, cache = hints.get("dag"), hints.setdefault("cache", {})
        if dag is None or dag.capped or "walk_plan" in cache:
            return cache.get("walk_plan")
        plan = None
        n, nnz = Ap.numel() - 1, Ai.numel()
        blocks = ops.sliced_blocks(n, dag.n_levels) if dag.n_levels > 0 else 1
        if blocks >= 8 and nnz - n <= ops.nat.load().lcd_small_max_entries() * n:
            try:
                plan = ops.SmallPlan(op_name, Ap, Ai, dag, blocks=blocks)
            except ops.NativeError as error:
                if error.code != ops.nat.ERR_TOO_LARGE:
                    raise
        cache["walk_plan"] = plan
        return plan

    def walk_solve(plan, Ax, b, x, cache):
        # the coefficients are gathered into slot order again only when the value array has other
        # contents than at the last solve (device checksum, as for the chain solver's tiles)
        stamp = ops.fingerprint(Ax.view(torch.int32))
        same = cache.get("walk_values") == stamp
        ops.sptrsv_small(plan, Ax, b, x, same_values=same, sync=True)
        cache["walk_values"] = stamp

    def ordered_plan_for(Ap, Ai, hints):
        dag, cache = hints.get("dag"), hints.setdefault("cache", {})
        if dag is None or dag.capped or "ordered_plan" in cache:
            return cache.get("ordered_plan")
        plan = None
        if ordered_solver_preferred(Ap.numel() - 1, dag.n_levels, average_row(Ap, Ai)):
            plan = ops.OrderedPlan(dag.wavefronts, dag.n_levels)
        cache["ordered_plan"] = plan
        return plan

    def chain_solve(Ap, Ai, Ax, b, x, cache):
        # the block tiles depend on the values (the structure is fixed per plan): they are
        # rebuilt unless the value array has the contents they were built from (position-keyed
        # 128-bit device checksum, as for the structure fingerprint of the plan cache)
        n = Ap.numel() - 1
        workspace = cache.get("chain_workspace")
        if workspace is None or workspace.device != Ax.device:
            workspace = cache["chain_workspace"] = ops.chain_workspace(n, Ax.device)
            cache.pop("chain_values", None)
        stamp = ops.fingerprint(Ax.view(torch.int32))
        if cache.get("chain_values") != stamp:
            # new values: preparation and solve pipelined over row ranges (the preparation is
            # throughput work on a second stream, the solve runs on one SM at a time)
            ops.chain_prepare_and_solve(Ap, Ai, Ax, b, workspace, x, upper=lowering.upper)
            cache["chain_values"] = stamp
            # explicit block inverses are only as accurate as the blocks are well conditioned
            cache["chain_stable"] = ops.chain_growth(workspace, n) <= ops.CHAIN_MAX_GROWTH
            if cache["chain_stable"]:
                return
        if cache["chain_stable"]:
            ops.sptrsv_csr_chain(Ap, Ai, Ax, b, workspace, x, upper=lowering.upper)
        else:           # substitution (still on the GPU): slower on such matrices, but stable
            ops.sptrsv_csr_syncfree(Ap, Ai, Ax, b, x, upper=lowering.upper)

    def chain_solve_streamed(Ap, Ai, Ax, pieces, b, x, cache, index_pieces=None, rhs_pieces=None,
                             result=None):
        # The value array is still being uploaded, piece by piece (pieces: elements uploaded
        # so far and the event that says so; index_pieces, rhs_pieces: the same for the column
        # indices when they travel beside the values and for a right-hand side sent in two parts;
        # result: the device array object of x, which can send finished rows to the host early).  The chain solver consumes the matrix front to
        # back, so tiles are prepared and rows solved as far as the entries have arrived: the
        # solve overlaps the upload instead of following it.  (No look at the tile cache: its
        # key needs the whole array, and the preparation hides under the upload anyway.)
        n = Ap.numel() - 1
        workspace = cache.get("chain_workspace")
        if workspace is None or workspace.device != Ax.device:
            workspace = cache["chain_workspace"] = ops.chain_workspace(n, Ax.device)
        cache.pop("chain_values", None)
        ends = torch.tensor([end for end, _ in pieces], dtype=Ap.dtype, device=Ap.device)
        # rows [0, r) are complete once Ap[r] entries are there
        # (the few numbers are finished on the host: every torch operator used here for the first
        # time in a process costs tens of milliseconds of module loading)
        found = torch.searchsorted(Ap, ends, right=True).tolist()
        complete = [min(max(r - 1, 0), n) // ops.CHAIN_SOLVE_ROWS * ops.CHAIN_SOLVE_ROWS for r in found]
        complete[-1] = n
        status = ops.new_status(Ax.device)
        stream = torch.cuda.current_stream()
        # as in ops.chain_prepare_and_solve: the tiles of a range are prepared on a second
        # stream (behind the upload of its entries), the range is solved on this stream behind
        # its tiles; a large piece is cut into ranges so that its preparation runs beside the
        # solve of the rows before it
        side = ops.side_stream(Ax.device)
        side.wait_stream(stream)
        step = ops.chain_pipeline_bounds(n)[1]
        begin = 0
        for (entries, event), end in zip(pieces, complete):
            if end <= begin and end != n:
                continue
            side.wait_event(event)
            if index_pieces:   # the first piece of the indices that covers these entries
                side.wait_event(next(e for upto, e in index_pieces if upto >= entries))
            cuts = list(range(begin, end, step)) + [end]
            tiles = []
            with torch.cuda.stream(side):
                for lo, hi in zip(cuts[:-1], cuts[1:]):
                    ops.chain_prepare(Ap, Ai, Ax, workspace, rows=(lo, hi))
                    tiles.append(torch.cuda.Event())
                    tiles[-1].record(side)
            for lo, hi, prepared in zip(cuts[:-1], cuts[1:], tiles):
                stream.wait_event(prepared)
                if rhs_pieces:
                    stream.wait_event(next(e for upto, e in rhs_pieces if upto >= hi))
                ops.sptrsv_csr_chain(Ap, Ai, Ax, b, workspace, x, status=status, rows=(lo, hi),
                                     sync=hi == n)
                if result is not None:
                    result.download_rows(lo, hi)
            begin = end
        if ops.chain_growth(workspace, n) > ops.CHAIN_MAX_GROWTH:
            # the block inverses grew: solve again by substitution (the whole array has arrived)
            if result is not None:
                result.forget_downloads()
            ops.sptrsv_csr_syncfree(Ap, Ai, Ax, b, x, upper=lowering.upper)

    def csr_solve(Ap, Ai, Ax, b, x, v, hints):
        lanes = _lanes_from_schedule(lowering, average_row(Ap, Ai))
        op_name = "csr_upper" if lowering.upper else "csr_lower"
        if lowering.execution_mode == "sync_free":
            if chain_solver_preferred(hints.get("rows", 0), hints.get("levels", 0),
                                      hints.get("arch")):
                chain_solve(Ap, Ai, Ax, b, x, hints.setdefault("cache", {}))
                return
            small = small_plan_for(op_name, Ap, Ai, hints)
            if small is not None:
                ops.sptrsv_small(small, Ax, b, x)
                return
            walk = walk_plan_for(op_name, Ap, Ai, hints) if lanes == 1 else None
            if walk is not None:
                walk_solve(walk, Ax, b, x, hints.setdefault("cache", {}))
                return
            ordered = ordered_plan_for(Ap, Ai, hints) if lanes == 1 else None
            if ordered is not None:
                ops.sptrsv_csr_ordered(Ap, Ai, Ax, b, ordered, x, upper=lowering.upper)
            else:
                ops.sptrsv_csr_syncfree(Ap, Ai, Ax, b, x, upper=lowering.upper, lanes=lanes)
        else:
            nodes, ptr_dev, ptr_host, tasks = wavefront_arrays(v, serves_tasks=True)
            small = small_plan_for(op_name, Ap, Ai, hints) if tasks is None else None
            if small is not None:          # the same level walk, inside one thread block
                ops.sptrsv_small(small, Ax, b, x)
                return
            mode = "per_level" if len(ptr_host) - 1 <= PER_LEVEL_MAX_LEVELS else "cooperative"
            ops.sptrsv_wavefront(op_name, Ap, Ai, Ax, b,
                                 nodes, ptr_dev, ptr_host, x, mode=mode, lanes=lanes, task_ptr=tasks)

    def sptrsv_csr(*args, _hints=None):
        v = split(args)
        hints = _hints or {}
        values = v[roles["val"]]
        if (lowering.execution_mode == "sync_free" and not lowering.upper and
                getattr(values, "arrival", None) and values._tensor.dtype == torch.float64 and
                chain_solver_preferred(hints.get("rows", 0), hints.get("levels", 0), hints.get("arch"))):
            Ax, pieces = values.take_arrival()
            indices, index_pieces = v[roles["idx"]], None
            if getattr(indices, "arrival", None) and indices._tensor.dtype == torch.int32:
                indices, index_pieces = indices.take_arrival()
            rhs, rhs_pieces = v[roles["rhs"]], None
            if getattr(rhs, "arrival", None) and rhs._tensor.dtype == torch.float64:
                rhs, rhs_pieces = rhs.take_arrival()
            result, x = v[roles["out"]], as_tensor(v[roles["out"]], torch.float64)
            if not (hasattr(result, "download_rows") and result._tensor.data_ptr() == x.data_ptr()):
                result = None
            chain_solve_streamed(as_tensor(v[roles["ptr"]], torch.int32), as_tensor(indices, torch.int32),
                                 Ax, pieces, as_tensor(rhs, torch.float64), x,
                                 hints.setdefault("cache", {}), index_pieces, rhs_pieces, result)
            return
        Ap, Ai, Ax = matrix(v)
        b = as_tensor(v[roles["rhs"]], torch.float64)
        x = as_tensor(v[roles["out"]], torch.float64)
        csr_solve(Ap, Ai, Ax, b, x, v, hints)

    def host_trip_count(v):
        """Product of the trip counts of the host loops around the block loop."""
        count = 1
        scalars = {k: val for k, val in v.items() if isinstance(val, (int, np.integer))}
        for call in lowering.host_loop_ranges:
            code = compile(ast.Expression(body=ast.fix_missing_locations(call)), "<host-loop>", "eval")
            count *= len(eval(code, {"__builtins__": {"range": range}}, scalars))
        return count

    def gauss_seidel(*args, _hints=None):
        # Sweeps over a lower-triangular matrix: every sweep recomputes x from b in row order,
        # i.e. it is the triangular solve on the diagonal-last form of the rows.  The structure
        # part of the conversion is kept with the plan, the values are converted every call.
        v = split(args)
        Ap, Ai, Ax = matrix(v)
        b = as_tensor(v[roles["rhs"]], torch.float64)
        x = as_tensor(v[roles["out"]], torch.float64)
        hints = _hints or {}
        cache = hints.setdefault("cache", {})
        separate = "diagonal" in roles
        layout = cache.get("gs_layout")
        if layout is None or layout.perm.device != Ap.device:
            layout = cache["gs_layout"] = ops.gs_layout(Ap, Ai, separate_diagonal=separate)
        diagonal = as_tensor(v[roles["diagonal"]], torch.float64) if separate else None
        values = ops.gs_values(layout, Ax, diagonal, out=cache.get("gs_values"))
        cache["gs_values"] = values
        for _ in range(host_trip_count(v)):
            csr_solve(layout.Ap, layout.Ai, values, b, x, v, hints)

    def sptrsv_csc(*args, _hints=None):
        v = split(args)
        hints = _hints or {}
        Ap, Ai, Ax = matrix(v)
        b = as_tensor(v[roles["rhs"]], torch.float64)
        x = as_tensor(v[roles["out"]], torch.float64)
        lanes = _lanes_from_schedule(lowering, average_row(Ap, Ai))
        band_chains = "task_ptr" in v and len(v["task_ptr"]) - 1 != len(v["task_nodes"])
        small = None if band_chains else small_plan_for(
            "csc_upper" if lowering.upper else "csc_lower", Ap, Ai, hints)
        if small is not None:
            # push into shared-memory accumulators, level by level inside one thread block
            ops.sptrsv_small(small, Ax, b, x)
            return
        if lowering.execution_mode == "sync_free":
            if lowering.dependence_protocol == PUSH_DEPENDENCE:
                # push protocol: the counters already hold edge multiplicities; the kernel
                # consumes them, the plan keeps the pristine ones
                dep = as_tensor(v["dep_count"], torch.int32).clone()
            else:
                # counter protocol counts distinct predecessors; the push kernel
                # decrements once per stored entry, so recount on the device
                dep = ops.csc_edge_count(Ap, Ai, upper=lowering.upper)
            ops.sptrsv_csc_syncfree(Ap, Ai, Ax, b, dep, x, upper=lowering.upper, lanes=lanes)
        else:
            nodes, ptr_dev, ptr_host, tasks = wavefront_arrays(v, serves_tasks=True)
            mode = "per_level" if len(ptr_host) - 1 <= PER_LEVEL_MAX_LEVELS else "cooperative"
            ops.sptrsv_wavefront("csc_upper" if lowering.upper else "csc_lower", Ap, Ai, Ax, b,
                                 nodes, ptr_dev, ptr_host, x, mode=mode, lanes=lanes, task_ptr=tasks)

    def ilu0_csr(*args, _hints=None):
        v = split(args)
        Ap, Ai, Ax = matrix(v)
        lookup = [name for name in names if name.startswith("_lcd_lookup_position_")]
        pos = as_tensor(v[lookup[0]], torch.int32) if lookup else ops.diag_positions(Ap, Ai)
        lanes = 0 if lowering.thread_loop_iterator is not None else 1
        dag = (_hints or {}).get("dag")
        if lowering.execution_mode == "sync_free":
            if dag is not None and dag.n_levels > 0 and dag.n / dag.n_levels >= 8:
                # rows in the order of the level sets: the rows of a level run side by side
                # (by index, a grid matrix keeps one grid line in flight)
                cache = (_hints or {}).get("cache", {})
                if "ilu0_max_row" not in cache:            # once per pattern: picks the lanes per row
                    cache["ilu0_max_row"] = int((Ap[1:] - Ap[:-1]).max()) if Ap.numel() > 1 else 0
                if cache.get("ilu0_scratch") is None or cache["ilu0_scratch"].numel() < Ai.numel():
                    cache["ilu0_scratch"] = torch.empty(max(Ai.numel(), 1), dtype=torch.float64,
                                                        device=Ax.device)
                ops.spilu0_csr(Ap, Ai, Ax, pos, mode="ordered", wavefronts=dag.wavefronts, lanes=lanes,
                               max_row=cache["ilu0_max_row"], scratch=cache["ilu0_scratch"])
            else:
                ops.spilu0_csr(Ap, Ai, Ax, pos, mode="sync_free", lanes=lanes)
        else:
            nodes, _, ptr_host = wavefront_arrays(v)
            ops.spilu0_csr(Ap, Ai, Ax, pos, mode="wavefront", wavefronts=nodes,
                           wavefront_ptr_host=ptr_host, lanes=lanes)

    def ilu0_csc(*args, _hints=None):
        # the column loop applies the row loop's updates in the row loop's order: gather the
        # values into row order, factor with the row kernel, scatter back (the row-ordered view
        # of the pattern is kept with the plan)
        v = split(args)
        Ap, Ai, Ax = matrix(v)
        cache = (_hints or {}).setdefault("cache", {})
        view = cache.get("csc_row_view")
        if view is None or view.Ap.device != Ap.device:
            view = cache["csc_row_view"] = ops.csc_row_view(Ap, Ai)
        dag = (_hints or {}).get("dag")
        if lowering.execution_mode == "sync_free":
            if dag is not None and dag.n_levels > 0 and dag.n / dag.n_levels >= 8:
                ops.spilu0_csc(Ap, Ai, Ax, view, mode="ordered", wavefronts=dag.wavefronts)
            else:
                ops.spilu0_csc(Ap, Ai, Ax, view, mode="sync_free")
        else:
            nodes, _, ptr_host = wavefront_arrays(v)
            ops.spilu0_csc(Ap, Ai, Ax, view, mode="wavefront", wavefronts=nodes,
                           wavefront_ptr_host=ptr_host)

    launcher = {"sptrsv_csr": sptrsv_csr, "sptrsv_csc": sptrsv_csc, "ilu0_csr": ilu0_csr,
                "ilu0_csc": ilu0_csc,
                "gauss_seidel_simple_csr": gauss_seidel, "gauss_seidel_full_csr": gauss_seidel}.get(
        lowering.operator)
    if launcher is None:
        raise CUDALoweringError(f"no native kernel for operator {lowering.operator!r}")
    launcher.__name__ = lowering.launcher_name
    launcher.accepts_hints = launcher in (sptrsv_csr, sptrsv_csc, gauss_seidel, ilu0_csr, ilu0_csc)

    def kernel(*args, **kwargs):
        raise CUDALoweringError(
            f"{lowering.kernel_name} is a native sm_100a kernel inside liblcd_b200.so "
            f"({lowering.entry_point}); launch it through {lowering.launcher_name}.")

    kernel.__name__ = lowering.kernel_name
    kernel.entry_point = lowering.entry_point
    return kernel, launcher
