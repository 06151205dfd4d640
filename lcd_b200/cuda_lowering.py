"""From a decorated loop nest to a native kernel binding.

The reference (``compiler/cuda_lowering.py``) rewrites the block loop into a
Numba-CUDA kernel plus a Python launcher (``CUDALowerer.lower`` ``:407-636``,
result record ``:72-98``).  Here nothing is generated: the loop nest is
*recognised* as one of the operators the hand-written sm_100a kernels implement
and the result record names that kernel and keeps the reference's launcher
contract -- launcher arguments are the original parameters, then lifted locals,
then structural-lookup tables, then the executor arrays of the chosen mode
(``:51-64``, ``:479-506``).  Loop nests outside the served family raise
:class:`CUDALoweringError`; there is no interpreter or CPU fallback.

Recognition is alpha-equivalence: identifiers are renamed in order of first
appearance and the block loop's AST is compared with the canonical forms below
(the operators of ``compiler/demo/sptrsv.py:26-43`` and
``compiler/demo/spilu0.py:21-47`` plus their backward-substitution forms, and the
Gauss-Seidel sweeps of ``compiler/demo/gauss_seidel.py:18-41``, whose block loop sits
inside a host sweep loop that the launcher runs).
"""

from __future__ import annotations

import ast
import builtins
from copy import deepcopy
from dataclasses import dataclass, field

COUNTER_DEPENDENCE = "counter"
PUSH_DEPENDENCE = "push"
PULL_DEPENDENCE = "pull"
DEPENDENCE_PROTOCOLS = (COUNTER_DEPENDENCE, PUSH_DEPENDENCE, PULL_DEPENDENCE)
CUDA_EXECUTION_MODES = frozenset({"plain", "sync_free", "wavefront"})
SYNC_FREE_ARGUMENTS = ("dep_count", "dag_ptr", "dag_index")
SYNC_FREE_RESET_ARGUMENT = "initial_dep_count"
WAVEFRONT_ARGUMENTS = ("wavefronts", "wave_start", "wave_end")
WARP_SYNC_FREE_ARGUMENTS = ("dep_count", "dag_ptr", "dag_index", "task_nodes", "task_ptr",
                            "task_counter")
WARP_PUSH_ARGUMENTS = ("dep_count", "task_nodes", "task_ptr", "task_counter")
WARP_PULL_ARGUMENTS = ("done", "task_nodes", "task_ptr", "task_counter")
WARP_WAVEFRONT_ARGUMENTS = ("task_nodes", "task_ptr", "band_start", "band_end")
WARP_SIZE = 32


class CUDALoweringError(Exception):
    """The loop nest cannot be served by the native kernels."""


class UnsupportedAtomicOperation(CUDALoweringError):
    """A reduction has no atomic counterpart on the device."""


# ---- canonical operator forms ---------------------------------------------------
# role of each parameter / local in the canonical spelling
_OPERATORS = {
    "sptrsv_csr_lower": (dict(Ap="ptr", Ai="idx", Ax="val", b="rhs", x="out", n="n"), """
for i in range(n):
    x[i] = b[i]
    for j in range(Ap[i], Ap[i + 1] - 1):
        x[i] -= Ax[j] * x[Ai[j]]
    x[i] /= Ax[Ap[i + 1] - 1]
"""),
    "sptrsv_csc_lower": (dict(Ap="ptr", Ai="idx", Ax="val", b="rhs", x="out", n="n"), """
for i in range(n):
    x[i] = (b[i] - x[i]) / Ax[Ap[i]]
    for j in range(Ap[i] + 1, Ap[i + 1]):
        x[Ai[j]] += Ax[j] * x[i]
"""),
    "sptrsv_csr_upper": (dict(Ap="ptr", Ai="idx", Ax="val", b="rhs", x="out", n="n"), """
for ii in range(n):
    x[n - 1 - ii] = b[n - 1 - ii]
    for j in range(Ap[n - 1 - ii] + 1, Ap[n - ii]):
        x[n - 1 - ii] -= Ax[j] * x[Ai[j]]
    x[n - 1 - ii] /= Ax[Ap[n - 1 - ii]]
"""),
    "sptrsv_csr_upper#alias": (dict(Ap="ptr", Ai="idx", Ax="val", b="rhs", x="out", n="n"), """
for ii in range(n):
    i = n - 1 - ii
    x[i] = b[i]
    for j in range(Ap[i] + 1, Ap[i + 1]):
        x[i] -= Ax[j] * x[Ai[j]]
    x[i] /= Ax[Ap[i]]
"""),
    "sptrsv_csc_upper": (dict(Ap="ptr", Ai="idx", Ax="val", b="rhs", x="out", n="n"), """
for ii in range(n):
    x[n - 1 - ii] = (b[n - 1 - ii] - x[n - 1 - ii]) / Ax[Ap[n - ii] - 1]
    for j in range(Ap[n - 1 - ii], Ap[n - ii] - 1):
        x[Ai[j]] += Ax[j] * x[n - 1 - ii]
"""),
    "sptrsv_csc_upper#alias": (dict(Ap="ptr", Ai="idx", Ax="val", b="rhs", x="out", n="n"), """
for ii in range(n):
    i = n - 1 - ii
    x[i] = (b[i] - x[i]) / Ax[Ap[i + 1] - 1]
    for j in range(Ap[i], Ap[i + 1] - 1):
        x[Ai[j]] += Ax[j] * x[i]
"""),
    "ilu0_csr": (dict(A_data="val", A_indices="idx", A_indptr="ptr", n="n"), """
for i in range(n):
    row_start = A_indptr[i]
    row_end = A_indptr[i + 1]
    for k_ptr in range(row_start, row_end):
        k = A_indices[k_ptr]
        if k >= i:
            break
        diag_val = 0.0
        for diag_ptr in range(A_indptr[k], A_indptr[k + 1]):
            if A_indices[diag_ptr] == k:
                diag_val = A_data[diag_ptr]
                break
        if diag_val != 0.0:
            A_data[k_ptr] = A_data[k_ptr] / diag_val
            l_ik = A_data[k_ptr]
            for j_ptr in range(k_ptr + 1, row_end):
                j = A_indices[j_ptr]
                for kj_ptr in range(A_indptr[k], A_indptr[k + 1]):
                    if A_indices[kj_ptr] == j:
                        u_kj = A_data[kj_ptr]
                        A_data[j_ptr] = A_data[j_ptr] - l_ik * u_kj
                        break
"""),
    "ilu0_csc": (dict(A_data="val", A_indices="idx", A_indptr="ptr", n="n"), """
for k in range(n):
    col_start = A_indptr[k]
    col_end = A_indptr[k + 1]
    diag_val = 0.0
    for dptr in range(col_start, col_end):
        if A_indices[dptr] == k:
            diag_val = A_data[dptr]
            break
    for i_ptr in range(col_start, col_end):
        i = A_indices[i_ptr]
        if i <= k:
            continue
        if diag_val != 0.0:
            A_data[i_ptr] = A_data[i_ptr] / diag_val
            l_ik = A_data[i_ptr]
            for j in range(k + 1, n):
                j_start = A_indptr[j]
                j_end = A_indptr[j + 1]
                u_kj = 0.0
                for kj_ptr in range(j_start, j_end):
                    if A_indices[kj_ptr] == k:
                        u_kj = A_data[kj_ptr]
                        break
                if u_kj != 0.0:
                    for ij_ptr in range(j_start, j_end):
                        if A_indices[ij_ptr] == i:
                            A_data[ij_ptr] = A_data[ij_ptr] - l_ik * u_kj
                            break
"""),
    "gauss_seidel_simple_csr": (dict(Ap="ptr", Ai="idx", Ax="val", D="diagonal", b="rhs", x="out", n="n"), """
for i in range(n):
    x[i] = b[i]
    for j in range(Ap[i], Ap[i + 1]):
        x[i] -= Ax[j] * x[Ai[j]]
    x[i] /= D[i]
"""),
    "gauss_seidel_full_csr": (dict(Ap="ptr", Ai="idx", Ax="val", b="rhs", x="out", n="n"), """
for i in range(n):
    sigma = 0.0
    diag = 1.0
    for j in range(Ap[i], Ap[i + 1]):
        if Ai[j] == i:
            diag = Ax[j]
        else:
            sigma += Ax[j] * x[Ai[j]]
    x[i] = (b[i] - sigma) / diag
"""),
}
# name of the inner loop a thread map may refer to, per operator
_THREAD_LOOPS = {"sptrsv_csr_lower": "j", "sptrsv_csc_lower": "j", "sptrsv_csr_upper": "j",
                 "sptrsv_csc_upper": "j", "ilu0_csr": "j_ptr", "ilu0_csc": "i_ptr", "gauss_seidel_simple_csr": "j",
                 "gauss_seidel_full_csr": "j"}
GAUSS_SEIDEL_OPERATORS = ("gauss_seidel_simple_csr", "gauss_seidel_full_csr")
# native entry point serving (operator, execution mode)
_ENTRY_POINTS = {
    ("sptrsv_csr", "sync_free"): "lcd_sptrsv_csr_syncfree",
    ("sptrsv_csr", "wavefront"): "lcd_sptrsv_wavefront",
    ("sptrsv_csc", "sync_free"): "lcd_sptrsv_csc_syncfree",
    ("sptrsv_csc", "wavefront"): "lcd_sptrsv_wavefront",
    ("ilu0_csr", "sync_free"): "lcd_spilu0_csr",
    ("ilu0_csr", "wavefront"): "lcd_spilu0_csr",
    # the column loop updates the same entries in the same order: row kernel on the row-ordered view
    ("ilu0_csc", "sync_free"): "lcd_spilu0_csr",
    ("ilu0_csc", "wavefront"): "lcd_spilu0_csr",
    # a sweep is a lower-triangular solve on the diagonal-last rows lcd_gs_layout/lcd_gs_values make
    ("gauss_seidel_simple_csr", "sync_free"): "lcd_sptrsv_csr_syncfree",
    ("gauss_seidel_simple_csr", "wavefront"): "lcd_sptrsv_wavefront",
    ("gauss_seidel_full_csr", "sync_free"): "lcd_sptrsv_csr_syncfree",
    ("gauss_seidel_full_csr", "wavefront"): "lcd_sptrsv_wavefront",
}
_BUILTIN_NAMES = frozenset(dir(builtins))


class _Canonicaliser(ast.NodeTransformer):
    """Renames every identifier that is not a builtin to v0, v1, ... in order of
    first appearance, and spells ``t op= v`` as ``t = t op v``."""

    def __init__(self):
        self.names = {}

    def visit_Name(self, node):
        if node.id in _BUILTIN_NAMES:
            return node
        new = self.names.setdefault(node.id, f"v{len(self.names)}")
        return ast.copy_location(ast.Name(id=new, ctx=node.ctx), node)

    def visit_AugAssign(self, node):
        target_load = deepcopy(node.target)
        target_load.ctx = ast.Load()
        assign = ast.Assign(targets=[node.target],
                            value=ast.BinOp(left=target_load, op=node.op, right=node.value))
        return self.generic_visit(ast.copy_location(assign, node))


def _canonical_dump(loop):
    canon = _Canonicaliser()
    tree = canon.visit(deepcopy(loop))
    return ast.dump(tree, annotate_fields=False, include_attributes=False), canon.names


def _canonical_library():
    library = {}
    for key, (roles, source) in _OPERATORS.items():
        loop = ast.parse(source.strip()).body[0]
        dump, names = _canonical_dump(loop)
        by_canonical = {canonical: roles.get(original, original)
                        for original, canonical in names.items()}
        thread_loop = names.get(_THREAD_LOOPS[key.split("#")[0]])
        library[dump] = (key.split("#")[0], by_canonical, thread_loop)
    return library


_LIBRARY = _canonical_library()


@dataclass
class _TargetLoop:
    loop: ast.For
    top_level_index: int
    host_loops: tuple = ()     # (iterator name, range expression) of enclosing host loops


def _find_block_loop(function, iterator):
    """The block loop: a top-level ``for``, or the only statement of a nest of top-level
    ``for ... in range(...)`` host loops (``compiler/cuda_lowering.py:1129-1140`` wraps the
    launch in those loops; here the launcher runs them)."""
    for index, statement in enumerate(function.body):
        host_loops = []
        node = statement
        while isinstance(node, ast.For) and isinstance(node.target, ast.Name) and not node.orelse:
            if node.target.id == iterator:
                return _TargetLoop(node, index, tuple(host_loops))
            call = node.iter
            if not (isinstance(call, ast.Call) and isinstance(call.func, ast.Name)
                    and call.func.id == "range" and not call.keywords and len(node.body) == 1):
                break
            host_loops.append((node.target.id, deepcopy(call)))
            node = node.body[0]
    for node in ast.walk(function):
        if (isinstance(node, ast.For) and isinstance(node.target, ast.Name)
                and node.target.id == iterator):
            raise CUDALoweringError(
                f"The block loop over {iterator!r} must be a top-level statement of the "
                "function or the only statement inside top-level `for ... in range(...)` "
                "host loops.")
    raise CUDALoweringError(f"No loop over the block iterator {iterator!r} was found.")


def _stored_names(statements):
    names = []
    for statement in statements:
        for node in ast.walk(statement):
            if isinstance(node, ast.Name) and isinstance(node.ctx, ast.Store) \
                    and node.id not in names:
                names.append(node.id)
    return names


def _loaded_names(node):
    return {n.id for n in ast.walk(node) if isinstance(n, ast.Name)}


@dataclass
class CUDALoweringResult:
    """What the runtime needs to serve one schedule of one operator.  Field names
    follow the reference's record; ``operator`` / ``roles`` / ``entry_point`` are
    the native additions, and ``source`` describes the binding in words."""

    kernel_name: str
    launcher_name: str
    kernel_arguments: list
    launcher_arguments: list
    lifted_variables: list
    lifted_loop_parameters: list
    host_prelude: list
    host_epilogue: list
    atomic_statement_ids: set
    execution_mode: str
    auxiliary_arguments: list
    operator: str = ""
    upper: bool = False
    roles: dict = field(default_factory=dict)
    entry_point: str = ""
    threads_per_block: int = 128
    thread_loop_iterator: str | None = None
    thread_unroll_factor: int = 1
    host_loop_iterators: tuple = ()
    host_loop_ranges: tuple = ()       # ast.Call `range(...)` of each host loop, outermost first
    n_warp: int | None = None
    warp_mapped: bool = False
    dependence_protocol: str = COUNTER_DEPENDENCE
    device_only_variables: tuple = ()
    module_ast: ast.Module | None = None
    kernel_ast: ast.AST | None = None
    launcher_ast: ast.AST | None = None

    @property
    def source(self):
        args = ", ".join(self.launcher_arguments)
        return (f"# native binding: {self.launcher_name}({args})\n"
                f"#   operator {self.operator}{' (upper)' if self.upper else ''}, "
                f"mode {self.execution_mode}, protocol {self.dependence_protocol}\n"
                f"#   -> {self.entry_point} in liblcd_b200.so (sm_100a)")


def _to_function(code):
    if isinstance(code, str):
        code = ast.parse(code)
    if isinstance(code, ast.Module):
        functions = [n for n in code.body if isinstance(n, (ast.FunctionDef, ast.AsyncFunctionDef))]
        if len(functions) != 1 or not isinstance(functions[0], ast.FunctionDef):
            raise CUDALoweringError("CUDA lowering expects exactly one synchronous function.")
        return functions[0]
    if isinstance(code, ast.FunctionDef):
        return code
    raise CUDALoweringError("CUDA lowering expects a function definition.")


def recognise_operator(code, loop_iterator):
    """(operator, upper, roles, thread_loop_name, target) for a decorated function."""
    function = _to_function(code)
    target = _find_block_loop(function, loop_iterator)
    dump, names = _canonical_dump(target.loop)
    match = _LIBRARY.get(dump)
    if match is None:
        raise CUDALoweringError(
            "The loop nest over %r is not one of the operators served by the native kernels "
            "(SpTRSV CSR/CSC lower/upper, SpILU0 CSR/CSC, Gauss-Seidel CSR sweeps); lcd_b200 does not interpret or "
            "fall back to the CPU." % loop_iterator)
    operator, by_canonical, thread_canonical = match
    roles = {}
    thread_loop = None
    for original, canonical in names.items():
        role = by_canonical.get(canonical)
        if role in ("ptr", "idx", "val", "rhs", "out", "n", "diagonal"):
            roles[role] = original
        if canonical == thread_canonical:
            thread_loop = original
    upper = operator.endswith("_upper")
    family = operator[:-6] if operator.endswith(("_lower", "_upper")) else operator
    return family, upper, roles, thread_loop, target, function


def lower_to_native(code, loop_iterator, reductions=None, kernel_name=None,
                    execution_mode="plain", sync_free_ready_count=0,
                    wavefront_threads_per_block=128, thread_loop_iterator=None,
                    thread_unroll_factor=1, n_warp=None,
                    dependence_protocol=COUNTER_DEPENDENCE, direct_dependence=None,
                    function_props=None, structural_lookups=()):
    """Bind one schedule of a recognised operator to its native kernel.

    Arguments and validation follow ``lower_to_numba_cuda`` of the reference
    (``compiler/cuda_lowering.py:2854-2884``, checks ``:313-406``)."""
    mode = execution_mode.replace("-", "_")
    if mode not in CUDA_EXECUTION_MODES:
        raise CUDALoweringError(f"Unknown execution mode {execution_mode!r}.")
    if not isinstance(sync_free_ready_count, int):
        raise CUDALoweringError("The sync-free readiness count must be an integer.")
    if not isinstance(wavefront_threads_per_block, int) or wavefront_threads_per_block <= 0:
        raise CUDALoweringError("The wavefront thread-block size must be a positive integer.")
    if not isinstance(thread_unroll_factor, int) or thread_unroll_factor <= 0:
        raise CUDALoweringError("The thread unroll factor must be a positive integer.")
    if thread_unroll_factor != 1 and thread_loop_iterator is None:
        raise CUDALoweringError("A thread unroll factor requires a thread-mapped loop.")
    if n_warp is not None and (not isinstance(n_warp, int) or n_warp <= 0):
        raise CUDALoweringError("n_warp must be a positive integer.")
    if dependence_protocol not in DEPENDENCE_PROTOCOLS:
        raise CUDALoweringError(f"Unknown dependence protocol {dependence_protocol!r}.")
    family, upper, roles, thread_loop, target, function = recognise_operator(code, loop_iterator)
    if thread_loop_iterator is not None and thread_loop_iterator != thread_loop:
        raise CUDALoweringError(
            f"The thread-mapped iterator {thread_loop_iterator!r} is not the inner loop "
            f"({thread_loop!r}) of the recognised operator.")
    if mode == "plain":
        raise CUDALoweringError("Loops with carried dependences need sync_free or wavefront.")
    warp_mapped = (n_warp == 1 and thread_loop_iterator is not None
                   and wavefront_threads_per_block % WARP_SIZE == 0)
    kind = getattr(direct_dependence, "kind", direct_dependence)
    protocol = (dependence_protocol
                if (kind is not None and kind == dependence_protocol and warp_mapped
                    and mode == "sync_free" and sync_free_ready_count == 0)
                else COUNTER_DEPENDENCE)

    host_prelude = deepcopy(function.body[:target.top_level_index])
    host_epilogue = deepcopy(function.body[target.top_level_index + 1:])
    parameters = [a.arg for a in function.args.args]
    loop_names = _loaded_names(target.loop) | set(_stored_names([target.loop]))
    prelude_names = _stored_names(host_prelude)
    lifted = [name for name in prelude_names if name in loop_names and name not in parameters]
    range_names = _loaded_names(target.loop.iter)
    lifted_loop_parameters = [name for name in lifted if name in range_names]
    lookup_names = [lookup.name for lookup in structural_lookups or ()]

    if mode == "sync_free":
        if not warp_mapped:
            executor = list(SYNC_FREE_ARGUMENTS)
        elif protocol == PUSH_DEPENDENCE:
            executor = list(WARP_PUSH_ARGUMENTS)
        elif protocol == PULL_DEPENDENCE:
            executor = list(WARP_PULL_ARGUMENTS)
        else:
            executor = list(WARP_SYNC_FREE_ARGUMENTS)
        launcher_executor = list(executor)
    else:
        executor = list(WARP_WAVEFRONT_ARGUMENTS if warp_mapped else WAVEFRONT_ARGUMENTS)
        launcher_executor = (["task_nodes", "task_ptr", "band_ptr"] if warp_mapped
                             else ["wavefronts", "wavefront_ptr"])
    base = parameters + [v for v in lifted if v not in parameters]
    kernel_arguments = base + [n for n in lookup_names + executor if n not in base]
    launcher_arguments = base + [n for n in lookup_names + launcher_executor if n not in base]
    name = kernel_name or function.name
    out_name = roles.get("out")
    return CUDALoweringResult(
        kernel_name=f"{name}_cuda_kernel", launcher_name=f"{name}_cuda_launch",
        kernel_arguments=kernel_arguments, launcher_arguments=launcher_arguments,
        lifted_variables=lifted, lifted_loop_parameters=lifted_loop_parameters,
        host_prelude=host_prelude, host_epilogue=host_epilogue,
        atomic_statement_ids=set(getattr(reductions, "atomic_statements", None) or ()),
        execution_mode=mode, auxiliary_arguments=lookup_names + executor,
        operator=family, upper=upper, roles=roles,
        entry_point=_ENTRY_POINTS[(family, mode)],
        threads_per_block=wavefront_threads_per_block,
        thread_loop_iterator=thread_loop_iterator, thread_unroll_factor=thread_unroll_factor,
        host_loop_iterators=tuple(name for name, _ in target.host_loops),
        host_loop_ranges=tuple(call for _, call in target.host_loops),
        n_warp=n_warp, warp_mapped=warp_mapped, dependence_protocol=protocol,
        device_only_variables=tuple(v for v in lifted if v == out_name),
        module_ast=ast.Module(body=[deepcopy(function)], type_ignores=[]),
        kernel_ast=deepcopy(target.loop), launcher_ast=None)


# The reference's entry point name, kept so call sites need no edit.
lower_to_numba_cuda = lower_to_native


def direct_protocol_of(operator, thread_loop_iterator):
    """Which direct (counter-free) protocol the edge rule of an operator admits
    when its inner loop is thread-mapped (``compiler/dag_codegen.py:1621-1664``):
    the column form pushes, the row form pulls, ILU0 has neither."""
    if thread_loop_iterator is None:
        return None
    return {"sptrsv_csc": PUSH_DEPENDENCE, "sptrsv_csr": PULL_DEPENDENCE}.get(operator)
