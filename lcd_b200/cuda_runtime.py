"""Prepare host values and device arrays for the native launchers, launch, and
restore the decorated function's return semantics.

Same contract as the reference's ``compiler/cuda_runtime.py``
(``compile_cuda_module`` ``:70-125``, ``prepare_cuda_arguments`` ``:128-181``,
``evaluate_host_prelude`` ``:184-199``, ``execute_cuda_call`` ``:202-228``):

* launcher arguments are positional, in ``lowering.launcher_arguments`` order;
* scalars stay host values, anything exposing ``__cuda_array_interface__`` passes
  through untouched, lists/tuples/ndarrays are copied to the device, everything
  else raises :class:`CUDARuntimePreparationError` (``:391-401``);
* ``wavefront_ptr`` and ``band_ptr`` stay on the host (``:16``);
* after the launch the runtime synchronises, copies returned arguments and lifted
  locals back (``copy_to_host`` when the value has it) and evaluates the removed
  host epilogue (``:215-228``, ``:267-304``).

Device memory and streams come from torch; the "module" bound by
``compile_cuda_module`` is the pair of Python callables that forward to the C ABI.
"""

from __future__ import annotations

import ast
from copy import deepcopy
from dataclasses import dataclass, field

import numpy as np

from .dag_preprocessing import (SyncFreeExecutionData, WarpTaskExecutionData,
                                WavefrontExecutionData)

HOST_LAUNCH_ARGUMENTS = frozenset({"wavefront_ptr", "band_ptr"})


class CUDARuntimePreparationError(Exception):
    """Lowered launcher arguments cannot be prepared."""


class CUDAModuleCompilationError(Exception):
    """A native kernel binding cannot be created."""


# Page-locked result buffers.  Allocating one costs about 12 ms per 32 MB, so a few are kept
# and handed out again - but only once the array that was returned to the caller is gone: the
# pool keeps a weak reference to that array, and every view or tensor made from it keeps it
# alive (a view's ``base`` is the array), so a dead reference means nobody can still read it.
_PINNED_BLOCKS = {}
_PINNED_BLOCKS_PER_SHAPE = 4


def _pinned_result(shape, dtype):
    """(page-locked tensor, its NumPy array) for a result of this shape; the array is what the
    caller receives."""
    import weakref
    import torch
    blocks = _PINNED_BLOCKS.setdefault((shape, dtype), [])
    for entry in blocks:
        block, alive = entry
        if alive() is None:
            array = block.numpy()
            entry[1] = weakref.ref(array)
            return block, array
    block = torch.empty(shape, dtype=dtype, pin_memory=True)
    array = block.numpy()
    if len(blocks) < _PINNED_BLOCKS_PER_SHAPE:
        blocks.append([block, weakref.ref(array)])
    return block, array


# Page-locked host arrays of at least twice this size are uploaded in pieces (a quarter of this
# size first, then doubling) on a copy stream of their own, with an event after each piece: a launcher that consumes its input
# front to back (the chain solver) starts on the first rows while the rest is still in flight.
STREAMED_UPLOAD_BYTES = 64 << 20
_COPY_STREAMS = {}


def _copy_stream(kind="upload"):
    import torch
    key = (torch.cuda.current_device(), kind)
    if key not in _COPY_STREAMS:
        _COPY_STREAMS[key] = torch.cuda.Stream(device=key[0])
    return _COPY_STREAMS[key]


class DeviceArray:
    """A CUDA tensor with the two members the runtime contract relies on:
    ``__cuda_array_interface__`` and ``copy_to_host()``.

    ``arrival`` is None, or the list of (elements uploaded so far, event) of an upload that is
    still in flight.  Reading ``tensor`` makes the current stream wait for the whole upload; a
    launcher that wants to follow the pieces takes the list with ``take_arrival()`` and waits
    for the events itself."""

    _early = None     # [page-locked tensor, its array, rows already on their way] of download_rows

    def __init__(self, tensor, arrival=None):
        self._tensor = tensor
        self.arrival = arrival

    @property
    def tensor(self):
        if self.arrival:
            import torch
            torch.cuda.current_stream().wait_event(self.arrival[-1][1])
            self.arrival = None
        return self._tensor

    def take_arrival(self):
        """(tensor, pieces) with the waiting left to the caller; pieces is None once awaited."""
        pieces, self.arrival = self.arrival, None
        return self._tensor, pieces

    @property
    def __cuda_array_interface__(self):
        return self.tensor.__cuda_array_interface__

    @property
    def shape(self):
        return tuple(self._tensor.shape)

    def copy_to_host(self):
        # through page-locked memory: a copy into a fresh pageable array runs at a few GB/s
        # (33 MB took 15 ms)
        if self._early is not None:
            # a launcher that produces the array front to back has sent most of it already
            (host, array, upto), self._early = self._early, None
            _copy_stream("download").synchronize()
            if upto < self._tensor.shape[0]:
                host[upto:].copy_(self.tensor[upto:])
            return array
        if self.tensor.numel() * self.tensor.element_size() < (1 << 16):
            return self.tensor.cpu().numpy()
        host, array = _pinned_result(tuple(self.tensor.shape), self.tensor.dtype)
        host.copy_(self.tensor)
        return array

    def download_rows(self, begin, end):
        """Start the copy of rows [begin, end) to the page-locked array that ``copy_to_host()``
        will return, behind the work queued on the current stream so far.  For launchers that
        finish their result front to back (ranges must follow one another from row 0; anything
        else is ignored and copied at the end)."""
        import torch
        if self._early is None:
            if begin != 0:
                return
            host, array = _pinned_result(tuple(self._tensor.shape), self._tensor.dtype)
            self._early = [host, array, 0]
        host, _, upto = self._early
        if begin != upto or end <= begin:
            return
        stream = _copy_stream("download")
        stream.wait_stream(torch.cuda.current_stream())
        self._tensor.record_stream(stream)
        with torch.cuda.stream(stream):
            host[begin:end].copy_(self._tensor[begin:end], non_blocking=True)
        self._early[2] = end

    def forget_downloads(self):
        """The rows sent so far are stale (the launcher computes the result again)."""
        if self._early is not None:
            _copy_stream("download").synchronize()
            self._early = None

    def __len__(self):
        return self._tensor.shape[0]


class LazyDeviceArray(DeviceArray):
    """A device array that is only computed when somebody reads it (executor arrays that the
    chosen kernel does not use, e.g. the level order next to a solver that ignores levels)."""

    def __init__(self, make, length):
        self._make, self._made, self._length = make, None, int(length)
        self.arrival = None

    @property
    def _tensor(self):
        if self._made is None:
            self._made = self._make()
        return self._made

    @property
    def shape(self):
        return (self._length,)

    def __len__(self):
        return self._length


class LazyHostArray:
    """Host counterpart: turns into a NumPy array on first use (``np.asarray`` and friends)."""

    def __init__(self, make):
        self._make, self._made = make, None

    def _array(self):
        if self._made is None:
            self._made = np.asarray(self._make())
        return self._made

    def __array__(self, dtype=None, copy=None):
        array = self._array()
        return array if dtype is None else array.astype(dtype, copy=False)

    def __len__(self):
        return len(self._array())

    def __getitem__(self, item):
        return self._array()[item]

    def copy(self):
        return self._array().copy()


class TorchCUDA:
    """The ``cuda`` object of a bound module: ``to_device`` and ``synchronize``
    (the two calls ``cuda_runtime`` makes on Numba's ``cuda`` in the reference)."""

    @staticmethod
    def to_device(array):
        import torch
        host = torch.from_numpy(np.ascontiguousarray(array))
        pinned = host.is_pinned()
        if not (pinned and host.dim() == 1 and
                host.numel() * host.element_size() >= 2 * STREAMED_UPLOAD_BYTES):
            return DeviceArray(host.to("cuda", non_blocking=pinned))
        return TorchCUDA.to_device_together([array])[0]

    @staticmethod
    def to_device_split(array, head):
        """Upload the first ``head`` elements of a page-locked 1-D array now; the returned
        ``finish()`` queues the rest (call it once, after whatever should travel in between).
        The ``DeviceArray`` carries both pieces in its arrival list."""
        import torch
        host = torch.from_numpy(np.ascontiguousarray(array))
        device = torch.empty(host.shape, dtype=host.dtype, device="cuda")
        copies = _copy_stream()
        copies.wait_stream(torch.cuda.current_stream())
        device.record_stream(copies)
        arrival = []

        def piece(start, end):
            with torch.cuda.stream(copies):
                device[start:end].copy_(host[start:end], non_blocking=True)
                event = torch.cuda.Event()
                event.record(copies)
            arrival.append((end, event))

        head = max(1, min(int(head), host.numel()))
        piece(0, head)
        if head == host.numel():
            return DeviceArray(device, arrival), lambda: None
        # (the list is complete before anybody can read it: finish() runs inside the same
        # start_large_uploads call)
        return DeviceArray(device, arrival), lambda: piece(head, host.numel())

    @staticmethod
    def to_device_together(arrays, after_first=None):
        """Streamed upload of page-locked 1-D arrays of one length (the column indices and the
        values of a sparse matrix): every array is cut at the same element positions and the
        pieces are issued in turn, so that after the k-th piece of the last array the first
        ``end_k`` elements of all of them are on the device.  One ``DeviceArray`` per array,
        each with its own list of (elements uploaded so far, event).  ``after_first()`` is called
        when the first pieces have been queued (for a copy that may wait until then)."""
        import torch
        hosts = [torch.from_numpy(np.ascontiguousarray(a)) for a in arrays]
        count = hosts[0].numel()
        if any(h.dim() != 1 or h.numel() != count or not h.is_pinned() for h in hosts):
            raise CUDARuntimePreparationError(
                "arrays uploaded together must be page-locked, one-dimensional and of one length")
        devices = [torch.empty(h.shape, dtype=h.dtype, device="cuda") for h in hosts]
        copies = _copy_stream()
        copies.wait_stream(torch.cuda.current_stream())   # the blocks may just have been in use there
        for device in devices:
            device.record_stream(copies)
        step = STREAMED_UPLOAD_BYTES // max(h.element_size() for h in hosts)
        arrivals = [[] for _ in hosts]
        with torch.cuda.stream(copies):
            start, piece = 0, step // 4
            while start < count:
                # (a short first piece: whoever follows the pieces starts early; then doubling:
                # the link is faster than any consumer here, and fewer pieces mean fewer launches)
                end = min(count, start + piece)
                piece *= 2
                for host, device, arrival in zip(hosts, devices, arrivals):
                    device[start:end].copy_(host[start:end], non_blocking=True)
                    event = torch.cuda.Event()
                    event.record(copies)
                    arrival.append((end, event))
                if start == 0 and after_first is not None:
                    after_first()           # (queues on the same copy stream)
                start = end
        return [DeviceArray(device, arrival) for device, arrival in zip(devices, arrivals)]

    @staticmethod
    def synchronize():
        import torch
        torch.cuda.synchronize()

    @staticmethod
    def device_array(shape, dtype):
        import torch
        torch_dtype = torch.from_numpy(np.zeros(0, dtype=dtype)).dtype
        return DeviceArray(torch.empty(shape, dtype=torch_dtype, device="cuda"))


def as_tensor(value, dtype=None):
    """View any device array of the contract as a torch tensor (no copy)."""
    import torch
    if isinstance(value, DeviceArray):
        tensor = value.tensor
    elif isinstance(value, torch.Tensor):
        tensor = value
    elif hasattr(value, "__cuda_array_interface__"):
        tensor = torch.as_tensor(value, device="cuda")
    else:
        raise CUDARuntimePreparationError(
            f"expected a device array, received {type(value).__name__}")
    if dtype is not None and tensor.dtype != dtype:
        tensor = tensor.to(dtype)
    return tensor.contiguous()


@dataclass
class CompiledCUDAModule:
    """Callables and globals belonging to one bound operator schedule."""

    kernel: object
    launcher: object
    namespace: dict


@dataclass
class CUDAPreparedArguments:
    """Host/device values ordered for a launcher."""

    launcher_argument_names: tuple
    values: dict
    host_values: dict
    lifted_variables: tuple
    hints: dict = field(default_factory=dict)   # what the inspector learnt (rows, levels, ...)
    verify: object = None   # set when the call started under a predicted plan: () -> plan was right

    @property
    def launcher_arguments(self):
        return tuple(self.values[name] for name in self.launcher_argument_names)

    def copy_to_host(self, name):
        if name not in self.values:
            raise CUDARuntimePreparationError(f"Unknown prepared CUDA argument {name!r}.")
        value = self.values[name]
        method = getattr(value, "copy_to_host", None)
        return method() if method is not None else value

    def copy_lifted_variables_to_host(self):
        return {name: self.copy_to_host(name) for name in self.lifted_variables}


def compile_cuda_module(lowering, function_globals=None, cuda_module=None):
    """Bind the native kernel and launcher of one lowering.

    Nothing is compiled at run time: the kernels were built ahead of time for
    sm_100a; a missing library raises (there is no other implementation)."""
    from . import _native, launchers
    namespace = dict(function_globals or {})
    namespace["cuda"] = cuda_module if cuda_module is not None else TorchCUDA
    try:
        _native.load()
        kernel, launcher = launchers.bind(lowering)
    except Exception as error:
        raise CUDAModuleCompilationError(
            f"Failed to bind the native kernel for {lowering.operator!r}: {error}") from error
    namespace[lowering.kernel_name] = kernel
    namespace[lowering.launcher_name] = launcher
    return CompiledCUDAModule(kernel=kernel, launcher=launcher, namespace=namespace)


def prepare_cuda_arguments(lowering, argument_values, execution_data, function_globals=None,
                           cuda_module=None):
    """Create lifted locals and prepare all launcher arguments."""
    if cuda_module is None:
        cuda_module = TorchCUDA
    host_values = dict(argument_values)
    prelude_names = _stored_names(lowering.host_prelude)
    if not all(name in host_values for name in prelude_names):
        # (callers that already evaluated the prelude pass its values along)
        host_values.update(_evaluate_host_prelude(lowering, host_values, function_globals or {}))
    host_values.update(_execution_values(lowering.execution_mode, execution_data))
    missing = [name for name in lowering.launcher_arguments if name not in host_values]
    if missing:
        raise CUDARuntimePreparationError(
            "Values are missing for generated launcher arguments: " + ", ".join(missing))
    device_only = set(getattr(lowering, "device_only_variables", ()))
    prepared = {}
    # small arrays first: an upload that is streamed in pieces must not sit in front of them on
    # the copy engine (the launcher that follows the pieces needs the other arguments complete)
    def upload_order(name):
        value = host_values[name]
        return value.nbytes if isinstance(value, np.ndarray) else 0
    for name in sorted(lowering.launcher_arguments, key=upload_order):
        value = host_values[name]
        if name in HOST_LAUNCH_ARGUMENTS:
            prepared[name] = value  # the host launcher reads the offsets
        elif (name in device_only and isinstance(value, np.ndarray)
              and hasattr(cuda_module, "device_array")):
            # an output the kernel overwrites completely: allocate, do not upload
            prepared[name] = cuda_module.device_array(value.shape, value.dtype)
        else:
            prepared[name] = _prepare_value(value, cuda_module)
    return CUDAPreparedArguments(tuple(lowering.launcher_arguments), prepared, host_values,
                                 tuple(lowering.lifted_variables))


def evaluate_host_prelude(lowering, argument_values, function_globals=None):
    """Evaluate the removed host statements (e.g. ``n = len(indptr) - 1``)."""
    return _evaluate_host_prelude(lowering, argument_values, function_globals or {})


def execute_cuda_call(compiled_module, lowering, prepared_arguments, function_globals=None):
    """Launch prepared work and restore the original return semantics."""
    launcher = compiled_module.launcher
    if prepared_arguments.hints and getattr(launcher, "accepts_hints", False):
        launcher(*prepared_arguments.launcher_arguments, _hints=prepared_arguments.hints)
    else:
        launcher(*prepared_arguments.launcher_arguments)
    cuda_module = compiled_module.namespace.get("cuda")
    if cuda_module is None or not hasattr(cuda_module, "synchronize"):
        raise CUDARuntimePreparationError(
            "The compiled CUDA module does not provide cuda.synchronize().")
    cuda_module.synchronize()
    results = dict(prepared_arguments.host_values)
    # returned arguments and lifted locals come back to the host; a name that is both
    # (the usual ``x``) is copied once
    names = [name for name in _returned_names(lowering.host_epilogue)
             if name in prepared_arguments.values]
    names += [name for name in prepared_arguments.lifted_variables if name not in names]
    results.update({name: prepared_arguments.copy_to_host(name) for name in names})
    return _evaluate_host_epilogue(lowering, results, function_globals or {})


_CODE_CACHE = {}


def _compiled(statements, build, filename):
    """Code object for a list of AST statements, compiled once (keyed by the list object, which
    belongs to a lowering that lives as long as its decorated function)."""
    entry = _CODE_CACHE.get(id(statements))
    if entry is None or entry[0] is not statements:
        if len(_CODE_CACHE) > 256:
            _CODE_CACHE.clear()
        entry = _CODE_CACHE[id(statements)] = (statements, compile(build(), filename=filename, mode="exec"))
    return entry[1]


def _evaluate_host_prelude(lowering, argument_values, function_globals):
    if not lowering.host_prelude:
        return {}
    namespace = dict(function_globals)
    namespace.update(argument_values)
    code = _compiled(lowering.host_prelude, lambda: ast.fix_missing_locations(
        ast.Module(body=deepcopy(lowering.host_prelude), type_ignores=[])), "<cuda-host-prelude>")
    exec(code, namespace, namespace)
    missing = [name for name in lowering.lifted_variables if name not in namespace]
    if missing:
        raise CUDARuntimePreparationError(
            "The removed host prelude did not define lifted variables: " + ", ".join(missing))
    return {name: namespace[name] for name in _stored_names(lowering.host_prelude)
            if name in namespace}


def _evaluate_host_epilogue(lowering, result_values, function_globals):
    if not lowering.host_epilogue:
        return None
    namespace = dict(function_globals)
    namespace.update(result_values)

    def build():
        helper = ast.FunctionDef(
            name="_lcd_host_epilogue",
            args=ast.arguments(posonlyargs=[], args=[], kwonlyargs=[], kw_defaults=[], defaults=[]),
            body=deepcopy(lowering.host_epilogue), decorator_list=[], returns=None,
            type_comment=None)
        if hasattr(helper, "type_params"):
            helper.type_params = []
        return ast.fix_missing_locations(ast.Module(body=[helper], type_ignores=[]))
    exec(_compiled(lowering.host_epilogue, build, "<cuda-host-epilogue>"), namespace, namespace)
    try:
        return namespace["_lcd_host_epilogue"]()
    finally:
        # the helper's globals are this namespace, which holds the helper: without this the
        # result arrays (and their page-locked buffers) would live until the next collection
        namespace.clear()


_NAME_CACHE = {}


def _cached_names(kind, statements, compute):
    """Name lists of a statement list, walked once (keyed like the compiled code above)."""
    key = (kind, id(statements))
    entry = _NAME_CACHE.get(key)
    if entry is None or entry[0] is not statements:
        if len(_NAME_CACHE) > 512:
            _NAME_CACHE.clear()
        entry = _NAME_CACHE[key] = (statements, tuple(compute(statements)))
    return list(entry[1])


def _returned_names(statements):
    return _cached_names("returned", statements, _walk_returned_names)


def _stored_names(statements):
    return _cached_names("stored", statements, _walk_stored_names)


def _walk_returned_names(statements):
    names = []
    for statement in statements:
        for node in ast.walk(statement):
            if isinstance(node, ast.Return) and node.value is not None:
                for value in ast.walk(node.value):
                    if (isinstance(value, ast.Name) and isinstance(value.ctx, ast.Load)
                            and value.id not in names):
                        names.append(value.id)
    return names


def _walk_stored_names(statements):
    names = []
    for statement in statements:
        for node in ast.walk(statement):
            if (isinstance(node, ast.Name) and isinstance(node.ctx, ast.Store)
                    and node.id not in names):
                names.append(node.id)
    return names


def _zeros_like_count(count_array, length=None, device_like=None):
    """int32 zeros next to an existing executor array (device or host)."""
    try:
        import torch
        if isinstance(count_array, torch.Tensor):
            n = count_array.numel() if length is None else length
            device = count_array.device
            if device.type == "cuda":
                # made when a launcher reads it (the native kernels that poll operands instead
                # of counting never do: two allocations and fills less per call)
                return LazyDeviceArray(lambda: torch.zeros(n, dtype=torch.int32, device=device), n)
            return torch.zeros(n, dtype=torch.int32, device=device)
    except ImportError:  # pragma: no cover
        pass
    n = len(count_array) if length is None else length
    return np.zeros(n, dtype=np.int32)


def _copy_of(array):
    return array.clone() if hasattr(array, "clone") else array.copy()


def _execution_values(execution_mode, execution_data):
    execution_mode = execution_mode.replace("-", "_")
    if isinstance(execution_data, WarpTaskExecutionData):
        initial = execution_data.initial_dep_count
        if initial is None:
            initial = _copy_of(execution_data.dep_count)
        return _with_auxiliary_values({
            "task_nodes": execution_data.task_nodes,
            "task_ptr": execution_data.task_ptr,
            "band_ptr": execution_data.band_ptr,
            "task_counter": _zeros_like_count(execution_data.dep_count, 1),
            "done": _zeros_like_count(execution_data.dep_count),
            "dep_count": execution_data.dep_count,
            "initial_dep_count": initial,
            "dag_ptr": execution_data.dag_ptr,
            "dag_index": execution_data.dag_index,
        }, execution_data)
    if execution_mode == "sync_free":
        if not isinstance(execution_data, SyncFreeExecutionData):
            raise CUDARuntimePreparationError(
                "Sync-free lowering requires SyncFreeExecutionData.")
        initial = execution_data.initial_dep_count
        if initial is None:
            initial = _copy_of(execution_data.dep_count)
        return _with_auxiliary_values({
            "dep_count": execution_data.dep_count,
            "initial_dep_count": initial,
            "dag_ptr": execution_data.dag_ptr,
            "dag_index": execution_data.dag_index,
        }, execution_data)
    if execution_mode == "wavefront":
        if not isinstance(execution_data, WavefrontExecutionData):
            raise CUDARuntimePreparationError(
                "Wavefront lowering requires WavefrontExecutionData.")
        return _with_auxiliary_values({
            "wavefronts": execution_data.wavefronts,
            "wavefront_ptr": execution_data.wavefront_ptr,
        }, execution_data)
    return {}


def _with_auxiliary_values(values, execution_data):
    auxiliary = getattr(execution_data, "auxiliary_values", {})
    collisions = set(values) & set(auxiliary)
    if collisions:
        raise CUDARuntimePreparationError(
            "Auxiliary values conflict with executor arguments: " + ", ".join(sorted(collisions)))
    values.update(auxiliary)
    return values


def _prepare_value(value, cuda_module):
    if _is_cuda_array(value) or np.isscalar(value) or value is None:
        return value
    if isinstance(value, (list, tuple)):
        value = np.asarray(value)
    if isinstance(value, np.ndarray):
        return cuda_module.to_device(value)
    raise CUDARuntimePreparationError(
        "CUDA launcher arguments must be scalars, NumPy arrays, sequences, or existing CUDA "
        f"arrays; received {type(value).__name__}.")


def _is_cuda_array(value):
    # (a DeviceArray first: asking it for the interface would wait for an upload in flight;
    # host arrays and scalars next, and a torch tensor by its own flag: torch builds the whole
    # interface dictionary for every look at the attribute, 4 us a time)
    if isinstance(value, DeviceArray):
        return True
    if value is None or isinstance(value, (np.ndarray, np.generic, int, float, list, tuple)):
        return False
    is_cuda = getattr(value, "is_cuda", None)
    if isinstance(is_cuda, bool):
        return is_cuda
    return hasattr(value, "__cuda_array_interface__")


def start_large_uploads(values, skip=(), together=(), late=()):
    """Begin the upload of the page-locked arrays among ``values`` (a dict, changed in place) if
    one of them is large enough to be streamed in pieces, so that the transfer overlaps the host
    work that follows.  Smaller arrays go first: the launcher that follows the pieces needs
    them complete.  The arrays named in ``together`` (one length, e.g. a matrix's column
    indices and values) go last and travel side by side, cut at the same element positions,
    so that a consumer that follows the pieces has whole rows early; of the arrays named in
    ``late`` (a right-hand side that the same consumer reads front to back) only the first
    sixteenth goes before them, the rest behind their first pieces.  Everything else stays as
    it is."""
    import torch
    pinned = [(value.nbytes, name) for name, value in values.items()
              if name not in skip and isinstance(value, np.ndarray) and value.ndim == 1
              and value.flags.c_contiguous and value.nbytes >= (1 << 20)
              and torch.from_numpy(value).is_pinned()]
    if not pinned or max(pinned)[0] < 2 * STREAMED_UPLOAD_BYTES:
        return
    side_by_side = [name for name in together if any(name == found for _, found in pinned)]
    if len(side_by_side) < 2:
        side_by_side = []
    finish = []
    for nbytes, name in sorted(pinned):
        if name in side_by_side:
            continue
        if side_by_side and name in late and nbytes >= STREAMED_UPLOAD_BYTES // 8:
            values[name], rest = TorchCUDA.to_device_split(values[name], len(values[name]) // 16)
            finish.append(rest)
        else:
            values[name] = TorchCUDA.to_device(values[name])
    if side_by_side:
        arrays = TorchCUDA.to_device_together([values[name] for name in side_by_side],
                                              after_first=lambda: [rest() for rest in finish])
        values.update(zip(side_by_side, arrays))
