"""Executor data structures of the dependence DAG.

Mirrors the interface of the reference's ``compiler/dag_preprocessing.py``
(``:12-51`` data classes, ``:54-112`` entry points, ``:115-143`` successor
compaction, ``:146-204`` wavefronts, ``:207-255`` warp tasks): the same names,
argument meaning, array dtypes (``int32``) and ``DAGPreprocessingError``
behaviour.  Two kinds of input are accepted everywhere:

* a :class:`lcd_b200.ops.DeviceDag` -- the arrays already built on the GPU by
  ``lcd_dag_build``; this is what the decorator passes (no host work at all);
* the reference's Python successor lists -- host-side format conversion for
  small inputs and for interface compatibility (validation and errors as in the
  reference).  This is list handling, not a solver path.
"""

from __future__ import annotations

from dataclasses import dataclass, field, replace

import numpy as np


class DAGPreprocessingError(Exception):
    """Raised when DAG data cannot form executor inputs."""


@dataclass(frozen=True)
class SyncFreeExecutionData:
    """CSR successors and mutable incoming-dependency counts."""

    dep_count: object
    dag_ptr: object
    dag_index: object
    initial_dep_count: object = None
    auxiliary_values: dict = field(default_factory=dict)

    @property
    def launcher_arguments(self):
        return self.dep_count, self.dag_ptr, self.dag_index


@dataclass(frozen=True)
class WavefrontExecutionData:
    """Flattened wavefront nodes and offsets for each wavefront."""

    wavefronts: object
    wavefront_ptr: object
    auxiliary_values: dict = field(default_factory=dict)

    @property
    def launcher_arguments(self):
        return self.wavefronts, self.wavefront_ptr


@dataclass(frozen=True)
class WarpTaskExecutionData:
    task_nodes: object
    task_ptr: object
    band_ptr: object
    dep_count: object
    dag_ptr: object
    dag_index: object
    initial_dep_count: object = None
    auxiliary_values: dict = field(default_factory=dict)


def _is_device_dag(value):
    # (asked of the class: reading the level arrays of a capped device DAG would build them)
    kind = type(value)
    return hasattr(value, "dag_ptr") and hasattr(kind, "wavefront_ptr") and hasattr(kind, "level")


def preprocess_dag_output(dag_successors, scheduling_data, execution_mode):
    """Convert inspector output to the selected executor format."""
    execution_mode = execution_mode.replace("-", "_")
    if execution_mode == "sync_free":
        return preprocess_sync_free(dag_successors, scheduling_data)
    if execution_mode == "wavefront":
        return preprocess_wavefront(dag_successors, scheduling_data)
    raise DAGPreprocessingError(
        f"Unknown execution mode {execution_mode!r}; expected sync_free or wavefront.")


def attach_auxiliary_values(execution_data, auxiliary_values):
    """Attach immutable inspector outputs (lookup tables) to executor data."""
    if not auxiliary_values:
        return execution_data
    if not isinstance(execution_data, (SyncFreeExecutionData, WavefrontExecutionData,
                                       WarpTaskExecutionData)):
        raise DAGPreprocessingError("Auxiliary values require recognized DAG execution data.")
    collisions = set(execution_data.auxiliary_values) & set(auxiliary_values)
    if collisions:
        raise DAGPreprocessingError(
            "Duplicate auxiliary execution values: " + ", ".join(sorted(collisions)))
    combined = dict(execution_data.auxiliary_values)
    combined.update(auxiliary_values)
    return replace(execution_data, auxiliary_values=combined)


# ---- host-side list handling ------------------------------------------------
def compact_successors(dag_successors):
    """Successor lists -> CSR ``dag_ptr`` / ``dag_index`` (ascending, distinct)."""
    node_count = len(dag_successors)
    dag_ptr = np.zeros(node_count + 1, dtype=np.int32)
    chunks = []
    for source, successors in enumerate(dag_successors):
        try:
            unique = np.unique(np.asarray([int(d) for d in successors], dtype=np.int64))
        except (TypeError, ValueError) as error:
            raise DAGPreprocessingError(f"Invalid successor list for node {source}.") from error
        if unique.size and (unique[0] < 0 or unique[-1] >= node_count):
            bad = int(unique[0] if unique[0] < 0 else unique[-1])
            raise DAGPreprocessingError(f"DAG edge {source} -> {bad} is out of bounds.")
        chunks.append(unique)
        dag_ptr[source + 1] = dag_ptr[source] + unique.size
    dag_index = (np.concatenate(chunks) if chunks else np.zeros(0)).astype(np.int32)
    return dag_ptr, dag_index


def wavefronts_from_dag(dag_successors, dep_count):
    """Kahn levels: a node joins the level after its last predecessor's level;
    each level lists its nodes in ascending order."""
    if _is_device_dag(dag_successors):
        dag = dag_successors
        nodes = dag.wavefronts.cpu().numpy()
        ptr = dag.wavefront_ptr_host
        return [nodes[ptr[k]:ptr[k + 1]].tolist() for k in range(len(ptr) - 1)]
    remaining = [int(c) for c in dep_count]
    levels = []
    frontier = [node for node, count in enumerate(remaining) if count == 0]
    while frontier:
        levels.append(frontier)
        released = set()
        for node in frontier:
            for successor in dag_successors[node]:
                remaining[successor] -= 1
                if remaining[successor] == 0:
                    released.add(successor)
        frontier = sorted(released)
    return levels


def preprocess_sync_free(dag_successors, dep_count=None):
    """CSR out-edge arrays plus (consumable and pristine) dependency counts."""
    if _is_device_dag(dag_successors):
        dag = dag_successors
        return SyncFreeExecutionData(dep_count=dag.dep_count.clone(),
                                     initial_dep_count=dag.dep_count,
                                     dag_ptr=dag.dag_ptr, dag_index=dag.dag_index)
    dag_ptr, dag_index = compact_successors(dag_successors)
    dep_count = np.asarray(dep_count, dtype=np.int32)
    if dep_count.ndim != 1 or len(dep_count) != len(dag_successors):
        raise DAGPreprocessingError("dep_count must contain one value for every DAG node.")
    if np.any(dep_count < 0):
        raise DAGPreprocessingError("Dependency counts cannot be negative.")
    return SyncFreeExecutionData(dep_count=dep_count.copy(), initial_dep_count=dep_count.copy(),
                                 dag_ptr=dag_ptr, dag_index=dag_index)


def preprocess_wavefront(dag_successors, wavefront_list=None):
    """Flatten wavefronts; every node must be scheduled exactly once."""
    if _is_device_dag(dag_successors):
        dag = dag_successors
        # wavefront_ptr stays on the host: the launcher reads it to size launches
        return WavefrontExecutionData(wavefronts=dag.wavefronts,
                                      wavefront_ptr=dag.wavefront_ptr_host)
    node_count = len(dag_successors)
    values = []
    wavefront_ptr = np.zeros(len(wavefront_list) + 1, dtype=np.int32)
    seen = np.zeros(node_count, dtype=bool)
    for number, wavefront in enumerate(wavefront_list):
        try:
            nodes = [int(node) for node in wavefront]
        except (TypeError, ValueError) as error:
            raise DAGPreprocessingError(f"Invalid node in wavefront {number}.") from error
        for node in nodes:
            if not 0 <= node < node_count:
                raise DAGPreprocessingError(f"Wavefront node {node} is out of bounds.")
            if seen[node]:
                raise DAGPreprocessingError(
                    f"DAG node {node} occurs in more than one wavefront.")
            seen[node] = True
        values.extend(nodes)
        wavefront_ptr[number + 1] = len(values)
    if not seen.all():
        missing = np.flatnonzero(~seen).tolist()
        raise DAGPreprocessingError(
            "Wavefront scheduling did not cover every DAG node; the DAG may "
            f"contain a cycle. Missing nodes: {missing}.")
    return WavefrontExecutionData(wavefronts=np.asarray(values, dtype=np.int32),
                                  wavefront_ptr=wavefront_ptr)


def preprocess_warp_tasks(dag_successors, wavefront_list=None, band_width=1, edge_count=None):
    """One task per node in wavefront order (``band_width == 1``) or chains of
    nodes connected inside ``band_width`` consecutive levels."""
    if not isinstance(band_width, int) or isinstance(band_width, bool) or band_width <= 0:
        raise DAGPreprocessingError("The band width must be a positive integer.")
    if _is_device_dag(dag_successors):
        dag = dag_successors
        if band_width != 1:
            from . import ops
            task_nodes, task_ptr, band_ptr = ops.band_chains(dag, band_width)
            band_ptr = band_ptr.cpu().numpy()          # band offsets stay on the host
        else:
            import torch
            task_ptr = torch.arange(dag.n + 1, dtype=torch.int32, device=dag.dep_count.device)
            if getattr(dag, "capped", False):
                # a deep DAG whose level sets were not built (the chain solver reads none): the
                # level order is computed only if somebody asks for it
                from .cuda_runtime import LazyDeviceArray, LazyHostArray
                task_nodes = LazyDeviceArray(lambda: dag.wavefronts, dag.n)
                band_ptr = LazyHostArray(lambda: dag.wavefront_ptr_host.copy())
            else:
                task_nodes = dag.wavefronts
                band_ptr = dag.wavefront_ptr_host.copy()
        count = dag.dep_count if edge_count is None else edge_count
        return WarpTaskExecutionData(task_nodes=task_nodes, task_ptr=task_ptr, band_ptr=band_ptr,
                                     dep_count=count.clone(), initial_dep_count=count,
                                     dag_ptr=dag.dag_ptr, dag_index=dag.dag_index)
    node_count = len(dag_successors)
    dag_ptr, dag_index = compact_successors(dag_successors)
    wavefront_data = preprocess_wavefront(dag_successors, wavefront_list)
    nodes, level_ptr = wavefront_data.wavefronts, wavefront_data.wavefront_ptr
    if edge_count is None:
        dep_count = np.bincount(dag_index, minlength=node_count).astype(np.int32)
    else:
        dep_count = np.asarray(edge_count, dtype=np.int32)
        if dep_count.shape != (node_count,):
            raise DAGPreprocessingError("edge_count must contain one value for every DAG node.")
    if band_width == 1:
        task_nodes = nodes
        task_ptr = np.arange(node_count + 1, dtype=np.int32)
        band_ptr = level_ptr.copy()
    else:
        task_nodes, task_ptr, band_ptr = _band_chains(nodes, level_ptr, dag_ptr, dag_index,
                                                      band_width)
    return WarpTaskExecutionData(task_nodes=task_nodes, task_ptr=task_ptr, band_ptr=band_ptr,
                                 dep_count=dep_count.copy(), initial_dep_count=dep_count.copy(),
                                 dag_ptr=dag_ptr, dag_index=dag_index)


def _band_chains(nodes, level_ptr, dag_ptr, dag_index, band_width):
    """Tasks for ``band_width`` > 1 from host arrays (the list form of the API): inside every band
    of ``band_width`` levels, the connected components of the DAG edges that stay in the band,
    listed by their first node in level order.  SciPy's connected-components labelling does the
    grouping; components are then ranked by the position of their first node."""
    from scipy.sparse import coo_matrix
    from scipy.sparse.csgraph import connected_components
    nodes = np.asarray(nodes, dtype=np.int64)
    level_ptr = np.asarray(level_ptr, dtype=np.int64)
    n = len(nodes)
    level_count = len(level_ptr) - 1
    n_bands = -(-level_count // band_width) if level_count else 0
    if n == 0:
        return (np.zeros(0, np.int32), np.zeros(1, np.int32), np.zeros(n_bands + 1, np.int32))
    position = np.empty(n, dtype=np.int64)
    position[nodes] = np.arange(n)
    level_of_position = np.repeat(np.arange(level_count), np.diff(level_ptr))
    band_of_node = (level_of_position // band_width)[position]
    source = np.repeat(np.arange(n), np.diff(np.asarray(dag_ptr, dtype=np.int64)))
    target = np.asarray(dag_index, dtype=np.int64)
    inside = band_of_node[source] == band_of_node[target]
    graph = coo_matrix((np.ones(int(inside.sum()), dtype=np.int8),
                        (position[source[inside]], position[target[inside]])), shape=(n, n))
    _, component = connected_components(graph, directed=False)
    first = np.full(component.max() + 1, n, dtype=np.int64)
    np.minimum.at(first, component, np.arange(n))
    label = first[component]                       # position of the component's first node
    order = np.argsort(label, kind="stable")
    heads = np.flatnonzero(np.r_[True, label[order][1:] != label[order][:-1]])
    task_ptr = np.r_[heads, n]
    band_first = level_ptr[np.minimum(np.arange(n_bands + 1) * band_width, level_count)]
    band_ptr = np.searchsorted(heads, band_first, side="left")
    return (nodes[order].astype(np.int32), task_ptr.astype(np.int32), band_ptr.astype(np.int32))
