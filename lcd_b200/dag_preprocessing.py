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
    return hasattr(value, "dag_ptr") and hasattr(value, "wavefront_ptr") and hasattr(value, "level")


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
            dag_ptr = dag.dag_ptr.cpu().numpy()
            dag_index = dag.dag_index.cpu().numpy()
            nodes = dag.wavefronts.cpu().numpy()
            task_nodes, task_ptr, band_ptr = _band_chains(nodes, dag.wavefront_ptr_host, dag_ptr,
                                                          dag_index, band_width)
        else:
            import torch
            task_nodes = dag.wavefronts
            task_ptr = torch.arange(dag.n + 1, dtype=torch.int32, device=dag.wavefronts.device)
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
    """Connected components (in order of first appearance) of each band of levels."""
    level_count = len(level_ptr) - 1
    task_nodes, task_ptr, band_ptr = [], [0], [0]
    for first in range(0, level_count, band_width):
        last = min(first + band_width, level_count)
        band = [int(v) for v in nodes[level_ptr[first]:level_ptr[last]]]
        position_of = {node: position for position, node in enumerate(band)}
        parent = list(range(len(band)))

        def find(position):
            root = position
            while parent[root] != root:
                root = parent[root]
            while parent[position] != root:
                parent[position], position = root, parent[position]
            return root

        for position, node in enumerate(band):
            for successor in dag_index[dag_ptr[node]:dag_ptr[node + 1]]:
                other = position_of.get(int(successor))
                if other is not None:
                    a, b = find(position), find(other)
                    if a != b:
                        parent[b] = a
        chains = {}
        for position, node in enumerate(band):
            chains.setdefault(find(position), []).append(node)
        for chain in chains.values():
            task_nodes.extend(chain)
            task_ptr.append(len(task_nodes))
        band_ptr.append(len(task_ptr) - 1)
    return (np.asarray(task_nodes, dtype=np.int32), np.asarray(task_ptr, dtype=np.int32),
            np.asarray(band_ptr, dtype=np.int32))
