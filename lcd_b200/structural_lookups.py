"""Diagonal-position tables ("structural lookups") built on the GPU.

Interface of the reference's ``compiler/structural_lookups.py``: a search of the
form ``for p in range(ptr[s], ptr[s + 1]): if idx[p] == s: ...; break`` over a
pair of arrays declared ``segmented_monotonically_increasing`` is replaced by a
table ``pos[s]`` (``int32``, ``-1`` when segment ``s`` does not store ``s``).
Plan creation (``:55-92``) is AST matching on the host; the table itself
(``:108-124``, ``:279-333``) is produced by the ``lcd_diag_positions`` kernel,
which also performs the reference's validation (monotone pointers, sorted
segments) and reports it as :class:`StructuralLookupError`.
"""

from __future__ import annotations

import ast
from dataclasses import dataclass

import numpy as np

SEGMENTED_MONOTONIC = "segmented_monotonically_increasing"
LOOKUP_NAME_PREFIX = "_lcd_lookup_position_"


class StructuralLookupError(Exception):
    """Concrete inputs violate a structural lookup plan."""


@dataclass(frozen=True)
class StructuralLookup:
    """One position table derived solely from sparse structure arrays."""

    name: str
    pointer_array: str
    index_array: str
    sorted_segments: bool = False

    @property
    def argument_names(self):
        return self.pointer_array, self.index_array


def _segmented_pairs(function_props):
    pairs = []
    for key, properties in (function_props or {}).items():
        if not (isinstance(key, tuple) and len(key) == 2):
            continue
        for prop in properties:
            tag = prop[0] if isinstance(prop, tuple) else prop
            if tag == SEGMENTED_MONOTONIC and tuple(key) not in pairs:
                pairs.append(tuple(key))
    return pairs


def _name(node):
    return node.id if isinstance(node, ast.Name) else None


def _subscript(node, array):
    return (isinstance(node, ast.Subscript) and _name(node.value) == array)


def _is_plus_one(node, base_dump):
    return (isinstance(node, ast.BinOp) and isinstance(node.op, ast.Add)
            and ast.dump(node.left) == base_dump
            and isinstance(node.right, ast.Constant) and node.right.value == 1)


def _self_lookup_pair(loop, pairs):
    """(pointer, index) when ``loop`` searches a segment for its own id."""
    call = loop.iter
    if not (isinstance(call, ast.Call) and _name(call.func) == "range" and len(call.args) == 2
            and isinstance(loop.target, ast.Name)):
        return None
    first, last = call.args
    for pointer, index in pairs:
        if not (_subscript(first, pointer) and _subscript(last, pointer)):
            continue
        segment = ast.dump(first.slice)
        if not _is_plus_one(last.slice, segment):
            continue
        for statement in loop.body:
            if not (isinstance(statement, ast.If) and isinstance(statement.test, ast.Compare)
                    and len(statement.test.ops) == 1 and isinstance(statement.test.ops[0], ast.Eq)):
                continue
            left, right = statement.test.left, statement.test.comparators[0]
            for entry, other in ((left, right), (right, left)):
                if (_subscript(entry, index) and _name(entry.slice) == loop.target.id
                        and ast.dump(other) == segment
                        and any(isinstance(s, ast.Break) for s in statement.body)):
                    return pointer, index
    return None


def create_structural_lookup_plan(function_ast, function_props=None):
    """Find the searches that a position table can replace."""
    pairs = _segmented_pairs(function_props)
    if not pairs:
        return ()
    used = {node.id for node in ast.walk(function_ast) if isinstance(node, ast.Name)}
    found = []
    for node in ast.walk(function_ast):
        if isinstance(node, ast.For):
            pair = _self_lookup_pair(node, pairs)
            if pair is not None and pair not in found:
                found.append(pair)
    plan = []
    for position, (pointer, index) in enumerate(found):
        suffix = position
        while f"{LOOKUP_NAME_PREFIX}{suffix}" in used:
            suffix += 1
        name = f"{LOOKUP_NAME_PREFIX}{suffix}"
        used.add(name)
        plan.append(StructuralLookup(name, pointer, index, sorted_segments=True))
    return tuple(plan)


def structural_argument_names(plan):
    """Structure inputs that must take part in cache fingerprints."""
    names = []
    for lookup in plan or ():
        for name in lookup.argument_names:
            if name not in names:
                names.append(name)
    return names


def structural_lookup_names(plan):
    return [lookup.name for lookup in plan or ()]


def _as_device_int32(value, what):
    import torch
    if isinstance(value, torch.Tensor):
        if value.dim() != 1:
            raise StructuralLookupError(f"{what} must be 1-D.")
        if value.dtype not in (torch.int32, torch.int64, torch.int16, torch.int8, torch.uint8):
            raise StructuralLookupError(f"{what} must contain integers.")
        return value.to(device="cuda", dtype=torch.int32).contiguous()
    array = np.asarray(value)
    if array.ndim != 1:
        raise StructuralLookupError(f"{what} must be 1-D.")
    if not np.issubdtype(array.dtype, np.integer):
        raise StructuralLookupError(f"{what} must contain integers.")
    return torch.from_numpy(np.ascontiguousarray(array, dtype=np.int32)).cuda()


def materialize_structural_lookups(plan, argument_values):
    """Build every planned table for one concrete sparsity structure (on the GPU).

    Returns ``{name: int32 CUDA tensor}``; unsorted segments or inconsistent
    pointers raise :class:`StructuralLookupError` like the reference."""
    from . import ops
    from ._native import ERR_BAD_POINTERS, ERR_UNSORTED, NativeError
    values = {}
    for lookup in plan or ():
        try:
            pointers = argument_values[lookup.pointer_array]
            indices = argument_values[lookup.index_array]
        except KeyError as error:
            raise StructuralLookupError(
                f"Missing structural argument {error.args[0]!r}.") from error
        pointers = _as_device_int32(pointers, lookup.pointer_array)
        indices = _as_device_int32(indices, lookup.index_array)
        if pointers.numel() == 0:
            raise StructuralLookupError(
                f"{lookup.pointer_array} must contain at least one offset.")
        try:
            values[lookup.name] = ops.diag_positions(pointers, indices)
        except NativeError as error:
            if error.code == ERR_UNSORTED:
                raise StructuralLookupError(
                    f"A segment of {lookup.index_array} violates the "
                    "segmented_monotonically_increasing property.") from error
            if error.code == ERR_BAD_POINTERS:
                raise StructuralLookupError(
                    f"Invalid pointer segment in {lookup.pointer_array}.") from error
            raise
    return values


__all__ = ["StructuralLookup", "StructuralLookupError", "create_structural_lookup_plan",
           "materialize_structural_lookups", "structural_argument_names",
           "structural_lookup_names"]
