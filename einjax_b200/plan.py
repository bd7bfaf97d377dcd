"""Sparse plan executor: a contraction plan's binary steps run on tile-COO
relations with every intermediate kept on the GPU.

The reference's ``ExecutionEngine.execute_plan`` (``execution/engine.py:264-324``)
walks a ``ContractionPlan``'s steps over dense arrays: each step contracts the
two operands named by ``input_indices`` with its ``formula``, removes them from
the working list and appends the result. ``execute_sparse_plan`` is the same
walk over ``SparseTensorRelation`` operands, each step an ``execute_sparse``
(or, differentiable, a ``sparse_einsum``) whose join and aggregation keys come
from the formula as ``infer_reduction_info`` derives them
(``optimizer/dp.py:50-95``): a label seen on both sides is a join key (first
occurrence, second occurrence); each output label aggregates from its first
occurrence. Intermediates never leave the device (no host round trip between
steps).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

from .sparse import SparseTensorRelation, as_relation


@dataclass
class PlanStep:
    """One binary contraction of a plan (the ``formula`` / ``input_indices`` of
    the reference's ``ContractionStep``)."""

    formula: str
    input_indices: tuple


def reduction_keys(formula: str):
    """(join_keys, kernel_string, agg_keys) of a binary formula ``"ab,bc->ac"``
    (``optimizer/dp.py:50-95``). Labels repeated inside one operand are not
    supported (the sparse path has no diagonal)."""
    f = formula.replace(" ", "")
    if "->" not in f or f.count(",") != 1:
        raise ValueError(f"binary formula with '->' expected, got {formula!r}")
    ins, out = f.split("->")
    lhs, rhs = ins.split(",")
    for t in (lhs, rhs, out):
        if len(set(t)) != len(t):
            raise ValueError(f"repeated label inside one term of {formula!r}")
    first = {}
    join_keys = []
    for side, labels in ((0, lhs), (1, rhs)):
        for i, c in enumerate(labels):
            if c in first:
                join_keys.append((first[c][1], i))
            else:
                first[c] = (side, i)
    missing = [c for c in out if c not in first]
    if missing:
        raise ValueError(f"output labels {missing} of {formula!r} are in neither operand")
    agg_keys = [first[c] for c in out]
    return join_keys, f, agg_keys


def plan_from_path(einsum_string: str, path: Sequence[Sequence[int]]) -> list:
    """Binary steps of an opt_einsum-style contraction path (pairs of positions
    in the current operand list; the first position is the step's lhs, as in
    ``optimizer/contraction_path.py:153-190``; the result is appended at the
    end), each keeping the labels that later operands or the output still
    need, in order of first appearance."""
    f = einsum_string.replace(" ", "")
    ins, out = f.split("->")
    terms = ins.split(",")
    steps = []
    for pair in path:
        i, j = (int(v) for v in pair)
        if i == j or not (0 <= i < len(terms) and 0 <= j < len(terms)):
            raise ValueError(f"bad path step {tuple(pair)} over {len(terms)} operands")
        a, b = terms[i], terms[j]
        rest = [t for k, t in enumerate(terms) if k not in (i, j)]
        keep = set(out).union(*[set(t) for t in rest]) if rest else set(out)
        res = "".join(c for c in dict.fromkeys(a + b) if c in keep)
        steps.append(PlanStep(f"{a},{b}->{res}", (i, j)))
        for k in sorted((i, j), reverse=True):
            del terms[k]
        terms.append(res)
    if len(terms) != 1:
        raise ValueError("the path does not reduce the operands to one")
    if sorted(terms[0]) != sorted(out):
        raise ValueError(f"the path yields {terms[0]!r}, not the output {out!r}")
    if terms[0] != out:
        steps[-1] = PlanStep(steps[-1].formula.split("->")[0] + "->" + out, steps[-1].input_indices)
    return steps


def _operand_order(formula, lhs, rhs, precision):
    """The step with its operands swapped (``"b,a->o"`` over (rhs, lhs)) when
    only that order maps the tile product onto the tensor-core kernel, e.g.
    ``"kl,ik->il"`` -> ``"ik,kl->il"``. The result relation is the same (a
    dense einsum's value does not depend on the operand order; coordinates come
    out sorted either way); the plan's choice of lhs is arbitrary."""
    from .sparse_dispatch import tile_einsum_path
    ins, out = formula.split("->")
    a, b = ins.split(",")
    swapped = f"{b},{a}->{out}"

    def path(ks, l, r):
        try:
            return tile_einsum_path(ks, l.tile_shape, r.tile_shape, l.values.dtype, r.values.dtype, precision)
        except ValueError:
            return "none"
    if path(formula, lhs, rhs) != "tc" and path(swapped, rhs, lhs) == "tc":
        return swapped, rhs, lhs
    return formula, lhs, rhs


def execute_sparse_plan(steps, operands: Sequence, *, differentiable: bool = False,
                        precision: str = "auto") -> SparseTensorRelation:
    """Runs ``steps`` (``PlanStep``s, objects with ``formula`` and
    ``input_indices`` such as the reference's ``ContractionStep``, or
    ``(formula, (i, j))`` pairs; a ``ContractionPlan`` is read through its
    ``steps``) over tile-COO operands
    (``execution/engine.py:264-324``): each step contracts operands i and j,
    removes them and appends the result; returns the last intermediate. A
    step whose tile product only the swapped operand order puts on the
    tensor cores runs swapped (same result relation). With
    ``differentiable`` the steps run through ``sparse_einsum`` so gradients
    flow to every operand's values."""
    from .autodiff import sparse_einsum
    from .sparse_dispatch import execute_sparse
    steps = getattr(steps, "steps", steps)  # a reference ContractionPlan
    work = [as_relation(o) for o in operands]
    for step in steps:
        formula, idx = (step.formula, step.input_indices) if hasattr(step, "formula") else step
        i, j = (int(v) for v in idx)
        lhs, rhs = work[i], work[j]
        formula, lhs, rhs = _operand_order(formula.replace(" ", ""), lhs, rhs, precision)
        jk, ks, ak = reduction_keys(formula)
        if differentiable:
            res = sparse_einsum(lhs, rhs, jk, ks, ak, precision=precision)
        else:
            res = execute_sparse(lhs, rhs, jk, ks, ak, precision=precision)
        for k in sorted((i, j), reverse=True):
            del work[k]
        work.append(res)
    if not work:
        raise ValueError("no operands")
    return work[-1]
