"""Numpy restatement of einjax's sparse-einsum hot path (CPU checker only).

TEST INFRASTRUCTURE: imported by ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU legs only. Parity is pinned: ``tests/test_oracle_golden.py``
checks every function here against golden vectors that
``tests/golden/make_golden.py`` produced by running the unmodified reference
modules (``tensor/sparse.py``, ``execution/sparse_dispatch.py``,
``kernels/pallas_*.py``, ``autodiff/custom_vjp.py``) under a numpy stand-in for
``jax.numpy``.

Two arithmetic modes, selected by ``compute_dtype``:

* ``"f64"`` — what the reference computes when ``jnp`` is numpy (its tile
  arrays are float64, ``tensor/sparse.py:210``);
* ``"f32"`` — what real JAX computes with x64 off, the library default:
  ``jnp.array(float64)`` becomes float32 at ``execution/sparse_dispatch.py:125``
  and ``segment_sum`` keeps that dtype (``:165``).

Paths in citations are relative to the einjax project root.
"""

from __future__ import annotations

from dataclasses import dataclass
from math import prod

import numpy as np

__all__ = [
    "Relation", "extract_coo", "to_relation", "relation_from_dense",
    "coordinate_join", "coordinate_join_hash", "coordinate_join_sorted",
    "add_batch_dim", "infer_output_tile_shape", "kernel_einsum",
    "compute_output_coords", "segment_sum", "execute_sparse",
    "partition_matched_pairs", "execute_sharded_sparse",
    "block_sparse_matmul_generic", "reverse_einsum_string",
    "sparse_einsum_raw_fwd", "sparse_einsum_raw_bwd", "canonical_pairs",
    "relation_allclose", "find_all_factors", "factor_tile_shapes", "compute_sparsity_stats_coo",
    "infer_reduction_keys", "execute_plan", "coalesce_coo",
]


@dataclass
class Relation:
    """Tile-COO relation; mirrors ``SparseTensorRelation`` (``tensor/sparse.py:27-90``)."""

    coords: np.ndarray
    values: np.ndarray
    shape: tuple
    tile_shape: tuple

    @property
    def num_tuples(self) -> int:
        return int(self.coords.shape[0])

    @property
    def ndim(self) -> int:
        return len(self.shape)

    def to_dense(self) -> np.ndarray:
        """Scatter tiles into a dense array (``tensor/sparse.py:75-90``)."""
        out = np.zeros(self.shape, dtype=self.values.dtype)
        for t in range(self.num_tuples):
            sl = tuple(slice(int(c) * s, (int(c) + 1) * s)
                       for c, s in zip(self.coords[t], self.tile_shape))
            out[sl] = self.values[t]
        return out


def extract_coo(data):
    """Dense or scipy input to (int32 indices, float64 values, shape).

    Follows ``tensor/sparse.py:234-270``: scipy matrices keep their COO
    entries (duplicates included); dense input goes through ``np.nonzero``.
    """
    try:
        import scipy.sparse as sp
        if sp.issparse(data):
            coo = sp.coo_matrix(data) if data.ndim == 2 else data.tocoo()
            idx = np.stack([coo.row, coo.col], axis=1).astype(np.int32)
            return idx, np.asarray(coo.data, dtype=np.float64), tuple(coo.shape)
    except ImportError:  # pragma: no cover
        pass
    arr = np.asarray(data, dtype=np.float64)
    nz = np.nonzero(arr)
    if len(nz[0]) == 0:
        return (np.zeros((0, arr.ndim), dtype=np.int32),
                np.zeros((0,), dtype=np.float64), tuple(arr.shape))
    return np.stack(nz, axis=1).astype(np.int32), arr[nz], tuple(arr.shape)


def to_relation(indices, values, shape, tile_shape) -> Relation:
    """COO to tile-COO, following ``SparseTensor.to_relation`` (``tensor/sparse.py:160-219``).

    Divisibility check (``:174-179``), zero filter (``:185-187``), tile and
    in-tile coordinates (``:200-201``), lexicographically sorted unique tile
    coordinates (``:204-206``), zero-filled float64 tiles with one scatter
    (``:210-212``): when a coordinate repeats, the entry that comes last in
    input order is the one that stays.
    """
    shape = tuple(int(s) for s in shape)
    tile_shape = tuple(int(t) for t in tile_shape)
    ndim = len(shape)
    for d in range(ndim):
        if shape[d] % tile_shape[d] != 0:
            raise ValueError(
                f"tile_shape[{d}]={tile_shape[d]} does not evenly divide shape[{d}]={shape[d]}")
    indices = np.asarray(indices)
    values = np.asarray(values, dtype=np.float64)
    nz = values != 0
    nz_idx = indices[nz]
    nz_val = values[nz]
    if nz_val.size == 0:
        return Relation(np.zeros((0, ndim), dtype=np.int32),
                        np.zeros((0, *tile_shape), dtype=np.float64), shape, tile_shape)
    ts = np.array(tile_shape, dtype=np.int32)
    tile_coords = nz_idx // ts
    within = nz_idx % ts
    uniq, inv = np.unique(tile_coords, axis=0, return_inverse=True)
    inv = inv.reshape(-1)
    vals = np.zeros((uniq.shape[0], *tile_shape), dtype=np.float64)
    vals[(inv,) + tuple(within[:, d] for d in range(ndim))] = nz_val
    return Relation(uniq.astype(np.int32), vals, shape, tile_shape)


def coalesce_coo(indices, values, shape, duplicates="sum"):
    """One entry per distinct coordinate with a non-zero value, row-major
    coordinate order. Zeros are dropped first (``tensor/sparse.py:185-187``);
    ``"last"`` keeps the last value in input order (the reference's NumPy
    assignment, ``tensor/sparse.py:211-212``), ``"sum"`` adds a coordinate's
    values in float64 in input order (``numpy.add.at``; what scipy's
    ``sum_duplicates`` computes). Returns ``(indices int32, values float64,
    number of non-zero inputs)``."""
    idx = np.asarray(indices, dtype=np.int64).reshape(-1, len(shape))
    val = np.asarray(values, dtype=np.float64).reshape(-1)
    nz = val != 0
    idx, val = idx[nz], val[nz]
    if len(val) and ((idx < 0).any() or (idx >= np.asarray(shape)).any()):
        raise ValueError("COO index outside the tensor shape")
    lin = np.ravel_multi_index(tuple(idx.T), shape) if len(val) else np.zeros(0, np.int64)
    uniq, inv = np.unique(lin, return_inverse=True)
    out = np.zeros(len(uniq))
    if duplicates == "sum":
        np.add.at(out, inv.reshape(-1), val)
    else:
        out[inv.reshape(-1)] = val  # sequential assignment: the last in input order stays
    coords = np.stack(np.unravel_index(uniq, shape), 1).astype(np.int32) if len(uniq) else \
        np.zeros((0, len(shape)), np.int32)
    return coords, out, int(len(val))


def relation_from_dense(dense, tile_shape) -> Relation:
    """The reference tests' helper ``SparseTensor(name, dense).to_relation(tile)``
    (``tests/test_sparse_dispatch.py:32-35``)."""
    idx, val, shape = extract_coo(dense)
    return to_relation(idx, val, shape, tile_shape)


def _key_ids(lhs_keys: np.ndarray, rhs_keys: np.ndarray):
    both = np.concatenate([lhs_keys, rhs_keys], axis=0)
    _, inv = np.unique(both, axis=0, return_inverse=True)
    inv = inv.reshape(-1)
    return inv[: lhs_keys.shape[0]], inv[lhs_keys.shape[0]:]


def coordinate_join(lhs_coords, rhs_coords, join_keys):
    """Hash join of tile coordinates, ``execution/sparse_dispatch.py:29-82``.

    Pair order is the reference's: for each RHS tile j in order, every LHS
    tile i with the same key, i ascending (``:75-80``). No keys gives the
    LHS-major cross product (``:53-59``). Both outputs are int64.
    """
    lhs_coords = np.asarray(lhs_coords)
    rhs_coords = np.asarray(rhs_coords)
    n_l, n_r = lhs_coords.shape[0], rhs_coords.shape[0]
    if not join_keys:
        return (np.repeat(np.arange(n_l), n_r).astype(np.int64),
                np.tile(np.arange(n_r), n_l).astype(np.int64))
    if n_l == 0 or n_r == 0:
        return np.array([], dtype=np.int64), np.array([], dtype=np.int64)
    ld = [k[0] for k in join_keys]
    rd = [k[1] for k in join_keys]
    lid, rid = _key_ids(lhs_coords[:, ld].astype(np.int64), rhs_coords[:, rd].astype(np.int64))
    nkeys = int(max(lid.max(initial=-1), rid.max(initial=-1))) + 1
    order = np.argsort(lid, kind="stable")
    cnt = np.bincount(lid, minlength=nkeys)
    start = np.concatenate([[0], np.cumsum(cnt)[:-1]])
    per_r = cnt[rid]
    total = int(per_r.sum())
    rhs_idx = np.repeat(np.arange(n_r, dtype=np.int64), per_r)
    offs = np.concatenate([[0], np.cumsum(per_r)[:-1]])
    within = np.arange(total, dtype=np.int64) - np.repeat(offs, per_r)
    lhs_idx = order[np.repeat(start[rid], per_r) + within].astype(np.int64)
    return lhs_idx, rhs_idx


def coordinate_join_hash(lhs_coords, rhs_coords, join_dims):
    """``kernels/pallas_gather.py:19-76``: as ``coordinate_join`` but accepts a
    list of ints as same-dimension shorthand and returns empty int64 arrays
    when either side is empty (``:39-48``)."""
    if join_dims and isinstance(join_dims[0], (int, np.integer)):
        keys = [(int(d), int(d)) for d in join_dims]
    else:
        keys = [tuple(k) for k in join_dims]
    lhs_coords = np.asarray(lhs_coords)
    rhs_coords = np.asarray(rhs_coords)
    if lhs_coords.shape[0] == 0 or rhs_coords.shape[0] == 0:
        return np.array([], dtype=np.int64), np.array([], dtype=np.int64)
    return coordinate_join(lhs_coords, rhs_coords, keys)


def coordinate_join_sorted(lhs_coords, rhs_coords, join_dims):
    """Sort-merge join, ``kernels/pallas_gather.py:79-174``.

    Both sides are stably sorted by key (``np.lexsort``, ``:131-132``); pairs
    come out key by key, LHS-major inside each key group (``:169-172``).
    """
    if join_dims and isinstance(join_dims[0], (int, np.integer)):
        keys = [(int(d), int(d)) for d in join_dims]
    else:
        keys = [tuple(k) for k in join_dims]
    lhs_coords = np.asarray(lhs_coords)
    rhs_coords = np.asarray(rhs_coords)
    n_l, n_r = lhs_coords.shape[0], rhs_coords.shape[0]
    if n_l == 0 or n_r == 0:
        return np.array([], dtype=np.int64), np.array([], dtype=np.int64)
    if not keys:
        return (np.repeat(np.arange(n_l), n_r).astype(np.int64),
                np.tile(np.arange(n_r), n_l).astype(np.int64))
    lk = lhs_coords[:, [k[0] for k in keys]].astype(np.int64)
    rk = rhs_coords[:, [k[1] for k in keys]].astype(np.int64)
    lid, rid = _key_ids(lk, rk)
    lo = np.lexsort(lk.T[::-1])
    ro = np.lexsort(rk.T[::-1])
    out_l, out_r = [], []
    # group boundaries in sorted order
    sl, sr = lid[lo], rid[ro]
    common = np.intersect1d(sl, sr)
    for key in common:  # ascending key order == lexicographic tuple order
        li = lo[np.searchsorted(sl, key, "left"):np.searchsorted(sl, key, "right")]
        ri = ro[np.searchsorted(sr, key, "left"):np.searchsorted(sr, key, "right")]
        out_l.append(np.repeat(li, ri.size))
        out_r.append(np.tile(ri, li.size))
    if not out_l:
        return np.array([], dtype=np.int64), np.array([], dtype=np.int64)
    return np.concatenate(out_l).astype(np.int64), np.concatenate(out_r).astype(np.int64)


def add_batch_dim(kernel_string: str, batch_label: str = "z") -> str:
    """``execution/sparse_dispatch.py:481-503``."""
    if "->" not in kernel_string:
        raise ValueError(f"kernel_string must contain '->': {kernel_string}")
    ins, out = kernel_string.split("->")
    return ",".join(batch_label + t for t in ins.split(",")) + "->" + batch_label + out


def infer_output_tile_shape(kernel_string, lhs_tile_shape, rhs_tile_shape):
    """``execution/sparse_dispatch.py:506-545`` (RHS sizes override LHS ones)."""
    if "->" not in kernel_string:
        raise ValueError(f"kernel_string must contain '->': {kernel_string}")
    ins, out = kernel_string.split("->")
    terms = ins.split(",")
    sizes = {}
    if len(terms) >= 1:
        for d, lab in enumerate(terms[0]):
            if d < len(lhs_tile_shape):
                sizes[lab] = lhs_tile_shape[d]
    if len(terms) >= 2:
        for d, lab in enumerate(terms[1]):
            if d < len(rhs_tile_shape):
                sizes[lab] = rhs_tile_shape[d]
    return tuple(sizes[lab] for lab in out)


def _cast(x, compute_dtype):
    if compute_dtype == "f32" and x.dtype == np.float64:
        return x.astype(np.float32)
    return x


def kernel_einsum(lhs_values, rhs_values, lhs_idx, rhs_idx, kernel_string,
                  compute_dtype="f64"):
    """Per-pair tile einsum, ``execution/sparse_dispatch.py:85-126``.

    Gathers the matched tiles (``:118-119``) and runs the ``z``-batched einsum
    (``:123-125``); no pairs gives zeros ``(0, *out_tile)`` in the input's own
    dtype, since that branch never reaches ``jnp`` (``:108-115``).
    """
    lhs_values = np.asarray(lhs_values)
    rhs_values = np.asarray(rhs_values)
    if len(lhs_idx) == 0:
        ots = infer_output_tile_shape(kernel_string, lhs_values.shape[1:], rhs_values.shape[1:])
        return np.zeros((0, *ots), dtype=lhs_values.dtype)
    a = _cast(lhs_values[np.asarray(lhs_idx)], compute_dtype)
    b = _cast(rhs_values[np.asarray(rhs_idx)], compute_dtype)
    if _is_matmul(kernel_string):
        # same contraction through BLAS (XLA's CPU backend also lowers it to
        # a batched GEMM); only the summation order inside a dot differs
        return np.matmul(a, b)
    return np.einsum(add_batch_dim(kernel_string), a, b)


def _is_matmul(ks: str) -> bool:
    ks = ks.replace(" ", "")
    if "->" not in ks:
        return False
    ins, out = ks.split("->")
    t = ins.split(",")
    if len(t) != 2 or len(t[0]) < 2 or len(t[0]) != len(t[1]) or len(out) != len(t[0]):
        return False
    batch = t[0][:-2]
    i, j = t[0][-2:]
    j2, k = t[1][-2:]
    labels = set(batch) | {i, j, k}
    return (t[1][:-2] == batch and j == j2 and out == batch + i + k
            and len(labels) == len(batch) + 3)


def compute_output_coords(lhs_coords, rhs_coords, lhs_idx, rhs_idx, agg_keys):
    """Output tile coordinate per pair, ``execution/sparse_dispatch.py:174-223``."""
    n = len(lhs_idx)
    out = np.zeros((n, len(agg_keys)), dtype=np.int32)
    if n == 0:
        return out
    for d, (src, dim) in enumerate(agg_keys):
        if src == 0:
            out[:, d] = np.asarray(lhs_coords)[np.asarray(lhs_idx), dim]
        else:
            out[:, d] = np.asarray(rhs_coords)[np.asarray(rhs_idx), dim]
    return out


def segment_sum(values, output_coords):
    """Group-by-sum, ``execution/sparse_dispatch.py:129-171``.

    Unique output coordinates come out lexicographically sorted (``:161``);
    each group is summed in pair order in the values' dtype (``:165-169``);
    ``np.add.at`` adds sequentially in index order, like the reference loop.
    """
    values = np.asarray(values)
    output_coords = np.asarray(output_coords)
    if len(values) == 0:
        ndim = output_coords.shape[1] if output_coords.ndim > 1 else 0
        tile = values.shape[1:] if values.ndim > 1 else ()
        return np.zeros((0, ndim), dtype=np.int32), np.zeros((0, *tile), dtype=values.dtype)
    uniq, inv = np.unique(output_coords.astype(np.int64), axis=0, return_inverse=True)
    inv = inv.reshape(-1)
    agg = np.zeros((uniq.shape[0], *values.shape[1:]), dtype=values.dtype)
    np.add.at(agg, inv, values)
    return uniq.astype(np.int32), agg


def _resolve_shapes(lhs, rhs, kernel_string, agg_keys, output_shape, output_tile_shape):
    if output_tile_shape is None:
        output_tile_shape = infer_output_tile_shape(kernel_string, lhs.tile_shape, rhs.tile_shape)
    if output_shape is None:
        output_shape = tuple(lhs.shape[d] if s == 0 else rhs.shape[d] for s, d in agg_keys)
    return tuple(output_shape), tuple(output_tile_shape)


def execute_sparse(lhs: Relation, rhs: Relation, join_keys, kernel_string, agg_keys,
                   output_shape=None, output_tile_shape=None, compute_dtype="f64") -> Relation:
    """Join, per-pair einsum, output coords, segment-sum: ``execution/sparse_dispatch.py:226-297``."""
    output_shape, output_tile_shape = _resolve_shapes(
        lhs, rhs, kernel_string, agg_keys, output_shape, output_tile_shape)
    li, ri = coordinate_join(lhs.coords, rhs.coords, join_keys)
    tiles = kernel_einsum(lhs.values, rhs.values, li, ri, kernel_string, compute_dtype)
    oc = compute_output_coords(lhs.coords, rhs.coords, li, ri, agg_keys)
    coords, vals = segment_sum(tiles, oc)
    return Relation(coords, vals, output_shape, output_tile_shape)


def infer_reduction_keys(formula: str):
    """Join keys, aggregation keys (as ``(side, dim)``) and output shape labels of a
    binary formula: ``optimizer/dp.py:50-95``. Scans lhs then rhs labels; a label
    seen before joins (its first position, this position); each output label
    aggregates from its first position."""
    ins, out = formula.replace(" ", "").split("->")
    terms = ins.split(",")
    first, join_keys = {}, []
    for side, labels in enumerate(terms):
        for i, c in enumerate(labels):
            if c in first:
                join_keys.append((first[c][1], i))
            else:
                first[c] = (side, i)
    return join_keys, [first[c] for c in out]


def execute_plan(steps, operands, compute_dtype="f64") -> Relation:
    """``ExecutionEngine.execute_plan`` (``execution/engine.py:264-324``) over
    tile-COO relations: ``steps`` are ``(formula, (i, j))``; each step contracts
    working operands i and j with ``execute_sparse``, deletes them (higher index
    first) and appends the result; the last intermediate is returned."""
    work = list(operands)
    for formula, (i, j) in steps:
        jk, ak = infer_reduction_keys(formula)
        res = execute_sparse(work[i], work[j], jk, formula.replace(" ", ""), ak, compute_dtype=compute_dtype)
        for k in sorted((i, j), reverse=True):
            del work[k]
        work.append(res)
    return work[-1]


def partition_matched_pairs(num_matches: int, num_devices: int):
    """Contiguous pair slices, first ``P % N`` get one more, ``execution/sparse_dispatch.py:300-327``."""
    if num_matches == 0:
        return [(0, 0)] * num_devices
    base, rem = divmod(num_matches, num_devices)
    parts, off = [], 0
    for d in range(num_devices):
        size = base + (1 if d < rem else 0)
        parts.append((off, off + size))
        off += size
    return parts


def execute_sharded_sparse(lhs, rhs, join_keys, kernel_string, agg_keys, output_shape=None,
                           output_tile_shape=None, num_devices=1, compute_dtype="f64"):
    """``execution/sparse_dispatch.py:330-478`` with the devices simulated.

    The pair list is split into contiguous slices (``:426``), each slice's
    per-pair tiles are computed, concatenated in slice order (what
    ``device_get`` returns, ``:466``) and segment-summed on the host (``:471``).
    """
    if num_devices <= 1:
        return execute_sparse(lhs, rhs, join_keys, kernel_string, agg_keys,
                              output_shape, output_tile_shape, compute_dtype)
    output_shape, output_tile_shape = _resolve_shapes(
        lhs, rhs, kernel_string, agg_keys, output_shape, output_tile_shape)
    li, ri = coordinate_join(lhs.coords, rhs.coords, join_keys)
    if len(li) == 0:
        return Relation(np.zeros((0, len(output_tile_shape)), dtype=np.int32),
                        np.zeros((0, *output_tile_shape), dtype=lhs.values.dtype),
                        output_shape, output_tile_shape)
    oc = compute_output_coords(lhs.coords, rhs.coords, li, ri, agg_keys)
    parts = partition_matched_pairs(len(li), num_devices)
    tiles = np.concatenate([kernel_einsum(lhs.values, rhs.values, li[s:e], ri[s:e],
                                          kernel_string, compute_dtype) for s, e in parts])
    coords, vals = segment_sum(tiles, oc)
    return Relation(coords, vals, output_shape, output_tile_shape)


def block_sparse_matmul_generic(lhs: Relation, rhs: Relation, block_shape=None,
                                compute_dtype="f64") -> Relation:
    """``kernels/pallas_matmul.py:33-113``: 2-D check (``:55-59``), inner-tile
    check (``:68-73``), join ``[(1,0)]``, ``ij,jk->ik``, agg ``[(0,0),(1,1)]``."""
    if lhs.ndim != 2 or rhs.ndim != 2:
        raise ValueError(f"block_sparse_matmul requires 2D tensors, got {lhs.ndim}D and {rhs.ndim}D")
    if block_shape is not None:
        m, _, n = block_shape
    else:
        m, n = lhs.tile_shape[0], rhs.tile_shape[1]
    if lhs.tile_shape[1] != rhs.tile_shape[0]:
        raise ValueError("Inner tile dimensions must match")
    li, ri = coordinate_join(lhs.coords, rhs.coords, [(1, 0)])
    oshape = (lhs.shape[0], rhs.shape[1])
    if len(li) == 0:
        return Relation(np.zeros((0, 2), dtype=np.int32), np.zeros((0, m, n), dtype=np.float64),
                        oshape, (m, n))
    tiles = kernel_einsum(lhs.values, rhs.values, li, ri, "ij,jk->ik", compute_dtype)
    oc = compute_output_coords(lhs.coords, rhs.coords, li, ri, [(0, 0), (1, 1)])
    coords, vals = segment_sum(tiles, oc)
    return Relation(coords, vals, oshape, (m, n))


def reverse_einsum_string(kernel_string: str):
    """``autodiff/custom_vjp.py:31-62``."""
    if "->" not in kernel_string:
        raise ValueError(f"kernel_string must contain '->': {kernel_string}")
    ins, out = kernel_string.split("->")
    terms = ins.split(",")
    return f"{out},{terms[1]}->{terms[0]}", f"{terms[0]},{out}->{terms[1]}"


def sparse_einsum_raw_fwd(lhs_values, rhs_values, lhs_idx, rhs_idx, kernel_string):
    """Forward of ``sparse_einsum_raw`` (``autodiff/custom_vjp.py:239-248``): per-pair tiles."""
    if len(lhs_idx) == 0:
        ots = infer_output_tile_shape(kernel_string, lhs_values.shape[1:], rhs_values.shape[1:])
        return np.zeros((0, *ots), dtype=lhs_values.dtype)
    return np.einsum(add_batch_dim(kernel_string), lhs_values[lhs_idx], rhs_values[rhs_idx])


def sparse_einsum_raw_bwd(lhs_values, rhs_values, lhs_idx, rhs_idx, kernel_string, g):
    """Backward of ``sparse_einsum_raw`` (``autodiff/custom_vjp.py:254-275``).

    Per-pair ``einsum(g, rhs)`` and ``einsum(lhs, g)`` with the reversed
    strings, scatter-added into zero arrays by input tile index.
    """
    gl_s, gr_s = reverse_einsum_string(kernel_string)
    gl = np.zeros_like(lhs_values)
    gr = np.zeros_like(rhs_values)
    if len(lhs_idx) > 0:
        pl = np.einsum(add_batch_dim(gl_s), g, rhs_values[rhs_idx])
        pr = np.einsum(add_batch_dim(gr_s), lhs_values[lhs_idx], g)
        np.add.at(gl, np.asarray(lhs_idx), pl)
        np.add.at(gr, np.asarray(rhs_idx), pr)
    return gl, gr


def canonical_pairs(lhs_idx, rhs_idx) -> np.ndarray:
    """Pairs as an (P, 2) int64 array sorted by (lhs, rhs): the canonical sort
    under which join results are compared bit for bit."""
    p = np.stack([np.asarray(lhs_idx, dtype=np.int64), np.asarray(rhs_idx, dtype=np.int64)], 1)
    if p.shape[0] == 0:
        return p.reshape(0, 2)
    return p[np.lexsort((p[:, 1], p[:, 0]))]


def relation_allclose(got_coords, got_values, ref: Relation, rtol, mag=None):
    """Coordinates bit-exact, values within ``rtol`` of ``ref``.

    The per-element bound is ``rtol * (|ref| + mag)`` where ``mag`` (same
    shape as the values) is the sum of |products| feeding each element — the
    standard error bound of a floating-point dot product. Without ``mag`` the
    bound is ``rtol * max(|ref|, max|ref| * 1e-3)``.
    """
    got_coords = np.asarray(got_coords)
    if got_coords.shape != ref.coords.shape or not np.array_equal(got_coords, ref.coords):
        return False, "coords differ"
    g = np.asarray(got_values, dtype=np.float64)
    r = np.asarray(ref.values, dtype=np.float64)
    if g.shape != r.shape:
        return False, f"value shape {g.shape} != {r.shape}"
    if r.size == 0:
        return True, "empty"
    if mag is None:
        scale = np.maximum(np.abs(r), np.abs(r).max() * 1e-3)
    else:
        scale = np.abs(r) + np.asarray(mag, dtype=np.float64)
    err = np.abs(g - r)
    bad = err > rtol * scale + 1e-30
    if bad.any():
        i = int(np.argmax(err / (scale + 1e-300)))
        return False, (f"{int(bad.sum())} elements out of tolerance; worst flat index {i}: "
                       f"got {g.flat[i]!r} ref {r.flat[i]!r}")
    return True, "ok"


# ------------------------------------------------------------ sparsity statistics


def find_all_factors(n: int) -> list:
    """Sorted divisors of n (``core/notation.py:27-43``)."""
    if n <= 0:
        raise ValueError(f"n must be positive, got {n}")
    out = set()
    for i in range(1, int(n ** 0.5) + 1):
        if n % i == 0:
            out.add(i)
            out.add(n // i)
    return sorted(out)


def factor_tile_shapes(shape) -> list:
    """Every tile shape whose sides divide the shape: the tiling schemes a
    tensor enumerates (``tensor/base.py:43-49``), in lexicographic order."""
    import itertools
    return sorted(itertools.product(*[find_all_factors(int(n)) for n in shape]))


def compute_sparsity_stats_coo(indices, values, shape, tile_shapes) -> dict:
    """T(U) (non-empty tiles) and V(l, U) (distinct tile coordinates along
    dimension l) per tiling scheme U, over the non-zero entries
    (``tensor/stats.py:25-80``; ``SparseTensor._compute_sparsity_metrics``,
    ``tensor/sparse.py:122-158``). Repeated coordinates count once."""
    idx = np.asarray(indices).reshape(len(values), -1).astype(np.int64)
    nz = idx[np.asarray(values) != 0]
    nd = len(shape)
    out = {}
    for ts in tile_shapes:
        ts = tuple(int(t) for t in ts)
        if len(nz) == 0:
            out[ts] = (0, tuple(0 for _ in range(nd)))
            continue
        tc = nz // np.array(ts, dtype=np.int64)
        out[ts] = (int(len(np.unique(tc, axis=0))), tuple(int(len(np.unique(tc[:, d]))) for d in range(nd)))
    return out
