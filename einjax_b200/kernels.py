"""Block-sparse matmul and coordinate-join entry points; mirrors einjax
``kernels/pallas_matmul.py`` and ``kernels/pallas_gather.py`` on the GPU."""

from __future__ import annotations

import numpy as np
import torch

from .sparse import SparseTensorRelation, as_relation, default_device, empty_relation
from .sparse_dispatch import _join_int32, execute_sparse


def block_sparse_matmul_generic(lhs, rhs, block_shape=None, *, precision="auto") -> SparseTensorRelation:
    """Block-sparse ``ij,jk->ik`` (``kernels/pallas_matmul.py:33-113``).

    Raises ValueError for non-2-D operands (``:55-59``) and mismatched inner
    tiles (``:68-73``). ``block_shape`` (M_tile, K_tile, N_tile) only labels
    the output tile shape, as in the reference.
    """
    lhs, rhs = as_relation(lhs), as_relation(rhs)
    if lhs.ndim != 2 or rhs.ndim != 2:
        raise ValueError(f"block_sparse_matmul requires 2D tensors, got {lhs.ndim}D and {rhs.ndim}D")
    if block_shape is not None:
        m, _, n = block_shape
    else:
        m, n = lhs.tile_shape[0], rhs.tile_shape[1]
    if lhs.tile_shape[1] != rhs.tile_shape[0]:
        raise ValueError(f"Inner tile dimensions must match: lhs.tile_shape[1]={lhs.tile_shape[1]} != "
                         f"rhs.tile_shape[0]={rhs.tile_shape[0]}")
    out_shape = (lhs.shape[0], rhs.shape[1])
    res = execute_sparse(lhs, rhs, [(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)], out_shape, (m, n), precision=precision)
    if res.num_tuples == 0:
        return empty_relation(out_shape, (m, n), torch.float32, lhs.device)
    return res


def block_sparse_matmul(lhs_coords, lhs_values, rhs_coords, rhs_values, block_shape, lhs_shape, rhs_shape,
                        *, precision="auto") -> SparseTensorRelation:
    """Raw-array variant (``kernels/pallas_matmul.py:116-158``)."""
    m, k, n = block_shape
    dev = default_device()
    lhs = SparseTensorRelation.from_arrays(lhs_coords, lhs_values, lhs_shape, (m, k), dev)
    rhs = SparseTensorRelation.from_arrays(rhs_coords, rhs_values, rhs_shape, (k, n), dev)
    return block_sparse_matmul_generic(lhs, rhs, block_shape, precision=precision)


def _coords_relation(coords, device):
    c = torch.as_tensor(np.asarray(coords, dtype=np.int32) if not torch.is_tensor(coords) else coords)
    c = c.to(device=device, dtype=torch.int32)
    if c.dim() == 1:
        c = c.reshape(-1, 1)
    nd = c.shape[1]
    ext = (c.amax(dim=0) + 1).tolist() if c.shape[0] else [1] * nd
    shape = tuple(max(1, int(e)) for e in ext)
    values = torch.zeros((c.shape[0],) + (1,) * nd, dtype=torch.float32, device=device)
    return SparseTensorRelation(c.contiguous(), values, shape, (1,) * nd)


def _normalize_dims(join_dims):
    if join_dims and isinstance(join_dims[0], (int, np.integer)):
        return [(int(d), int(d)) for d in join_dims]
    return [tuple(int(x) for x in k) for k in join_dims]


def coordinate_join_hash(lhs_coords, rhs_coords, join_dims):
    """``kernels/pallas_gather.py:19-76``: same pairs and order as
    ``coordinate_join``; ints are same-dimension shorthand; an empty side gives
    empty int64 results."""
    dev = default_device()
    keys = _normalize_dims(join_dims)
    L = _coords_relation(lhs_coords, dev)
    R = _coords_relation(rhs_coords, dev)
    if L.num_tuples == 0 or R.num_tuples == 0:
        e = torch.zeros(0, dtype=torch.int64, device=dev)
        return e, e.clone()
    _equalize_grids(L, R, keys)
    li, ri = _join_int32(L, R, keys)
    return li.long(), ri.long()


def _equalize_grids(L, R, keys):
    # key extents come from the relations' grids; coordinate-only relations
    # take their shape from the largest coordinate seen on either side
    ls, rs = list(L.shape), list(R.shape)
    for a, b in keys:
        m = max(ls[a], rs[b])
        ls[a], rs[b] = m, m
    L.shape, R.shape = tuple(ls), tuple(rs)


def coordinate_join_sorted(lhs_coords, rhs_coords, join_dims):
    """Sort-merge join order (``kernels/pallas_gather.py:79-174``): pairs by key
    ascending, then LHS index, then RHS index — the hash-join pairs regrouped
    by (key, lhs) with a stable device sort (inside one (key, lhs) group the
    hash order already has RHS ascending)."""
    dev = default_device()
    keys = _normalize_dims(join_dims)
    L = _coords_relation(lhs_coords, dev)
    R = _coords_relation(rhs_coords, dev)
    if L.num_tuples == 0 or R.num_tuples == 0:
        e = torch.zeros(0, dtype=torch.int64, device=dev)
        return e, e.clone()
    if not keys:
        li, ri = _join_int32(L, R, keys)
        return li.long(), ri.long()
    _equalize_grids(L, R, keys)
    # augmented lhs coords: join columns then the row index, grouped through
    # the output-grouping machinery (stable radix sort on the packed key)
    from .sparse_dispatch import plan_pairs
    n = L.num_tuples
    cols = [L.coords[:, a] for a, _ in keys] + [torch.arange(n, dtype=torch.int32, device=dev)]
    aug = SparseTensorRelation(torch.stack(cols, 1).contiguous(), L.values,
                               tuple(L.shape[a] for a, _ in keys) + (n,), (1,) * (len(keys) + 1))
    Rk = SparseTensorRelation(R.coords, R.values, R.shape, R.tile_shape)
    plan = plan_pairs(aug, Rk, [(q, b) for q, (_, b) in enumerate(keys)],
                      [(0, q) for q in range(len(keys) + 1)])
    return plan.seg_lhs.long(), plan.seg_rhs.long()
