"""Differentiable sparse contraction; mirrors einjax ``autodiff/custom_vjp.py``
with ``torch.autograd.Function`` in place of ``jax.custom_vjp``.

Coordinates and join indices are static structure; gradients flow through
tile values only (``custom_vjp.py:1-15``). The backward rule is the
reference's (``:254-275``): the per-pair gradient of the LHS tile is
``einsum(g, rhs)`` with the reversed string ``"{out},{rhs}->{lhs}"`` and of
the RHS tile ``einsum(lhs, g)`` with ``"{lhs},{out}->{rhs}"``, scatter-added
by input tile index. Here the scatter-add is fused: pairs are grouped by
input tile (stable, so each group keeps pair order) and each group's
per-pair contractions are summed into that tile in one segmented tile
einsum, without materialising per-pair gradient tiles.
"""

from __future__ import annotations

import torch

from .sparse import SparseTensorRelation, as_relation, empty_relation
from .sparse_dispatch import _resolve_shapes, plan_pairs, tile_einsum


def _reverse_einsum_string(kernel_string: str):
    """``autodiff/custom_vjp.py:31-62``."""
    if "->" not in kernel_string:
        raise ValueError(f"kernel_string must contain '->': {kernel_string}")
    ins, out = kernel_string.split("->")
    lhs_l, rhs_l = ins.split(",")
    return f"{out},{rhs_l}->{lhs_l}", f"{lhs_l},{out}->{rhs_l}"


def _group_by(index: torch.Tensor, n_rows: int):
    """Stable grouping of pair positions by ``index`` (int32 in [0, n_rows)).

    Returns (perm int32 — original positions in grouped order, offsets int64
    (G+1), group values int32 (G,)).
    """
    from . import _lib as L
    from .sparse import read_counts, stream_ptr, workspace
    dev = index.device
    P = int(index.shape[0])
    # the output-grouping entry point keyed by coordinate 0 of an arange
    # "relation": the output coordinate of pair p is index[p] itself
    rows = torch.arange(n_rows, dtype=torch.int32, device=dev).reshape(-1, 1)
    lib = L.lib()
    ws = workspace(lib.es_segments_workspace_size(P), dev)
    cnt = torch.zeros(2, dtype=torch.int64, device=dev)
    zero = torch.zeros(P, dtype=torch.int32, device=dev)
    idx = index.to(torch.int32).contiguous()
    st = stream_ptr(dev)
    ext = L.i64arr([n_rows])
    L.check("es_segments_plan", lib.es_segments_plan(
        rows.data_ptr(), 1, rows.data_ptr(), 1, idx.data_ptr(), zero.data_ptr(), P, L.i32arr([0, 0]),
        1, ext, ws.data_ptr(), ws.numel(), cnt.data_ptr(), cnt[1:].data_ptr(), st))
    G, err = read_counts(cnt)
    L.device_error("es_segments_plan", err, "pair index outside its relation")
    oc = torch.empty((G, 1), dtype=torch.int32, device=dev)
    so = torch.empty(G + 1, dtype=torch.int64, device=dev)
    sp = torch.empty(P, dtype=torch.int32, device=dev)
    L.check("es_segments_fill", lib.es_segments_fill(
        idx.data_ptr(), zero.data_ptr(), P, 1, ext, ws.data_ptr(), ws.numel(), G, oc.data_ptr(), so.data_ptr(),
        None, None, sp.data_ptr(), 0, None, st))
    return sp, so, oc.reshape(-1)


def _vjp_tiles(kernel_string, lhs_values, rhs_values, g_values, g_index, lhs_idx, rhs_idx, need_l, need_r,
               precision):
    """Gradients of the tile values.

    ``g_values`` holds cotangent tiles; pair p's cotangent is
    ``g_values[g_index[p]]`` (per-pair: g_index = arange(P); aggregated: the
    pair's output segment). Returns (grad_lhs, grad_rhs), float32, shaped like
    the value arrays.
    """
    gl_s, gr_s = _reverse_einsum_string(kernel_string)
    gl = gr = None
    if need_l:
        perm, offs, grp = _group_by(lhs_idx, lhs_values.shape[0])
        pl = g_index.index_select(0, perm.long())
        pr = rhs_idx.index_select(0, perm.long())
        gl = torch.zeros(lhs_values.shape, dtype=torch.float32, device=lhs_values.device)
        tile_einsum(gl_s, g_values, rhs_values, pl, pr, offs, seg_out_index=grp, out=gl, precision=precision)
    if need_r:
        perm, offs, grp = _group_by(rhs_idx, rhs_values.shape[0])
        pl = lhs_idx.index_select(0, perm.long())
        pr = g_index.index_select(0, perm.long())
        gr = torch.zeros(rhs_values.shape, dtype=torch.float32, device=rhs_values.device)
        tile_einsum(gr_s, lhs_values, g_values, pl, pr, offs, seg_out_index=grp, out=gr, precision=precision)
    return gl, gr


class _SparseEinsumRaw(torch.autograd.Function):
    @staticmethod
    def forward(ctx, lhs_values, rhs_values, lhs_idx, rhs_idx, kernel_string, precision):
        ctx.save_for_backward(lhs_values, rhs_values, lhs_idx, rhs_idx)
        ctx.kernel_string, ctx.precision = kernel_string, precision
        return tile_einsum(kernel_string, lhs_values, rhs_values, lhs_idx, rhs_idx, precision=precision)

    @staticmethod
    def backward(ctx, g):
        lv, rv, li, ri = ctx.saved_tensors
        P = li.shape[0]
        if P == 0:
            return torch.zeros_like(lv), torch.zeros_like(rv), None, None, None, None
        gidx = torch.arange(P, dtype=torch.int32, device=lv.device)
        gl, gr = _vjp_tiles(ctx.kernel_string, lv, rv, g.contiguous(), gidx, li, ri, ctx.needs_input_grad[0],
                            ctx.needs_input_grad[1], ctx.precision)
        return (gl.to(lv.dtype) if gl is not None else None, gr.to(rv.dtype) if gr is not None else None,
                None, None, None, None)


def sparse_einsum_raw(lhs_values, rhs_values, lhs_coords, rhs_coords, lhs_indices, rhs_indices, kernel_string,
                      precision="auto"):
    """Differentiable per-pair tile contraction (``autodiff/custom_vjp.py:204-278``).

    Returns ``(P, *out_tile)`` per-pair tiles; ``torch.autograd`` gradients
    w.r.t. both value arrays follow the reference's backward rule.
    """
    dev = lhs_values.device
    li = torch.as_tensor(lhs_indices, device=dev).to(torch.int32)
    ri = torch.as_tensor(rhs_indices, device=dev).to(torch.int32)
    return _SparseEinsumRaw.apply(lhs_values, rhs_values, li, ri, kernel_string, precision)


class _SparseEinsumAgg(torch.autograd.Function):
    @staticmethod
    def forward(ctx, lhs_values, rhs_values, plan, kernel_string, precision):
        ctx.plan, ctx.kernel_string, ctx.precision = plan, kernel_string, precision
        ctx.save_for_backward(lhs_values, rhs_values)
        return tile_einsum(kernel_string, lhs_values, rhs_values, plan.seg_lhs, plan.seg_rhs, plan.seg_offsets,
                           precision=precision)

    @staticmethod
    def backward(ctx, g):
        lv, rv = ctx.saved_tensors
        plan = ctx.plan
        dev = lv.device
        counts = plan.seg_offsets[1:] - plan.seg_offsets[:-1]
        seg_of_sorted = torch.repeat_interleave(torch.arange(plan.num_segments, device=dev), counts)
        if plan.seg_pair is None:  # pairs already in grouped order
            gidx = seg_of_sorted.to(torch.int32)
        else:
            gidx = torch.empty(plan.num_pairs, dtype=torch.int32, device=dev)
            gidx[plan.seg_pair.long()] = seg_of_sorted.to(torch.int32)
        gl, gr = _vjp_tiles(ctx.kernel_string, lv, rv, g.contiguous(), gidx, plan.lhs_idx, plan.rhs_idx,
                            ctx.needs_input_grad[0], ctx.needs_input_grad[1], ctx.precision)
        return (gl.to(lv.dtype) if gl is not None else None, gr.to(rv.dtype) if gr is not None else None,
                None, None, None)


def sparse_einsum(lhs, rhs, join_keys, kernel_string, agg_keys, output_shape=None, output_tile_shape=None,
                  precision="auto") -> SparseTensorRelation:
    """Differentiable ``execute_sparse`` (``autodiff/custom_vjp.py:124-201``):
    the output relation's ``values`` carries an autograd graph back to
    ``lhs.values`` and ``rhs.values`` (set ``requires_grad`` on them)."""
    lhs, rhs = as_relation(lhs), as_relation(rhs)
    output_shape, output_tile_shape = _resolve_shapes(lhs, rhs, kernel_string, agg_keys, output_shape,
                                                      output_tile_shape)
    plan = plan_pairs(lhs, rhs, join_keys, agg_keys)
    if plan.num_pairs == 0:
        return empty_relation(output_shape, output_tile_shape, lhs.values.dtype, lhs.device)
    vals = _SparseEinsumAgg.apply(lhs.values, rhs.values, plan, kernel_string, precision)
    return SparseTensorRelation(plan.out_coords, vals, output_shape, output_tile_shape)
