"""Multi-GPU execution of the sparse path: one process per GPU, torch.distributed.

Two ways to split one binary contraction over N ranks
(``execute_sharded_sparse``, ``execution/sparse_dispatch.py:330-478``):

* ``shard="output"`` — output tiles are independent. Every rank plans the
  join and output grouping (small, replicated metadata), then computes a
  contiguous range of output tiles chosen so each rank gets ~P/N pairs
  (``balanced_segment_ranges``). No collective touches the data path; the
  optional ``gather`` all-gathers the shards in rank order, which keeps the
  coordinates globally sorted.
* ``shard="contracted"`` — the contracted (join-key) tile range is split into
  N contiguous key ranges holding ~equal numbers of LHS tiles
  (``balanced_key_ranges``); each rank contracts its slice into partial output
  tiles, and the partials are summed across ranks by a reduce-scatter over
  the union of output coordinates (``sparse_reduce_scatter``).

The reference instead slices the pair list contiguously (``:300-327``) and
sums on the host; results agree after the canonical (lexicographic) order.
Host-side pieces here run on CPU tensors with the gloo backend as well, which
is how they are tested without GPUs.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist


def world(group=None):
    if not (dist.is_available() and dist.is_initialized()):
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def balanced_segment_ranges(seg_offsets, n_ranks: int):
    """Split segments [0, O) into n contiguous ranges with ~equal pair counts.

    ``seg_offsets``: (O+1) non-decreasing pair offsets. Rank r gets the
    segments whose first pair index falls in [r*P/n, (r+1)*P/n).
    """
    so = np.asarray(seg_offsets, dtype=np.int64)
    O = so.shape[0] - 1
    P = int(so[-1]) if O >= 0 else 0
    if O <= 0:
        return [(0, 0)] * n_ranks
    starts = so[:-1]
    bounds = [0]
    for r in range(1, n_ranks):
        target = (P * r) // n_ranks
        bounds.append(int(np.searchsorted(starts, target, side="left")))
    bounds.append(O)
    for r in range(1, len(bounds)):
        bounds[r] = max(bounds[r], bounds[r - 1])
    return [(bounds[r], bounds[r + 1]) for r in range(n_ranks)]


def balanced_key_ranges(key_counts, n_ranks: int):
    """Split key values [0, K) into n contiguous ranges with ~equal counts."""
    c = np.asarray(key_counts, dtype=np.int64)
    K = c.shape[0]
    csum = np.concatenate([[0], np.cumsum(c)])
    total = int(csum[-1])
    bounds = [0]
    for r in range(1, n_ranks):
        bounds.append(int(np.searchsorted(csum, (total * r) // n_ranks, side="left")))
    bounds.append(K)
    for r in range(1, len(bounds)):
        bounds[r] = min(max(bounds[r], bounds[r - 1]), K)
    return [(bounds[r], bounds[r + 1]) for r in range(n_ranks)]


def all_gather_rows(t: torch.Tensor, group=None) -> list:
    """All-gather tensors whose first dimension differs per rank."""
    rank, n = world(group)
    if n == 1:
        return [t]
    cnt = torch.tensor([t.shape[0]], dtype=torch.int64, device=t.device)
    cnts = [torch.zeros_like(cnt) for _ in range(n)]
    dist.all_gather(cnts, cnt, group=group)
    sizes = [int(c.item()) for c in cnts]
    mx = max(sizes) if sizes else 0
    pad = torch.zeros((mx, *t.shape[1:]), dtype=t.dtype, device=t.device)
    pad[: t.shape[0]] = t
    outs = [torch.empty_like(pad) for _ in range(n)]
    dist.all_gather(outs, pad, group=group)
    return [o[:s] for o, s in zip(outs, sizes)]


def _reduce_scatter_sum(chunks: list, group=None) -> torch.Tensor:
    """Sum-reduce equal-shape chunks, rank r keeps chunk r (NCCL reduce-scatter;
    all-reduce + slice on backends without reduce_scatter, e.g. gloo)."""
    rank, n = world(group)
    if n == 1:
        return chunks[0]
    if dist.get_backend(group) == "nccl":
        out = torch.empty_like(chunks[rank])
        dist.reduce_scatter(out, chunks, op=dist.ReduceOp.SUM, group=group)
        return out
    full = torch.stack(chunks)
    dist.all_reduce(full, op=dist.ReduceOp.SUM, group=group)
    return full[rank].clone()


def sparse_reduce_scatter(coords: torch.Tensor, values: torch.Tensor, group=None, gather=True):
    """Sum partial output tiles across ranks.

    Each rank holds (coords (O_r, nd) lexicographically sorted, values
    (O_r, *tile)). The union of coordinates is formed on every rank, each rank
    lays its partials into a zero (U, *tile) buffer in union order, the buffer
    is reduce-scattered in N contiguous row chunks, and (with ``gather``) the
    summed chunks are all-gathered back. Returns (coords, values) — the full
    union with ``gather``, else this rank's chunk.
    """
    rank, n = world(group)
    if n == 1:
        return coords, values
    nd = coords.shape[1]
    allc = torch.cat(all_gather_rows(coords.contiguous(), group))
    # lexicographic unique via a packed int64 key (coords are small, non-negative)
    ext = (allc.amax(dim=0).to(torch.int64) + 1) if allc.shape[0] else torch.ones(nd, dtype=torch.int64)
    mult = torch.ones(nd, dtype=torch.int64, device=coords.device)
    for d in range(nd - 2, -1, -1):
        mult[d] = mult[d + 1] * ext[d + 1]
    key_all = (allc.to(torch.int64) * mult).sum(1)
    ukeys = torch.unique(key_all, sorted=True)
    U = int(ukeys.shape[0])
    per = (U + n - 1) // n
    buf = torch.zeros((per * n, *values.shape[1:]), dtype=values.dtype, device=values.device)
    if coords.shape[0]:
        my = (coords.to(torch.int64) * mult).sum(1)
        pos = torch.searchsorted(ukeys, my)
        buf[pos] = values
    chunks = list(buf.split(per))
    mine = _reduce_scatter_sum(chunks, group)
    ucoords = torch.stack([(ukeys // mult[d]) % ext[d] for d in range(nd)], 1).to(torch.int32)
    if not gather:
        lo, hi = min(rank * per, U), min((rank + 1) * per, U)
        return ucoords[lo:hi], mine[: hi - lo]
    full = torch.cat(all_gather_rows(mine.contiguous(), group))[:U]
    return ucoords, full


def execute_sharded_sparse(lhs, rhs, join_keys, kernel_string, agg_keys, output_shape=None, output_tile_shape=None,
                           *, num_devices=None, group=None, gather=True, precision="auto", shard="output"):
    """See ``einjax_b200.sparse_dispatch.execute_sharded_sparse``."""
    from .sparse import SparseTensorRelation, as_relation, empty_relation
    from .sparse_dispatch import _resolve_shapes, execute_sparse, plan_pairs, tile_einsum

    rank, n = world(group)
    if num_devices is not None and num_devices <= 1 or n == 1:
        return execute_sparse(lhs, rhs, join_keys, kernel_string, agg_keys, output_shape, output_tile_shape,
                              precision=precision)
    lhs, rhs = as_relation(lhs), as_relation(rhs)
    output_shape, output_tile_shape = _resolve_shapes(lhs, rhs, kernel_string, agg_keys, output_shape,
                                                      output_tile_shape)
    if shard == "contracted":
        if len(join_keys) != 1:
            raise ValueError("contracted sharding needs exactly one join key")
        ld = join_keys[0][0]
        kext = lhs.grid()[ld]
        counts = torch.bincount(lhs.coords[:, ld].long(), minlength=kext).cpu().numpy()
        k0, k1 = balanced_key_ranges(counts, n)[rank]
        keep = (lhs.coords[:, ld] >= k0) & (lhs.coords[:, ld] < k1)
        idx = torch.nonzero(keep).squeeze(1)
        local = SparseTensorRelation(lhs.coords.index_select(0, idx), lhs.values.index_select(0, idx),
                                     lhs.shape, lhs.tile_shape)
        part = execute_sparse(local, rhs, join_keys, kernel_string, agg_keys, output_shape, output_tile_shape,
                              precision=precision)
        c, v = sparse_reduce_scatter(part.coords, part.values, group, gather=gather)
        return SparseTensorRelation(c, v, output_shape, output_tile_shape)
    plan = plan_pairs(lhs, rhs, join_keys, agg_keys)
    if plan.num_pairs == 0:
        return empty_relation(output_shape, output_tile_shape, lhs.values.dtype, lhs.device)
    s0, s1 = balanced_segment_ranges(plan.seg_offsets.cpu().numpy(), n)[rank]
    if s1 > s0:
        vals = tile_einsum(kernel_string, lhs.values, rhs.values, plan.seg_lhs, plan.seg_rhs,
                           plan.seg_offsets[s0:s1 + 1], precision=precision,
                           seg_strip=plan.seg_strip[s0:s1] if plan.seg_strip is not None else None,
                           pair_key=plan.seg_key, key_extent=plan.key_extent)
    else:
        vals = tile_einsum(kernel_string, lhs.values, rhs.values, plan.seg_lhs[:0], plan.seg_rhs[:0],
                           None, num_out_rows=0, precision=precision)
    coords = plan.out_coords[s0:s1]
    if not gather:
        return SparseTensorRelation(coords, vals, output_shape, output_tile_shape)
    coords = torch.cat(all_gather_rows(coords.contiguous(), group))
    vals = torch.cat(all_gather_rows(vals.contiguous(), group))
    return SparseTensorRelation(coords, vals, output_shape, output_tile_shape)
