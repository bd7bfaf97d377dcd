"""Multi-GPU execution of the sparse path: one process per GPU, torch.distributed.

Two ways to split one binary contraction over N ranks
(``execute_sharded_sparse``, ``execution/sparse_dispatch.py:330-478``):

* ``shard="output"`` — output tiles are independent. The lhs tiles are split
  into N contiguous ranges of output strips (the lhs-derived output
  coordinates) holding ~P/N join pairs each (``output_strip_ranges``); every
  rank joins, groups and contracts only its own lhs tiles against the full
  rhs, so tiling, join, grouping and the tile GEMM are all sharded. No
  collective touches the data path; the optional ``gather`` all-gathers the
  shards in rank order, which keeps the coordinates globally sorted. Element
  COO input can be split before tiling with ``balanced_row_ranges`` (each
  rank then tiles only its rows and passes ``lhs_sharded=True``).
* ``shard="contracted"`` — the contracted (join-key) tile range is split into
  N contiguous key ranges holding ~equal numbers of lhs tiles
  (``balanced_key_ranges``); each rank contracts its slice into partial output
  tiles, written by the tile GEMM straight into the order of the union of all
  ranks' output coordinates (``coordinate_union``: an all-gather of the
  coordinates, then the library's own sort-and-group), and the partials are
  summed by one NCCL reduce-scatter over that buffer.

The reference instead slices the pair list contiguously (``:300-327``) and
sums on the host; results agree after the canonical (lexicographic) order.
The host-side pieces here (ranges, all-gather, reduce-scatter) also run on
CPU tensors with the gloo backend, which is how they are tested without GPUs;
the coordinate union itself runs in the CUDA library (a caller may pass its
own ``union`` function, as the CPU tests do).
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


def balanced_row_ranges(indices, shape, tile_shape, n_ranks: int, dim: int = 0):
    """Split an element COO along ``dim`` into n contiguous, tile-aligned index
    ranges ``[(lo, hi), ...]`` holding ~equal numbers of non-empty tiles.

    A rank that takes the entries with ``lo <= indices[:, dim] < hi`` owns
    whole tile strips (tile rows along ``dim``), so with ``dim`` the leading
    output dimension its output tiles are disjoint from every other rank's.
    When every lhs tile meets the same number of rhs tiles (a dense rhs, as in
    an SpMM) the tile count is the pair count, so the ranges balance the
    contraction too. Host-side planning over the COO (numpy)."""
    idx = np.asarray(indices)
    shape = tuple(int(s) for s in shape)
    tile_shape = tuple(int(t) for t in tile_shape)
    grid = [s // t for s, t in zip(shape, tile_shape)]
    t = idx.astype(np.int64) // np.asarray(tile_shape, dtype=np.int64)
    key = np.zeros(idx.shape[0], dtype=np.int64)
    for d in range(len(shape)):
        key = key * grid[d] + t[:, d]
    # strip of each distinct tile: `dim` first in the packing keeps it exact
    strip = np.unique(key)
    if dim != 0:
        tiles = np.stack(np.unravel_index(strip, grid), axis=1)
        strip_of = tiles[:, dim]
    else:
        strip_of = strip // int(np.prod(grid[1:], dtype=np.int64))
    counts = np.bincount(strip_of, minlength=grid[dim])
    ranges = balanced_key_ranges(counts, n_ranks)
    return [(a * tile_shape[dim], b * tile_shape[dim]) for a, b in ranges]


def _packed(coords: torch.Tensor, dims, ext) -> torch.Tensor:
    k = torch.zeros(coords.shape[0], dtype=torch.int64, device=coords.device)
    for d, e in zip(dims, ext):
        k = k * int(e) + coords[:, d].to(torch.int64)
    return k


def output_strip_ranges(lhs, rhs, join_keys, agg_keys, n_ranks: int):
    """Contiguous lhs tile ranges ``[(t0, t1), ...]``, one per rank, cut at
    output-strip boundaries and balanced by join pairs, or None when the
    output has no strip layout this split covers.

    A strip is a run of lhs tiles sharing the lhs-derived output coordinates
    (the leading ``agg_keys`` with source 0). The split needs them to be the
    leading lhs dimensions in order, so that a strip is a contiguous run of
    the lexicographically sorted lhs and the concatenated rank outputs stay
    sorted. The pairs of lhs tile t are the rhs tiles whose join key equals
    t's, counted from a histogram of rhs keys (no join needed)."""
    nlead = 0
    while nlead < len(agg_keys) and int(agg_keys[nlead][0]) == 0:
        nlead += 1
    if nlead == 0 or [int(d) for _, d in agg_keys[:nlead]] != list(range(nlead)):
        return None
    if any(int(s) != 1 for s, _ in agg_keys[nlead:]):
        return None
    T = lhs.num_tuples
    if T == 0:
        return [(0, 0)] * n_ranks
    lc, rc = lhs.coords, rhs.coords
    if join_keys:
        lg, rg = lhs.grid(), rhs.grid()
        ext = [max(lg[int(a)], rg[int(b)]) for a, b in join_keys]
        rk = _packed(rc, [int(b) for _, b in join_keys], ext)
        lk = _packed(lc, [int(a) for a, _ in join_keys], ext)
        uk, cnt = torch.unique(rk, return_counts=True)
        pos = torch.searchsorted(uk, lk).clamp_(max=max(int(uk.shape[0]) - 1, 0))
        w = torch.where(uk[pos] == lk, cnt[pos], torch.zeros_like(cnt[pos])) if uk.numel() else \
            torch.zeros(T, dtype=torch.int64, device=lc.device)
    else:
        w = torch.full((T,), rhs.num_tuples, dtype=torch.int64, device=lc.device)
    head = torch.ones(T, dtype=torch.bool, device=lc.device)
    if T > 1:
        head[1:] = (lc[1:, :nlead] != lc[:-1, :nlead]).any(dim=1)
    starts = torch.nonzero(head).squeeze(1)  # first tile of every strip
    before = torch.cumsum(w, 0) - w          # pairs before each tile
    sb = before[starts]                      # pairs before each strip
    P = int(w.sum().item())
    targets = torch.tensor([(P * r) // n_ranks for r in range(1, n_ranks)], dtype=torch.int64,
                           device=lc.device)
    j = torch.searchsorted(sb, targets, side="left")
    cut = torch.where(j < starts.shape[0], starts[j.clamp(max=starts.shape[0] - 1)],
                      torch.full_like(j, T)).cpu().tolist()
    bounds = [0] + [int(x) for x in cut] + [T]
    for r in range(1, len(bounds)):
        bounds[r] = max(bounds[r], bounds[r - 1])
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


def coordinate_union(coords: torch.Tensor, extents, group=None):
    """Union of every rank's output coordinates and this rank's place in it.

    ``coords`` (O_r, nd) int32 on this rank's GPU, coordinates in
    ``[0, extents)``. All ranks' coordinates are all-gathered, then grouped by
    the library (``es_segsum_plan`` + ``es_segsum_groups``: radix sort of the
    packed coordinates, group heads, scan). Returns ``(union (U, nd) int32
    sorted lexicographically, pos (O_r,) int32 = row of each local coordinate
    in the union)``."""
    from . import _lib as L
    from .sparse import read_counts, stream_ptr, workspace
    rank, n = world(group)
    parts = all_gather_rows(coords.contiguous(), group)
    off = sum(int(p.shape[0]) for p in parts[:rank])
    allc = torch.cat(parts).contiguous()
    nrows, nd = int(allc.shape[0]), int(coords.shape[1])
    dev = allc.device
    if nrows == 0:
        return torch.zeros((0, nd), dtype=torch.int32, device=dev), torch.zeros(0, dtype=torch.int32, device=dev)
    lib = L.lib()
    e = L.i64arr([int(x) for x in extents])
    ws = workspace(lib.es_segsum_workspace_size(nrows), dev)
    cnt = torch.zeros(2, dtype=torch.int64, device=dev)
    st = stream_ptr(dev)
    L.check("es_segsum_plan", lib.es_segsum_plan(allc.data_ptr(), nrows, nd, e, ws.data_ptr(), ws.numel(),
                                                 cnt.data_ptr(), cnt[1:].data_ptr(), st))
    U, err = read_counts(cnt)
    L.device_error("es_segsum_plan", err, "output coordinate outside the output grid")
    uc = torch.empty((U, nd), dtype=torch.int32, device=dev)
    grp = torch.empty(nrows, dtype=torch.int32, device=dev)
    L.check("es_segsum_groups", lib.es_segsum_groups(nrows, nd, e, ws.data_ptr(), ws.numel(), U, uc.data_ptr(),
                                                     grp.data_ptr(), st))
    return uc, grp[off:off + int(coords.shape[0])]


def _union_chunk(U: int, n: int):
    per = (U + n - 1) // n
    return max(per, 1)


def sparse_reduce_scatter(coords: torch.Tensor, values: torch.Tensor, group=None, gather=True, extents=None,
                          union=None):
    """Sum partial output tiles across ranks.

    Each rank holds (coords (O_r, nd), values (O_r, *tile)). The union of
    coordinates is formed on every rank (``union(coords, extents, group)``,
    default ``coordinate_union``), each rank places its partials in a zero
    (U, *tile) buffer in union order, the buffer is reduce-scattered in N
    contiguous row chunks, and (with ``gather``) the summed chunks are
    all-gathered back. Returns (coords, values) — the full union with
    ``gather``, else this rank's chunk.
    """
    rank, n = world(group)
    if n == 1:
        return coords, values
    if extents is None:
        mx = coords.amax(dim=0).to(torch.int64) if coords.shape[0] else torch.zeros(coords.shape[1],
                                                                                     dtype=torch.int64,
                                                                                     device=coords.device)
        dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
        extents = (mx + 1).tolist()
    ucoords, pos = (union or coordinate_union)(coords, extents, group)
    U = int(ucoords.shape[0])
    per = _union_chunk(U, n)
    buf = torch.zeros((per * n, *values.shape[1:]), dtype=values.dtype, device=values.device)
    if coords.shape[0]:
        buf.index_copy_(0, pos.to(torch.int64), values)
    return _scatter_partials(buf, ucoords, per, group, gather)


def _scatter_partials(buf, ucoords, per, group, gather):
    rank, n = world(group)
    U = int(ucoords.shape[0])
    mine = _reduce_scatter_sum(list(buf.split(per)), group)
    if not gather:
        lo, hi = min(rank * per, U), min((rank + 1) * per, U)
        return ucoords[lo:hi], mine[: hi - lo]
    full = torch.cat(all_gather_rows(mine.contiguous(), group))[:U]
    return ucoords, full


def _slice(rel, t0: int, t1: int):
    from .sparse import SparseTensorRelation
    return SparseTensorRelation(rel.coords[t0:t1], rel.values[t0:t1], rel.shape, rel.tile_shape)


def contracted_key_range(lhs, join_keys, n_ranks: int, rank: int):
    """This rank's contiguous range of the (single) join key's tile
    coordinate, balanced by lhs tile count."""
    if len(join_keys) != 1:
        raise ValueError("contracted sharding needs exactly one join key")
    ld = int(join_keys[0][0])
    kext = lhs.grid()[ld]
    counts = torch.bincount(lhs.coords[:, ld].long(), minlength=kext).cpu().numpy()
    return balanced_key_ranges(counts, n_ranks)[rank]


def execute_sharded_sparse(lhs, rhs, join_keys, kernel_string, agg_keys, output_shape=None, output_tile_shape=None,
                           *, num_devices=None, group=None, gather=True, precision="auto", shard="output",
                           lhs_sharded=False, timings=None):
    """See ``einjax_b200.sparse_dispatch.execute_sharded_sparse``.

    ``lhs_sharded``: ``lhs`` already holds only this rank's share (its output
    strips for ``shard="output"``, e.g. the tiles of its ``balanced_row_ranges``
    rows; its contracted key range for ``"contracted"``). ``timings``: a list
    that receives ``(label, CUDA event)`` marks around the collective."""
    from .sparse import SparseTensorRelation, as_relation, empty_relation, latest_ready, mark
    from .sparse_dispatch import _out_extents, _resolve_shapes, execute_sparse, plan_pairs, tile_einsum

    rank, n = world(group)
    if num_devices is not None and num_devices <= 1 or n == 1:
        return execute_sparse(lhs, rhs, join_keys, kernel_string, agg_keys, output_shape, output_tile_shape,
                              precision=precision)
    if shard not in ("output", "contracted"):
        raise ValueError(f"shard must be 'output' or 'contracted', got {shard!r}")
    lhs, rhs = as_relation(lhs), as_relation(rhs)
    output_shape, output_tile_shape = _resolve_shapes(lhs, rhs, kernel_string, agg_keys, output_shape,
                                                      output_tile_shape)
    if shard == "contracted":
        if lhs_sharded:
            local = lhs
        else:
            k0, k1 = contracted_key_range(lhs, join_keys, n, rank)
            ld = int(join_keys[0][0])
            keep = (lhs.coords[:, ld] >= k0) & (lhs.coords[:, ld] < k1)
            idx = torch.nonzero(keep).squeeze(1)
            local = SparseTensorRelation(lhs.coords.index_select(0, idx), lhs.values.index_select(0, idx),
                                         lhs.shape, lhs.tile_shape)
        odt = torch.bfloat16 if lhs.values.dtype == rhs.values.dtype == torch.bfloat16 else torch.float32
        if local.num_tuples and rhs.num_tuples:
            plan = plan_pairs(local, rhs, join_keys, agg_keys)
            oc = plan.out_coords
        else:
            plan = None
            oc = torch.zeros((0, len(agg_keys)), dtype=torch.int32, device=lhs.device)
        ext = _out_extents(lhs, rhs, agg_keys)
        ucoords, pos = coordinate_union(oc, ext, group)
        U = int(ucoords.shape[0])
        per = _union_chunk(U, n)
        buf = torch.zeros((per * n, *output_tile_shape), dtype=odt, device=lhs.device)
        if plan is not None and plan.num_pairs:
            # the fused GEMM writes each partial output tile at its union row
            lv, lr = local.values_and_ready()
            rv, rr = rhs.values_and_ready()
            tile_einsum(kernel_string, lv, rv, plan.seg_lhs, plan.seg_rhs, plan.seg_offsets,
                        seg_out_index=pos, out=buf, precision=precision, seg_strip=plan.seg_strip,
                        pair_key=plan.seg_key, key_extent=plan.key_extent, ready=latest_ready(lr, rr))
        mark(timings, "collective0")
        c, v = _scatter_partials(buf, ucoords, per, group, gather)
        mark(timings, "collective1")
        return SparseTensorRelation(c, v, output_shape, output_tile_shape)
    # output-tile sharding
    if lhs_sharded:
        local = lhs
    else:
        ranges = output_strip_ranges(lhs, rhs, join_keys, agg_keys, n)
        if ranges is None:
            return _replicated_plan_shard(lhs, rhs, join_keys, kernel_string, agg_keys, output_shape,
                                          output_tile_shape, group, gather, precision)
        local = _slice(lhs, *ranges[rank])
    if local.num_tuples and rhs.num_tuples:
        part = execute_sparse(local, rhs, join_keys, kernel_string, agg_keys, output_shape, output_tile_shape,
                              precision=precision)
    else:
        part = empty_relation(output_shape, output_tile_shape, lhs.values.dtype, lhs.device)
    if not gather:
        return part
    mark(timings, "collective0")
    coords = torch.cat(all_gather_rows(part.coords.contiguous(), group))
    vals = torch.cat(all_gather_rows(part.values.contiguous(), group))
    mark(timings, "collective1")
    return SparseTensorRelation(coords, vals, output_shape, output_tile_shape)


def _replicated_plan_shard(lhs, rhs, join_keys, kernel_string, agg_keys, output_shape, output_tile_shape, group,
                           gather, precision):
    """Output sharding for outputs without a strip layout: every rank plans
    the whole join and grouping, then contracts a contiguous range of output
    tiles balanced by pair count."""
    from .sparse import SparseTensorRelation, empty_relation, latest_ready
    from .sparse_dispatch import plan_pairs, tile_einsum
    rank, n = world(group)
    plan = plan_pairs(lhs, rhs, join_keys, agg_keys)
    if plan.num_pairs == 0:
        return empty_relation(output_shape, output_tile_shape, lhs.values.dtype, lhs.device)
    s0, s1 = balanced_segment_ranges(plan.seg_offsets.cpu().numpy(), n)[rank]
    if s1 > s0:
        lv, lr = lhs.values_and_ready()
        rv, rr = rhs.values_and_ready()
        vals = tile_einsum(kernel_string, lv, rv, plan.seg_lhs, plan.seg_rhs,
                           plan.seg_offsets[s0:s1 + 1], precision=precision,
                           seg_strip=plan.seg_strip[s0:s1] if plan.seg_strip is not None else None,
                           pair_key=plan.seg_key, key_extent=plan.key_extent, ready=latest_ready(lr, rr))
    else:
        vals = tile_einsum(kernel_string, lhs.values, rhs.values, plan.seg_lhs[:0], plan.seg_rhs[:0],
                           None, num_out_rows=0, precision=precision)
    coords = plan.out_coords[s0:s1]
    if not gather:
        return SparseTensorRelation(coords, vals, output_shape, output_tile_shape)
    coords = torch.cat(all_gather_rows(coords.contiguous(), group))
    vals = torch.cat(all_gather_rows(vals.contiguous(), group))
    return SparseTensorRelation(coords, vals, output_shape, output_tile_shape)
