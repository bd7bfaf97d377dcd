"""Sparse tensor-relational execution on the GPU; mirrors einjax
``execution/sparse_dispatch.py`` function by function.

``execute_sparse`` runs join -> output grouping -> fused tile einsum with the
segment-sum folded into the contraction, so the ``(P, *tile)`` per-pair
partials of the reference (``kernel_einsum`` at :85-126 then ``segment_sum``
at :129-171) are never materialised. The unfused pieces stay available under
their reference names for callers that want them.

Arguments keep the reference's meaning; relations may be this package's
``SparseTensorRelation`` (device tensors) or the reference's numpy ones
(converted on entry). Results are device relations in float32 (bfloat16 when
both inputs are bfloat16), the dtype JAX computes in with x64 off.
"""

from __future__ import annotations

from dataclasses import dataclass
from math import prod

import torch

from . import _lib as L
from .sparse import (_DEFERRED, SparseTensorRelation, as_relation, empty_relation, es_dtype, latest_ready, mark,
                     read_counts, stream_ptr, workspace)

_PREC = {"auto": L.ES_PREC_AUTO, "exact": L.ES_PREC_EXACT, "tc": L.ES_PREC_TC}


def _add_batch_dim(kernel_string: str, batch_label: str = "z") -> str:
    """``execution/sparse_dispatch.py:481-503``."""
    if "->" not in kernel_string:
        raise ValueError(f"kernel_string must contain '->': {kernel_string}")
    ins, out = kernel_string.split("->")
    return ",".join(batch_label + t for t in ins.split(",")) + "->" + batch_label + out


def _infer_output_tile_shape(kernel_string, lhs_tile_shape, rhs_tile_shape) -> tuple:
    """``execution/sparse_dispatch.py:506-545``: label sizes from the lhs tile,
    then the rhs tile, read off in output order."""
    if "->" not in kernel_string:
        raise ValueError(f"kernel_string must contain '->': {kernel_string}")
    ins, out = kernel_string.split("->")
    terms = ins.split(",")
    sizes = {}
    for d, lab in enumerate(terms[0]):
        if d < len(lhs_tile_shape):
            sizes[lab] = lhs_tile_shape[d]
    if len(terms) >= 2:
        for d, lab in enumerate(terms[1]):
            if d < len(rhs_tile_shape):
                sizes[lab] = rhs_tile_shape[d]
    return tuple(sizes[lab] for lab in out)


def _partition_matched_pairs(num_matches: int, num_devices: int):
    """Contiguous pair slices, the first ``P % N`` one longer
    (``execution/sparse_dispatch.py:300-327``)."""
    if num_matches == 0:
        return [(0, 0)] * num_devices
    base, rem = divmod(num_matches, num_devices)
    parts, off = [], 0
    for d in range(num_devices):
        size = base + (1 if d < rem else 0)
        parts.append((off, off + size))
        off += size
    return parts


def _key_extents(lhs: SparseTensorRelation, rhs: SparseTensorRelation, join_keys):
    lg, rg = lhs.grid(), rhs.grid()
    return [max(lg[a], rg[b]) for a, b in join_keys]


def _join_int32(lhs: SparseTensorRelation, rhs: SparseTensorRelation, join_keys):
    """Join on the GPU; returns (lhs_idx, rhs_idx) int32 device tensors."""
    dev = lhs.device
    lib = L.lib()
    nl, nr = lhs.num_tuples, rhs.num_tuples
    keys = [(int(a), int(b)) for a, b in join_keys]
    for a, b in keys:
        if not (0 <= a < lhs.ndim and 0 <= b < rhs.ndim):
            raise ValueError(f"join key {(a, b)} outside operand ranks {lhs.ndim}, {rhs.ndim}")
    flat = [v for k in keys for v in k]
    ext = _key_extents(lhs, rhs, keys) if keys else []
    ws = workspace(lib.es_join_workspace_size(nl, nr), dev)
    cnt = torch.zeros(2, dtype=torch.int64, device=dev)
    st = stream_ptr(dev)
    lc = lhs.coords.contiguous()
    rc = rhs.coords.contiguous()
    L.check("es_join_plan", lib.es_join_plan(
        lc.data_ptr(), nl, lhs.ndim, rc.data_ptr(), nr, rhs.ndim, L.i32arr(flat), len(keys), L.i64arr(ext),
        ws.data_ptr(), ws.numel(), cnt.data_ptr(), cnt[1:].data_ptr(), st))
    P, err = read_counts(cnt, launch_pending=True)
    L.device_error("es_join_plan", err, "tile coordinate outside the relation's tile grid")
    li = torch.empty(P, dtype=torch.int32, device=dev)
    ri = torch.empty(P, dtype=torch.int32, device=dev)
    L.check("es_join_fill", lib.es_join_fill(nl, nr, len(keys), ws.data_ptr(), ws.numel(), P, li.data_ptr(),
                                             ri.data_ptr(), L.ES_I32, st))
    return li, ri


def coordinate_join(lhs, rhs, join_keys):
    """Match tiles on join-key coordinates (``execution/sparse_dispatch.py:29-82``).

    Returns int64 device tensors ``(lhs_indices, rhs_indices)`` in the
    reference's order: RHS tile ascending, and for each RHS tile the matching
    LHS tiles in ascending index; no keys gives the LHS-major cross product.
    """
    lhs, rhs = as_relation(lhs), as_relation(rhs)
    li, ri = _join_int32(lhs, rhs, join_keys)
    return li.long(), ri.long()


def _out_dtype(*dts):
    return torch.bfloat16 if all(d == torch.bfloat16 for d in dts) else torch.float32


def _es_out(dt):
    return L.ES_BF16 if dt == torch.bfloat16 else L.ES_F32


_OUT_TILES = {}


def _out_tile(kernel_string, lt, rt):
    """(encoded kernel string, output tile shape) of a tile einsum, cached."""
    key = (kernel_string, lt, rt)
    hit = _OUT_TILES.get(key)
    if hit is None:
        ks = kernel_string.replace(" ", "").encode()
        ot = L.i64arr([0] * 8)
        nd = L.lib().es_out_tile_shape(ks, L.i64arr(lt), len(lt), L.i64arr(rt), len(rt), ot)
        if nd < 0:
            raise ValueError(f"invalid kernel string {kernel_string!r} for tiles {lt} and {rt}")
        hit = (ks, tuple(int(ot[i]) for i in range(nd)))
        if len(_OUT_TILES) < 4096:
            _OUT_TILES[key] = hit
    return hit


def tile_einsum(kernel_string, lhs_values, rhs_values, pair_lhs, pair_rhs, seg_offsets=None, seg_out_index=None,
                out=None, num_out_rows=None, out_dtype=None, precision="auto", seg_strip=None, pair_key=None,
                key_extent=0, check=True, ready=None):
    """Segmented tile einsum through ``es_tile_einsum``.

    Without ``seg_offsets`` every pair is its own segment (per-pair output,
    ``kernel_einsum``); with it, each segment's pairs are summed in fp32 into
    one output tile (row ``seg_out_index[s]`` of ``out`` if given, else row s).
    ``seg_strip`` (strip key per segment, from the output grouping) lets the
    tensor-core path batch the segments of one output strip; ``pair_key`` (the
    contracted tile coordinate of each pair, in ``[0, key_extent)``) lets it
    block the contracted range so the re-read operand stays in L2. With
    ``check`` the device error flag is read back (one 4-byte copy and a wait);
    ``check="defer"`` queues it for the next count read or
    ``check_device_errors()`` (no wait here); False skips it. ``ready``: a
    ``(sequence, event)`` from ``SparseTensorRelation.values_and_ready``
    that the call waits for right before its first launch reading the
    values (its pair grouping runs before that, overlapping the fill).
    """
    lib = L.lib()
    dev = lhs_values.device
    lt = tuple(lhs_values.shape[1:])
    rt = tuple(rhs_values.shape[1:])
    ks, out_tile = _out_tile(kernel_string, lt, rt)
    P = int(pair_lhs.shape[0])
    nseg = int(seg_offsets.shape[0]) - 1 if seg_offsets is not None else P
    odt = out_dtype or _out_dtype(lhs_values.dtype, rhs_values.dtype)
    if out is None:
        rows = num_out_rows if num_out_rows is not None else nseg
        out = (torch.zeros if seg_out_index is not None else torch.empty)((rows, *out_tile), dtype=odt, device=dev)
    if P == 0 or nseg == 0:
        return out
    if ready is not None and not (lhs_values.is_contiguous() and rhs_values.is_contiguous()):
        # a copy would read the values now: wait here instead
        torch.cuda.current_stream(dev).wait_event(ready[1])
        ready = None
    lv, rv = lhs_values.contiguous(), rhs_values.contiguous()
    pl = pair_lhs.to(torch.int32).contiguous()
    pr = pair_rhs.to(torch.int32).contiguous()
    so = seg_offsets.contiguous() if seg_offsets is not None else None
    sx = seg_out_index.to(torch.int32).contiguous() if seg_out_index is not None else None
    sg = seg_strip.contiguous() if (seg_strip is not None and so is not None) else None
    pk = pair_key.to(torch.int32).contiguous() if (pair_key is not None and so is not None) else None
    lti, rti = L.i64arr(lt), L.i64arr(rt)
    prec = _PREC[precision]
    kext = int(key_extent) if pk is not None else 0
    wsb = lib.es_tile_einsum_workspace_size(ks, lti, len(lt), rti, len(rt), es_dtype(lv), es_dtype(rv),
                                            int(lv.shape[0]), int(rv.shape[0]), P, nseg, kext, prec)
    ws = workspace(wsb, dev) if wsb else None
    err = torch.empty(1, dtype=torch.int32, device=dev)  # cleared by the call
    # deferred check: the call copies its status into a pinned slot itself
    status_host, commit = _DEFERRED.reserve("es_tile_einsum") if check == "defer" else (None, None)
    L.check("es_tile_einsum", lib.es_tile_einsum_ev(
        ks, lti, len(lt), rti, len(rt), lv.data_ptr(), es_dtype(lv), int(lv.shape[0]), rv.data_ptr(), es_dtype(rv),
        int(rv.shape[0]), pl.data_ptr(), pr.data_ptr(), P, so.data_ptr() if so is not None else None, nseg,
        sx.data_ptr() if sx is not None else None, sg.data_ptr() if sg is not None else None,
        pk.data_ptr() if pk is not None else None, kext, out.data_ptr(),
        _es_out(out.dtype), prec, ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
        err.data_ptr(), stream_ptr(dev), ready[1].cuda_event if ready is not None else None, status_host))
    if check == "defer":
        commit()
    elif check:
        e = int(err.item())
        if e:
            L.check("es_tile_einsum (device)", e)
    return out


def tile_einsum_path(kernel_string, lhs_tile, rhs_tile, lhs_dtype=torch.float32, rhs_dtype=torch.float32,
                     precision="auto") -> str:
    """"tc" or "simt": the path ``tile_einsum`` takes for these tiles."""
    lib = L.lib()
    ks = kernel_string.replace(" ", "").encode()
    r = lib.es_tile_einsum_path(ks, L.i64arr(lhs_tile), len(lhs_tile), L.i64arr(rhs_tile), len(rhs_tile),
                                L._dtype_code(lhs_dtype), L._dtype_code(rhs_dtype), _PREC[precision])
    if r < 0:
        raise ValueError(f"tile_einsum_path: {lib.es_status_string(-r).decode()}")
    return "tc" if r == 1 else "simt"


def kernel_einsum(lhs_values, rhs_values, lhs_indices, rhs_indices, kernel_string, precision="auto"):
    """Per-pair tile einsum, output ``(P, *out_tile)``
    (``execution/sparse_dispatch.py:85-126``)."""
    if "->" not in kernel_string:
        raise ValueError(f"kernel_string must contain '->': {kernel_string}")
    return tile_einsum(kernel_string, lhs_values, rhs_values, torch.as_tensor(lhs_indices, device=lhs_values.device),
                       torch.as_tensor(rhs_indices, device=lhs_values.device), precision=precision)


def _compute_output_coords(lhs, rhs, lhs_indices, rhs_indices, join_keys, agg_keys, output_shape,
                           output_tile_shape):
    """Output tile coordinate per pair, int32 ``(P, out_ndim)``
    (``execution/sparse_dispatch.py:174-223``)."""
    lhs, rhs = as_relation(lhs), as_relation(rhs)
    dev = lhs.device
    li = torch.as_tensor(lhs_indices, device=dev).to(torch.int32).contiguous()
    ri = torch.as_tensor(rhs_indices, device=dev).to(torch.int32).contiguous()
    P = int(li.shape[0])
    out = torch.zeros((P, len(output_tile_shape)), dtype=torch.int32, device=dev)
    if P == 0:
        return out
    flat = [int(v) for k in agg_keys for v in k]
    L.check("es_output_coords", L.lib().es_output_coords(
        lhs.coords.contiguous().data_ptr(), lhs.ndim, rhs.coords.contiguous().data_ptr(), rhs.ndim, li.data_ptr(),
        ri.data_ptr(), P, L.i32arr(flat), len(agg_keys), out.data_ptr(), stream_ptr(dev)))
    return out


def segment_sum(values: torch.Tensor, output_coords: torch.Tensor, marks=None):
    """Group rows by coordinate and sum them (``execution/sparse_dispatch.py:129-171``).

    Returns (unique coords int32 sorted lexicographically, summed values in
    the input's dtype); rows of a group are added in row order, in fp32.
    ``marks``: see ``sparse.mark`` (plan0/1 around the grouping, fill0/1
    around the reduction).
    """
    dev = values.device
    oc = torch.as_tensor(output_coords, device=dev).to(torch.int32)
    if values.shape[0] == 0:
        nd = oc.shape[1] if oc.dim() > 1 else 0
        return (torch.zeros((0, nd), dtype=torch.int32, device=dev),
                torch.zeros((0, *values.shape[1:]), dtype=values.dtype, device=dev))
    oc = oc.reshape(values.shape[0], -1).contiguous()
    nd = oc.shape[1]
    ext = (oc.amax(dim=0).to(torch.int64) + 1).tolist()
    if int(oc.amin().item()) < 0:
        raise ValueError("segment_sum: negative output coordinate")
    lib = L.lib()
    n = int(values.shape[0])
    te = prod(values.shape[1:])
    ws = workspace(lib.es_segsum_workspace_size(n), dev)
    cnt = torch.zeros(2, dtype=torch.int64, device=dev)
    st = stream_ptr(dev)
    e = L.i64arr(ext)
    mark(marks, "plan0")
    L.check("es_segsum_plan", lib.es_segsum_plan(oc.data_ptr(), n, nd, e, ws.data_ptr(), ws.numel(), cnt.data_ptr(),
                                                 cnt[1:].data_ptr(), st))
    mark(marks, "plan1")
    O, err = read_counts(cnt)
    L.device_error("es_segsum_plan", err, "segment_sum: coordinate outside its extent")
    vals = values.contiguous()
    odt = torch.bfloat16 if vals.dtype == torch.bfloat16 else torch.float32
    uc = torch.empty((O, nd), dtype=torch.int32, device=dev)
    uv = torch.empty((O, *values.shape[1:]), dtype=odt, device=dev)
    mark(marks, "fill0")
    L.check("es_segsum_fill", lib.es_segsum_fill(vals.data_ptr(), es_dtype(vals), n, te, nd, e, ws.data_ptr(),
                                                 ws.numel(), O, uc.data_ptr(), uv.data_ptr(), _es_out(odt), st))
    mark(marks, "fill1")
    return uc, uv


@dataclass
class PairPlan:
    """Join + output grouping of one binary contraction, all on the device."""

    lhs_idx: torch.Tensor       # int32 (P,), join order
    rhs_idx: torch.Tensor
    out_coords: torch.Tensor    # int32 (O, out_nd), lexicographic
    seg_offsets: torch.Tensor   # int64 (O+1,)
    seg_lhs: torch.Tensor       # int32 (P,), pairs grouped by output tile
    seg_rhs: torch.Tensor
    seg_pair: torch.Tensor | None  # int32 (P,), original pair index (None: identity)
    seg_strip: torch.Tensor | None = None  # int64 (O,), strip key (lhs-derived output coords)
    seg_key: torch.Tensor | None = None    # int32 (P,), contracted tile coordinate of each grouped pair
    key_extent: int = 0

    @property
    def num_pairs(self) -> int:
        return int(self.lhs_idx.shape[0])

    @property
    def num_segments(self) -> int:
        return int(self.out_coords.shape[0])


def _out_extents(lhs, rhs, agg_keys):
    lg, rg = lhs.grid(), rhs.grid()
    return [lg[d] if s == 0 else rg[d] for s, d in agg_keys]


def _direct_batch_dims(lhs, rhs, join_keys, agg_keys):
    """Number of leading batch dims when the call has the shape
    lhs (batch..., strip..., k) x rhs (batch..., k, col...) ->
    (batch..., strip..., col...): join keys = the batch dims paired (d, d)
    plus (last lhs dim, first rhs dim after the batch ones), output = the
    other lhs then the other rhs coordinates, and a small ((batch, k), col)
    rhs table. None for any other shape."""
    keys = {tuple(int(v) for v in k) for k in join_keys}
    if len(keys) != len(join_keys) or not keys:
        return None
    nb = len(keys) - 1
    if nb >= lhs.ndim or nb >= rhs.ndim or keys != {(d, d) for d in range(nb)} | {(lhs.ndim - 1, nb)}:
        return None
    want = [(0, d) for d in range(lhs.ndim - 1)] + [(1, d) for d in range(nb + 1, rhs.ndim)]
    if [tuple(int(v) for v in k) for k in agg_keys] != want or not want:
        return None
    lg, rg = lhs.grid(), rhs.grid()
    cext = prod(rg[nb + 1:])
    kext = max(lg[-1], rg[nb]) * prod(max(lg[d], rg[d]) for d in range(nb))
    # pairs <= lhs tiles x present columns fit the int32 pair arrays
    if kext * cext <= (1 << 26) and min(cext, max(rhs.num_tuples, 1)) * max(lhs.num_tuples, 1) < (1 << 31) - 1:
        return nb
    return None


def _direct_shape(lhs, rhs, join_keys, agg_keys) -> bool:
    """True when ``_plan_direct`` covers the call (``_direct_batch_dims``)."""
    return _direct_batch_dims(lhs, rhs, join_keys, agg_keys) is not None


def _plan_direct(lhs, rhs, join_keys, agg_keys, marks=None, nb=None):
    """Join + grouping without sorts (``es_direct_*``); None when a relation
    is not in lexicographic order (the general path then runs). ``marks``:
    see ``sparse.mark``; ``nb``: ``_direct_batch_dims`` when known."""
    dev = lhs.device
    lib = L.lib()
    if nb is None:
        nb = _direct_batch_dims(lhs, rhs, join_keys, agg_keys)
    lg, rg = L.i64arr(lhs.grid()), L.i64arr(rhs.grid())
    nl, nr = lhs.num_tuples, rhs.num_tuples
    ws = workspace(lib.es_direct_workspace_size(nl, lhs.ndim, nr, rhs.ndim, nb, lg, rg), dev)
    # P, O, out of order (all written by the plan), status (cleared by it)
    cnt = torch.empty(4, dtype=torch.int64, device=dev)
    st = stream_ptr(dev)
    lc, rc = lhs.coords.contiguous(), rhs.coords.contiguous()
    mark(marks, "plan0")
    L.check("es_direct_plan", lib.es_direct_plan(
        lc.data_ptr(), nl, lhs.ndim, rc.data_ptr(), nr, rhs.ndim, nb, lg, rg, ws.data_ptr(), ws.numel(),
        cnt.data_ptr(), cnt[3:].data_ptr(), st))
    mark(marks, "plan1")
    P, O, unordered, err = read_counts(cnt, launch_pending=True)
    L.device_error("es_direct_plan", err, "tile coordinate outside the tensor grid")
    if unordered:
        return None
    out_nd = len(agg_keys)
    oc = torch.empty((O, out_nd), dtype=torch.int32, device=dev)
    so = torch.empty(O + 1, dtype=torch.int64, device=dev)
    sl = torch.empty(P, dtype=torch.int32, device=dev)
    sr = torch.empty(P, dtype=torch.int32, device=dev)
    sg = torch.empty(O, dtype=torch.int64, device=dev)
    # the contracted coordinate names the lhs tile of a strip only without
    # batch dims (the general path's rule): the tensor-core path may then
    # merge strips on it
    sk = torch.empty(P, dtype=torch.int32, device=dev) if nb == 0 else None
    mark(marks, "fill0")
    L.check("es_direct_fill", lib.es_direct_fill(
        lc.data_ptr(), nl, lhs.ndim, nr, rhs.ndim, nb, lg, rg, ws.data_ptr(), ws.numel(), P, O, oc.data_ptr(),
        so.data_ptr(), sl.data_ptr(), sr.data_ptr(), sg.data_ptr(), sk.data_ptr() if sk is not None else None, st))
    mark(marks, "fill1")
    kext = _key_extents(lhs, rhs, [(lhs.ndim - 1, nb)])[0] if nb == 0 else 0
    # pairs come grouped; "join order" is taken to be this grouped order
    # (seg_pair None: the identity)
    return PairPlan(sl, sr, oc, so, sl, sr, None, sg, sk, kext)


def plan_pairs(lhs: SparseTensorRelation, rhs: SparseTensorRelation, join_keys, agg_keys,
               marks=None) -> PairPlan:
    """Join the relations and group the pairs by output tile.

    Host waits: one for the operands' tile counts when they come unresolved
    from ``tile_coo`` / ``tile_dense`` (both resolved together), and one for
    the pair and output-tile counts (matmul-like shapes; the general path
    reads them one after the other). The operands' pending value fills are
    launched behind that count copy, so they run while the host sizes the
    pair arrays and launches what follows.

    Matmul-like shapes (``_direct_shape``) group without sorting; the pairs of
    each output tile are in join order either way, and ``lhs_idx``/``rhs_idx``
    then hold the grouped order."""
    dev = lhs.device
    nb = _direct_batch_dims(lhs, rhs, join_keys, agg_keys) if lhs.num_tuples > 0 and rhs.num_tuples > 0 else None
    if nb is not None:
        plan = _plan_direct(lhs, rhs, join_keys, agg_keys, marks, nb)
        if plan is not None:
            return plan
    li, ri = _join_int32(lhs, rhs, join_keys)
    P = int(li.shape[0])
    out_nd = len(agg_keys)
    if P == 0:
        z = torch.zeros(0, dtype=torch.int32, device=dev)
        return PairPlan(li, ri, torch.zeros((0, out_nd), dtype=torch.int32, device=dev),
                        torch.zeros(1, dtype=torch.int64, device=dev), z, z, z)
    for s, d in agg_keys:
        if s not in (0, 1) or not (0 <= d < (lhs.ndim if s == 0 else rhs.ndim)):
            raise ValueError(f"agg key {(s, d)} invalid")
    lib = L.lib()
    ext = L.i64arr(_out_extents(lhs, rhs, agg_keys))
    flat = L.i32arr([int(v) for k in agg_keys for v in k])
    ws = workspace(lib.es_segments_workspace_size(P), dev)
    cnt = torch.zeros(2, dtype=torch.int64, device=dev)
    st = stream_ptr(dev)
    L.check("es_segments_plan", lib.es_segments_plan(
        lhs.coords.contiguous().data_ptr(), lhs.ndim, rhs.coords.contiguous().data_ptr(), rhs.ndim, li.data_ptr(),
        ri.data_ptr(), P, flat, out_nd, ext, ws.data_ptr(), ws.numel(), cnt.data_ptr(), cnt[1:].data_ptr(), st))
    O, err = read_counts(cnt, launch_pending=True)
    L.device_error("es_segments_plan", err, "output tile coordinate outside the output grid")
    oc = torch.empty((O, out_nd), dtype=torch.int32, device=dev)
    so = torch.empty(O + 1, dtype=torch.int64, device=dev)
    sl = torch.empty(P, dtype=torch.int32, device=dev)
    sr = torch.empty(P, dtype=torch.int32, device=dev)
    sp = torch.empty(P, dtype=torch.int32, device=dev)
    # segments sharing the leading lhs-derived output coordinates form a strip
    nlead = 0
    while nlead < out_nd and agg_keys[nlead][0] == 0:
        nlead += 1
    strips = nlead > 0 and all(s == 1 for s, _ in agg_keys[nlead:])
    sg = torch.empty(O, dtype=torch.int64, device=dev) if strips else None
    L.check("es_segments_fill", lib.es_segments_fill(
        li.data_ptr(), ri.data_ptr(), P, out_nd, ext, ws.data_ptr(), ws.numel(), O, oc.data_ptr(), so.data_ptr(),
        sl.data_ptr(), sr.data_ptr(), sp.data_ptr(), nlead, sg.data_ptr() if sg is not None else None, st))
    # contracted coordinate of each grouped pair, when it names the lhs tile
    # of a strip (one join key; lhs coordinates = leading output dims + that
    # key): the tensor-core path may then merge strips on it
    sk, kext = None, 0
    lhs_dims = {int(d) for s, d in agg_keys[:nlead]}
    if strips and len(join_keys) == 1 and lhs_dims | {int(join_keys[0][0])} == set(range(lhs.ndim)) \
            and len(lhs_dims) == nlead and int(join_keys[0][0]) not in lhs_dims:
        jd = int(join_keys[0][0])
        sk = torch.empty((P, 1), dtype=torch.int32, device=dev)
        L.check("es_output_coords", lib.es_output_coords(
            lhs.coords.contiguous().data_ptr(), lhs.ndim, rhs.coords.contiguous().data_ptr(), rhs.ndim,
            sl.data_ptr(), sr.data_ptr(), P, L.i32arr([0, jd]), 1, sk.data_ptr(), st))
        sk = sk.reshape(-1)
        kext = _key_extents(lhs, rhs, [tuple(join_keys[0])])[0]
    return PairPlan(li, ri, oc, so, sl, sr, sp, sg, sk, kext)


def _resolve_shapes(lhs, rhs, kernel_string, agg_keys, output_shape, output_tile_shape):
    if output_tile_shape is None:
        output_tile_shape = _infer_output_tile_shape(kernel_string, lhs.tile_shape, rhs.tile_shape)
    if output_shape is None:
        output_shape = tuple(lhs.shape[d] if s == 0 else rhs.shape[d] for s, d in agg_keys)
    return tuple(output_shape), tuple(output_tile_shape)


def execute_sparse(lhs, rhs, join_keys, kernel_string, agg_keys, output_shape=None, output_tile_shape=None,
                   *, precision="auto", plan: PairPlan | None = None) -> SparseTensorRelation:
    """Join -> fused tile einsum + segment-sum (``execution/sparse_dispatch.py:226-297``).

    Output coordinates are sorted lexicographically; each output tile is the
    fp32 sum over its pairs in join order. ``precision``: "auto" (tensor cores
    where a kernel covers the shape, fp32-level accuracy), "exact" (fp32 FFMA)
    or "tc" (tensor cores or error).
    """
    if "->" not in kernel_string:
        raise ValueError(f"kernel_string must contain '->': {kernel_string}")
    lhs, rhs = as_relation(lhs), as_relation(rhs)
    output_shape, output_tile_shape = _resolve_shapes(lhs, rhs, kernel_string, agg_keys, output_shape,
                                                      output_tile_shape)
    plan = plan or plan_pairs(lhs, rhs, join_keys, agg_keys)
    if plan.num_pairs == 0:
        return empty_relation(output_shape, output_tile_shape, lhs.values.dtype, lhs.device)
    # deferred tile fills finish under the GEMM's pair grouping; the GEMM's
    # device status is read at the next count read (no wait here)
    lv, lr = lhs.values_and_ready()
    rv, rr = rhs.values_and_ready()
    vals = tile_einsum(kernel_string, lv, rv, plan.seg_lhs, plan.seg_rhs, plan.seg_offsets,
                       precision=precision, seg_strip=plan.seg_strip, pair_key=plan.seg_key,
                       key_extent=plan.key_extent, check="defer", ready=latest_ready(lr, rr))
    return SparseTensorRelation(plan.out_coords, vals, output_shape, output_tile_shape)


def execute_sharded_sparse(lhs, rhs, join_keys, kernel_string, agg_keys, output_shape=None, output_tile_shape=None,
                           mesh=None, num_devices=None, *, group=None, gather=True, precision="auto",
                           shard="output", lhs_sharded=False, timings=None):
    """Multi-GPU ``execute_sparse`` (``execution/sparse_dispatch.py:330-478``).

    One process per GPU (``torch.distributed``). With no process group, or a
    single rank, this is ``execute_sparse`` (the reference's fallback at
    :377-393). ``shard="output"``: each rank takes a contiguous range of
    output strips (lhs tiles sharing their lhs-derived output coordinates)
    balanced by join pairs, and joins, groups and contracts only those —
    output tiles are independent, so no collective touches the data path.
    ``shard="contracted"``: each rank contracts a contiguous range of the
    (single) join key and the partial tiles are summed by a reduce-scatter
    over the union of output coordinates. With ``gather`` every rank returns
    the full relation, as the reference does; without it, its own share.
    ``lhs_sharded``: ``lhs`` is already this rank's share (e.g. tiled from its
    ``distributed.balanced_row_ranges`` rows of an element COO).
    ``mesh`` is accepted for signature compatibility; ranks come from ``group``.
    """
    from . import distributed as D
    return D.execute_sharded_sparse(lhs, rhs, join_keys, kernel_string, agg_keys, output_shape, output_tile_shape,
                                    num_devices=num_devices, group=group, gather=gather, precision=precision,
                                    shard=shard, lhs_sharded=lhs_sharded, timings=timings)
