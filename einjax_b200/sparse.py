"""Tile-COO relations on the GPU; mirrors einjax ``tensor/sparse.py``.

``SparseTensorRelation`` keeps the reference's layout (``tensor/sparse.py:27-90``):
``coords`` int32 ``(T, ndim)`` in lexicographic order and ``values``
``(T, *tile_shape)`` row-major, here as CUDA tensors in float32 (the dtype the
reference's JAX path computes in with x64 off) or bfloat16.
``SparseTensor(name, data).to_relation(tile_shape)`` runs the tiling on the
GPU through ``es_tile_coo_*`` / ``es_tile_dense_*``.
"""

from __future__ import annotations

from math import prod
from typing import Any

import numpy as np
import torch

from . import _lib as L

_TORCH_TO_ES = {torch.float32: L.ES_F32, torch.bfloat16: L.ES_BF16, torch.float64: L.ES_F64}
_ES_TO_TORCH = {L.ES_F32: torch.float32, L.ES_BF16: torch.bfloat16}


def es_dtype(t: torch.Tensor) -> int:
    try:
        return _TORCH_TO_ES[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported value dtype {t.dtype}") from None


def default_device() -> torch.device:
    if not torch.cuda.is_available():
        raise L.EinsparseUnavailable("einjax_b200 needs a CUDA device (sm_100a); no CPU fallback exists")
    return torch.device("cuda", torch.cuda.current_device())


def _device_index(device) -> int:
    if isinstance(device, torch.device):
        return device.index if device.index is not None else torch.cuda.current_device()
    return torch.cuda.current_device() if device is None else int(device)


def stream_ptr(device=None) -> int:
    """cudaStream_t of the current stream of ``device``."""
    return _raw_stream(_device_index(device))


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None) or (
    lambda i: torch.cuda.current_stream(i).cuda_stream)


def workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def mark(marks, label: str) -> None:
    """Appends (label, CUDA event recorded on the current stream) to ``marks``
    when it is a list: lets a caller time the launches of one call without
    the host reads of counts between them."""
    if marks is not None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        marks.append((label, ev))


class _DeferredErrors:
    """Device error slots read back later, without a sync of their own.

    ``defer`` queues an asynchronous copy of a call's int32 error slot into a
    pinned host ring and records an event; ``flush`` (run after every host
    read of counts, which waits on the stream anyway, and by
    ``check_device_errors``) reads the copies that have landed and raises for
    the first non-zero one. A failure of a call is then reported by the next
    call that reads counts back, as CUDA reports asynchronous errors."""

    SLOTS = 256

    def __init__(self):
        self.host = None
        self.next = 0
        self.pending = []  # (function name, slot, event)

    def _slot(self) -> int:
        if self.host is None:
            self.host = torch.zeros(self.SLOTS, dtype=torch.int32, pin_memory=True)
            self.events = [None] * self.SLOTS
        # a slot (and its event) is reused SLOTS allocations later, always
        # after a flush has consumed its previous entry
        if len(self.pending) >= self.SLOTS - 1:
            self.flush()
        slot = self.next
        self.next = (self.next + 1) % self.SLOTS
        return slot

    def _commit(self, fn: str, slot: int) -> None:
        ev = self.events[slot]
        if ev is None:
            ev = self.events[slot] = torch.cuda.Event()
        ev.record()
        self.pending.append((fn, slot, ev))

    def defer(self, fn: str, err: torch.Tensor) -> None:
        slot = self._slot()
        self.host[slot:slot + 1].copy_(err.reshape(1), non_blocking=True)
        self._commit(fn, slot)

    def reserve(self, fn: str):
        """``(host_address, commit)`` for a call that copies its own status
        into the pinned slot (``es_tile_einsum_ev``'s ``status_host``);
        ``commit()`` after the call queues the slot for the next flush."""
        slot = self._slot()
        return self.host.data_ptr() + 4 * slot, (lambda: self._commit(fn, slot))

    def flush(self) -> None:
        pending, self.pending = self.pending, []
        first = None
        for fn, slot, ev in pending:
            ev.synchronize()
            e = int(self.host[slot])
            if e and first is None:
                first = (fn, e)
        if first is not None:
            L.check(first[0] + " (device)", first[1])


_DEFERRED = _DeferredErrors()


def defer_device_error(fn: str, err: torch.Tensor) -> None:
    """Check ``err`` (device int32 status) at the next count read or
    ``check_device_errors`` instead of now."""
    _DEFERRED.defer(fn, err)


def check_device_errors() -> None:
    """Wait for the deferred device error slots of earlier calls and raise
    for the first failure (``ValueError`` for bad input, ``EinsparseError``
    otherwise, e.g. a bounded wait that ran out)."""
    _DEFERRED.flush()


class _PendingFills:
    """Relations whose tile values are not written yet, oldest first.

    The tiling calls write a relation's coordinates at once and queue the
    launch of its value fill here. The pair plan's count reads launch the
    queued fills between the copy of their counts and their wait, so the GPU
    fills tiles (the largest writes of a step) while the host waits for the
    counts and then sizes and launches what follows; a relation's first
    ``values`` access launches its own fill."""

    def __init__(self):
        self.rels = []  # weak references, creation order

    def add(self, rel) -> None:
        import weakref
        self.rels.append(weakref.ref(rel))

    def __bool__(self) -> bool:
        return bool(self.rels)

    def flush(self) -> None:
        rels, self.rels = self.rels, []
        for r in rels:
            rel = r()
            if rel is not None:
                rel.materialize()


_PENDING = _PendingFills()


class _PendingTilings:
    """Tile counts of tiling calls not read yet. Each call copies its counts
    into a slot of a pinned ring right after its plan launches and records
    an event (no wait); the first use of any such relation waits for the
    copies and resolves every pending tiling in call order."""

    SLOTS = 1024

    def __init__(self):
        self.host = None
        self.next = 0
        self.items = []  # (weak relation, slot, n, event)

    def add(self, rel, counts: torch.Tensor) -> None:
        import weakref
        n = int(counts.numel())
        if self.host is None:
            self.host = torch.empty(self.SLOTS, dtype=torch.int64, pin_memory=True)
        if self.next + n > self.SLOTS:
            self.resolve_all()
            self.next = 0
        slot = self.next
        self.next += n
        self.host[slot:slot + n].copy_(counts, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self.items.append((weakref.ref(rel), slot, n, ev))

    def __bool__(self) -> bool:
        return bool(self.items)

    def resolve_all(self) -> None:
        items, self.items = self.items, []
        if not items:
            return
        for _, _, _, ev in items:
            ev.synchronize()
        vals = self.host[:max(slot + n for _, slot, n, _ in items)].tolist()
        self.next = 0
        for r, slot, n, _ in items:
            rel = r()
            if rel is not None and rel._finish is not None:
                rel._complete(vals[slot:slot + n])


_TILINGS = _PendingTilings()


def resolve_tilings() -> None:
    """Read the tile counts of every unresolved relation (one wait) and
    launch their coordinate writes."""
    _TILINGS.resolve_all()


def latest_ready(*readies):
    """The newest of ``(sequence, event)`` pairs (None entries skipped): the
    fill stream runs in order, so its event covers the older ones."""
    rs = [r for r in readies if r is not None]
    return max(rs, key=lambda r: r[0]) if rs else None


def launch_pending_fills() -> None:
    """Launch the value fills of every relation whose values are pending
    (stream-ordered like any launch; nothing waits)."""
    _PENDING.flush()


class _CountReader:
    """Pinned host buffer for count reads: the copy goes in asynchronously,
    pending fills are launched behind it, and the host waits on an event
    recorded right after the copy, not on the whole stream."""

    def __init__(self):
        self.host = None

    def read(self, t: torch.Tensor, launch_pending: bool):
        n = int(t.numel())
        if self.host is None or self.host.numel() < n:
            self.host = torch.empty(max(n, 16), dtype=torch.int64, pin_memory=True)
        h = self.host[:n]
        h.copy_(t.reshape(-1).to(torch.int64), non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        if launch_pending and _PENDING:
            _PENDING.flush()
        ev.synchronize()
        return [int(v) for v in h.tolist()]


_COUNTS = _CountReader()


def read_counts(t: torch.Tensor, launch_pending: bool = False):
    """Read a small device int64 tensor (count, error, ...): one wait, on the
    copy alone; deferred error slots of earlier calls are checked after it.
    ``launch_pending``: launch the pending value fills behind the copy first
    (the pair plan's reads do, since the most host work of a contraction --
    sizing the pairs and launching the tile einsum -- follows them, and the
    fills keep the GPU busy meanwhile)."""
    vals = _COUNTS.read(t, launch_pending)
    if _DEFERRED.pending:
        _DEFERRED.flush()
    return vals


def value_dtype_for(dtype) -> torch.dtype:
    """Device storage dtype for an input dtype: bf16 stays bf16, else float32."""
    if dtype in (torch.bfloat16, "bf16", "bfloat16"):
        return torch.bfloat16
    return torch.float32


class SparseTensorRelation:
    """Tile-COO relation held on the GPU (``tensor/sparse.py:27-90``).

    ``tile_coo`` and ``tile_dense`` return relations in two deferred states.
    Unresolved: the tile count is still on its way to the host; the first
    use of ``coords``, ``values`` or ``num_tuples`` of any unresolved
    relation waits once and resolves all of them (allocation and coordinate
    launch), so the operands of a contraction share one host wait; a bad
    input (e.g. a COO index outside the shape) raises there. Pending
    values: the value fill is launched by the first read of ``values``, by
    ``materialize()``, or by the next count read of a pair plan
    (``plan_pairs``), whichever comes first; it reads the tiling's input
    until then, and raises if that input was changed in place meanwhile."""

    __slots__ = ("_coords", "_values", "shape", "tile_shape", "_pending", "_finish", "_failed", "_dev", "_ready",
                 "__weakref__")

    def __init__(self, coords: torch.Tensor, values: torch.Tensor, shape, tile_shape, pending=None):
        self._coords = coords
        self._values = values
        self.shape = tuple(int(s) for s in shape)
        self.tile_shape = tuple(int(t) for t in tile_shape)
        self._pending = pending
        self._finish = None
        self._failed = None
        self._dev = None
        self._ready = None  # (sequence, event) behind the value fill on the fill stream
        if pending is not None:
            _PENDING.add(self)

    @classmethod
    def _unresolved(cls, shape, tile_shape, device, counts: torch.Tensor, finish) -> "SparseTensorRelation":
        """A relation whose tile count is on the device (``counts``):
        ``finish(host_counts)`` returns ``(coords, values, pending_fill)``."""
        rel = cls(None, None, shape, tile_shape)
        rel._finish = finish
        rel._dev = device
        _TILINGS.add(rel, counts)
        return rel

    def _resolve(self) -> None:
        if self._finish is not None:
            _TILINGS.resolve_all()
        if self._failed is not None:
            raise self._failed

    def _complete(self, host_counts) -> None:
        finish, self._finish = self._finish, None
        try:
            coords, values, pending = finish(host_counts)
        except Exception as e:  # kept: every later use raises it again
            self._failed = e
            return
        self._coords, self._values = coords, values
        if pending is not None:
            self._pending = pending
            _PENDING.add(self)

    @property
    def coords(self) -> torch.Tensor:
        if self._finish is not None or self._failed is not None:
            self._resolve()
        return self._coords

    @coords.setter
    def coords(self, c: torch.Tensor) -> None:
        self._finish = self._failed = None
        self._coords = c

    @property
    def values(self) -> torch.Tensor:
        """The tile values; the current stream waits for a deferred fill."""
        v, ready = self.values_and_ready()
        if ready is not None:
            torch.cuda.current_stream(v.device).wait_event(ready[1])
        return v

    @values.setter
    def values(self, v: torch.Tensor) -> None:
        self._pending = None
        self._ready = None
        self._values = v

    def values_and_ready(self):
        """``(values, ready)`` without waiting: ``ready`` is ``(sequence,
        event)`` behind the value fill on the device's fill stream, or None
        when the values are written in stream order. A caller that reads the
        values on a stream must make it wait for the event first (e.g.
        ``tile_einsum(..., ready=...)``, which waits just before the launch
        that reads them)."""
        if self._finish is not None or self._failed is not None:
            self._resolve()
        if self._pending is not None:
            self.materialize()
        return self._values, self._ready

    @property
    def pending(self) -> bool:
        """True while the tile count is unread or the value fill has not been
        launched."""
        return self._finish is not None or self._pending is not None

    def materialize_count(self) -> "SparseTensorRelation":
        """Resolve the tile count (and with it every unresolved relation);
        the value fill stays pending."""
        if self._finish is not None or self._failed is not None:
            self._resolve()
        return self

    def materialize(self) -> "SparseTensorRelation":
        """Resolve the tile count and launch the pending value fill (no-op
        when neither is pending)."""
        if self._finish is not None or self._failed is not None:
            self._resolve()
        fill, self._pending = self._pending, None
        if fill is not None:
            self._ready = fill()
        return self

    def __repr__(self) -> str:
        if self._finish is not None:
            return f"SparseTensorRelation(unresolved, shape={self.shape}, tile_shape={self.tile_shape})"
        return (f"SparseTensorRelation(tuples={self.num_tuples}, shape={self.shape}, "
                f"tile_shape={self.tile_shape}, dtype={self._values.dtype}, pending={self.pending})")

    @property
    def num_tuples(self) -> int:
        return int(self.coords.shape[0])

    @property
    def ndim(self) -> int:
        return len(self.shape)

    @property
    def tile_size(self) -> int:
        return prod(self.tile_shape)

    @property
    def nnz(self) -> int:
        return int(torch.count_nonzero(self.values).item())

    @property
    def density(self) -> float:
        total = prod(self.shape)
        return self.nnz / total if total > 0 else 0.0

    @property
    def device(self) -> torch.device:
        return self._dev if self._finish is not None else self.coords.device

    def grid(self) -> tuple:
        """Tile-grid extent per dimension (ceil(shape / tile), at least 1)."""
        return tuple(max(1, -(-s // t)) for s, t in zip(self.shape, self.tile_shape))

    def to_dense(self) -> torch.Tensor:
        """Scatter tiles into a dense device tensor (``tensor/sparse.py:75-90``)."""
        out = torch.zeros(self.shape, dtype=self.values.dtype, device=self.values.device)
        if self.num_tuples == 0:
            return out
        g = self.grid()
        view_shape = []
        for gd, td in zip(g, self.tile_shape):
            view_shape += [gd, td]
        perm = list(range(0, 2 * self.ndim, 2)) + list(range(1, 2 * self.ndim, 2))
        blocked = out.view(*view_shape).permute(*perm)  # (g0, g1, ..., t0, t1, ...)
        idx = tuple(self.coords[:, d].long() for d in range(self.ndim))
        blocked[idx] = self.values.reshape(self.num_tuples, *self.tile_shape)
        return out

    def to_numpy(self):
        """``(coords int32, values)`` as numpy arrays (values float32)."""
        return (self.coords.cpu().numpy(), self.values.float().cpu().numpy())

    @staticmethod
    def from_arrays(coords, values, shape, tile_shape, device=None, dtype=None) -> "SparseTensorRelation":
        """Move host (numpy) or device tile-COO arrays onto the GPU.

        float64 values become float32 (JAX's x64-off default), bfloat16 stays.
        """
        device = device or default_device()
        vt = value_dtype_for(dtype if dtype is not None else getattr(values, "dtype", None))
        c = torch.as_tensor(np.asarray(coords, dtype=np.int32) if not torch.is_tensor(coords) else coords)
        c = c.to(device=device, dtype=torch.int32).reshape(-1, len(shape)).contiguous()
        if torch.is_tensor(values):
            v = values.to(device=device, dtype=vt)
        else:
            v = torch.from_numpy(np.ascontiguousarray(values)).to(device=device).to(vt)
        v = v.reshape(c.shape[0], *tile_shape).contiguous()
        return SparseTensorRelation(c, v, tuple(shape), tuple(tile_shape))

    @staticmethod
    def from_reference(rel, device=None, dtype=None) -> "SparseTensorRelation":
        """Convert any object with ``coords, values, shape, tile_shape`` (e.g. the
        reference's numpy ``SparseTensorRelation``)."""
        return SparseTensorRelation.from_arrays(rel.coords, rel.values, rel.shape, rel.tile_shape, device, dtype)


def as_relation(x, device=None) -> SparseTensorRelation:
    if isinstance(x, SparseTensorRelation):
        return x
    return SparseTensorRelation.from_reference(x, device)


def empty_relation(shape, tile_shape, dtype, device) -> SparseTensorRelation:
    return SparseTensorRelation(torch.zeros((0, len(shape)), dtype=torch.int32, device=device),
                                torch.zeros((0, *tile_shape), dtype=dtype, device=device), shape, tile_shape)


def _check_divisible(shape, tile_shape):
    if len(tile_shape) != len(shape):
        raise ValueError(f"tile_shape rank {len(tile_shape)} != tensor rank {len(shape)}")
    for d, (s, t) in enumerate(zip(shape, tile_shape)):
        if t <= 0 or s % t != 0:
            raise ValueError(f"tile_shape[{d}]={t} does not evenly divide shape[{d}]={s}")


DUPLICATE_POLICIES = ("last", "sum", "error")


def as_device_tensor(x, device=None) -> torch.Tensor:
    """A torch tensor for ``x``: torch tensors as they are, objects exporting
    DLPack (JAX / CuPy arrays; zero-copy when they already live on the GPU)
    through ``torch.from_dlpack``, anything else through numpy; then moved
    to ``device`` when given (no copy if it is already there)."""
    if torch.is_tensor(x):
        t = x
    elif hasattr(x, "__dlpack__") and not isinstance(x, np.ndarray):
        t = torch.from_dlpack(x)
    else:
        t = torch.as_tensor(np.asarray(x))
    return t if device is None else t.to(device)


def coalesce_coo(indices, values, shape, duplicates="sum", out_dtype=torch.float64, marks=None):
    """One entry per distinct coordinate holding a non-zero value, in row-major
    coordinate order, on the GPU (``es_coo_coalesce``): ``duplicates="sum"``
    adds repeated coordinates (float64, input order; scipy / torch sparse
    semantics), ``"last"`` keeps the last in input order (the reference's
    tiling, ``tensor/sparse.py:211-212``). Zero entries are dropped first.
    Returns ``(indices int32 (n, ndim), values (n,), nonzero_inputs)``.
    ``marks``: see ``mark`` (coalesce0/coalesce1 around the launches)."""
    if duplicates not in ("sum", "last"):
        raise ValueError(f"duplicates must be 'sum' or 'last', got {duplicates!r}")
    shape = tuple(int(s) for s in shape)
    nd = len(shape)
    vals = as_device_tensor(values)
    dev = vals.device if vals.is_cuda else default_device()
    vals = vals.to(dev)
    if vals.dtype not in _TORCH_TO_ES:
        vals = vals.to(torch.float64)
    vals = vals.reshape(-1).contiguous()
    idx = as_device_tensor(indices, dev).to(torch.int32).reshape(-1, nd).contiguous()
    n = int(vals.shape[0])
    if int(idx.shape[0]) != n:
        raise ValueError("values and indices disagree in length")
    lib = L.lib()
    sh = L.i64arr(shape)
    ws = workspace(lib.es_coo_coalesce_workspace_size(n, nd, sh), dev)
    oi = torch.empty((max(n, 1), nd), dtype=torch.int32, device=dev)
    ov = torch.empty(max(n, 1), dtype=out_dtype, device=dev)
    cnt = torch.zeros(3, dtype=torch.int64, device=dev)
    mark(marks, "coalesce0")
    L.check("es_coo_coalesce", lib.es_coo_coalesce(
        idx.data_ptr(), vals.data_ptr(), es_dtype(vals), n, nd, sh,
        L.ES_DUP_SUM if duplicates == "sum" else L.ES_DUP_LAST, ws.data_ptr(), ws.numel(), oi.data_ptr(),
        ov.data_ptr(), es_dtype(ov), cnt.data_ptr(), cnt[2:].data_ptr(), stream_ptr(dev)))
    mark(marks, "coalesce1")
    u, nz, err = read_counts(cnt)
    L.device_error("es_coo_coalesce", err, "COO index outside the tensor shape")
    return oi[:u], ov[:u], nz


def tile_coo(indices: torch.Tensor, values: torch.Tensor, shape, tile_shape,
             out_dtype=torch.float32, marks=None, duplicates="last") -> SparseTensorRelation:
    """Element COO (device tensors) -> tile-COO relation (``tensor/sparse.py:160-219``).

    ``indices`` int32 ``(nnz, ndim)``, ``values`` (nnz,) float32/float64/bf16.
    Zeros are dropped. Repeated coordinates: ``duplicates="last"`` (the
    reference's behaviour) keeps the last in input order, ``"sum"`` adds them
    (``coalesce_coo`` first), ``"error"`` raises ``ValueError``. ``marks``:
    see ``mark`` (plan0/plan1 around the plan launches, fill0/fill1 around the
    fill).

    The relation comes back unresolved (``SparseTensorRelation``): the tile
    count is read, and an index outside ``shape`` raises ``ValueError``, at
    its first use, together with every other unresolved relation; the tile
    values are then a pending fill launched at the first use of ``values``
    or the next pair plan's count read. ``values`` (the input) must stay
    unchanged until then (``materialize()`` does both now). With ``marks``
    the tiling is complete before returning.
    """
    if duplicates not in DUPLICATE_POLICIES:
        raise ValueError(f"duplicates must be one of {DUPLICATE_POLICIES}, got {duplicates!r}")
    if duplicates != "last":
        ci, cv, nz = coalesce_coo(indices, values, shape, "sum" if duplicates == "sum" else "last")
        if duplicates == "error" and int(ci.shape[0]) != nz:
            raise ValueError(f"{nz - int(ci.shape[0])} repeated COO coordinates (duplicates='error')")
        indices, values = ci, cv
    shape = tuple(int(s) for s in shape)
    tile_shape = tuple(int(t) for t in tile_shape)
    _check_divisible(shape, tile_shape)
    dev = values.device
    lib = L.lib()
    nnz = int(values.shape[0])
    idx = indices.to(device=dev, dtype=torch.int32).contiguous()
    vals = values.contiguous()
    if nnz == 0:
        return empty_relation(shape, tile_shape, out_dtype, dev)
    sh, tl = L.i64arr(shape), L.i64arr(tile_shape)
    nd = len(shape)
    wsb = lib.es_tile_coo_workspace_size(nnz, nd, sh, tl)
    ws = workspace(wsb, dev)
    cnt = torch.empty(2, dtype=torch.int64, device=dev)  # cleared by the plan call
    st = stream_ptr(dev)
    mark(marks, "plan0")
    L.check("es_tile_coo_plan", lib.es_tile_coo_plan(
        idx.data_ptr(), vals.data_ptr(), es_dtype(vals), nnz, nd, sh, tl, ws.data_ptr(), ws.numel(),
        cnt.data_ptr(), cnt[1:].data_ptr(), st))
    mark(marks, "plan1")
    oc = L.ES_F32 if out_dtype == torch.float32 else L.ES_BF16
    vd = es_dtype(vals)
    stream = torch.cuda.current_stream(dev)
    version = vals._version

    def finish(counts):
        T, err = counts
        L.device_error("es_tile_coo_plan", err, "COO index outside the tensor shape")
        with _on(stream):
            coords = torch.empty((T, nd), dtype=torch.int32, device=dev)
            out = torch.empty((T, *tile_shape), dtype=out_dtype, device=dev)
            L.check("es_tile_coo_fill", lib.es_tile_coo_fill(
                vals.data_ptr(), vd, nnz, nd, sh, tl, ws.data_ptr(), ws.numel(), T, coords.data_ptr(), None, oc,
                stream.cuda_stream))
        if T == 0:
            return coords, out, None
        after = torch.cuda.Event()
        after.record(stream)

        def launch(sp):
            L.check("es_tile_coo_fill", lib.es_tile_coo_fill(
                vals.data_ptr(), vd, nnz, nd, sh, tl, ws.data_ptr(), ws.numel(), T, None, out.data_ptr(), oc, sp))
        return coords, out, _deferred_fill(dev, vals, launch, "tile_coo", after, version, (out, ws, vals))

    if marks is None:
        return SparseTensorRelation._unresolved(shape, tile_shape, dev, cnt, finish)
    # timed callers get the tiling done now, between their marks
    coords, out, fill = finish(read_counts(cnt))
    mark(marks, "fill0")
    if fill is not None:
        torch.cuda.current_stream(dev).wait_event(fill()[1])
    mark(marks, "fill1")
    return SparseTensorRelation(coords, out, shape, tile_shape)


class _on:
    """``torch.cuda.stream(s)`` when ``s`` is not already current (entering
    the context costs a few microseconds)."""

    def __init__(self, stream):
        self.stream = stream
        self.ctx = None

    def __enter__(self):
        if _raw_stream(self.stream.device_index) != self.stream.cuda_stream:
            self.ctx = torch.cuda.stream(self.stream)
            self.ctx.__enter__()

    def __exit__(self, *a):
        if self.ctx is not None:
            self.ctx.__exit__(*a)


def tile_dense(dense: torch.Tensor, tile_shape, out_dtype=torch.float32) -> SparseTensorRelation:
    """Dense device array -> tile-COO of its non-zero tiles (``to_relation`` of a
    dense ``SparseTensor``, ``tensor/sparse.py:104-117,160-219``). As with
    ``tile_coo``, the relation comes back unresolved and its values are a
    pending fill that reads ``dense`` when it runs."""
    shape = tuple(int(s) for s in dense.shape)
    tile_shape = tuple(int(t) for t in tile_shape)
    _check_divisible(shape, tile_shape)
    dev = dense.device
    lib = L.lib()
    d = dense.contiguous()
    sh, tl = L.i64arr(shape), L.i64arr(tile_shape)
    nd = len(shape)
    ws = workspace(lib.es_tile_dense_workspace_size(nd, sh, tl), dev)
    cnt = torch.empty(1, dtype=torch.int64, device=dev)  # cleared by the plan call
    st = stream_ptr(dev)
    L.check("es_tile_dense_plan", lib.es_tile_dense_plan(
        d.data_ptr(), es_dtype(d), nd, sh, tl, ws.data_ptr(), ws.numel(), cnt.data_ptr(), st))
    oc = L.ES_F32 if out_dtype == torch.float32 else L.ES_BF16
    stream = torch.cuda.current_stream(dev)
    version = d._version

    def finish(counts):
        T = counts[0]
        with _on(stream):
            coords = torch.empty((T, nd), dtype=torch.int32, device=dev)
            out = torch.empty((T, *tile_shape), dtype=out_dtype, device=dev)
            L.check("es_tile_dense_fill", lib.es_tile_dense_fill(
                d.data_ptr(), es_dtype(d), nd, sh, tl, ws.data_ptr(), ws.numel(), T, coords.data_ptr(), None, oc,
                stream.cuda_stream))
        if T == 0:
            return coords, out, None
        after = torch.cuda.Event()
        after.record(stream)

        def launch(sp):
            L.check("es_tile_dense_fill", lib.es_tile_dense_fill(
                d.data_ptr(), es_dtype(d), nd, sh, tl, ws.data_ptr(), ws.numel(), T, None, out.data_ptr(), oc, sp))
        return coords, out, _deferred_fill(dev, d, launch, "tile_dense", after, version, (out, ws, d))

    return SparseTensorRelation._unresolved(shape, tile_shape, dev, cnt, finish)


_FILL_STREAMS = {}
_FILL_SEQ = [0]


def _fill_stream(dev) -> torch.cuda.Stream:
    """The device's stream for deferred value fills (one per device), at the
    lowest priority: a caller on a higher-priority stream gets its kernels
    scheduled ahead of a running fill's remaining CTAs, so the two overlap
    (on a default-priority stream the fill's CTAs go first)."""
    i = _device_index(dev)
    st = _FILL_STREAMS.get(i)
    if st is None:
        st = _FILL_STREAMS[i] = torch.cuda.Stream(device=i, priority=torch.cuda.Stream.priority_range()[0])
    return st


def _deferred_fill(dev, source: torch.Tensor, launch, name: str, after: torch.cuda.Event, version: int, keep):
    """Pending value fill of a tiling call. ``launch(stream)`` runs on the
    device's fill stream once ``after`` (recorded behind the tiling's
    coordinate write) has passed, so the fill overlaps whatever the tiling's
    stream does next; the returned callable launches it and gives back
    ``(sequence, event)``, the event recorded behind it. The tensors in
    ``keep`` (output, workspace, input) are marked used on the fill stream
    so their memory is not reused before the fill ends. ``source``, the
    tiling's input, must not be changed in place before the fill runs
    (checked through its version counter against ``version``, taken when the
    tiling was called)."""

    def fill():
        if source._version != version:
            raise RuntimeError(f"{name}: the input was changed in place before the tile values were filled; "
                               "call materialize() on the relation before changing it")
        side = _fill_stream(dev)
        side.wait_event(after)
        launch(side.cuda_stream)
        ev = torch.cuda.Event()
        ev.record(side)
        for t in keep:
            t.record_stream(side)
        _FILL_SEQ[0] += 1
        return (_FILL_SEQ[0], ev)
    return fill


def _extract_coo(data: Any):
    """Input -> (indices int32 (nnz, ndim), values, shape) on the host, as
    ``_extract_coo`` (``tensor/sparse.py:234-270``); dense input is kept dense
    (it is tiled on the GPU without a COO detour)."""
    try:
        import scipy.sparse as sp
        if sp.issparse(data):
            coo = sp.coo_matrix(data) if data.ndim == 2 else data.tocoo()
            idx = np.stack([coo.row, coo.col], axis=1).astype(np.int32)
            return "coo", idx, np.asarray(coo.data, dtype=np.float64), tuple(coo.shape)
    except ImportError:  # pragma: no cover
        pass
    if isinstance(data, tuple) and len(data) == 3:
        idx, val, shape = data
        return "coo", idx, val, tuple(int(s) for s in shape)
    if torch.is_tensor(data) and data.layout != torch.strided:
        coo = data if data.layout == torch.sparse_coo else data.to_sparse_coo()
        return "coo", coo._indices().t(), coo._values(), tuple(coo.shape)
    if torch.is_tensor(data):
        return "dense", data, None, tuple(data.shape)
    if hasattr(data, "coords") and hasattr(data, "data") and hasattr(data, "shape"):
        # COO objects with (ndim, nnz) coordinates, e.g. pydata sparse's COO
        return "coo", as_device_tensor(data.coords).t(), data.data, tuple(int(s) for s in data.shape)
    if hasattr(data, "__dlpack__") and not isinstance(data, np.ndarray):
        t = torch.from_dlpack(data)  # JAX / CuPy arrays: zero-copy on the device
        return "dense", t, None, tuple(t.shape)
    arr = np.asarray(data)
    if arr.dtype not in (np.float32, np.float64):
        arr = arr.astype(np.float64)
    return "dense", arr, None, tuple(arr.shape)


def find_all_factors(n: int) -> list:
    """Sorted divisors of n (``core/notation.py:27-43``)."""
    n = int(n)
    if n <= 0:
        raise ValueError(f"n must be positive, got {n}")
    out = set()
    for i in range(1, int(n ** 0.5) + 1):
        if n % i == 0:
            out.update((i, n // i))
    return sorted(out)


def factor_tile_shapes(shape) -> list:
    """The tiling schemes a tensor of this shape enumerates: every tile shape
    whose sides divide the shape (``tensor/base.py:43-49``), sorted."""
    import itertools
    return sorted(itertools.product(*[find_all_factors(n) for n in shape]))


def _sparsity_stats(indices, values, shape, tile_shapes, device):
    lib = L.lib()
    shape = tuple(int(s) for s in shape)
    nd = len(shape)
    ts = [tuple(int(t) for t in x) for x in tile_shapes]
    for t in ts:
        if len(t) != nd or min(t) <= 0:
            raise ValueError(f"tile shape {t} does not fit a tensor of shape {shape}")
    dev = torch.device(device) if device is not None else default_device()
    if indices is not None:
        idx = as_device_tensor(indices).to(device=dev, dtype=torch.int32).reshape(-1, nd).contiguous()
        n = int(idx.shape[0])
    else:
        idx = None
        n = prod(shape)
    vals = None
    if values is not None:
        vals = as_device_tensor(values)
        if vals.dtype not in (torch.float32, torch.float64, torch.bfloat16):
            vals = vals.to(torch.float64)
        vals = vals.to(dev).reshape(-1).contiguous()
        if int(vals.shape[0]) != n:
            raise ValueError("values and indices disagree in length")
    S = len(ts)
    sh, tl = L.i64arr(shape), L.i64arr([v for t in ts for v in t])
    ws = workspace(lib.es_sparsity_stats_workspace_size(n, nd, sh, tl, S), dev)
    nt = torch.zeros(max(S, 1), dtype=torch.int64, device=dev)
    vc = torch.zeros((max(S, 1), nd), dtype=torch.int64, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    L.check("es_sparsity_stats", lib.es_sparsity_stats(
        idx.data_ptr() if idx is not None else None, vals.data_ptr() if vals is not None else None,
        es_dtype(vals) if vals is not None else L.ES_F32, n, nd, sh, tl, S, ws.data_ptr(), ws.numel(),
        nt.data_ptr(), vc.data_ptr(), err.data_ptr(), stream_ptr(dev)))
    nt_h, vc_h, e = nt.cpu().tolist(), vc.cpu().tolist(), int(err.item())
    L.device_error("es_sparsity_stats", e, "COO index outside the tensor shape")
    return {t: (int(nt_h[i]), tuple(int(v) for v in vc_h[i])) for i, t in enumerate(ts)}


def compute_sparsity_stats_coo(indices, values, shape, tile_shapes, device=None) -> dict:
    """T(U) and V(l, U) for every tile shape U (``tensor/stats.py:25-80``):
    ``{tile_shape: (num_tuples, value_count)}``, computed on the GPU. Zero
    values do not count; repeated coordinates count once."""
    return _sparsity_stats(indices, values, shape, tile_shapes, device)


def compute_sparsity_stats_dense(data, tile_shapes, device=None) -> dict:
    """``compute_sparsity_stats_coo`` of a dense array's non-zeros
    (``tensor/stats.py:81-117``), reading the dense array directly."""
    d = data if torch.is_tensor(data) else torch.as_tensor(np.asarray(data))
    return _sparsity_stats(None, d, tuple(d.shape), tile_shapes, device)


class SparseTensor:
    """User-facing sparse tensor (``tensor/sparse.py:93-231``) whose tiling runs on the GPU.

    ``data``: a scipy sparse matrix, a dense numpy array / torch tensor, a
    torch sparse (COO / CSR) tensor, a COO object with ``coords`` ``(ndim,
    nnz)``, ``data`` and ``shape`` (pydata sparse), any DLPack exporter (JAX
    / CuPy arrays, taken without a copy when on the GPU), or an ``(indices,
    values, shape)`` COO triple (indices ``(nnz, ndim)``; any rank, unlike
    scipy; its arrays may be torch tensors or DLPack exporters too).

    ``duplicates`` says what repeated coordinates mean: ``"last"`` (the
    reference's tiling: the last in input order wins), ``"sum"`` (scipy /
    torch sparse semantics) or ``"error"``; the default is ``"sum"`` for
    torch sparse tensors and ``"last"`` for everything else.

    The reference computes per-scheme sparsity statistics
    (``_compute_sparsity_metrics``, planner input) in its constructor; here
    ``sparsity_stats()`` computes them on the GPU on demand.
    """

    def __init__(self, name: str, data: Any, device=None, dtype=None, duplicates=None):
        self.name = name
        self.device = device or default_device()
        self._kind, self._a, self._b, self.shape = _extract_coo(data)
        self.data = data
        self._out_dtype = value_dtype_for(dtype)
        if duplicates is None:
            duplicates = "sum" if torch.is_tensor(data) and data.layout != torch.strided else "last"
        if duplicates not in DUPLICATE_POLICIES:
            raise ValueError(f"duplicates must be one of {DUPLICATE_POLICIES}, got {duplicates!r}")
        self.duplicates = duplicates

    @property
    def ndim(self) -> int:
        return len(self.shape)

    def sparsity_stats(self, tile_shapes=None) -> dict:
        """``{tile_shape: (num_tuples, value_count)}`` for the given tile shapes,
        by default every tiling scheme of the shape (the ``num_tuples`` and
        ``value_count`` of the reference's ``self.schemes``,
        ``tensor/sparse.py:122-158``)."""
        ts = factor_tile_shapes(self.shape) if tile_shapes is None else tile_shapes
        if self._kind == "coo":
            return _sparsity_stats(self._a, self._b, self.shape, ts, self.device)
        return _sparsity_stats(None, self._a, self.shape, ts, self.device)

    def to_relation(self, tile_shape) -> SparseTensorRelation:
        tile_shape = tuple(int(t) for t in tile_shape)
        _check_divisible(self.shape, tile_shape)
        if self._kind == "coo":
            idx = as_device_tensor(self._a).to(self.device, non_blocking=True).reshape(-1, len(self.shape))
            val = as_device_tensor(self._b).to(self.device, non_blocking=True)
            if val.dtype not in _TORCH_TO_ES:
                val = val.to(torch.float64)
            # resolved here, so that bad input raises from to_relation as in
            # the reference; the values stay a pending fill
            return tile_coo(idx, val, self.shape, tile_shape, self._out_dtype,
                            duplicates=self.duplicates).materialize_count()
        dense = self._a if torch.is_tensor(self._a) else torch.from_numpy(np.ascontiguousarray(self._a))
        return tile_dense(dense.to(self.device, non_blocking=True), tile_shape, self._out_dtype).materialize_count()
