"""Seeded synthetic inputs for the five benchmark configurations.

The reference publishes no dataset or benchmark inputs for its sparse path;
every input here is synthetic, drawn with ``numpy.random.default_rng(seed)``
so that the CPU checker and the GPU path see the same numbers.

Each generator takes a ``scale`` knob that shrinks the problem while keeping
its distributions (tile size, density, skew), so the same code produces the
full-size benchmark inputs and the small parity-test cases.

Configurations (kernel strings and key lists as the reference's
``execute_sparse`` takes them, ``execution/sparse_dispatch.py:226-234``):

* C1  block-sparse ``ij,jk->ik``: 4096^2 fp32, 128^2 tiles, 10% of tile
  positions (``rng.choice``), N(0,1) values, tile-COO given directly.
* C2  element-sparse SpMM ``ij,jk->ik``: A 65536^2 COO with 4,294,967 unique
  coordinates, rows Zipf(s=1.1) through a seeded permutation, columns uniform,
  N(0,1); B dense 65536x256 N(0,1); tile 32.
* C3  batched ``bij,bjk->bik``: b=16, 8192^2 per batch, bf16, tiles (1,64,64),
  band of 8 elements (tile offsets -1,0,+1) then uniform fill to 5% (819
  tiles per batch), values N(0,0.02).
* C4  chain ``ij,jk,kl->il``: 16384^2 operands, 128^2 tiles at 2%/5%/2%.
* C5  order-3 ``ijk,kl->ijl``: X 4096^3 COO with 50M unique coordinates,
  each index Zipf(s=1.2); W dense 4096x128; tiles 16^3 / 16x16.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass
class TileCOO:
    """Tile-COO operand on the host: coords int32 (T, ndim), values (T, *tile)."""

    coords: np.ndarray
    values: np.ndarray
    shape: tuple
    tile_shape: tuple


@dataclass
class ElementCOO:
    """Element COO operand on the host: indices int32 (nnz, ndim), values (nnz,)."""

    indices: np.ndarray
    values: np.ndarray
    shape: tuple


@dataclass
class Workload:
    """One binary sparse contraction, in the argument order of ``execute_sparse``."""

    name: str
    lhs: object
    rhs: object
    join_keys: list
    kernel_string: str
    agg_keys: list
    lhs_tile: tuple
    rhs_tile: tuple
    dtype: str = "f32"
    extra: dict = field(default_factory=dict)


def _bounded_zipf_cdf(n: int, s: float) -> np.ndarray:
    w = np.arange(1, n + 1, dtype=np.float64) ** (-s)
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    return cdf


def _unique_in_draw_order(draw, target: int, max_rounds: int = 64) -> np.ndarray:
    """Keep drawing int64 keys until ``target`` distinct ones are seen.

    Returns the first ``target`` distinct keys in draw order. ``draw(n)``
    returns ``n`` fresh keys.
    """
    keys = np.zeros(0, dtype=np.int64)
    for _ in range(max_rounds):
        need = target - keys.size
        if need <= 0:
            break
        batch = draw(max(2 * need, 1024))
        allk = np.concatenate([keys, batch])
        _, first = np.unique(allk, return_index=True)
        first.sort()
        keys = allk[first]
    if keys.size < target:
        raise RuntimeError("could not draw enough distinct coordinates")
    return keys[:target]


def c1_block_sparse(seed: int = 0, scale: int = 1) -> Workload:
    """C1: 4096^2 x 4096^2 block-sparse matmul, 128^2 tiles, 10% tiles."""
    rng = np.random.default_rng(seed)
    n = 4096 // scale
    t = 128 if scale == 1 else max(8, 128 // scale)
    g = n // t
    ntile = int(round(0.1 * g * g))
    ops = []
    for _ in range(2):
        pos = np.sort(rng.choice(g * g, ntile, replace=False))
        coords = np.stack([pos // g, pos % g], axis=1).astype(np.int32)
        vals = rng.standard_normal((ntile, t, t)).astype(np.float32)
        ops.append(TileCOO(coords, vals, (n, n), (t, t)))
    return Workload("C1", ops[0], ops[1], [(1, 0)], "ij,jk->ik",
                    [(0, 0), (1, 1)], (t, t), (t, t))


def c2_spmm(seed: int = 0, scale: int = 1, n_cols: int = 256) -> Workload:
    """C2: A 65536^2 element COO (Zipf rows) times dense B, tile 32.

    ``scale`` divides the matrix side and the nnz target (density kept at
    0.1%/scale). B stays ``n_cols`` wide.
    """
    rng = np.random.default_rng(seed)
    n = 65536 // scale
    target = int(round(4294967 / (scale * scale)))
    perm = rng.permutation(n)
    cdf = _bounded_zipf_cdf(n, 1.1)

    def draw(k):
        ranks = np.searchsorted(cdf, rng.random(k), side="right")
        ranks = np.minimum(ranks, n - 1)
        rows = perm[ranks].astype(np.int64)
        cols = rng.integers(0, n, k, dtype=np.int64)
        return rows * n + cols

    keys = _unique_in_draw_order(draw, target)
    idx = np.stack([keys // n, keys % n], axis=1).astype(np.int32)
    vals = rng.standard_normal(target).astype(np.float32)
    b = rng.standard_normal((n, n_cols)).astype(np.float32)
    t = 32
    return Workload("C2", ElementCOO(idx, vals, (n, n)), b, [(1, 0)],
                    "ij,jk->ik", [(0, 0), (1, 1)], (t, t), (t, t))


def c3_batched_bf16(seed: int = 0, scale: int = 1, batch: int = 16) -> Workload:
    """C3: batched block-sparse ``bij,bjk->bik`` in bf16, tiles (1,64,64).

    Band 8 elements wide (touches tile offsets -1, 0, +1), then a uniform
    random fill of distinct tiles up to 5% of tile positions per batch.
    Values N(0, 0.02) rounded to bf16 (kept as float32 holding bf16 values).
    """
    rng = np.random.default_rng(seed)
    n = 8192 // scale
    t = 64
    g = n // t
    per_batch = int(round(0.05 * g * g))
    ops = []
    for _ in range(2):
        all_coords = []
        for b in range(batch):
            band = set()
            for i in range(g):
                for d in (-1, 0, 1):
                    j = i + d
                    if 0 <= j < g:
                        band.add(i * g + j)
            chosen = np.array(sorted(band), dtype=np.int64)
            if chosen.size > per_batch:
                chosen = np.sort(rng.choice(chosen, per_batch, replace=False))
            rest = np.setdiff1d(np.arange(g * g, dtype=np.int64), chosen)
            fill = rng.choice(rest, per_batch - chosen.size, replace=False)
            pos = np.sort(np.concatenate([chosen, fill]))
            c = np.stack([np.full(pos.size, b), pos // g, pos % g], axis=1)
            all_coords.append(c)
        coords = np.concatenate(all_coords).astype(np.int32)
        vals = (rng.standard_normal((coords.shape[0], 1, t, t)) * 0.02).astype(np.float32)
        vals = round_to_bf16(vals)
        ops.append(TileCOO(coords, vals, (batch, n, n), (1, t, t)))
    return Workload("C3", ops[0], ops[1], [(0, 0), (2, 1)], "bij,bjk->bik",
                    [(0, 0), (0, 1), (1, 2)], (1, t, t), (1, t, t), dtype="bf16")


def c4_chain(seed: int = 0, scale: int = 1) -> dict:
    """C4: three 16384^2 block-sparse operands (128^2 tiles, 2%/5%/2%).

    Returns a dict with the three tile-COO operands. The contraction order is
    fixed to (A B) C.
    """
    rng = np.random.default_rng(seed)
    n = 16384 // scale
    t = 128 if scale == 1 else max(8, 128 // scale)
    g = n // t
    ops = []
    for dens in (0.02, 0.05, 0.02):
        k = max(1, int(round(dens * g * g)))
        pos = np.sort(rng.choice(g * g, k, replace=False))
        coords = np.stack([pos // g, pos % g], axis=1).astype(np.int32)
        vals = rng.standard_normal((k, t, t)).astype(np.float32)
        ops.append(TileCOO(coords, vals, (n, n), (t, t)))
    return {"A": ops[0], "B": ops[1], "C": ops[2], "tile": (t, t)}


def c5_order3(seed: int = 0, scale: int = 1, n_out: int = 128) -> Workload:
    """C5: X 4096^3 element COO (Zipf s=1.2 per mode) times dense W, tiles 16.

    ``scale`` divides the side and divides the nnz target by scale^3.
    """
    rng = np.random.default_rng(seed)
    n = 4096 // scale
    target = int(round(50_000_000 / scale ** 3))
    cdf = _bounded_zipf_cdf(n, 1.2)

    def draw(k):
        parts = []
        for _ in range(3):
            r = np.searchsorted(cdf, rng.random(k), side="right")
            parts.append(np.minimum(r, n - 1).astype(np.int64))
        return (parts[0] * n + parts[1]) * n + parts[2]

    keys = _unique_in_draw_order(draw, target)
    i = keys // (n * n)
    j = (keys // n) % n
    k = keys % n
    idx = np.stack([i, j, k], axis=1).astype(np.int32)
    vals = rng.standard_normal(target).astype(np.float32)
    w = rng.standard_normal((n, n_out)).astype(np.float32)
    return Workload("C5", ElementCOO(idx, vals, (n, n, n)), w, [(2, 0)],
                    "ijk,kl->ijl", [(0, 0), (0, 1), (1, 1)], (16, 16, 16), (16, 16))


def c5_order3_device(seed: int = 0, scale: int = 1, n_out: int = 128, device=None) -> Workload:
    """C5 drawn on the GPU: the same distributions as ``c5_order3`` (each index
    bounded-Zipf(s=1.2) by inverse-CDF sampling, the first ``target`` distinct
    coordinates in draw order, N(0,1) values, dense N(0,1) W), with torch's
    seeded CUDA generator instead of numpy's, so the 50M-entry tensor takes
    seconds instead of many minutes. The arrays stay on ``device``
    (``lhs.indices`` int32 (nnz, 3), ``lhs.values`` float32, ``rhs`` float32);
    the same seed on the same GPU model and torch build gives the same draw,
    and checkers read the arrays back instead of redrawing them."""
    import torch
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev)
    g.manual_seed(int(seed))
    n = 4096 // scale
    target = int(round(50_000_000 / scale ** 3))
    cdf = torch.from_numpy(_bounded_zipf_cdf(n, 1.2)).to(dev)
    keys = torch.zeros(0, dtype=torch.int64, device=dev)
    for _ in range(256):
        need = target - int(keys.numel())
        if need <= 0:
            break
        k = max(4 * need, 1 << 22)
        parts = []
        for _ in range(3):
            r = torch.searchsorted(cdf, torch.rand(k, generator=g, device=dev, dtype=torch.float64), right=True)
            parts.append(r.clamp_(max=n - 1))
        batch = (parts[0] * n + parts[1]) * n + parts[2]
        allk = torch.cat([keys, batch])
        uk, inv = torch.unique(allk, return_inverse=True)
        first = torch.full((uk.numel(),), allk.numel(), dtype=torch.int64, device=dev)
        first.scatter_reduce_(0, inv, torch.arange(allk.numel(), device=dev), reduce="amin")
        keys = allk[torch.sort(first).values]
        del allk, uk, inv, first, batch, parts
    if keys.numel() < target:
        raise RuntimeError("could not draw enough distinct coordinates")
    keys = keys[:target]
    idx = torch.stack([keys // (n * n), (keys // n) % n, keys % n], dim=1).to(torch.int32)
    del keys
    vals = torch.randn(target, generator=g, device=dev, dtype=torch.float32)
    w = torch.randn((n, n_out), generator=g, device=dev, dtype=torch.float32)
    return Workload("C5", ElementCOO(idx, vals, (n, n, n)), w, [(2, 0)],
                    "ijk,kl->ijl", [(0, 0), (0, 1), (1, 1)], (16, 16, 16), (16, 16))


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even), kept as float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    return r.astype(np.uint32).view(np.float32).reshape(x.shape)
