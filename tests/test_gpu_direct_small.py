"""The one-CTA direct join + grouping plan (small inputs) against the
multi-launch plan on the same relations: pair lists, segment offsets, output
coordinates and strips bit-identical, and both against the oracle's join."""

import numpy as np
import pytest
import torch

import einjax_b200 as E
import oracle as O
from einjax_b200 import sparse_dispatch as SD

pytestmark = pytest.mark.gpu


def _rel(seed, shape, tile, density):
    g = np.random.default_rng(seed)
    grid = [s // t for s, t in zip(shape, tile)]
    n = int(np.prod(grid))
    pick = np.sort(g.choice(n, max(1, int(n * density)), replace=False))
    coords = np.stack(np.unravel_index(pick, grid), 1).astype(np.int32)
    vals = g.standard_normal((len(pick), *tile)).astype(np.float32)
    return coords, vals


def _plan(lc, rc, join, agg):
    torch.cuda.synchronize()
    return SD.plan_pairs(lc, rc, join, agg)


@pytest.mark.parametrize("case", [
    # (lhs shape, rhs shape, tile lhs, tile rhs, densities, join keys, output keys (operand, dim))
    ((512, 1024), (1024, 256), (32, 32), (32, 32), (0.3, 0.5), [(1, 0)], [(0, 0), (1, 1)]),
    ((2048, 2048), (2048, 512), (32, 32), (32, 32), (0.05, 0.9), [(1, 0)], [(0, 0), (1, 1)]),
    ((4, 256, 256), (4, 256, 128), (1, 32, 32), (1, 32, 32), (0.4, 0.6), [(0, 0), (2, 1)], [(0, 0), (0, 1), (1, 2)]),
    ((16, 16, 4096), (4096, 64), (4, 4, 32), (32, 32), (0.1, 0.7), [(2, 0)], [(0, 0), (0, 1), (1, 1)]),
])
def test_small_plan_matches_multi_launch_plan(case, monkeypatch):
    ls, rs, lt, rt, (dl, dr), join, agg = case
    lc, lv = _rel(1, ls, lt, dl)
    rc, rv = _rel(2, rs, rt, dr)
    A = E.SparseTensorRelation.from_arrays(lc, lv, ls, lt)
    B = E.SparseTensorRelation.from_arrays(rc, rv, rs, rt)
    assert A.num_tuples + B.num_tuples <= 8192
    small = _plan(A, B, join, agg)
    monkeypatch.setenv("EINSPARSE_NO_SMALL_PLAN", "1")
    multi = _plan(A, B, join, agg)
    for name in ("lhs_idx", "rhs_idx", "out_coords", "seg_offsets", "seg_lhs", "seg_rhs"):
        assert torch.equal(getattr(small, name), getattr(multi, name)), name
    for name in ("seg_strip", "seg_key"):
        a, b = getattr(small, name), getattr(multi, name)
        assert (a is None) == (b is None)
        if a is not None:
            assert torch.equal(a, b), name
    # the pair set against the oracle's join (canonical order)
    li, ri = O.coordinate_join(lc, rc, join)
    got = sorted(zip(small.lhs_idx.cpu().tolist(), small.rhs_idx.cpu().tolist()))
    assert got == sorted(zip(np.asarray(li).tolist(), np.asarray(ri).tolist()))
