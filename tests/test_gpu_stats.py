"""Per-tiling-scheme sparsity statistics on the GPU (``es_sparsity_stats``)
against the reference's own values (golden vectors from ``tensor/stats.py``
and ``SparseTensor``'s metrics) and against the oracle on larger inputs.
Counts are integers: every comparison is exact."""

import numpy as np
import pytest
import torch

import einjax_b200 as E
import oracle as O
from golden_io import cases_of_kind, load_cases

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(cases_of_kind("stats", "golden_stats.npz")))
def test_sparsity_stats_golden(name):
    c = load_cases("golden_stats.npz")[name]
    shape = tuple(int(v) for v in c["shape"])
    ts = [tuple(int(v) for v in t) for t in c["tile_shapes"]]
    assert ts == E.factor_tile_shapes(shape)
    if "dense" in c:
        got = E.SparseTensor("t", c["dense"]).sparsity_stats()
        got2 = E.compute_sparsity_stats_dense(torch.from_numpy(c["dense"]).cuda(), ts)
        assert got == got2
    else:
        got = E.SparseTensor("t", (c["indices"], c["values"], shape)).sparsity_stats()
    np.testing.assert_array_equal([got[t][0] for t in ts], c["num_tuples"])
    np.testing.assert_array_equal([got[t][1] for t in ts], c["value_count"])


def _random_coo(rng, shape, nnz):
    idx = np.stack([rng.integers(0, n, nnz) for n in shape], 1).astype(np.int32)
    idx[rng.choice(nnz, nnz // 8, replace=False)] = idx[rng.choice(nnz, nnz // 8)]
    val = rng.standard_normal(nnz)
    val[rng.random(nnz) < 0.05] = 0.0
    return idx, val


@pytest.mark.parametrize("shape,nnz", [((4096, 2048), 200_000), ((96, 128, 60), 50_000), ((10_000,), 3_000)])
def test_sparsity_stats_all_schemes_vs_oracle(shape, nnz):
    rng = np.random.default_rng(len(shape))
    idx, val = _random_coo(rng, shape, nnz)
    ts = E.factor_tile_shapes(shape)
    got = E.compute_sparsity_stats_coo(idx, val, shape, ts)
    ref = O.compute_sparsity_stats_coo(idx, val, shape, ts)
    assert got == ref


def test_sparsity_stats_sort_path_and_values_dtypes():
    """Tile grids too large for a bitmap (2^40 tiles) take the sort path;
    bf16 / fp32 values and no values at all."""
    rng = np.random.default_rng(9)
    shape = (1 << 20, 1 << 20)
    idx, val = _random_coo(rng, shape, 100_000)
    ts = [(1, 1), (2, 1), (1, 1 << 10), (1 << 10, 1 << 10), (3, 7)]
    ref = O.compute_sparsity_stats_coo(idx, val, shape, ts)
    assert E.compute_sparsity_stats_coo(idx, val, shape, ts) == ref
    v32 = torch.from_numpy(val.astype(np.float32))
    assert E.compute_sparsity_stats_coo(idx, v32, shape, ts) == ref
    vbf = torch.from_numpy(val).to(torch.bfloat16)  # N(0,1) values stay non-zero in bf16
    assert E.compute_sparsity_stats_coo(idx, vbf, shape, ts) == ref
    ones = np.ones(len(val))
    assert E.compute_sparsity_stats_coo(idx, None, shape, ts) == O.compute_sparsity_stats_coo(idx, ones, shape, ts)


def test_sparsity_stats_dense_3d_and_errors():
    rng = np.random.default_rng(4)
    d = rng.standard_normal((24, 18, 10)) * (rng.random((24, 18, 10)) < 0.07)
    ts = E.factor_tile_shapes(d.shape)
    nz = np.nonzero(d)
    ref = O.compute_sparsity_stats_coo(np.stack(nz, 1), d[nz], d.shape, ts)
    assert E.compute_sparsity_stats_dense(torch.from_numpy(d).cuda(), ts) == ref
    assert E.compute_sparsity_stats_dense(np.zeros((6, 4)), [(2, 2)]) == {(2, 2): (0, (0, 0))}
    with pytest.raises(ValueError):
        E.compute_sparsity_stats_coo(np.array([[0, 9]], np.int32), np.ones(1), (4, 4), [(2, 2)])
