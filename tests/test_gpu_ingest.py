"""GPU parity of COO ingestion (``coalesce_coo``, ``tile_coo(duplicates=...)``,
``SparseTensor`` over torch sparse / DLPack / pydata-style COO inputs) against
the reference's tiling of repeated coordinates (golden vectors:
``SparseTensor.to_relation`` of a COO matrix, where the last repeat wins, and
of scipy's CSR of it, where repeats are added) and against the oracle.

Coordinates and counts are compared exactly; coalesced float64 values exactly
against the oracle (both add in input order); float32 tiles to 1e-6 relative
against the reference's float64 tiles.
"""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

import einjax_b200 as E
import oracle as O
from golden_io import cases_of_kind, load_cases

pytestmark = pytest.mark.gpu

INGEST = load_cases("golden_ingest.npz")


def _tiles_close(rel, coords, values):
    c, v = rel.to_numpy()
    np.testing.assert_array_equal(c, coords)
    np.testing.assert_allclose(v, values, rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("name", sorted(cases_of_kind("ingest", "golden_ingest.npz")))
def test_duplicate_policies_golden(name):
    c = INGEST[name]
    shape, tile = tuple(c.meta["shape"]), tuple(c.meta["tile"])
    last = E.SparseTensor("t", (c["indices"], c["values"], shape)).to_relation(tile)
    _tiles_close(last, c["last_coords"], c["last_values"])
    summed = E.SparseTensor("t", (c["indices"], c["values"], shape), duplicates="sum").to_relation(tile)
    _tiles_close(summed, c["sum_coords"], c["sum_values"])
    with pytest.raises(ValueError, match="repeated"):
        E.SparseTensor("t", (c["indices"], c["values"], shape), duplicates="error").to_relation(tile)
    idx = torch.from_numpy(c["indices"]).cuda()
    val = torch.from_numpy(c["values"]).cuda()
    for pol in ("sum", "last"):
        gi, gv, nz = E.coalesce_coo(idx, val, shape, pol)
        ri, rv, rnz = O.coalesce_coo(c["indices"], c["values"], shape, pol)
        assert nz == rnz
        np.testing.assert_array_equal(gi.cpu().numpy(), ri)
        np.testing.assert_array_equal(gv.cpu().numpy(), rv)


def _dup_coo(rng, shape, nnz, frac_rep=0.3):
    idx = np.stack([rng.integers(0, n, nnz) for n in shape], 1).astype(np.int32)
    rep = rng.choice(nnz, int(nnz * frac_rep), replace=False)
    idx[rep] = idx[rng.choice(nnz, len(rep))]
    val = rng.standard_normal(nnz)
    val[rng.random(nnz) < 0.05] = 0.0
    return idx, val


@pytest.mark.parametrize("shape,nnz,tile", [((4096, 4096), 1_000_000, (32, 32)), ((64, 96, 80), 300_000, (8, 16, 16)),
                                            ((50_000,), 200_000, (100,)), ((6, 10, 12, 8), 20_000, (3, 5, 4, 8))])
@pytest.mark.parametrize("vdtype", [torch.float64, torch.float32, torch.bfloat16])
def test_coalesce_vs_oracle(shape, nnz, tile, vdtype):
    rng = np.random.default_rng(nnz % 97)
    idx, val = _dup_coo(rng, shape, nnz)
    tv = torch.from_numpy(val).to(vdtype)
    v_in = tv.double().numpy()  # the values as the GPU sees them
    for pol in ("sum", "last"):
        gi, gv, nz = E.coalesce_coo(torch.from_numpy(idx).cuda(), tv.cuda(), shape, pol)
        ri, rv, rnz = O.coalesce_coo(idx, v_in, shape, pol)
        assert nz == rnz and gi.shape[0] == len(rv)
        np.testing.assert_array_equal(gi.cpu().numpy(), ri)
        np.testing.assert_array_equal(gv.cpu().numpy(), rv)
    rel = E.tile_coo(torch.from_numpy(idx).cuda(), tv.cuda(), shape, tile, duplicates="sum")
    si, sv, _ = O.coalesce_coo(idx, v_in, shape, "sum")
    ref = O.to_relation(si, sv, shape, tile)
    c, v = rel.to_numpy()
    np.testing.assert_array_equal(c, ref.coords)
    np.testing.assert_array_equal(v, ref.values.astype(np.float32))


def test_coalesce_edges():
    e = torch.zeros((0, 2), dtype=torch.int32, device="cuda")
    gi, gv, nz = E.coalesce_coo(e, torch.zeros(0, device="cuda"), (4, 4))
    assert gi.shape == (0, 2) and nz == 0
    gi, gv, nz = E.coalesce_coo(torch.tensor([[1, 1], [2, 2]], device="cuda"), torch.zeros(2, device="cuda"), (4, 4))
    assert gi.shape[0] == 0 and nz == 0
    one = torch.tensor([[3, 3]] * 5000, dtype=torch.int32, device="cuda")
    gi, gv, nz = E.coalesce_coo(one, torch.full((5000,), 0.5, dtype=torch.float64, device="cuda"), (4, 4))
    assert gi.tolist() == [[3, 3]] and gv.item() == 2500.0 and nz == 5000
    with pytest.raises(ValueError):
        E.coalesce_coo(torch.tensor([[0, 4]], device="cuda"), torch.ones(1, device="cuda"), (4, 4))
    with pytest.raises(ValueError):
        E.tile_coo(one, torch.ones(5000, device="cuda"), (4, 4), (2, 2), duplicates="bogus")
    with pytest.raises(ValueError, match="repeated"):
        E.tile_coo(one, torch.ones(5000, device="cuda"), (4, 4), (2, 2), duplicates="error")


def test_torch_sparse_input_sums_repeats():
    rng = np.random.default_rng(2)
    idx, val = _dup_coo(rng, (96, 128), 5000)
    ts = torch.sparse_coo_tensor(torch.from_numpy(idx.T.astype(np.int64)), torch.from_numpy(val), (96, 128))
    assert not ts.is_coalesced()
    st = E.SparseTensor("t", ts)
    assert st.duplicates == "sum"
    rel = st.to_relation((16, 32))
    si, sv, _ = O.coalesce_coo(idx, val, (96, 128), "sum")
    ref = O.to_relation(si, sv, (96, 128), (16, 32))
    c, v = rel.to_numpy()
    np.testing.assert_array_equal(c, ref.coords)
    np.testing.assert_array_equal(v, ref.values.astype(np.float32))
    np.testing.assert_allclose(rel.to_dense().cpu().numpy(), ts.to_dense().numpy(), rtol=1e-6, atol=1e-6)
    csr = ts.coalesce().to_sparse_csr().cuda()
    np.testing.assert_array_equal(E.SparseTensor("t", csr).to_relation((16, 32)).to_numpy()[0], ref.coords)


class _DLPackOnly:
    """Exposes a tensor only through the DLPack protocol (as a JAX or CuPy array does)."""

    def __init__(self, t):
        self._t = t

    def __dlpack__(self, **kw):
        return self._t.__dlpack__(**kw)

    def __dlpack_device__(self):
        return self._t.__dlpack_device__()


def test_dlpack_and_pydata_inputs():
    rng = np.random.default_rng(8)
    idx, val = _dup_coo(rng, (32, 40, 24), 20_000)
    ti = torch.from_numpy(idx).cuda()
    tv = torch.from_numpy(val).cuda()
    assert E.as_device_tensor(_DLPackOnly(tv)).data_ptr() == tv.data_ptr()  # zero-copy
    ref = O.to_relation(idx, val, (32, 40, 24), (8, 8, 8))
    rel = E.SparseTensor("t", (_DLPackOnly(ti), _DLPackOnly(tv), (32, 40, 24))).to_relation((8, 8, 8))
    c, v = rel.to_numpy()
    np.testing.assert_array_equal(c, ref.coords)
    np.testing.assert_array_equal(v, ref.values.astype(np.float32))
    pyd = SimpleNamespace(coords=idx.T.copy(), data=val, shape=(32, 40, 24))
    c2, v2 = E.SparseTensor("t", pyd).to_relation((8, 8, 8)).to_numpy()
    np.testing.assert_array_equal(c2, ref.coords)
    np.testing.assert_array_equal(v2, v)
    dense = torch.from_numpy(ref.to_dense()).cuda()
    c3, v3 = E.SparseTensor("t", _DLPackOnly(dense)).to_relation((8, 8, 8)).to_numpy()
    np.testing.assert_array_equal(c3, ref.coords)
    np.testing.assert_array_equal(v3, v)


@pytest.mark.parametrize("n", [1, 2, 31, 4095, 4096, 4097, 3 * 4096 + 5, 70_001])
@pytest.mark.parametrize("shape", [(7, 3), (1 << 20, 1 << 20, 1 << 20), (3, 1 << 30, 5), (1 << 16, 1 << 16)])
def test_coalesce_sort_sizes_and_key_widths(n, shape):
    """The radix sort under coalescing at tile-boundary sizes (4096 keys per
    tile) and key widths from 5 to 61 bits (1 to 8 passes), heavy repeats."""
    rng = np.random.default_rng(n + len(shape))
    idx = np.stack([rng.integers(0, s, n) for s in shape], 1).astype(np.int32)
    rep = rng.choice(n, n // 2, replace=False) if n > 1 else np.zeros(0, np.int64)
    idx[rep] = idx[rng.choice(n, len(rep))]
    val = rng.standard_normal(n)
    for pol in ("sum", "last"):
        gi, gv, nz = E.coalesce_coo(torch.from_numpy(idx).cuda(), torch.from_numpy(val).cuda(), shape, pol)
        ri, rv, rnz = O.coalesce_coo(idx, val, shape, pol)
        assert nz == rnz
        np.testing.assert_array_equal(gi.cpu().numpy(), ri)
        np.testing.assert_array_equal(gv.cpu().numpy(), rv)
