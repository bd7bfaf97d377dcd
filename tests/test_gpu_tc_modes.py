"""Tensor-core tile GEMM launch modes, through the public tile einsum.

* Fused key blocks: when the rhs operand is split into key blocks, one
  launch takes every (key block, item) unit and a last pass adds the blocks'
  partial sums in block order; it must give the same bits as one launch per
  block (``EINSPARSE_NO_FUSED_BLOCKS``), with output rows scattered through
  ``seg_out_index`` too.
* Accumulation chains (fp32): the tensor core truncates when it adds into its
  accumulator, so a long contraction is summed in chains of at most a few
  hundred products per accumulator, the chains added in fp32 with rounding to
  nearest. A long dense strip must then be as close to float64 as a plain
  fp32 computation, and clearly closer than without chains
  (``EINSPARSE_CHAIN_KSTEPS=0``).
* bf16 with a sparse rhs whose panel slots are sometimes one consecutive copy
  and sometimes zero-filled in shared memory (a stage's slots must be zeroed
  again after a consecutive copy overwrote them).
"""

import numpy as np
import pytest
import torch

import einjax_b200 as E
import oracle as O
from einjax_b200 import sparse_dispatch as SD

pytestmark = pytest.mark.gpu

MM = ([(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])


def _c2_like(seed, n=8192, m=256, nnz=160_000, dense_rows=()):
    rng = np.random.default_rng(seed)
    rows = rng.permutation(n)[np.minimum(rng.zipf(1.1, nnz) - 1, n - 1)]
    cols = rng.integers(0, n, nnz)
    key = np.unique(rows.astype(np.int64) * n + cols)
    idx = np.stack([key // n, key % n], 1).astype(np.int32)
    for r in dense_rows:
        extra = np.stack([np.full(n, r), np.arange(n)], 1).astype(np.int32)
        idx = np.unique(np.concatenate([idx, extra]), axis=0)
    val = rng.standard_normal(len(idx)).astype(np.float32)
    b = rng.standard_normal((n, m)).astype(np.float32)
    return idx, val, b


def _run(idx, val, b, n):
    A = E.tile_coo(torch.from_numpy(idx).cuda(), torch.from_numpy(val).cuda(), (n, n), (32, 32))
    B = E.tile_dense(torch.from_numpy(b).cuda(), (32, 32))
    return A, B, SD.plan_pairs(A, B, MM[0], MM[2])


def _einsum(A, B, plan, seg_out=None, rows=None):
    out = None
    if seg_out is not None:
        out = torch.zeros((rows, 32, 32), dtype=torch.float32, device="cuda")
    return SD.tile_einsum(MM[1], A.values, B.values, plan.seg_lhs, plan.seg_rhs, plan.seg_offsets,
                          seg_out_index=seg_out, out=out, precision="tc", seg_strip=plan.seg_strip,
                          pair_key=plan.seg_key, key_extent=plan.key_extent)


@pytest.mark.parametrize("chains", ["0", "64"])
def test_fused_key_blocks_match_sequential_launches(monkeypatch, chains):
    n = 8192
    idx, val, b = _c2_like(3, n)
    A, B, plan = _run(idx, val, b, n)
    monkeypatch.setenv("EINSPARSE_KBLOCK_BYTES", str(1 << 20))  # 16 key blocks
    monkeypatch.setenv("EINSPARSE_CHAIN_KSTEPS", chains)
    fused = _einsum(A, B, plan)
    O_ = plan.num_segments
    perm = torch.randperm(O_ + 7, generator=torch.Generator().manual_seed(1))[:O_].to(torch.int32).cuda()
    fused_sc = _einsum(A, B, plan, perm, O_ + 7)
    monkeypatch.setenv("EINSPARSE_NO_FUSED_BLOCKS", "1")
    seq = _einsum(A, B, plan)
    seq_sc = _einsum(A, B, plan, perm, O_ + 7)
    torch.cuda.synchronize()
    if chains == "0":
        # same summation order: ((block 0 + block 1) + block 2) + ...
        assert torch.equal(fused.view(torch.int32), seq.view(torch.int32))
        assert torch.equal(fused_sc.view(torch.int32), seq_sc.view(torch.int32))
    else:
        # chains inside a block are added into the block's partial first
        tol = 1e-5 * (seq.abs() + 1.0)
        assert bool(((fused - seq).abs() <= tol).all())
        assert bool(((fused_sc - seq_sc).abs() <= 1e-5 * (seq_sc.abs() + 1.0)).all())
    assert torch.equal(fused_sc[perm.long()].view(torch.int32), fused.view(torch.int32))
    untouched = torch.ones(O_ + 7, dtype=torch.bool, device="cuda")
    untouched[perm.long()] = False
    assert bool((fused_sc[untouched] == 0).all())


def _f64_err(got, idx, val, b, n):
    import scipy.sparse as sp
    a = sp.csr_matrix((val.astype(np.float64), (idx[:, 0], idx[:, 1])), shape=(n, n))
    ref = a @ b.astype(np.float64)
    a32 = sp.csr_matrix((val, (idx[:, 0], idx[:, 1])), shape=(n, n))
    f32 = a32 @ b  # float32 accumulation in row order
    return ref, np.abs(got - ref), np.abs(f32.astype(np.float64) - ref)


def _dense(res, n, m):
    coords, vals = res
    g = np.zeros((n, m))
    g.reshape(n // 32, 32, m // 32, 32)[coords[:, 0], :, coords[:, 1], :] = vals
    return g


def test_chains_keep_long_contractions_at_fp32_accuracy(monkeypatch):
    n, m = 16384, 256
    idx, val, b = _c2_like(4, n, m, nnz=60_000, dense_rows=(5, 77, 4000))
    A, B, plan = _run(idx, val, b, n)
    oc = plan.out_coords.cpu().numpy()
    errs = {}
    for ch in ("64", "0"):
        monkeypatch.setenv("EINSPARSE_CHAIN_KSTEPS", ch)
        got = _dense((oc, _einsum(A, B, plan).cpu().numpy()), n, m)
        ref, err, err32 = _f64_err(got, idx, val, b, n)
        errs[ch] = err
    dense = np.array([5, 77, 4000])
    # the dense rows sum 16384 products per element: chained accumulation
    # stays within twice a plain fp32 sum's error, the unchained one does not
    e_ch, e_no, e32 = errs["64"][dense], errs["0"][dense], err32[dense]
    assert e_ch.max() <= 2 * e32.max() + 1e-6, (e_ch.max(), e32.max())
    assert np.sqrt((e_ch ** 2).mean()) <= 3 * np.sqrt((e32 ** 2).mean())
    assert e_no.max() > e_ch.max()


@pytest.mark.parametrize("dens", [(0.3, 0.5), (0.5, 0.8)])
def test_bf16_sparse_rhs_panel_slots(dens):
    rng = np.random.default_rng(11)

    def rel(shape, tile, d):
        g = [s // t for s, t in zip(shape, tile)]
        n = int(np.prod(g))
        pos = np.sort(rng.choice(n, max(1, int(round(d * n))), replace=False))
        coords = np.stack(np.unravel_index(pos, g), 1).astype(np.int32)
        from einjax_b200 import workloads as W
        vals = W.round_to_bf16(rng.standard_normal((len(pos), *tile)).astype(np.float32)).astype(np.float64)
        return O.Relation(coords, vals, shape, tile)
    lhs = rel((2, 1024, 1024), (1, 64, 64), dens[0])
    rhs = rel((2, 1024, 1024), (1, 64, 64), dens[1])
    jk, ks, ak = [(0, 0), (2, 1)], "bij,bjk->bik", [(0, 0), (0, 1), (1, 2)]
    dl = E.SparseTensorRelation.from_arrays(lhs.coords, lhs.values, lhs.shape, lhs.tile_shape, dtype=torch.bfloat16)
    dr = E.SparseTensorRelation.from_arrays(rhs.coords, rhs.values, rhs.shape, rhs.tile_shape, dtype=torch.bfloat16)
    res = E.execute_sparse(dl, dr, jk, ks, ak, precision="tc")
    ref = O.execute_sparse(lhs, rhs, jk, ks, ak)
    mag = O.execute_sparse(O.Relation(lhs.coords, np.abs(lhs.values), lhs.shape, lhs.tile_shape),
                           O.Relation(rhs.coords, np.abs(rhs.values), rhs.shape, rhs.tile_shape), jk, ks, ak)
    c, v = res.to_numpy()
    np.testing.assert_array_equal(c, ref.coords)
    assert np.all(np.abs(v.astype(np.float64) - ref.values) <= 2e-2 * (np.abs(ref.values) + mag.values))


def test_deferred_device_error_reported_later():
    """A device-side error of a call made with check="defer" (here a pair
    index past the lhs rows, which the kernel reports and reads as a zero
    tile) is raised by the next count read or by check_device_errors, not
    by the call itself."""
    n = 2048
    idx, val, b = _c2_like(7, n, nnz=8000)
    A, B, plan = _run(idx, val, b, n)
    bad = plan.seg_lhs.clone()
    bad[0] = A.num_tuples + 5
    out = SD.tile_einsum(MM[1], A.values, B.values, bad, plan.seg_rhs, plan.seg_offsets, precision="tc",
                         seg_strip=plan.seg_strip, pair_key=plan.seg_key, key_extent=plan.key_extent,
                         check="defer")
    assert out.shape[0] == plan.num_segments
    with pytest.raises(ValueError):
        E.check_device_errors()
    E.check_device_errors()  # reported once
    # a good call afterwards is unaffected
    SD.tile_einsum(MM[1], A.values, B.values, plan.seg_lhs, plan.seg_rhs, plan.seg_offsets, precision="tc",
                   seg_strip=plan.seg_strip, pair_key=plan.seg_key, key_extent=plan.key_extent, check="defer")
    E.check_device_errors()
