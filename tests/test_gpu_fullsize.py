"""Parity at the benchmark sizes (BASELINE configurations at full size).

The small golden cases pin every function bit for bit; these tests run the
configurations the benchmark times, at their full sizes, and check the
results through what the domain offers at that size:

* C2 (the headline, 1.83M A tiles, 14.6M pairs, the tile GEMM's contracted
  range split into key blocks that fit in L2): tile coordinates and a sample
  of tile values exactly; join pairs bit-exact against the oracle after a
  canonical sort; every output element against scipy's float64 A @ B.
* C3 (bf16, batched): join pairs and output coordinates exactly against the
  oracle, a sample of output tiles against float64 per-tile products.
* C4 (three 16384^2 operands, (A B) C): forward output and the gradients of
  all three operands against the oracle's forward and backward rules.
* C5 (X 4096^3 with 50M entries, drawn on the GPU): a random sample of
  output tile positions against float64 sums over X's entries; linearity
  (the result over all k equals the sum of the results over even and odd k
  tiles); a k slice against the oracle tile for tile.

Values use the fp32 error bound |got - ref| <= rtol * (|ref| + sum |a*b|)
with rtol = 1e-5 (bf16: 2e-2); C2 additionally must be about as close to
float64 as a plain fp32 SpMM of the same inputs (the share of elements
within plain rtol 1e-5, the largest error, the relative Frobenius error).
"""

import numpy as np
import pytest
import torch

import bench
import einjax_b200 as E
import oracle as O
from einjax_b200 import sparse_dispatch as SD
from einjax_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _bound(got, ref, mag, rtol=1e-5):
    return bool(np.all(np.abs(np.asarray(got, np.float64) - ref) <= rtol * (np.abs(ref) + mag)))


@pytest.mark.timeout(900)
def test_c2_full_size():
    w = W.c2_spmm(seed=0)
    n, m = w.lhs.shape[0], w.rhs.shape[1]
    idx = torch.from_numpy(w.lhs.indices).cuda()
    val = torch.from_numpy(w.lhs.values).cuda()
    A = E.tile_coo(idx, val, w.lhs.shape, (32, 32))
    B = E.tile_dense(torch.from_numpy(w.rhs).cuda(), (32, 32))
    # tiling: coordinates exactly, a sample of tiles element for element
    tk = (w.lhs.indices[:, 0].astype(np.int64) // 32) * (n // 32) + w.lhs.indices[:, 1] // 32
    ut = np.unique(tk)
    want = np.stack([ut // (n // 32), ut % (n // 32)], 1).astype(np.int32)
    got_c = A.coords.cpu().numpy()
    np.testing.assert_array_equal(got_c, want)
    pick = np.random.default_rng(0).choice(len(ut), 2000, replace=False)
    sel = np.isin(tk, ut[pick])
    ref_t = np.zeros((len(ut), 32, 32), np.float32)
    pos = np.searchsorted(ut, tk[sel])
    ref_t[pos, w.lhs.indices[sel, 0] % 32, w.lhs.indices[sel, 1] % 32] = w.lhs.values[sel]
    np.testing.assert_array_equal(A.values[torch.from_numpy(pick).cuda()].cpu().numpy(), ref_t[pick])
    # join: pairs bit-exact after a canonical sort
    plan = SD.plan_pairs(A, B, w.join_keys, w.agg_keys)
    li, ri = O.coordinate_join(want, B.coords.cpu().numpy(), w.join_keys)
    assert plan.num_pairs == len(li)
    np.testing.assert_array_equal(O.canonical_pairs(plan.seg_lhs.cpu().numpy(), plan.seg_rhs.cpu().numpy()),
                                  O.canonical_pairs(li, ri))
    del plan
    # the whole product: every element against float64
    res = E.execute_sparse(A, B, w.join_keys, w.kernel_string, w.agg_keys)
    st = bench.c2_parity(w, (0, n), res.coords.cpu().numpy(), res.values.cpu().numpy())
    assert st["elements"] == n * m
    assert st["bound_ok"], st
    # as close to float64 as a plain fp32 SpMM of the same inputs, within the
    # 3-pass TF32 products' own error (~2^-22 per product against fp32's 2^-24)
    assert st["within_rtol"] >= st["fp32_spmm_within_rtol"] - 5e-3, st
    assert st["max_abs_err"] <= 4 * st["fp32_spmm_max_abs_err"], st
    assert st["rel_fro"] < 1e-5, st


@pytest.mark.timeout(900)
def test_c3_full_size_bf16():
    w = W.c3_batched_bf16(seed=0)
    kw = dict(dtype=torch.bfloat16)
    lhs = E.SparseTensorRelation.from_arrays(w.lhs.coords, w.lhs.values, w.lhs.shape, w.lhs.tile_shape, **kw)
    rhs = E.SparseTensorRelation.from_arrays(w.rhs.coords, w.rhs.values, w.rhs.shape, w.rhs.tile_shape, **kw)
    plan = SD.plan_pairs(lhs, rhs, w.join_keys, w.agg_keys)
    li, ri = O.coordinate_join(w.lhs.coords, w.rhs.coords, w.join_keys)
    np.testing.assert_array_equal(O.canonical_pairs(plan.seg_lhs.cpu().numpy(), plan.seg_rhs.cpu().numpy()),
                                  O.canonical_pairs(li, ri))
    oc = O.compute_output_coords(w.lhs.coords, w.rhs.coords, li, ri, w.agg_keys)
    res = E.execute_sparse(lhs, rhs, w.join_keys, w.kernel_string, w.agg_keys)
    c, v = res.to_numpy()
    np.testing.assert_array_equal(c, np.unique(oc, axis=0))
    pick = np.random.default_rng(1).choice(len(c), 1024, replace=False)
    ref, mag = bench.blocksparse_ref(w.lhs.coords, w.lhs.values, w.rhs.coords, w.rhs.values, 1, c[pick])
    assert _bound(v[pick].reshape(ref.shape), ref, mag, 2e-2)


def _agg_grads(lhs, rhs, jk, ks, ak, g_out):
    """Reference backward of one aggregated step: per-pair gradients of the
    output tile's cotangent (autodiff/custom_vjp.py:254-275) scatter-added
    into the operands' tiles."""
    li, ri = O.coordinate_join(lhs.coords, rhs.coords, jk)
    oc = O.compute_output_coords(lhs.coords, rhs.coords, li, ri, ak)
    uc, inv = np.unique(oc, axis=0, return_inverse=True)
    g = g_out[inv.reshape(-1)]
    gl = np.zeros_like(lhs.values)
    gr = np.zeros_like(rhs.values)
    for s in range(0, len(li), 512):  # chunks keep the gathered tiles small
        sl = slice(s, s + 512)
        np.add.at(gl, li[sl], np.matmul(g[sl], np.swapaxes(rhs.values[ri[sl]], 1, 2)))
        np.add.at(gr, ri[sl], np.matmul(np.swapaxes(lhs.values[li[sl]], 1, 2), g[sl]))
    return gl, gr


@pytest.mark.timeout(900)
def test_c4_full_size_forward_and_grads():
    w = W.c4_chain(seed=0)
    rels = {k: O.Relation(w[k].coords, w[k].values.astype(np.float64), w[k].shape, w[k].tile_shape) for k in "ABC"}
    dev = {k: E.SparseTensorRelation.from_arrays(r.coords, r.values, r.shape, r.tile_shape, dtype=torch.float32)
           for k, r in rels.items()}
    for d in dev.values():
        d.values.requires_grad_(True)
    plan = E.plan_from_path("ij,jk,kl->il", [(0, 1), (0, 1)])
    D = E.execute_sparse_plan(plan, [dev["A"], dev["B"], dev["C"]], differentiable=True)
    D.values.sum().backward()
    mm = ([(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
    ab = O.execute_sparse(rels["A"], rels["B"], *mm)
    abc = O.execute_sparse(ab, rels["C"], *mm)
    absr = {k: O.Relation(r.coords, np.abs(r.values), r.shape, r.tile_shape) for k, r in rels.items()}
    ab_abs = O.execute_sparse(absr["A"], absr["B"], *mm)
    abc_abs = O.execute_sparse(ab_abs, absr["C"], *mm)
    np.testing.assert_array_equal(D.coords.cpu().numpy(), abc.coords)
    assert _bound(D.values.detach().cpu().numpy(), abc.values, abc_abs.values)
    g = np.ones_like(abc.values)
    g_ab, g_c = _agg_grads(ab, rels["C"], *mm, g)
    g_a, g_b = _agg_grads(rels["A"], rels["B"], *mm, g_ab)
    m_ab, m_c = _agg_grads(ab_abs, absr["C"], *mm, g)
    m_a, m_b = _agg_grads(absr["A"], absr["B"], *mm, m_ab)
    assert _bound(dev["C"].values.grad.cpu().numpy(), g_c, m_c)
    assert _bound(dev["A"].values.grad.cpu().numpy(), g_a, m_a)
    assert _bound(dev["B"].values.grad.cpu().numpy(), g_b, m_b)


def _c5_run(w, idx, val, wd=None):
    X = E.tile_coo(idx, val, w.lhs.shape, w.lhs_tile)
    Wt = E.tile_dense(w.rhs if wd is None else wd, w.rhs_tile)
    return E.execute_sparse(X, Wt, w.join_keys, w.kernel_string, w.agg_keys)


@pytest.mark.timeout(900)
def test_c5_full_size():
    w = W.c5_order3_device(seed=0)
    idx, val = w.lhs.indices, w.lhs.values
    assert idx.shape[0] == 50_000_000
    res = _c5_run(w, idx, val)
    c = res.coords.cpu().numpy()
    # sampled output tile positions, all l tiles, against float64 sums
    ij = np.unique(c[:, :2], axis=0)
    want = ij[np.random.default_rng(2).choice(len(ij), 128, replace=False)]
    idx_h, val_h, w_h = idx.cpu().numpy(), val.cpu().numpy(), w.rhs.cpu().numpy()
    ref, mag = bench.c5_sample_ref(idx_h, val_h, w_h, want)
    rowmap = {tuple(x): r for r, x in enumerate(c)}
    rows = [rowmap[(a, b, l)] for a, b in want for l in range(8)]
    got = res.values[torch.tensor(rows, device=res.values.device)].cpu().numpy()
    got = got.reshape(len(want), 8, 16, 16, 16).transpose(0, 2, 3, 1, 4).reshape(ref.shape)
    assert _bound(got, ref, mag)
    # linearity over a split of the contracted range
    odd = ((idx[:, 2] // 16) % 2).bool()
    r_even = _c5_run(w, idx[~odd].contiguous(), val[~odd].contiguous())
    r_odd = _c5_run(w, idx[odd].contiguous(), val[odd].contiguous())
    u = torch.cat([r_even.coords, r_odd.coords])
    key = lambda t: (t[:, 0].long() * 256 + t[:, 1].long()) * 8 + t[:, 2].long()  # noqa: E731
    full_key = key(res.coords)
    tot = torch.zeros_like(res.values)
    for part in (r_even, r_odd):
        pos = torch.searchsorted(full_key, key(part.coords))
        assert torch.equal(full_key[pos], key(part.coords))
        tot.index_add_(0, pos, part.values)
    assert torch.equal(torch.unique(key(u)), full_key)
    del r_even, r_odd
    mag_full = _c5_run(w, idx, val.abs(), w.rhs.abs())
    assert torch.equal(mag_full.coords, res.coords)
    assert bool(((res.values - tot).abs() <= 2e-5 * (res.values.abs() + mag_full.values)).all())
    del tot, mag_full
    # one k slice tile for tile against the oracle
    ks = idx[:, 2] >= 255 * 16  # the last k tile: a few thousand entries
    si, sv = idx[ks].contiguous(), val[ks].contiguous()
    got = _c5_run(w, si, sv)
    X = O.to_relation(si.cpu().numpy(), sv.cpu().numpy().astype(np.float64), w.lhs.shape, w.lhs_tile)
    Wr = O.relation_from_dense(w_h.astype(np.float64), w.rhs_tile)
    ref = O.execute_sparse(X, Wr, w.join_keys, w.kernel_string, w.agg_keys)
    refm = O.execute_sparse(O.Relation(X.coords, np.abs(X.values), X.shape, X.tile_shape),
                            O.Relation(Wr.coords, np.abs(Wr.values), Wr.shape, Wr.tile_shape),
                            w.join_keys, w.kernel_string, w.agg_keys)
    gc, gv = got.to_numpy()
    np.testing.assert_array_equal(gc, ref.coords)
    assert _bound(gv, ref.values, refm.values)
