"""GPU autodiff parity: ``sparse_einsum_raw`` / ``sparse_einsum`` backward
against the reference's own backward rule (golden vectors produced by
calling ``autodiff/custom_vjp.py``'s bwd) and against the oracle for the
aggregated (segment-summed) case and the C4 chain."""

import numpy as np
import pytest
import torch

import einjax_b200 as E
import oracle as O
from golden_io import cases_of_kind, load_cases

pytestmark = pytest.mark.gpu

UNIT = load_cases()
CFG = load_cases("golden_configs.npz")


def _bound(got, ref, mag, rtol=1e-5):
    return np.all(np.abs(got - ref) <= rtol * (np.abs(ref) + mag) + 1e-12)


@pytest.mark.parametrize("name", sorted(cases_of_kind("vjp")))
def test_raw_vjp_golden(name):
    c = UNIT[name]
    ks = c.meta["kernel"]
    lv = torch.from_numpy(c["lhs_values"]).float().cuda().requires_grad_(True)
    rv = torch.from_numpy(c["rhs_values"]).float().cuda().requires_grad_(True)
    out = E.sparse_einsum_raw(lv, rv, c["lhs_coords"], c["rhs_coords"], c["li"], c["ri"], ks)
    fmag = O.sparse_einsum_raw_fwd(np.abs(c["lhs_values"]), np.abs(c["rhs_values"]), c["li"], c["ri"], ks)
    assert _bound(out.detach().cpu().numpy(), c["fwd"], fmag)
    g = torch.from_numpy(c["g"]).float().cuda()
    out.backward(g)
    gl_mag, gr_mag = O.sparse_einsum_raw_bwd(np.abs(c["lhs_values"]), np.abs(c["rhs_values"]), c["li"], c["ri"], ks,
                                             np.abs(c["g"]))
    assert _bound(lv.grad.cpu().numpy(), c["grad_lhs"], gl_mag)
    assert _bound(rv.grad.cpu().numpy(), c["grad_rhs"], gr_mag)


def _agg_grads_oracle(lhs, rhs, jk, ks, ak, g_out):
    """Gradients of sum(out * g_out) for out = execute_sparse(lhs, rhs): the
    reference backward rule applied with each pair's cotangent being its
    output tile's cotangent."""
    li, ri = O.coordinate_join(lhs.coords, rhs.coords, jk)
    oc = O.compute_output_coords(lhs.coords, rhs.coords, li, ri, ak)
    _, inv = np.unique(oc, axis=0, return_inverse=True)
    g = g_out[inv.reshape(-1)]
    return O.sparse_einsum_raw_bwd(lhs.values, rhs.values, li, ri, ks, g)


def test_aggregated_grad_vs_oracle():
    rng = np.random.default_rng(5)
    A = rng.standard_normal((64, 96)) * (rng.random((64, 96)) < 0.2)
    B = rng.standard_normal((96, 48)) * (rng.random((96, 48)) < 0.2)
    lhs, rhs = O.relation_from_dense(A, (16, 16)), O.relation_from_dense(B, (16, 16))
    jk, ks, ak = [(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)]
    dl = E.SparseTensorRelation.from_arrays(lhs.coords, lhs.values, lhs.shape, lhs.tile_shape)
    dr = E.SparseTensorRelation.from_arrays(rhs.coords, rhs.values, rhs.shape, rhs.tile_shape)
    dl.values.requires_grad_(True)
    dr.values.requires_grad_(True)
    out = E.sparse_einsum(dl, dr, jk, ks, ak)
    ref = O.execute_sparse(lhs, rhs, jk, ks, ak)
    np.testing.assert_array_equal(out.coords.cpu().numpy(), ref.coords)
    g_out = rng.standard_normal(ref.values.shape)
    (out.values * torch.from_numpy(g_out).float().cuda()).sum().backward()
    gl, gr = _agg_grads_oracle(lhs, rhs, jk, ks, ak, g_out)
    glm, grm = _agg_grads_oracle(O.Relation(lhs.coords, np.abs(lhs.values), lhs.shape, lhs.tile_shape),
                                 O.Relation(rhs.coords, np.abs(rhs.values), rhs.shape, rhs.tile_shape),
                                 jk, ks, ak, np.abs(g_out))
    assert _bound(dl.values.grad.cpu().numpy(), gl, glm)
    assert _bound(dr.values.grad.cpu().numpy(), gr, grm)
    # finite-difference spot check on one stored element, as the reference tests do
    # (tests/test_autodiff.py:160-190, eps 1e-4, atol 1e-3)
    t, i, j = 0, 3, 5
    eps = 1e-3

    def f(delta):
        v = lhs.values.copy()
        v[t, i, j] += delta
        r = O.execute_sparse(O.Relation(lhs.coords, v, lhs.shape, lhs.tile_shape), rhs, jk, ks, ak)
        return float((r.values * g_out).sum())
    fd = (f(eps) - f(-eps)) / (2 * eps)
    assert abs(fd - float(dl.values.grad[t, i, j])) < 1e-3 * max(1.0, abs(fd))


def test_chain_backward():
    """C4 shape (scaled): grads of all three operands through two steps."""
    c = CFG["C4_small"]
    rels = {k: O.Relation(c[f"{k}_coords"], c[f"{k}_values"].astype(np.float64),
                          tuple(int(x) for x in c[f"{k}_shape"]), tuple(int(x) for x in c[f"{k}_tile"]))
            for k in "ABC"}
    dev = {k: E.SparseTensorRelation.from_arrays(r.coords, r.values, r.shape, r.tile_shape) for k, r in rels.items()}
    for d in dev.values():
        d.values.requires_grad_(True)
    mm = ([(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
    ab = E.sparse_einsum(dev["A"], dev["B"], *mm)
    abc = E.sparse_einsum(ab, dev["C"], *mm)
    abc.values.sum().backward()
    # oracle: dL/dC = AB^T ones, dL/d(AB) = ones C^T, then through AB
    ab_ref = O.execute_sparse(rels["A"], rels["B"], *mm)
    abc_ref = O.execute_sparse(ab_ref, rels["C"], *mm)
    np.testing.assert_array_equal(abc.coords.cpu().numpy(), abc_ref.coords)
    g_abc = np.ones_like(abc_ref.values)
    g_ab, g_c = _agg_grads_oracle(ab_ref, rels["C"], *mm, g_abc)
    g_a, g_b = _agg_grads_oracle(rels["A"], rels["B"], *mm, g_ab)
    absr = {k: O.Relation(r.coords, np.abs(r.values), r.shape, r.tile_shape) for k, r in rels.items()}
    ab_abs = O.execute_sparse(absr["A"], absr["B"], *mm)
    m_ab, m_c = _agg_grads_oracle(ab_abs, absr["C"], *mm, g_abc)
    m_a, m_b = _agg_grads_oracle(absr["A"], absr["B"], *mm, m_ab)
    assert _bound(dev["C"].values.grad.cpu().numpy(), g_c, m_c)
    assert _bound(dev["A"].values.grad.cpu().numpy(), g_a, m_a)
    assert _bound(dev["B"].values.grad.cpu().numpy(), g_b, m_b)


def test_chain_backward_128_tiles():
    """The C4 tile size (128 x 128, fp32 tensor cores without strips in the
    autodiff forward): grads of all three operands through two steps."""
    rng = np.random.default_rng(4)

    def rel(shape, dens):
        g = (shape[0] // 128, shape[1] // 128)
        n = g[0] * g[1]
        pos = np.sort(rng.choice(n, max(1, int(round(dens * n))), replace=False))
        coords = np.stack([pos // g[1], pos % g[1]], 1).astype(np.int32)
        vals = rng.standard_normal((len(pos), 128, 128)).astype(np.float32).astype(np.float64)
        return O.Relation(coords, vals, shape, (128, 128))

    rels = {"A": rel((1024, 1536), 0.3), "B": rel((1536, 1024), 0.4), "C": rel((1024, 768), 0.3)}
    dev = {k: E.SparseTensorRelation.from_arrays(r.coords, r.values, r.shape, r.tile_shape, dtype=torch.float32)
           for k, r in rels.items()}
    for d in dev.values():
        d.values.requires_grad_(True)
    mm = ([(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
    ab = E.sparse_einsum(dev["A"], dev["B"], *mm)
    abc = E.sparse_einsum(ab, dev["C"], *mm)
    abc.values.sum().backward()
    ab_ref = O.execute_sparse(rels["A"], rels["B"], *mm)
    abc_ref = O.execute_sparse(ab_ref, rels["C"], *mm)
    np.testing.assert_array_equal(abc.coords.cpu().numpy(), abc_ref.coords)
    g_abc = np.ones_like(abc_ref.values)
    g_ab, g_c = _agg_grads_oracle(ab_ref, rels["C"], *mm, g_abc)
    g_a, g_b = _agg_grads_oracle(rels["A"], rels["B"], *mm, g_ab)
    absr = {k: O.Relation(r.coords, np.abs(r.values), r.shape, r.tile_shape) for k, r in rels.items()}
    ab_abs = O.execute_sparse(absr["A"], absr["B"], *mm)
    m_ab, m_c = _agg_grads_oracle(ab_abs, absr["C"], *mm, g_abc)
    m_a, m_b = _agg_grads_oracle(absr["A"], absr["B"], *mm, m_ab)
    assert _bound(dev["C"].values.grad.cpu().numpy(), g_c, m_c)
    assert _bound(dev["A"].values.grad.cpu().numpy(), g_a, m_a)
    assert _bound(dev["B"].values.grad.cpu().numpy(), g_b, m_b)
