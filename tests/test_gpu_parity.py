"""GPU parity: the CUDA path (through the C ABI) against golden vectors from the
reference and against the CPU oracle.

Tolerances: join pairs, tile coordinates and segment structure bit-exact
(pairs in the reference's own order, not only after a canonical sort);
fp32 values within  |got - ref| <= 1e-5 * (|ref| + sum|a*b|)  per element,
where sum|a*b| is the same contraction over absolute values (the standard
dot-product error bound); bf16 inputs within 2e-2 of the same bound.
"""

import numpy as np
import pytest
import torch

import einjax_b200 as E
import oracle as O
from golden_io import cases_of_kind, load_cases

pytestmark = pytest.mark.gpu

UNIT = load_cases()
CFG = load_cases("golden_configs.npz")
RTOL32 = 1e-5
RTOL_BF16 = 2e-2


def _rel(c, p):
    return O.Relation(c[f"{p}_coords"], c[f"{p}_values"], tuple(int(x) for x in c[f"{p}_shape"]),
                      tuple(int(x) for x in c[f"{p}_tile"]))


def _dev(r: O.Relation, dtype=None):
    return E.SparseTensorRelation.from_arrays(r.coords, r.values, r.shape, r.tile_shape, dtype=dtype)


def _mag(lhs, rhs, jk, ks, ak, osh=None, ots=None):
    a = O.Relation(lhs.coords, np.abs(lhs.values.astype(np.float64)), lhs.shape, lhs.tile_shape)
    b = O.Relation(rhs.coords, np.abs(rhs.values.astype(np.float64)), rhs.shape, rhs.tile_shape)
    return O.execute_sparse(a, b, jk, ks, ak, osh, ots).values


def _assert_rel(res, ref, mag, rtol=RTOL32):
    c, v = res.to_numpy()
    ok, msg = O.relation_allclose(c, v, ref, rtol=rtol, mag=mag)
    assert ok, msg


# ----------------------------------------------------------------- tiling

@pytest.mark.parametrize("name", sorted(cases_of_kind("to_relation")))
def test_to_relation_golden(name):
    c = UNIT[name]
    st = E.SparseTensor("t", (c["indices"], c["values"], tuple(c.meta["shape"])))
    rel = st.to_relation(tuple(c.meta["tile"]))
    coords, vals = rel.to_numpy()
    np.testing.assert_array_equal(coords, c["out_coords"])
    np.testing.assert_array_equal(vals, c["out_values"].astype(np.float32))


@pytest.mark.parametrize("name", ["torel_roundtrip", "torel_three_d", "torel_random2", "torel_one_d"])
def test_dense_tiling_golden(name):
    c = UNIT[name]
    dense = np.zeros(tuple(c.meta["shape"]))
    dense[tuple(c["indices"].T)] = c["values"]
    rel = E.SparseTensor("t", dense).to_relation(tuple(c.meta["tile"]))
    coords, vals = rel.to_numpy()
    np.testing.assert_array_equal(coords, c["out_coords"])
    np.testing.assert_array_equal(vals, c["out_values"].astype(np.float32))
    np.testing.assert_array_equal(rel.to_dense().cpu().numpy(), dense.astype(np.float32))


def test_tiling_rejects_bad_input():
    with pytest.raises(ValueError):
        E.SparseTensor("t", np.eye(5)).to_relation((2, 2))
    idx = np.array([[0, 0], [4, 1]], dtype=np.int32)
    with pytest.raises(ValueError):
        E.SparseTensor("t", (idx, np.ones(2), (4, 4))).to_relation((2, 2))


@pytest.mark.parametrize("seed,shape,tile,nnz,dup", [
    (0, (256, 384), (32, 16), 3000, 0.0), (1, (64, 64, 64), (8, 4, 16), 20000, 0.2),
    (2, (4096, 4096), (32, 32), 50000, 0.05), (3, (1000,), (8,), 400, 0.5), (4, (96, 96), (96, 96), 500, 0.1),
    # scans over many 4096-element tiles (several look-back windows)
    (5, (4096, 8192), (16, 16), 1_500_000, 0.1)])
def test_tile_coo_random(seed, shape, tile, nnz, dup):
    rng = np.random.default_rng(seed)
    idx = np.stack([rng.integers(0, s, nnz) for s in shape], 1).astype(np.int32)
    ndup = int(dup * nnz)
    if ndup:
        idx[rng.choice(nnz, ndup, replace=False)] = idx[rng.choice(nnz, ndup)]
    val = rng.standard_normal(nnz)
    val[rng.random(nnz) < 0.05] = 0.0
    ref = O.to_relation(idx, val, shape, tile)
    rel = E.SparseTensor("t", (idx, val, shape)).to_relation(tile)
    coords, vals = rel.to_numpy()
    np.testing.assert_array_equal(coords, ref.coords)
    np.testing.assert_array_equal(vals, ref.values.astype(np.float32))


# ------------------------------------------------------------------- joins

@pytest.mark.parametrize("name", sorted(cases_of_kind("join")))
def test_join_golden(name):
    c = UNIT[name]
    keys = [tuple(k) for k in c.meta["join_keys"]]
    li, ri = E.coordinate_join_hash(c["lhs_coords"], c["rhs_coords"], keys)
    np.testing.assert_array_equal(li.cpu().numpy(), c["hash_li"])
    np.testing.assert_array_equal(ri.cpu().numpy(), c["hash_ri"])
    assert li.dtype == torch.int64
    sl, sr = E.coordinate_join_sorted(c["lhs_coords"], c["rhs_coords"], keys)
    np.testing.assert_array_equal(sl.cpu().numpy(), c["sorted_li"])
    np.testing.assert_array_equal(sr.cpu().numpy(), c["sorted_ri"])


def test_join_int_shorthand():
    c = UNIT["join_int_shorthand"]
    li, ri = E.coordinate_join_hash(c["lhs_coords"], c["rhs_coords"], c.meta["join_dims"])
    np.testing.assert_array_equal(li.cpu().numpy(), c["hash_li"])
    np.testing.assert_array_equal(ri.cpu().numpy(), c["hash_ri"])


@pytest.mark.parametrize("nl,nr,hi,keys", [(20000, 30000, 300, [(1, 0)]), (5000, 7000, 12, [(0, 0), (2, 1)]),
                                           (100000, 3, 2, [(1, 1)]), (3, 100000, 2, [(0, 0)])])
def test_join_random_exact_order(nl, nr, hi, keys):
    rng = np.random.default_rng(nl + nr)
    nd = 3
    lc = rng.integers(0, hi, (nl, nd)).astype(np.int32)
    rc = rng.integers(0, hi, (nr, nd)).astype(np.int32)
    want_l, want_r = O.coordinate_join(lc, rc, keys)
    li, ri = E.coordinate_join_hash(lc, rc, keys)
    np.testing.assert_array_equal(li.cpu().numpy(), want_l)
    np.testing.assert_array_equal(ri.cpu().numpy(), want_r)


# --------------------------------------------------------- segment sum etc.

@pytest.mark.parametrize("name", sorted(cases_of_kind("segment_sum")))
def test_segment_sum_golden(name):
    c = UNIT[name]
    v = torch.from_numpy(c["values"]).float().cuda()
    uc, uv = E.segment_sum(v, torch.from_numpy(c["out_coords"]).cuda())
    np.testing.assert_array_equal(uc.cpu().numpy(), c["res_coords"])
    mag = O.segment_sum(np.abs(c["values"].astype(np.float64)), c["out_coords"])[1]
    err = np.abs(uv.cpu().numpy() - c["res_values"])
    assert np.all(err <= RTOL32 * (np.abs(c["res_values"]) + mag) + 1e-30)


@pytest.mark.parametrize("name", sorted(cases_of_kind("kernel_einsum")))
@pytest.mark.parametrize("precision", ["exact", "auto"])
def test_kernel_einsum_golden(name, precision):
    c = UNIT[name]
    lv = torch.from_numpy(c["lhs_values"]).float().cuda()
    rv = torch.from_numpy(c["rhs_values"]).float().cuda()
    out = E.kernel_einsum(lv, rv, c["li"], c["ri"], c.meta["kernel"], precision=precision).cpu().numpy()
    ref = c["out"]
    assert out.shape == ref.shape
    mag = O.kernel_einsum(np.abs(c["lhs_values"]), np.abs(c["rhs_values"]), c["li"], c["ri"], c.meta["kernel"])
    assert np.all(np.abs(out - ref) <= RTOL32 * (np.abs(ref) + mag) + 1e-30)


def test_output_coords():
    c = UNIT["exec_rand_order3"]
    lhs, rhs = _rel(c, "lhs"), _rel(c, "rhs")
    ak = [tuple(k) for k in c.meta["agg_keys"]]
    got = E._compute_output_coords(_dev(lhs), _dev(rhs), c["li"], c["ri"], [(2, 0)], ak, None, (2, 4, 6))
    np.testing.assert_array_equal(got.cpu().numpy(), O.compute_output_coords(lhs.coords, rhs.coords, c["li"],
                                                                              c["ri"], ak))


# ------------------------------------------------------------ end to end

@pytest.mark.parametrize("name", sorted(cases_of_kind("execute")))
@pytest.mark.parametrize("precision", ["exact", "auto"])
def test_execute_sparse_golden(name, precision):
    c = UNIT[name]
    m = c.meta
    lhs, rhs = _rel(c, "lhs"), _rel(c, "rhs")
    jk = [tuple(k) for k in m["join_keys"]]
    ak = [tuple(k) for k in m["agg_keys"]]
    osh = None if m["output_shape"] is None else tuple(m["output_shape"])
    ots = None if m["output_tile_shape"] is None else tuple(m["output_tile_shape"])
    li, ri = E.coordinate_join(_dev(lhs), _dev(rhs), jk)
    np.testing.assert_array_equal(li.cpu().numpy(), c["li"])
    np.testing.assert_array_equal(ri.cpu().numpy(), c["ri"])
    res = E.execute_sparse(_dev(lhs), _dev(rhs), jk, m["kernel"], ak, osh, ots, precision=precision)
    assert list(res.shape) == m["res_shape"] and list(res.tile_shape) == m["res_tile"]
    ref = O.Relation(c["res_coords"], c["res_values"], tuple(m["res_shape"]), tuple(m["res_tile"]))
    _assert_rel(res, ref, _mag(lhs, rhs, jk, m["kernel"], ak, osh, ots))
    # the reference's own dense check
    if res.num_tuples:
        np.testing.assert_allclose(res.to_dense().cpu().numpy(), O.Relation(
            c["res_coords"], c["res_values"], tuple(m["res_shape"]), tuple(m["res_tile"])).to_dense(),
            atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("name", sorted(cases_of_kind("bsm")))
def test_block_sparse_matmul_golden(name):
    c = UNIT[name]
    lhs, rhs = _rel(c, "lhs"), _rel(c, "rhs")
    res = E.block_sparse_matmul_generic(_dev(lhs), _dev(rhs))
    ref = O.Relation(c["res_coords"], c["res_values"], res.shape, res.tile_shape)
    _assert_rel(res, ref, _mag(lhs, rhs, [(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)]))
    raw = E.block_sparse_matmul(lhs.coords, lhs.values, rhs.coords, rhs.values,
                                tuple(c.meta["block_shape"]), lhs.shape, rhs.shape)
    _assert_rel(raw, O.Relation(c["raw_coords"], c["raw_values"], raw.shape, raw.tile_shape),
                _mag(lhs, rhs, [(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)]))


def test_block_sparse_matmul_errors():
    a = _dev(O.relation_from_dense(np.ones((4, 4)), (2, 2)))
    b3 = E.SparseTensorRelation.from_arrays(np.zeros((1, 3), np.int32), np.ones((1, 1, 1, 1)), (1, 1, 1), (1, 1, 1))
    with pytest.raises(ValueError):
        E.block_sparse_matmul_generic(a, b3)
    b = _dev(O.relation_from_dense(np.ones((4, 4)), (1, 2)))
    with pytest.raises(ValueError):
        E.block_sparse_matmul_generic(a, b)


@pytest.mark.parametrize("name", ["C1_small", "C2_small", "C3_small", "C5_small"])
def test_config_golden(name):
    c = CFG[name]
    m = c.meta
    jk = [tuple(k) for k in m["join_keys"]]
    ak = [tuple(k) for k in m["agg_keys"]]
    bf16 = name == "C3_small"
    if "lhs_values" in c:
        lhs, rhs = _rel(c, "lhs"), _rel(c, "rhs")
        dl = _dev(lhs, torch.bfloat16 if bf16 else None)
        dr = _dev(rhs, torch.bfloat16 if bf16 else None)
    else:
        pfx = "a" if "a_indices" in c else "x"
        shape = tuple(int(s) for s in c[f"{pfx}_shape"])
        dense_b = c["b_dense"] if pfx == "a" else c["w_dense"]
        tl, tr = ((32, 32), (32, 32)) if pfx == "a" else ((16, 16, 16), (16, 16))
        dl = E.SparseTensor("A", (c[f"{pfx}_indices"], c[f"{pfx}_values"], shape)).to_relation(tl)
        dr = E.SparseTensor("B", torch.from_numpy(dense_b).cuda()).to_relation(tr)
        np.testing.assert_array_equal(dl.coords.cpu().numpy(), c["lhs_coords"])
        np.testing.assert_array_equal(dr.coords.cpu().numpy(), c["rhs_coords"])
        lhs = O.Relation(dl.coords.cpu().numpy(), dl.values.cpu().numpy().astype(np.float64), dl.shape, tl)
        rhs = O.Relation(dr.coords.cpu().numpy(), dr.values.cpu().numpy().astype(np.float64), dr.shape, tr)
    li, ri = E.coordinate_join(dl, dr, jk)
    np.testing.assert_array_equal(li.cpu().numpy(), c["li"])
    np.testing.assert_array_equal(ri.cpu().numpy(), c["ri"])
    res = E.execute_sparse(dl, dr, jk, m["kernel"], ak)
    ref = O.Relation(c["res_coords"], c["res_values"], tuple(m["res_shape"]), tuple(m["res_tile"]))
    _assert_rel(res, ref, _mag(lhs, rhs, jk, m["kernel"], ak), RTOL_BF16 if bf16 else RTOL32)


def test_chain_golden():
    c = CFG["C4_small"]
    A, B, C = _rel(c, "A"), _rel(c, "B"), _rel(c, "C")
    mm = ([(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
    ab = E.execute_sparse(_dev(A), _dev(B), *mm)
    abc = E.execute_sparse(ab, _dev(C), *mm)
    ab_ref = O.Relation(c["ab_coords"], c["ab_values"], ab.shape, ab.tile_shape)
    _assert_rel(ab, ab_ref, _mag(A, B, *mm))
    absA = O.execute_sparse(O.Relation(A.coords, np.abs(A.values), A.shape, A.tile_shape),
                            O.Relation(B.coords, np.abs(B.values), B.shape, B.tile_shape), *mm)
    mag = _mag(absA, C, *mm)
    _assert_rel(abc, O.Relation(c["abc_coords"], c["abc_values"], abc.shape, abc.tile_shape), mag)


# ------------------------------------------------------------- edge cases

def test_empty_and_no_match():
    e = E.SparseTensorRelation.from_arrays(np.zeros((0, 2), np.int32), np.zeros((0, 2, 2)), (4, 4), (2, 2))
    res = E.execute_sparse(e, e, [(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
    assert res.num_tuples == 0 and tuple(res.values.shape) == (0, 2, 2)
    A = np.zeros((4, 4)); A[0, 0] = 1
    B = np.zeros((4, 4)); B[2, 2] = 1
    res = E.execute_sparse(_dev(O.relation_from_dense(A, (2, 2))), _dev(O.relation_from_dense(B, (2, 2))),
                           [(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
    assert res.num_tuples == 0
    li, ri = E.coordinate_join(e, e, [])
    assert li.numel() == 0


def test_large_cross_product_order():
    a = _dev(O.relation_from_dense(np.ones((64, 2)), (1, 2)))
    b = _dev(O.relation_from_dense(np.ones((2, 48)), (2, 1)))
    li, ri = E.coordinate_join(a, b, [])
    wl, wr = O.coordinate_join(a.coords.cpu().numpy(), b.coords.cpu().numpy(), [])
    np.testing.assert_array_equal(li.cpu().numpy(), wl)
    np.testing.assert_array_equal(ri.cpu().numpy(), wr)


@pytest.mark.parametrize("ks,jk,ak,sa,sb,ta,tb", [
    ("ij,jk->ik", [(1, 0)], [(0, 0), (1, 1)], (256, 512), (512, 192), (64, 32), (32, 96)),
    ("ij,jk->ik", [(1, 0)], [(0, 0), (1, 1)], (512, 512), (512, 512), (128, 128), (128, 128)),
    ("ijk,kl->ijl", [(2, 0)], [(0, 0), (0, 1), (1, 1)], (64, 64, 64), (64, 32), (16, 16, 16), (16, 16)),
    ("bij,bjk->bik", [(0, 0), (2, 1)], [(0, 0), (0, 1), (1, 2)], (3, 256, 256), (3, 256, 256), (1, 64, 64),
     (1, 64, 64)),
    ("ij,kj->ik", [(1, 1)], [(0, 0), (1, 0)], (256, 256), (128, 256), (32, 32), (32, 32)),
])
@pytest.mark.parametrize("precision", ["exact", "auto"])
def test_random_vs_oracle(ks, jk, ak, sa, sb, ta, tb, precision):
    rng = np.random.default_rng(len(ks) + sa[0])
    ga = tuple(s // t for s, t in zip(sa, ta))
    gb = tuple(s // t for s, t in zip(sb, tb))

    def rel(shape, tile, grid, dens):
        n = int(np.prod(grid))
        pos = np.sort(rng.choice(n, max(1, int(dens * n)), replace=False))
        coords = np.stack(np.unravel_index(pos, grid), 1).astype(np.int32)
        return O.Relation(coords, rng.standard_normal((len(pos), *tile)), shape, tile)
    lhs, rhs = rel(sa, ta, ga, 0.3), rel(sb, tb, gb, 0.3)
    ref = O.execute_sparse(lhs, rhs, jk, ks, ak, compute_dtype="f64")
    res = E.execute_sparse(_dev(lhs), _dev(rhs), jk, ks, ak, precision=precision)
    lhs32 = O.Relation(lhs.coords, lhs.values.astype(np.float32).astype(np.float64), lhs.shape, lhs.tile_shape)
    rhs32 = O.Relation(rhs.coords, rhs.values.astype(np.float32).astype(np.float64), rhs.shape, rhs.tile_shape)
    ref = O.execute_sparse(lhs32, rhs32, jk, ks, ak)
    _assert_rel(res, ref, _mag(lhs, rhs, jk, ks, ak))


def test_bf16_batched_vs_oracle():
    from einjax_b200 import workloads as W
    w = W.c3_batched_bf16(seed=1, scale=8, batch=3)
    dl = E.SparseTensorRelation.from_arrays(w.lhs.coords, w.lhs.values, w.lhs.shape, w.lhs.tile_shape,
                                            dtype=torch.bfloat16)
    dr = E.SparseTensorRelation.from_arrays(w.rhs.coords, w.rhs.values, w.rhs.shape, w.rhs.tile_shape,
                                            dtype=torch.bfloat16)
    res = E.execute_sparse(dl, dr, w.join_keys, w.kernel_string, w.agg_keys)
    assert res.values.dtype == torch.bfloat16
    lhs = O.Relation(w.lhs.coords, w.lhs.values.astype(np.float64), w.lhs.shape, w.lhs.tile_shape)
    rhs = O.Relation(w.rhs.coords, w.rhs.values.astype(np.float64), w.rhs.shape, w.rhs.tile_shape)
    ref = O.execute_sparse(lhs, rhs, w.join_keys, w.kernel_string, w.agg_keys)
    _assert_rel(res, ref, _mag(lhs, rhs, w.join_keys, w.kernel_string, w.agg_keys), RTOL_BF16)


# ------------------------------------------------- tensor-core path geometry

def _random_block_sparse(rng, shape, tile, dens, dtype=np.float64):
    grid = tuple(s // t for s, t in zip(shape, tile))
    n = int(np.prod(grid))
    pos = np.sort(rng.choice(n, max(1, int(round(dens * n))), replace=False))
    coords = np.stack(np.unravel_index(pos, grid), 1).astype(np.int32)
    return O.Relation(coords, rng.standard_normal((len(pos), *tile)).astype(dtype), shape, tile)


TC_CASES = [
    # (kernel, join, agg, lhs shape, lhs tile, rhs shape, rhs tile, density A, density B, note)
    ("ij,jk->ik", [(1, 0)], [(0, 0), (1, 1)], (1024, 1024), (128, 128), (1024, 1024), (128, 128), 0.2, 0.3, "C1-like"),
    ("ij,jk->ik", [(1, 0)], [(0, 0), (1, 1)], (2048, 1024), (32, 32), (1024, 256), (32, 32), 0.02, 1.0, "C2-like"),
    ("ij,jk->ik", [(1, 0)], [(0, 0), (1, 1)], (1024, 1024), (32, 32), (1024, 256), (32, 32), 0.05, 0.5, "C2 sparse B"),
    ("ij,jk->ik", [(1, 0)], [(0, 0), (1, 1)], (256, 512), (16, 16), (512, 192), (16, 16), 0.1, 0.3, "16 tiles"),
    ("ij,jk->ik", [(1, 0)], [(0, 0), (1, 1)], (512, 256), (256, 64), (256, 640), (64, 128), 0.5, 0.6, "M=256"),
    ("ijk,kl->ijl", [(2, 0)], [(0, 0), (0, 1), (1, 1)], (128, 128, 256), (16, 16, 16), (256, 128), (16, 16), 0.01,
     1.0, "C5-like"),
    ("bij,bjk->bik", [(0, 0), (2, 1)], [(0, 0), (0, 1), (1, 2)], (3, 512, 512), (1, 64, 64), (3, 512, 512),
     (1, 64, 64), 0.1, 0.1, "C3-like f32"),
    ("ij,jk->ik", [(1, 0)], [(0, 0), (1, 1)], (1024, 1024), (64, 32), (1024, 512), (32, 64), 0.1, 0.6,
     "stacked Mt=64"),
    ("ij,jk->ik", [(1, 0)], [(0, 0), (1, 1)], (512, 1024), (16, 32), (1024, 256), (32, 16), 0.1, 0.5,
     "stacked Mt=16"),
    ("ij,jk->ik", [(1, 0)], [(0, 0), (1, 1)], (2048, 2048), (32, 64), (2048, 512), (64, 32), 0.03, 0.8,
     "stacked Kt=64"),
]


@pytest.mark.parametrize("case", TC_CASES, ids=[c[-1] for c in TC_CASES])
def test_tensor_core_path(case):
    ks, jk, ak, sa, ta, sb, tb, da, db, _ = case
    rng = np.random.default_rng(abs(hash(case[-1])) % 1000)
    lhs, rhs = _random_block_sparse(rng, sa, ta, da), _random_block_sparse(rng, sb, tb, db)
    from einjax_b200.sparse_dispatch import tile_einsum_path
    assert tile_einsum_path(ks, ta, tb) == "tc"
    res = E.execute_sparse(_dev(lhs), _dev(rhs), jk, ks, ak, precision="tc")
    lhs32 = O.Relation(lhs.coords, lhs.values.astype(np.float32).astype(np.float64), lhs.shape, lhs.tile_shape)
    rhs32 = O.Relation(rhs.coords, rhs.values.astype(np.float32).astype(np.float64), rhs.shape, rhs.tile_shape)
    ref = O.execute_sparse(lhs32, rhs32, jk, ks, ak)
    _assert_rel(res, ref, _mag(lhs, rhs, jk, ks, ak))
    exact = E.execute_sparse(_dev(lhs), _dev(rhs), jk, ks, ak, precision="exact")
    _assert_rel(exact, ref, _mag(lhs, rhs, jk, ks, ak))


DIRECT_CASES = [
    # (kernel, join, agg, lhs shape, lhs tile, rhs shape, rhs tile, density A, density B)
    ("ij,jk->ik", [(1, 0)], [(0, 0), (1, 1)], (1024, 2048), (32, 32), (2048, 256), (32, 32), 0.05, 1.0),
    ("ij,jk->ik", [(1, 0)], [(0, 0), (1, 1)], (512, 768), (16, 16), (768, 640), (16, 32), 0.2, 0.3),
    ("ijk,kl->ijl", [(2, 0)], [(0, 0), (0, 1), (1, 1)], (64, 64, 128), (16, 16, 16), (128, 96), (16, 16), 0.05, 0.8),
    ("ij,j->i", [(1, 0)], [(0, 0)], (256, 512), (16, 16), (512,), (16,), 0.3, 0.7),
    # strips longer than one 128-tile warp step, two rhs column dims
    ("ij,jk->ik", [(1, 0)], [(0, 0), (1, 1)], (128, 16384), (16, 32), (16384, 96), (32, 32), 0.5, 0.6),
    ("ij,jkl->ikl", [(1, 0)], [(0, 0), (1, 1), (1, 2)], (64, 4096), (8, 16), (4096, 24, 40), (16, 8, 8), 0.6, 0.3),
    # batch dims joined pairwise (C3's shape), keys listed in either order
    ("bij,bjk->bik", [(0, 0), (2, 1)], [(0, 0), (0, 1), (1, 2)], (4, 512, 512), (1, 32, 32), (4, 512, 384),
     (1, 32, 32), 0.1, 0.2),
    ("bij,bjk->bik", [(2, 1), (0, 0)], [(0, 0), (0, 1), (1, 2)], (3, 256, 2048), (1, 16, 16), (3, 2048, 64),
     (1, 16, 16), 0.3, 0.4),
    ("abij,abjk->abik", [(0, 0), (1, 1), (3, 2)], [(0, 0), (0, 1), (0, 2), (1, 3)], (2, 3, 128, 256),
     (1, 1, 16, 16), (2, 3, 256, 128), (1, 1, 16, 16), 0.2, 0.3),
]


@pytest.mark.parametrize("case", DIRECT_CASES, ids=[f"{c[0]}-{c[4]}" for c in DIRECT_CASES])
def test_direct_grouping_matches_sorted(case, monkeypatch):
    """The sort-free join + grouping gives the same segments, pairs (in join
    order inside each segment), strips and keys as join + radix grouping."""
    from einjax_b200 import sparse_dispatch as SD
    ks, jk, ak, sa, ta, sb, tb, da, db = case
    rng = np.random.default_rng(5)
    lhs, rhs = _dev(_random_block_sparse(rng, sa, ta, da)), _dev(_random_block_sparse(rng, sb, tb, db))
    assert SD._direct_shape(lhs, rhs, jk, ak)
    d = SD.plan_pairs(lhs, rhs, jk, ak)
    monkeypatch.setattr(SD, "_direct_shape", lambda *a: False)
    g = SD.plan_pairs(lhs, rhs, jk, ak)
    for name in ("out_coords", "seg_offsets", "seg_lhs", "seg_rhs", "seg_key"):
        a, b = getattr(d, name), getattr(g, name)
        assert (a is None) == (b is None), name
        assert a is None or torch.equal(a.cpu(), b.cpu()), name
    assert d.key_extent == g.key_extent
    # strips: same grouping of segments (labels may differ)
    ds, gs = d.seg_strip.cpu().numpy(), g.seg_strip.cpu().numpy()
    assert np.array_equal(np.diff(ds) != 0, np.diff(gs) != 0)
    res = E.execute_sparse(lhs, rhs, jk, ks, ak, precision="exact")
    ref = O.execute_sparse(*(O.Relation(r.coords.cpu().numpy(), r.values.cpu().double().numpy(), r.shape,
                                        r.tile_shape) for r in (lhs, rhs)), jk, ks, ak)
    np.testing.assert_array_equal(res.coords.cpu().numpy(), ref.coords)


@pytest.mark.parametrize("side", ["lhs", "rhs"])
def test_direct_grouping_unsorted_falls_back(side):
    """A relation out of lexicographic order takes the general path."""
    from einjax_b200 import sparse_dispatch as SD
    rng = np.random.default_rng(8)
    lhs = _random_block_sparse(rng, (256, 256), (32, 32), 0.3)
    rhs = _random_block_sparse(rng, (256, 128), (32, 32), 0.5)
    rel = lhs if side == "lhs" else rhs
    perm = rng.permutation(rel.coords.shape[0])
    shuffled = O.Relation(rel.coords[perm], rel.values[perm], rel.shape, rel.tile_shape)
    lhs, rhs = (shuffled, rhs) if side == "lhs" else (lhs, shuffled)
    jk, ks, ak = [(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)]
    assert SD._plan_direct(_dev(lhs), _dev(rhs), jk, ak) is None
    res = E.execute_sparse(_dev(lhs), _dev(rhs), jk, ks, ak, precision="exact")
    ref = O.execute_sparse(lhs, rhs, jk, ks, ak)
    np.testing.assert_array_equal(res.coords.cpu().numpy(), ref.coords)
    np.testing.assert_allclose(res.values.cpu().numpy(), ref.values, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("tile,bands", [((64, 64), 2), ((32, 32), 4), ((128, 128), 1)])
def test_tensor_core_bf16(tile, bands):
    from einjax_b200 import workloads as W
    rng = np.random.default_rng(tile[0])
    n = tile[0] * 8
    lhs = _random_block_sparse(rng, (2, n, n), (1, *tile), 0.2)
    rhs = _random_block_sparse(rng, (2, n, n), (1, *tile), 0.2)
    lhs.values = W.round_to_bf16(lhs.values.astype(np.float32)).astype(np.float64)
    rhs.values = W.round_to_bf16(rhs.values.astype(np.float32)).astype(np.float64)
    jk, ks, ak = [(0, 0), (2, 1)], "bij,bjk->bik", [(0, 0), (0, 1), (1, 2)]
    res = E.execute_sparse(_dev(lhs, torch.bfloat16), _dev(rhs, torch.bfloat16), jk, ks, ak, precision="auto")
    ref = O.execute_sparse(lhs, rhs, jk, ks, ak)
    _assert_rel(res, ref, _mag(lhs, rhs, jk, ks, ak), RTOL_BF16)


@pytest.mark.parametrize("case", [TC_CASES[1], TC_CASES[2], TC_CASES[0], TC_CASES[5], TC_CASES[7]],
                         ids=["C2-like", "C2 sparse B", "C1-like", "C5-like", "stacked Mt=64"])
def test_tensor_core_key_blocks(case, monkeypatch):
    """Force many contracted-range blocks (later blocks add into the output)."""
    monkeypatch.setenv("EINSPARSE_KBLOCK_BYTES", "65536")
    ks, jk, ak, sa, ta, sb, tb, da, db, _ = case
    rng = np.random.default_rng(99)
    lhs, rhs = _random_block_sparse(rng, sa, ta, da), _random_block_sparse(rng, sb, tb, db)
    res = E.execute_sparse(_dev(lhs), _dev(rhs), jk, ks, ak, precision="tc")
    lhs32 = O.Relation(lhs.coords, lhs.values.astype(np.float32).astype(np.float64), lhs.shape, lhs.tile_shape)
    rhs32 = O.Relation(rhs.coords, rhs.values.astype(np.float32).astype(np.float64), rhs.shape, rhs.tile_shape)
    ref = O.execute_sparse(lhs32, rhs32, jk, ks, ak)
    _assert_rel(res, ref, _mag(lhs, rhs, jk, ks, ak))


def test_tensor_core_key_blocks_bf16(monkeypatch):
    monkeypatch.setenv("EINSPARSE_KBLOCK_BYTES", "32768")
    from einjax_b200 import workloads as W
    rng = np.random.default_rng(7)
    lhs = _random_block_sparse(rng, (2, 1024, 1024), (1, 64, 64), 0.2)
    rhs = _random_block_sparse(rng, (2, 1024, 1024), (1, 64, 64), 0.2)
    lhs.values = W.round_to_bf16(lhs.values.astype(np.float32)).astype(np.float64)
    rhs.values = W.round_to_bf16(rhs.values.astype(np.float32)).astype(np.float64)
    jk, ks, ak = [(0, 0), (2, 1)], "bij,bjk->bik", [(0, 0), (0, 1), (1, 2)]
    res = E.execute_sparse(_dev(lhs, torch.bfloat16), _dev(rhs, torch.bfloat16), jk, ks, ak, precision="tc")
    ref = O.execute_sparse(lhs, rhs, jk, ks, ak)
    _assert_rel(res, ref, _mag(lhs, rhs, jk, ks, ak), RTOL_BF16)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("tile", [(32, 32), (4, 4, 4), (3, 5)])
def test_segment_sum_vector_path(dtype, tile):
    """segment_sum's 4-element vector reduction (aligned rows) gives the same
    bits as the scalar reduction (rows off a 16-byte boundary), and both
    match the oracle's grouping and sums."""
    from math import prod
    g = torch.Generator().manual_seed(5)
    n, te = 3000, prod(tile)
    oc = torch.randint(0, 13, (n, 2), generator=g, dtype=torch.int32)
    host = torch.randn(n, *tile, generator=g).to(dtype)
    aligned = host.cuda()
    buf = torch.empty(n * te + 8, dtype=dtype, device="cuda")
    shifted = buf[1:1 + n * te].view(n, *tile)
    shifted.copy_(aligned)
    assert shifted.data_ptr() % 16 != 0
    uc1, uv1 = E.segment_sum(aligned, oc.cuda())
    uc2, uv2 = E.segment_sum(shifted, oc.cuda())
    assert torch.equal(uc1, uc2) and torch.equal(uv1.view(torch.int16 if dtype == torch.bfloat16 else torch.int32),
                                                  uv2.view(torch.int16 if dtype == torch.bfloat16 else torch.int32))
    v64 = host.double().numpy()
    rc, rv = O.segment_sum(v64, oc.numpy())
    mag = O.segment_sum(np.abs(v64), oc.numpy())[1]
    np.testing.assert_array_equal(uc1.cpu().numpy(), rc)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    got = uv1.float().cpu().numpy().astype(np.float64)
    assert np.all(np.abs(got - rv) <= tol * (np.abs(rv) + mag))


@pytest.mark.timeout(600)
def test_c2_like_large_vs_scipy():
    """C2's shape at 1/4 of its rows and columns: COO -> tiles -> direct join
    -> stacked tensor-core GEMM, against scipy's float64 sparse x dense."""
    import scipy.sparse as sp
    rng = np.random.default_rng(21)
    n, m, nnz = 16384, 256, 268_000
    rows = rng.permutation(n)[np.minimum(rng.zipf(1.1, nnz) - 1, n - 1)]
    cols = rng.integers(0, n, nnz)
    a = sp.coo_matrix((rng.standard_normal(nnz).astype(np.float32).astype(np.float64), (rows, cols)), shape=(n, n))
    a.sum_duplicates()
    a = a.tocoo()
    b = rng.standard_normal((n, m)).astype(np.float32)
    idx = np.stack([a.row, a.col], 1).astype(np.int32)
    A = E.SparseTensor("A", (idx, a.data.astype(np.float32), (n, n))).to_relation((32, 32))
    B = E.SparseTensor("B", torch.from_numpy(b).cuda()).to_relation((32, 32))
    res = E.execute_sparse(A, B, [(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
    ref = a.tocsr() @ b.astype(np.float64)
    mag = abs(a.tocsr()) @ np.abs(b.astype(np.float64))
    coords, vals = res.to_numpy()
    got = np.zeros((n, m))
    for t, (i, j) in enumerate(coords):
        got[i * 32:(i + 1) * 32, j * 32:(j + 1) * 32] = vals[t]
    present = np.zeros((n // 32, m // 32), bool)
    present[coords[:, 0], coords[:, 1]] = True
    want = np.zeros_like(present)
    want[np.unique(a.row // 32)[:, None], np.arange(m // 32)[None, :]] = True
    assert np.array_equal(present, want)
    assert np.all(np.abs(got - ref) <= 1e-5 * (np.abs(ref) + mag))


@pytest.mark.parametrize("ks,lt,rt", [("ik,jk->ij", (64, 32), (128, 32)), ("ij,ik->jk", (32, 64), (32, 128)),
                                      ("ki,kj->ij", (32, 128), (32, 64)), ("bik,bjk->bij", (1, 64, 32), (1, 128, 32))])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_tile_einsum_transposed_operands(ks, lt, rt, dtype):
    """Contractions that are a plain tile matmul after swapping an operand's
    last two dims (the autodiff strings) take the tensor-core path through a
    transposed copy and agree with the exact SIMT path."""
    from einjax_b200 import sparse_dispatch as SD
    assert SD.tile_einsum_path(ks, lt, rt, dtype, dtype) == "tc"
    g = torch.Generator().manual_seed(3)
    nl, nr, P, nseg = 37, 29, 400, 61
    lv = torch.randn(nl, *lt, generator=g).to(dtype).cuda()
    rv = torch.randn(nr, *rt, generator=g).to(dtype).cuda()
    pl = torch.randint(0, nl, (P,), generator=g, dtype=torch.int32)
    pr = torch.randint(0, nr, (P,), generator=g, dtype=torch.int32)
    cuts = torch.sort(torch.randperm(P - 1, generator=g)[:nseg - 1] + 1).values
    so = torch.cat([torch.zeros(1, dtype=torch.int64), cuts.to(torch.int64), torch.full((1,), P, dtype=torch.int64)])
    args = (ks, lv, rv, pl.cuda(), pr.cuda(), so.cuda())
    got = SD.tile_einsum(*args, out_dtype=torch.float32, precision="tc")
    ref = SD.tile_einsum(*args, out_dtype=torch.float32, precision="exact")
    mag = SD.tile_einsum(ks, lv.float().abs(), rv.float().abs(), pl.cuda(), pr.cuda(), so.cuda(),
                         out_dtype=torch.float32, precision="exact")
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert torch.all((got - ref).abs() <= tol * (ref.abs() + mag) + 1e-6)
