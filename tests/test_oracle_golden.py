"""Pin the CPU oracle against golden vectors from the unmodified reference.

Integer results (pairs, coordinates, partitions) must match bit for bit,
including order; float64 values to 1e-12 relative (both sides are numpy,
possibly with a different summation order inside ``einsum``).
"""

import numpy as np
import pytest

import oracle as O
from golden_io import cases_of_kind, load_cases

UNIT = load_cases()
CFG = load_cases("golden_configs.npz")


def _close(a, b, rtol=1e-12, atol=1e-12):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    assert a.shape == b.shape
    np.testing.assert_allclose(a, b, rtol=rtol, atol=atol)


@pytest.mark.parametrize("name", sorted(cases_of_kind("to_relation")))
def test_to_relation(name):
    c = UNIT[name]
    rel = O.to_relation(c["indices"], c["values"], c.meta["shape"], c.meta["tile"])
    assert rel.coords.dtype == np.int32
    np.testing.assert_array_equal(rel.coords, c["out_coords"])
    assert rel.values.dtype == c["out_values"].dtype
    np.testing.assert_array_equal(rel.values, c["out_values"])


def test_to_relation_non_divisible():
    with pytest.raises(ValueError):
        O.relation_from_dense(np.eye(5), (2, 2))


@pytest.mark.parametrize("name", sorted(cases_of_kind("join")))
def test_joins(name):
    c = UNIT[name]
    keys = [tuple(k) for k in c.meta["join_keys"]]
    li, ri = O.coordinate_join(c["lhs_coords"], c["rhs_coords"], keys)
    assert li.dtype == np.int64 and ri.dtype == np.int64
    np.testing.assert_array_equal(li, c["li"])
    np.testing.assert_array_equal(ri, c["ri"])
    hl, hr = O.coordinate_join_hash(c["lhs_coords"], c["rhs_coords"], keys)
    np.testing.assert_array_equal(hl, c["hash_li"])
    np.testing.assert_array_equal(hr, c["hash_ri"])
    sl, sr = O.coordinate_join_sorted(c["lhs_coords"], c["rhs_coords"], keys)
    np.testing.assert_array_equal(sl, c["sorted_li"])
    np.testing.assert_array_equal(sr, c["sorted_ri"])


def test_join_int_shorthand():
    c = UNIT["join_int_shorthand"]
    hl, hr = O.coordinate_join_hash(c["lhs_coords"], c["rhs_coords"], c.meta["join_dims"])
    np.testing.assert_array_equal(hl, c["hash_li"])
    np.testing.assert_array_equal(hr, c["hash_ri"])


@pytest.mark.parametrize("name", sorted(cases_of_kind("segment_sum")))
def test_segment_sum(name):
    c = UNIT[name]
    uc, uv = O.segment_sum(c["values"], c["out_coords"])
    np.testing.assert_array_equal(uc, c["res_coords"])
    assert uv.dtype == c["res_values"].dtype
    np.testing.assert_array_equal(uv, c["res_values"])


@pytest.mark.parametrize("name", sorted(cases_of_kind("kernel_einsum")))
def test_kernel_einsum(name):
    c = UNIT[name]
    out = O.kernel_einsum(c["lhs_values"], c["rhs_values"], c["li"], c["ri"], c.meta["kernel"])
    _close(out, c["out"])
    out32 = O.kernel_einsum(c["lhs_values"], c["rhs_values"], c["li"], c["ri"], c.meta["kernel"], "f32")
    assert out32.dtype == c["out_f32"].dtype
    _close(out32, c["out_f32"], rtol=1e-6, atol=1e-6)


def test_helpers():
    h = UNIT["helpers"].meta
    for s, want in h["add_batch_dim"].items():
        assert O.add_batch_dim(s) == want
    for s, a, b, want in h["infer_tile"]:
        assert list(O.infer_output_tile_shape(s, tuple(a), tuple(b))) == want
    for s, want in h["reverse"].items():
        assert list(O.reverse_einsum_string(s)) == want
    for n, d, want in h["partition"]:
        assert [list(p) for p in O.partition_matched_pairs(n, d)] == want
    with pytest.raises(ValueError):
        O.add_batch_dim("ij,jk")


def _rel(c, p):
    return O.Relation(c[f"{p}_coords"], c[f"{p}_values"], tuple(int(x) for x in c[f"{p}_shape"]),
                      tuple(int(x) for x in c[f"{p}_tile"]))


@pytest.mark.parametrize("name", sorted(cases_of_kind("execute")))
def test_execute_sparse(name):
    c = UNIT[name]
    m = c.meta
    lhs, rhs = _rel(c, "lhs"), _rel(c, "rhs")
    jk = [tuple(k) for k in m["join_keys"]]
    ak = [tuple(k) for k in m["agg_keys"]]
    osh = None if m["output_shape"] is None else tuple(m["output_shape"])
    ots = None if m["output_tile_shape"] is None else tuple(m["output_tile_shape"])
    li, ri = O.coordinate_join(lhs.coords, rhs.coords, jk)
    np.testing.assert_array_equal(li, c["li"])
    np.testing.assert_array_equal(ri, c["ri"])
    res = O.execute_sparse(lhs, rhs, jk, m["kernel"], ak, osh, ots)
    assert list(res.shape) == m["res_shape"] and list(res.tile_shape) == m["res_tile"]
    np.testing.assert_array_equal(res.coords, c["res_coords"])
    _close(res.values, c["res_values"])
    res32 = O.execute_sparse(lhs, rhs, jk, m["kernel"], ak, osh, ots, compute_dtype="f32")
    np.testing.assert_array_equal(res32.coords, c["res32_coords"])
    assert res32.values.dtype == c["res32_values"].dtype
    _close(res32.values, c["res32_values"], rtol=1e-5, atol=1e-5)
    for nd in (2, 4, 8):
        shr = O.execute_sharded_sparse(lhs, rhs, jk, m["kernel"], ak, osh, ots, num_devices=nd)
        np.testing.assert_array_equal(shr.coords, c[f"sharded{nd}_coords"])
        _close(shr.values, c[f"sharded{nd}_values"])


@pytest.mark.parametrize("name", sorted(cases_of_kind("bsm")))
def test_block_sparse_matmul(name):
    c = UNIT[name]
    res = O.block_sparse_matmul_generic(_rel(c, "lhs"), _rel(c, "rhs"))
    np.testing.assert_array_equal(res.coords, c["res_coords"])
    _close(res.values, c["res_values"])
    np.testing.assert_array_equal(c["raw_coords"], c["res_coords"])


@pytest.mark.parametrize("name", sorted(cases_of_kind("vjp")))
def test_vjp(name):
    c = UNIT[name]
    fwd = O.sparse_einsum_raw_fwd(c["lhs_values"], c["rhs_values"], c["li"], c["ri"], c.meta["kernel"])
    _close(fwd, c["fwd"])
    gl, gr = O.sparse_einsum_raw_bwd(c["lhs_values"], c["rhs_values"], c["li"], c["ri"], c.meta["kernel"], c["g"])
    _close(gl, c["grad_lhs"])
    _close(gr, c["grad_rhs"])


@pytest.mark.parametrize("name", ["C1_small", "C2_small", "C3_small", "C5_small"])
def test_config_cases(name):
    c = CFG[name]
    m = c.meta
    jk = [tuple(k) for k in m["join_keys"]]
    ak = [tuple(k) for k in m["agg_keys"]]
    if "lhs_values" in c:
        lhs, rhs = _rel(c, "lhs"), _rel(c, "rhs")
    else:
        pfx = "a" if "a_indices" in c else "x"
        shape = tuple(int(s) for s in c[f"{pfx}_shape"])
        dense_b = c["b_dense"] if pfx == "a" else c["w_dense"]
        tile = (32, 32) if pfx == "a" else (16, 16, 16)
        lhs = O.to_relation(c[f"{pfx}_indices"], c[f"{pfx}_values"], shape, tile)
        rhs = O.relation_from_dense(dense_b.astype(np.float64), (32, 32) if pfx == "a" else (16, 16))
        np.testing.assert_array_equal(lhs.coords, c["lhs_coords"])
        np.testing.assert_array_equal(rhs.coords, c["rhs_coords"])
    li, ri = O.coordinate_join(lhs.coords, rhs.coords, jk)
    np.testing.assert_array_equal(li, c["li"])
    np.testing.assert_array_equal(ri, c["ri"])
    res = O.execute_sparse(lhs, rhs, jk, m["kernel"], ak, compute_dtype="f32")
    np.testing.assert_array_equal(res.coords, c["res_coords"])
    _close(res.values, c["res_values"], rtol=1e-5, atol=1e-5)


def test_config_chain():
    c = CFG["C4_small"]
    A, B, C = _rel(c, "A"), _rel(c, "B"), _rel(c, "C")
    mm = ([(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
    ab = O.execute_sparse(A, B, mm[0], mm[1], mm[2], compute_dtype="f32")
    np.testing.assert_array_equal(ab.coords, c["ab_coords"])
    _close(ab.values, c["ab_values"], rtol=1e-5, atol=1e-5)
    abc = O.execute_sparse(ab, C, mm[0], mm[1], mm[2], compute_dtype="f32")
    np.testing.assert_array_equal(abc.coords, c["abc_coords"])
    _close(abc.values, c["abc_values"], rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("name", sorted(cases_of_kind("stats", "golden_stats.npz")))
def test_sparsity_stats(name):
    """T(U) and V(l, U) of every tiling scheme, against the reference's own
    SparseTensor metrics / compute_sparsity_stats_coo."""
    c = load_cases("golden_stats.npz")[name]
    shape = tuple(int(v) for v in c["shape"])
    if "dense" in c:
        nzi = np.nonzero(c["dense"])
        idx, val = np.stack(nzi, 1).astype(np.int32), c["dense"][nzi]
    else:
        idx, val = c["indices"], c["values"]
    ts = [tuple(int(v) for v in t) for t in c["tile_shapes"]]
    assert ts == O.factor_tile_shapes(shape)
    res = O.compute_sparsity_stats_coo(idx, val, shape, ts)
    np.testing.assert_array_equal([res[t][0] for t in ts], c["num_tuples"])
    np.testing.assert_array_equal([res[t][1] for t in ts], c["value_count"])


PLAN = load_cases("golden_plan.npz")


def _plan_ops(c):
    return [O.Relation(c[f"op{i}_coords"], c[f"op{i}_values"].astype(np.float64),
                       tuple(int(v) for v in c[f"op{i}_shape"]), tuple(int(v) for v in c[f"op{i}_tile"]))
            for i in range(c.meta["n_ops"])]


@pytest.mark.parametrize("name", sorted(cases_of_kind("keys", "golden_plan.npz")))
def test_reduction_keys(name):
    """Join / aggregation keys against the reference's infer_reduction_info."""
    m = PLAN[name].meta
    assert all(s == [0, 1] for s in m["join_sides"])
    jk, ak = O.infer_reduction_keys(m["formula"])
    assert [list(k) for k in jk] == m["join_keys"]
    assert [list(k) for k in ak] == m["agg_keys"]


@pytest.mark.parametrize("name", sorted(cases_of_kind("plan", "golden_plan.npz")))
def test_execute_plan(name):
    """The plan walk over tile-COO relations against the reference's sparse
    chain (coordinates bit-exact, in order) and against its dense
    ExecutionEngine.execute_plan result."""
    c = PLAN[name]
    steps = [(s["formula"], tuple(s["input_indices"])) for s in c.meta["steps"]]
    for i in range(c.meta["n_ops"]):
        ops = _plan_ops(c)
        np.testing.assert_array_equal(ops[i].to_dense(), c[f"op{i}_dense"].astype(np.float32))
    res = O.execute_plan(steps, _plan_ops(c), compute_dtype="f32")
    np.testing.assert_array_equal(res.coords, c["res_coords"])
    _close(res.values, c["res_values"], rtol=1e-5, atol=1e-5)
    assert list(res.shape) == c.meta["res_shape"] and list(res.tile_shape) == c.meta["res_tile"]
    res64 = O.execute_plan(steps, _plan_ops(c))
    _close(res64.to_dense(), c["out_dense"], rtol=1e-5, atol=1e-6)


INGEST = load_cases("golden_ingest.npz")


@pytest.mark.parametrize("name", sorted(cases_of_kind("ingest", "golden_ingest.npz")))
def test_coalesce_and_duplicate_policies(name):
    """Repeated COO coordinates: "last" against the reference's tiling of the
    COO matrix (bit-exact), "sum" against its tiling of scipy's CSR of it and
    against scipy's coalesced COO (float64 sums to 1e-12: scipy may add a
    row's repeats in another order)."""
    c = INGEST[name]
    shape, tile = tuple(c.meta["shape"]), tuple(c.meta["tile"])
    r = O.to_relation(c["indices"], c["values"], shape, tile)
    np.testing.assert_array_equal(r.coords, c["last_coords"])
    np.testing.assert_array_equal(r.values, c["last_values"])
    li, lv, nz = O.coalesce_coo(c["indices"], c["values"], shape, "last")
    assert nz == int((c["values"] != 0).sum()) and len(lv) < nz
    r = O.to_relation(li, lv, shape, tile)
    np.testing.assert_array_equal(r.coords, c["last_coords"])
    np.testing.assert_array_equal(r.values, c["last_values"])
    si, sv, _ = O.coalesce_coo(c["indices"], c["values"], shape, "sum")
    np.testing.assert_array_equal(si, li)
    ref = {tuple(i): v for i, v in zip(c["coalesced_indices"].tolist(), c["coalesced_values"])}
    assert all(ref.pop(tuple(i)) == pytest.approx(v, rel=1e-12, abs=1e-12) for i, v in zip(si.tolist(), sv))
    assert all(v == 0 for v in ref.values())  # coordinates whose inputs were all zero
    r = O.to_relation(si, sv, shape, tile)
    np.testing.assert_array_equal(r.coords, c["sum_coords"])
    _close(r.values, c["sum_values"])
