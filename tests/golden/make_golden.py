"""Generate golden vectors by running the unmodified einjax reference.

Run in a container where the reference source tree is available (pass its
path with ``--reference``; it is read, never written). The reference needs
``jax``; the stand-in under ``tests/golden/_jaxstub`` maps ``jax.numpy`` onto
numpy so the reference's own functions run unchanged:

* ``tensor/sparse.py``             SparseTensor, to_relation, _extract_coo
* ``execution/sparse_dispatch.py`` coordinate_join, kernel_einsum, segment_sum,
                                   execute_sparse, execute_sharded_sparse, ...
* ``kernels/pallas_matmul.py``, ``kernels/pallas_gather.py``
* ``autodiff/custom_vjp.py``       sparse_einsum_raw forward and backward rule
* ``sharding/partition.py``        tile_shape_to_partition_spec

Cases: the inputs of the reference's own hot-path unit tests, seeded random
relations over several kernel strings, and scaled-down instances of the five
benchmark configurations. Outputs go to ``tests/golden/*.npz`` (keys
``<case>__<field>``, with a JSON ``<case>__meta``).

Usage:  python tests/golden/make_golden.py --reference <path-to-einjax>
        python tests/golden/make_golden.py --reference <path> --stats-only
            (only ``golden_stats.npz``: per-tiling-scheme sparsity statistics
            from ``tensor/stats.py`` and ``SparseTensor``'s metrics)
        python tests/golden/make_golden.py --reference <path> --plan-only
            (only ``golden_plan.npz``: join / aggregation keys from
            ``optimizer/dp.py``'s ``infer_reduction_info`` and multi-step plans
            run by ``execution/engine.py``'s ``ExecutionEngine.execute_plan``)
        python tests/golden/make_golden.py --reference <path> --ingest-only
            (only ``golden_ingest.npz``: COO input with repeated coordinates
            tiled by ``SparseTensor.to_relation``, given as a COO matrix --
            the last repeat wins -- and as scipy's CSR of it -- repeats added)
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(root: str):
    sys.path.insert(0, os.path.join(HERE, "_jaxstub"))
    import jax  # noqa: F401  (the stand-in)
    pkg = types.ModuleType("einjax")
    pkg.__path__ = [root]
    sys.modules["einjax"] = pkg
    if "opt_einsum" not in sys.modules:
        # optimizer/contraction_path.py imports opt_einsum at module level but only
        # get_contraction_order calls it; the plans below give their steps explicitly.
        sys.modules["opt_einsum"] = types.ModuleType("opt_einsum")
    for sub in ("core", "tensor", "execution", "kernels", "autodiff", "sharding", "optimizer"):
        m = types.ModuleType(f"einjax.{sub}")
        m.__path__ = [os.path.join(root, sub)]
        sys.modules[f"einjax.{sub}"] = m
    mods = {}
    for name in ("tensor.sparse", "tensor.stats", "execution.sparse_dispatch", "kernels.pallas_matmul",
                 "kernels.pallas_gather", "kernels.registry", "autodiff.custom_vjp",
                 "sharding.partition"):
        mods[name] = importlib.import_module(f"einjax.{name}")
    return mods


class Store:
    def __init__(self):
        self.arrays = {}

    def put(self, case: str, meta: dict, **arrays):
        assert case not in {k.split("__")[0] for k in self.arrays}, case
        self.arrays[f"{case}__meta"] = np.array(json.dumps(meta))
        for k, v in arrays.items():
            self.arrays[f"{case}__{k}"] = np.asarray(v)

    def save(self, path):
        np.savez_compressed(path, **self.arrays)


def make_stats(mods):
    """Sparsity statistics T(U), V(l, U) per tiling scheme: the reference's
    SparseTensor metrics (tensor/sparse.py:122-158, all factor tile shapes of
    the shape) and compute_sparsity_stats_coo (tensor/stats.py:25-80), on
    seeded inputs with explicit zeros and repeated coordinates."""
    sp_mod, stats = mods["tensor.sparse"], mods["tensor.stats"]
    st = Store()
    rng = np.random.default_rng(31)
    dense_cases = {"dense2d": (12, 18), "dense3d": (8, 12, 6), "dense1d": (30,)}
    for name, shape in dense_cases.items():
        d = rng.standard_normal(shape) * (rng.random(shape) < 0.15)
        t = sp_mod.SparseTensor(name, d)
        ts = sorted(t.schemes)
        st.put(f"stats_{name}", {"kind": "stats", "source": "SparseTensor"}, dense=d,
               shape=np.array(shape, dtype=np.int64), tile_shapes=np.array(ts, dtype=np.int64),
               num_tuples=np.array([t.schemes[k].num_tuples for k in ts], dtype=np.int64),
               value_count=np.array([t.schemes[k].value_count for k in ts], dtype=np.int64))
    coo_cases = {"coo2d": ((64, 48), 300), "coo3d": ((16, 24, 10), 500), "coo2d_large": ((256, 512), 4000)}
    for name, (shape, nnz) in coo_cases.items():
        idx = np.stack([rng.integers(0, n, nnz) for n in shape], 1).astype(np.int32)
        idx[rng.choice(nnz, nnz // 10, replace=False)] = idx[rng.choice(nnz, nnz // 10)]  # repeats
        val = rng.standard_normal(nnz)
        val[rng.random(nnz) < 0.1] = 0.0  # explicit zeros do not count
        factors = [mods["core.notation"].find_all_factors(n) for n in shape]
        import itertools
        ts = sorted(itertools.product(*factors))
        res = stats.compute_sparsity_stats_coo(idx, val, tuple(shape), ts)
        st.put(f"stats_{name}", {"kind": "stats", "source": "compute_sparsity_stats_coo"}, indices=idx, values=val,
               shape=np.array(shape, dtype=np.int64), tile_shapes=np.array(ts, dtype=np.int64),
               num_tuples=np.array([res[k][0] for k in ts], dtype=np.int64),
               value_count=np.array([res[k][1] for k in ts], dtype=np.int64))
    st.save(os.path.join(HERE, "golden_stats.npz"))
    print("wrote", len(st.arrays), "arrays to golden_stats.npz")


KEY_FORMULAS = ["ij,jk->ik", "bij,bjk->bik", "ijk,kl->ijl", "ij,kj->ik", "ij,ij->ij", "i,j->ij", "ijk,jk->i",
                "abc,cab->b", "jk,kl->jl", "bkl,bik->bil", "jm,ijl->ilm", "ji,jk->ki", "ij,jk->ki"]

# (einsum string, operand shapes, operand tile shapes, element density, path, step formulas)
PLANS = {
    "plan_chain3": ("ij,jk,kl->il", [(96, 64), (64, 80), (80, 48)], [(16, 16), (16, 16), (16, 16)], 0.05,
                    [(1, 2), (0, 1)], ["jk,kl->jl", "ij,jl->il"]),
    "plan_chain4": ("ij,jk,kl,lm->im", [(64, 48), (48, 32), (32, 40), (40, 24)], [(8, 8)] * 4, 0.08,
                    [(0, 1), (0, 1), (0, 1)], ["ij,jk->ik", "kl,lm->km", "ik,km->im"]),
    "plan_batched": ("bij,jk,bkl->bil", [(3, 32, 24), (24, 40), (3, 40, 16)], [(1, 8, 8), (8, 8), (1, 8, 8)], 0.1,
                     [(0, 1), (0, 1)], ["bij,jk->bik", "bkl,bik->bil"]),
    "plan_order3": ("ijk,kl,jm->ilm", [(16, 24, 32), (32, 20), (24, 12)], [(4, 8, 8), (8, 4), (8, 4)], 0.1,
                    [(0, 1), (0, 1)], ["ijk,kl->ijl", "jm,ijl->ilm"]),
}


def make_plan(mods):
    """Join / aggregation keys from the reference's infer_reduction_info
    (optimizer/dp.py:50-95) for single binary formulas, and multi-operand plans
    executed two ways by the reference: ExecutionEngine.execute_plan
    (execution/engine.py:264-324) over the dense operands, and the same steps
    as a chain of its sparse execute_sparse over tile-COO relations."""
    import jax
    dp = importlib.import_module("einjax.optimizer.dp")
    base = importlib.import_module("einjax.tensor.base")
    cp = importlib.import_module("einjax.optimizer.contraction_path")
    eng = importlib.import_module("einjax.execution.engine")
    sp_mod, sd = mods["tensor.sparse"], mods["execution.sparse_dispatch"]
    st = Store()

    def keys(formula, lshape, rshape):
        ins, out = formula.split("->")
        a, b = ins.split(",")
        lt, rt = base.BaseTensor("L", lshape), base.BaseTensor("R", rshape)
        info = dp.infer_reduction_info(out, base.IndexedTerm(lt, a), base.IndexedTerm(rt, b))
        side = lambda t: 0 if t is lt else 1  # noqa: E731
        return info, {"join_keys": [[jl[1], jr[1]] for jl, jr in info.join_keys],
                      "join_sides": [[side(jl[0]), side(jr[0])] for jl, jr in info.join_keys],
                      "agg_keys": [[side(t), i] for t, i in info.aggregation_keys],
                      "output_shape": list(info.output_shape)}

    for n, f in enumerate(KEY_FORMULAS):
        ins = f.split("->")[0].split(",")
        dims = {}
        for c in "".join(ins):
            dims.setdefault(c, 2 + len(dims))
        _, meta = keys(f, tuple(dims[c] for c in ins[0]), tuple(dims[c] for c in ins[1]))
        st.put(f"keys_{n}", {"kind": "keys", "formula": f, **meta})

    rng = np.random.default_rng(77)
    for name, (es, shapes, tiles, dens, path, formulas) in PLANS.items():
        dense = [rng.standard_normal(s) * (rng.random(s) < dens) for s in shapes]
        tensors = [base.BaseTensor(f"x{i}", s) for i, s in enumerate(shapes)]
        ops_t, steps, metas = list(tensors), [], []
        for k, ((i, j), f) in enumerate(zip(path, formulas)):
            ins, out = f.split("->")
            a, b = ins.split(",")
            info, meta = keys(f, ops_t[i].shape, ops_t[j].shape)
            res_t = base.BaseTensor(f"_t{k}", info.output_shape)
            steps.append(cp.ContractionStep(k, f, (i, j), a, b, out, res_t, info))
            metas.append({"formula": f, "input_indices": [i, j], **meta})
            for idx in sorted((i, j), reverse=True):
                del ops_t[idx]
            ops_t.append(res_t)
        plan = cp.ContractionPlan(es, steps, 0.0, [])
        out_dense = np.asarray(eng.ExecutionEngine().execute_plan(plan, [np.asarray(d) for d in dense]))
        # the same steps over tile-COO relations through the reference's sparse path
        work = [sp_mod.SparseTensor(f"x{i}", d).to_relation(t) for i, (d, t) in enumerate(zip(dense, tiles))]
        arrays = {}
        for i, r in enumerate(work):
            arrays[f"op{i}_coords"] = r.coords
            arrays[f"op{i}_values"] = r.values.astype(np.float32)
            arrays[f"op{i}_shape"] = np.array(r.shape, np.int64)
            arrays[f"op{i}_tile"] = np.array(r.tile_shape, np.int64)
            arrays[f"op{i}_dense"] = dense[i]
        jax.F32 = True
        for m in metas:
            i, j = m["input_indices"]
            res = sd.execute_sparse(work[i], work[j], [tuple(k) for k in m["join_keys"]], m["formula"],
                                    [tuple(k) for k in m["agg_keys"]])
            for idx in sorted((i, j), reverse=True):
                del work[idx]
            work.append(res)
        jax.F32 = False
        fin = work[-1]
        st.put(name, {"kind": "plan", "einsum": es, "path": [list(p) for p in path], "steps": metas,
                      "n_ops": len(shapes), "res_shape": list(fin.shape), "res_tile": list(fin.tile_shape)},
               **arrays, out_dense=out_dense, res_coords=fin.coords, res_values=np.asarray(fin.values, np.float32))
    st.save(os.path.join(HERE, "golden_plan.npz"))
    print("wrote", len(st.arrays), "arrays to golden_plan.npz")


def make_ingest(mods):
    """COO input with repeated coordinates, explicit zeros and repeats that
    cancel: SparseTensor(coo_matrix).to_relation (tensor/sparse.py:160-270;
    the last repeat wins) and SparseTensor(coo_matrix.tocsr()).to_relation
    (scipy adds repeats first), plus scipy's coalesced COO of the same input."""
    import scipy.sparse as ssp
    sp_mod = mods["tensor.sparse"]
    st = Store()
    rng = np.random.default_rng(41)
    for name, (shape, nnz, tile) in {"ingest_small": ((12, 16), 60, (4, 4)),
                                     "ingest_rect": ((64, 48), 900, (8, 16)),
                                     "ingest_dense_dups": ((8, 8), 400, (2, 4))}.items():
        idx = np.stack([rng.integers(0, n, nnz) for n in shape], 1).astype(np.int32)
        rep = rng.choice(nnz, nnz // 4, replace=False)
        idx[rep] = idx[rng.choice(nnz, nnz // 4)]
        val = np.round(rng.standard_normal(nnz), 3)
        val[rng.random(nnz) < 0.1] = 0.0
        # a repeated coordinate whose values cancel, alone in its tile
        in_last = (idx[:, 0] // tile[0] == shape[0] // tile[0] - 1) & (idx[:, 1] // tile[1] == shape[1] // tile[1] - 1)
        idx[in_last] = 0
        idx[:2] = [shape[0] - 1, shape[1] - 1]
        val[:2] = [1.25, -1.25]
        coo = ssp.coo_matrix((val, (idx[:, 0], idx[:, 1])), shape=shape)
        last = sp_mod.SparseTensor("t", coo).to_relation(tile)
        csr = coo.tocsr()
        summed = sp_mod.SparseTensor("t", csr).to_relation(tile)
        cc = csr.tocoo()
        st.put(name, {"kind": "ingest", "shape": list(shape), "tile": list(tile)}, indices=idx, values=val,
               last_coords=last.coords, last_values=last.values, sum_coords=summed.coords, sum_values=summed.values,
               coalesced_indices=np.stack([cc.row, cc.col], 1).astype(np.int32), coalesced_values=cc.data)
    st.save(os.path.join(HERE, "golden_ingest.npz"))
    print("wrote", len(st.arrays), "arrays to golden_ingest.npz")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--stats-only", action="store_true")
    ap.add_argument("--plan-only", action="store_true")
    ap.add_argument("--ingest-only", action="store_true")
    args = ap.parse_args()
    mods = load_reference(os.path.abspath(args.reference))
    mods["core.notation"] = importlib.import_module("einjax.core.notation")
    if args.plan_only:
        make_plan(mods)
        return
    if args.ingest_only:
        make_ingest(mods)
        return
    make_stats(mods)
    if args.stats_only:
        return
    make_plan(mods)
    make_ingest(mods)
    import jax
    sp_mod = mods["tensor.sparse"]
    sd = mods["execution.sparse_dispatch"]
    pm = mods["kernels.pallas_matmul"]
    pg = mods["kernels.pallas_gather"]
    cv = mods["autodiff.custom_vjp"]
    part = mods["sharding.partition"]
    STR = sp_mod.SparseTensorRelation

    def rel_from_dense(dense, tile):
        return sp_mod.SparseTensor("t", dense).to_relation(tile)

    def rel_arrays(prefix, rel, vdtype=None):
        vals = rel.values if vdtype is None else rel.values.astype(vdtype)
        return {f"{prefix}_coords": rel.coords, f"{prefix}_values": vals,
                f"{prefix}_shape": np.array(rel.shape, dtype=np.int64),
                f"{prefix}_tile": np.array(rel.tile_shape, dtype=np.int64)}

    # ------------------------------------------------------------------ unit cases
    st = Store()

    # to_relation (tests/test_sparse.py:219-295, tests/test_rigorous.py:438-463)
    d44 = np.zeros((4, 4)); d44[0, 0] = 1.0
    d3 = np.zeros((4, 4, 4)); d3[0, 0, 0] = 1.0; d3[3, 3, 3] = 2.0
    rt = np.array([[1.0, 0, 0, 2], [0, 3, 0, 0], [0, 0, 4, 0], [5, 0, 0, 6]])
    trel_cases = {
        "identity": (np.array([[1.0, 0.0], [0.0, 2.0]]), (2, 2)),
        "diagonal": (np.diag([1.0, 2.0, 3.0, 4.0]), (2, 2)),
        "skip_empty": (d44, (2, 2)),
        "roundtrip": (rt, (2, 2)),
        "empty": (np.zeros((4, 4)), (2, 2)),
        "three_d": (d3, (2, 2, 2)),
        "element_tiling": (np.eye(3), (1, 1)),
        "one_d": (np.array([0.0, 1.0, 0.0, 3.0, 0.0, 0.0, 7.0, 0.0]), (2,)),
    }
    rng = np.random.default_rng(7)
    for i, (shape, tile, dens) in enumerate([((16, 16), (4, 4), 0.1), ((12, 18), (3, 6), 0.3),
                                              ((8, 8, 8), (2, 4, 2), 0.05), ((64, 32), (16, 8), 0.01)]):
        d = rng.standard_normal(shape) * (rng.random(shape) < dens)
        trel_cases[f"random{i}"] = (d, tile)
    for name, (dense, tile) in trel_cases.items():
        idx, val, shape = sp_mod._extract_coo(dense)
        rel = sp_mod.SparseTensor("t", dense).to_relation(tile)
        st.put(f"torel_{name}", {"kind": "to_relation", "tile": list(tile), "shape": list(shape)},
               indices=idx, values=val, out_coords=rel.coords, out_values=rel.values)
    # duplicates through scipy COO: the last entry in input order survives
    import scipy.sparse as ssp
    rows = np.array([0, 1, 0, 3, 0, 2, 3]); cols = np.array([1, 2, 1, 3, 1, 0, 3])
    vals = np.array([1.0, 2.0, 3.0, 4.0, 5.0, 0.0, -6.0])
    coo = ssp.coo_matrix((vals, (rows, cols)), shape=(4, 4))
    idx, val, shape = sp_mod._extract_coo(coo)
    rel = sp_mod.SparseTensor("dup", coo).to_relation((2, 2))
    st.put("torel_duplicates", {"kind": "to_relation", "tile": [2, 2], "shape": [4, 4]},
           indices=idx, values=val, out_coords=rel.coords, out_values=rel.values)

    # joins (tests/test_sparse_dispatch.py:43-129, tests/test_pallas.py:232-338,
    #        tests/test_rigorous.py:884-933, 1275-1300)
    join_cases = {
        "matmul": (np.array([[0, 0], [0, 1]]), np.array([[0, 0], [1, 0]]), [(1, 0)]),
        "cross": (np.array([[0, 0], [1, 1]]), np.array([[0, 0], [1, 1]]), []),
        "nomatch": (np.array([[0, 0]]), np.array([[1, 0]]), [(1, 0)]),
        "multi": (np.array([[0, 0], [1, 0]]), np.array([[0, 0]]), [(1, 0)]),
        "empty": (np.zeros((0, 2)), np.zeros((0, 2)), [(1, 0)]),
        "pallas_matmul": (np.array([[0, 0], [0, 1], [1, 0]]), np.array([[0, 0], [1, 0]]), [(1, 0)]),
        "pallas_cross": (np.array([[0], [1]]), np.array([[0], [1], [2]]), []),
        "same_dim": (np.array([[0, 0], [1, 1]]), np.array([[0, 0], [1, 1]]), [(0, 0), (1, 1)]),
        "many_to_many": (np.array([[0, 0], [0, 1]]), np.array([[0, 0], [0, 1]]), [(0, 0)]),
        "multi_sorted": (np.array([[0, 0], [1, 0]]), np.array([[0, 0], [0, 1]]), [(1, 0)]),
        "consistency": (np.array([[0, 0], [0, 1], [1, 0]]), np.array([[0, 0], [1, 0], [1, 1]]), [(1, 0)]),
    }
    r42 = np.random.RandomState(42)
    join_cases["hash_vs_sorted50"] = (r42.randint(0, 5, size=(50, 2)), r42.randint(0, 5, size=(50, 2)), [(1, 0)])
    rng = np.random.default_rng(11)
    for i, (nl, nr, ndl, ndr, keys, hi) in enumerate([
            (200, 150, 2, 2, [(1, 0)], 12), (300, 300, 3, 2, [(2, 0)], 20),
            (100, 120, 3, 3, [(0, 0), (2, 1)], 6), (64, 64, 2, 2, [(0, 1), (1, 0)], 8),
            (1, 500, 2, 2, [(1, 0)], 3), (400, 1, 2, 2, [(1, 1)], 4)]):
        join_cases[f"random{i}"] = (rng.integers(0, hi, (nl, ndl)), rng.integers(0, hi, (nr, ndr)), keys)
    for name, (lc, rc, keys) in join_cases.items():
        lc = np.asarray(lc, dtype=np.int32); rc = np.asarray(rc, dtype=np.int32)
        L = STR(coords=lc, values=np.zeros((lc.shape[0], 1)), shape=(1,) * lc.shape[1], tile_shape=(1,) * lc.shape[1])
        R = STR(coords=rc, values=np.zeros((rc.shape[0], 1)), shape=(1,) * rc.shape[1], tile_shape=(1,) * rc.shape[1])
        li, ri = sd.coordinate_join(L, R, keys)
        hl, hr = pg.coordinate_join_hash(lc, rc, keys)
        sl, sr = pg.coordinate_join_sorted(lc, rc, keys)
        st.put(f"join_{name}", {"kind": "join", "join_keys": [list(k) for k in keys]},
               lhs_coords=lc, rhs_coords=rc, li=np.asarray(li, np.int64), ri=np.asarray(ri, np.int64),
               hash_li=np.asarray(hl, np.int64), hash_ri=np.asarray(hr, np.int64),
               sorted_li=np.asarray(sl, np.int64), sorted_ri=np.asarray(sr, np.int64))
    # integer shorthand of the hash join (tests/test_pallas.py:268-274)
    lc = np.array([[0, 0], [1, 1]], dtype=np.int32)
    hl, hr = pg.coordinate_join_hash(lc, lc, [0, 1])
    st.put("join_int_shorthand", {"kind": "join_hash_only", "join_dims": [0, 1]},
           lhs_coords=lc, rhs_coords=lc, hash_li=np.asarray(hl, np.int64), hash_ri=np.asarray(hr, np.int64))

    # segment_sum (tests/test_sparse_dispatch.py:204-257, tests/test_rigorous.py:955-971)
    seg_cases = {
        "single": (np.array([[[1.0, 2.0], [3.0, 4.0]]]), np.array([[0, 0]])),
        "sum_two": (np.array([[[1.0, 0.0], [0.0, 1.0]], [[2.0, 0.0], [0.0, 2.0]]]), np.array([[0, 0], [0, 0]])),
        "mixed": (np.array([[[1.0]], [[2.0]], [[3.0]]]), np.array([[0, 0], [0, 0], [1, 0]])),
        "empty": (np.zeros((0, 2, 2)), np.zeros((0, 2), dtype=np.int32)),
        "sorted": (np.array([[[1.0]], [[2.0]], [[3.0]]]), np.array([[2, 0], [0, 0], [1, 0]])),
        "three_same": (np.ones((3, 2, 2)), np.array([[0, 0], [0, 0], [0, 0]])),
    }
    rng = np.random.default_rng(13)
    for i, (p, nd, hi, tile) in enumerate([(500, 2, 6, (4, 4)), (300, 3, 4, (2, 3, 2)), (1000, 1, 50, (8,))]):
        seg_cases[f"random{i}"] = (rng.standard_normal((p, *tile)), rng.integers(0, hi, (p, nd)))
        seg_cases[f"random{i}_f32"] = (rng.standard_normal((p, *tile)).astype(np.float32), rng.integers(0, hi, (p, nd)))
    for name, (v, c) in seg_cases.items():
        uc, uv = sd.segment_sum(v, np.asarray(c, dtype=np.int32))
        st.put(f"segsum_{name}", {"kind": "segment_sum"}, values=v, out_coords=np.asarray(c, np.int32),
               res_coords=uc, res_values=uv)

    # kernel_einsum (tests/test_sparse_dispatch.py:137-196, tests/test_rigorous.py:935-952)
    ker_cases = {
        "matmul": (np.array([[[1.0, 0.0], [0.0, 1.0]], [[2.0, 0.0], [0.0, 2.0]]]),
                   np.array([[[3.0, 0.0], [0.0, 3.0]], [[4.0, 0.0], [0.0, 4.0]]]), [0, 1], [0, 1], "ij,jk->ik"),
        "outer": (np.array([[1.0, 2.0]]), np.array([[3.0, 4.0]]), [0], [0], "i,j->ij"),
        "dot": (np.array([[1.0, 2.0, 3.0]]), np.array([[4.0, 5.0, 6.0]]), [0], [0], "i,i->"),
        "empty": (np.zeros((2, 3, 3)), np.zeros((2, 3, 3)), [], [], "ij,jk->ik"),
        "single_pair": (np.eye(2).reshape(1, 2, 2), np.array([[[1.0, 2.0], [3.0, 4.0]]]), [0], [0], "ij,jk->ik"),
    }
    rng = np.random.default_rng(17)
    for i, (ks, ls, rs) in enumerate([("ij,jk->ik", (4, 6), (6, 5)), ("ij,kj->ik", (4, 6), (5, 6)),
                                      ("ji,jk->ik", (6, 4), (6, 5)), ("ijk,kl->ijl", (3, 4, 5), (5, 2)),
                                      ("bij,bjk->bik", (1, 4, 3), (1, 3, 5)), ("ij,ij->ij", (3, 3), (3, 3)),
                                      ("ij,kl->ij", (2, 3), (4, 2)), ("ii,ij->j", (3, 3), (3, 4)),
                                      ("ij,jk->ki", (3, 4), (4, 5)), ("ijk,jkl->il", (2, 3, 4), (3, 4, 5))]):
        nl, nr, p = 5, 6, 12
        ker_cases[f"random{i}"] = (rng.standard_normal((nl, *ls)), rng.standard_normal((nr, *rs)),
                                   rng.integers(0, nl, p), rng.integers(0, nr, p), ks)
    for name, (lv, rv, li, ri, ks) in ker_cases.items():
        li = np.asarray(li, np.int64); ri = np.asarray(ri, np.int64)
        out = sd.kernel_einsum(lv, rv, li, ri, ks)
        jax.F32 = True
        out32 = sd.kernel_einsum(lv, rv, li, ri, ks)
        jax.F32 = False
        st.put(f"kernel_{name}", {"kind": "kernel_einsum", "kernel": ks}, lhs_values=lv, rhs_values=rv,
               li=li, ri=ri, out=out, out_f32=np.asarray(out32))

    # helpers (tests/test_sparse_dispatch.py:434-468)
    helper = {"add_batch_dim": {s: sd._add_batch_dim(s) for s in ("ij,jk->ik", "i,j->ij", "i,i->", "bij,bjk->bik")},
              "infer_tile": [[s, list(a), list(b), list(sd._infer_output_tile_shape(s, a, b))] for s, a, b in [
                  ("ij,jk->ik", (2, 3), (3, 4)), ("i,j->ij", (3,), (4,)), ("i,i->", (5,), (5,)),
                  ("ii,ij->j", (3, 3), (3, 4)), ("ijk,kl->ijl", (16, 16, 16), (16, 16))]],
              "reverse": {s: list(cv._reverse_einsum_string(s)) for s in ("ij,jk->ik", "i,j->ij", "i,i->", "ijk,kl->ijl")},
              "partition": [[n, d, [list(p) for p in sd._partition_matched_pairs(n, d)]]
                            for n in (0, 1, 3, 7, 8, 10, 15, 64, 100) for d in (1, 2, 4, 8)]}
    pspec = []
    for shape, tile in [((8, 8), (2, 8)), ((8, 8), (8, 8)), ((8, 8), (2, 2)), ((4, 6, 8), (2, 6, 4)),
                        ((8,), (16,)), ((8, 8), (3, 8)), ((8, 8), (0, 8)), ((8, 8, 8, 8, 8), (1, 1, 1, 1, 1)),
                        ((8, 8), (2,))]:
        try:
            res = list(part.tile_shape_to_partition_spec(shape, tile))
        except ValueError:
            res = "ValueError"
        pspec.append([list(shape), list(tile), res])
    helper["partition_spec"] = pspec
    st.put("helpers", helper)

    # execute_sparse end to end (tests/test_sparse_dispatch.py:263-426,
    # tests/test_rigorous.py:1069-1136, tests/test_pallas.py:53-223)
    A_t = np.array([[1.0, 2, 0, 0], [3, 4, 0, 0], [0, 0, 5, 6], [0, 0, 7, 8]])
    Ae = np.zeros((4, 4)); Ae[0, 0] = 1.0
    Be = np.zeros((4, 4)); Be[2, 2] = 1.0
    Aag = np.zeros((4, 4)); Aag[0, 0] = 1; Aag[0, 2] = 2; Aag[1, 1] = 3; Aag[1, 3] = 4
    Bag = np.zeros((4, 4)); Bag[0, 0] = 5; Bag[2, 0] = 6; Bag[1, 1] = 7; Bag[3, 1] = 8
    Bnum = np.array([[1.0, 2, 0, 0], [0, 3, 4, 0], [0, 0, 5, 6], [0, 0, 0, 7]])
    MM = ([(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
    exe = {
        "identity": (np.array([[1.0, 2.0], [3.0, 4.0]]), np.eye(2), (1, 1), (1, 1), MM, (2, 2), (1, 1)),
        "diagonal": (np.diag([1.0, 2, 3, 4]), np.diag([5.0, 6, 7, 8]), (1, 1), (1, 1), MM, (4, 4), (1, 1)),
        "tiled": (A_t, np.eye(4), (2, 2), (2, 2), MM, (4, 4), (2, 2)),
        "outer": (np.array([1.0, 0.0, 3.0]).reshape(3, 1), np.array([0.0, 2.0, 4.0]).reshape(1, 3), (1, 1), (1, 1),
                  ([], "ij,kl->ij", [(0, 0), (1, 1)]), (3, 3), (1, 1)),
        "elementwise": (np.diag([1.0, 2, 3]), np.diag([4.0, 5, 6]), (1, 1), (1, 1),
                        ([(0, 0), (1, 1)], "ij,ij->ij", [(0, 0), (0, 1)]), (3, 3), (1, 1)),
        "empty_result": (Ae, Be, (2, 2), (2, 2), MM, (4, 4), (2, 2)),
        "inferred": (np.diag([1.0, 2.0]), np.diag([3.0, 4.0]), (1, 1), (1, 1), MM, None, None),
        "num_vs_dense": (np.eye(4), Bnum, (2, 2), (2, 2), MM, None, None),
        "aggregation": (Aag, Bag, (2, 2), (2, 2), MM, None, None),
        "ones_agg": (np.ones((4, 4)), np.ones((4, 4)), (2, 2), (2, 2), MM, (4, 4), (2, 2)),
        "non_square": (np.array([[1.0, 0, 2, 0], [0, 3, 0, 4], [5, 0, 6, 0]]),
                       np.array([[1.0, 0], [0, 2], [3, 0], [0, 4]]), (1, 1), (1, 1), MM, None, None),
    }
    np.random.seed(42)
    S1 = np.random.randn(8, 8); S2 = np.random.randn(8, 8)
    S1[S1 < 0] = 0.0; S2[S2 < 0] = 0.0
    exe["sharded_match"] = (S1, S2, (2, 2), (2, 2), MM, (8, 8), (2, 2))
    rng = np.random.default_rng(23)

    def rnd(shape, dens):
        return rng.standard_normal(shape) * (rng.random(shape) < dens)
    rand_specs = [
        ("mm", (32, 48), (48, 40), (4, 8), (8, 5), MM, 0.05),
        ("mm_t16", (64, 64), (64, 32), (16, 16), (16, 16), MM, 0.02),
        ("mm_rect", (24, 36), (36, 20), (6, 4), (4, 10), MM, 0.1),
        ("ij_kj", (32, 40), (24, 40), (4, 8), (6, 8), ([(1, 1)], "ij,kj->ik", [(0, 0), (1, 0)]), 0.05),
        ("ji_jk", (40, 32), (40, 24), (8, 4), (8, 6), ([(0, 0)], "ji,jk->ik", [(0, 1), (1, 1)]), 0.05),
        ("ij_jk_ki", (32, 48), (48, 40), (4, 8), (8, 5), ([(1, 0)], "ij,jk->ki", [(1, 1), (0, 0)]), 0.05),
        ("batched", (3, 16, 24), (3, 24, 16), (1, 4, 8), (1, 8, 4),
         ([(0, 0), (2, 1)], "bij,bjk->bik", [(0, 0), (0, 1), (1, 2)]), 0.05),
        ("order3", (8, 8, 16), (16, 12), (2, 4, 4), (4, 6), ([(2, 0)], "ijk,kl->ijl", [(0, 0), (0, 1), (1, 1)]), 0.05),
        ("hadamard", (16, 16), (16, 16), (4, 4), (4, 4), ([(0, 0), (1, 1)], "ij,ij->ij", [(0, 0), (0, 1)]), 0.2),
        ("cross_sum", (6, 4), (4, 6), (2, 2), (2, 3), ([], "ij,kl->ij", [(0, 0), (1, 1)]), 0.2),
        ("two_key", (12, 16, 8), (16, 8, 10), (3, 4, 2), (4, 2, 5),
         ([(1, 0), (2, 1)], "ijk,jkl->il", [(0, 0), (1, 2)]), 0.1),
    ]
    for name, sa, sb, ta, tb, spec, dens in rand_specs:
        exe[f"rand_{name}"] = (rnd(sa, dens), rnd(sb, dens), ta, tb, spec, None, None)
    for name, (A, B, ta, tb, (jk, ks, ak), osh, ots) in exe.items():
        lhs = rel_from_dense(A, ta); rhs = rel_from_dense(B, tb)
        li, ri = sd.coordinate_join(lhs, rhs, jk)
        res = sd.execute_sparse(lhs, rhs, jk, ks, ak, osh, ots)
        jax.F32 = True
        res32 = sd.execute_sparse(lhs, rhs, jk, ks, ak, osh, ots)
        jax.F32 = False
        meta = {"kind": "execute", "join_keys": [list(k) for k in jk], "kernel": ks, "agg_keys": [list(k) for k in ak],
                "output_shape": None if osh is None else list(osh),
                "output_tile_shape": None if ots is None else list(ots),
                "res_shape": list(res.shape), "res_tile": list(res.tile_shape)}
        sharded = {}
        for nd in (2, 4, 8):
            jax.NUM_FAKE_DEVICES = nd
            mesh = jax.sharding.Mesh(np.array(jax.local_devices()).reshape(-1), ("x",))
            shr = sd.execute_sharded_sparse(lhs, rhs, jk, ks, ak, osh, ots, mesh=mesh)
            jax.NUM_FAKE_DEVICES = 1
            sharded[f"sharded{nd}_coords"] = shr.coords
            sharded[f"sharded{nd}_values"] = shr.values
        st.put(f"exec_{name}", meta, **rel_arrays("lhs", lhs), **rel_arrays("rhs", rhs), li=np.asarray(li, np.int64),
               ri=np.asarray(ri, np.int64), res_coords=res.coords, res_values=res.values,
               res32_coords=res32.coords, res32_values=res32.values, **sharded)
        if ks == "ij,jk->ik" and jk == [(1, 0)]:
            bsm = pm.block_sparse_matmul_generic(lhs, rhs)
            raw = pm.block_sparse_matmul(lhs.coords, lhs.values, rhs.coords, rhs.values,
                                         (ta[0], ta[1], tb[1]), lhs.shape, rhs.shape)
            st.put(f"bsm_{name}", {"kind": "bsm", "block_shape": [ta[0], ta[1], tb[1]]},
                   **rel_arrays("lhs", lhs), **rel_arrays("rhs", rhs), res_coords=bsm.coords,
                   res_values=bsm.values, raw_coords=raw.coords, raw_values=raw.values)

    # autodiff: sparse_einsum_raw forward and the reference's own backward rule
    # (tests/test_autodiff.py:160-403)
    vjp_cases = {
        "t2": (np.array([[1.0, 2.0], [3.0, 4.0]]), np.array([[5.0, 6.0], [7.0, 8.0]]), (2, 2), (2, 2), MM),
        "diag": (np.diag([1.0, 2, 3, 4]), np.diag([5.0, 6, 7, 8]), (2, 2), (2, 2), MM),
        "accum": (Aag, Bag, (2, 2), (2, 2), MM),
        "t1": (np.array([[1.0, 0.0], [0.0, 2.0]]), np.array([[3.0, 0.0], [0.0, 4.0]]), (1, 1), (1, 1), MM),
    }
    for name, sa, sb, ta, tb, spec, dens in rand_specs[:8]:
        vjp_cases[f"rand_{name}"] = (rnd(sa, max(dens, 0.1)), rnd(sb, max(dens, 0.1)), ta, tb, spec)
    for name, (A, B, ta, tb, (jk, ks, ak)) in vjp_cases.items():
        lhs = rel_from_dense(A, ta); rhs = rel_from_dense(B, tb)
        li, ri = sd.coordinate_join(lhs, rhs, jk)
        jax.LAST_VJP.clear()
        fwd = cv.sparse_einsum_raw(lhs.values, rhs.values, lhs.coords, rhs.coords, li, ri, ks)
        obj = jax.LAST_VJP[-1]
        g = rng.standard_normal(np.asarray(fwd).shape)
        _, resid = obj.fwd(lhs.values, rhs.values)
        gl, gr = obj.bwd(resid, g)
        st.put(f"vjp_{name}", {"kind": "vjp", "kernel": ks, "join_keys": [list(k) for k in jk]},
               lhs_values=lhs.values, rhs_values=rhs.values, lhs_coords=lhs.coords, rhs_coords=rhs.coords,
               li=np.asarray(li, np.int64), ri=np.asarray(ri, np.int64), fwd=np.asarray(fwd), g=g,
               grad_lhs=np.asarray(gl), grad_rhs=np.asarray(gr))
    st.save(os.path.join(HERE, "golden_unit.npz"))

    # ------------------------------------------------------------ config-shaped cases
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from einjax_b200 import workloads as wl
    cs = Store()

    def run_exec(name, lhs, rhs, jk, ks, ak, extra_inputs):
        li, ri = sd.coordinate_join(lhs, rhs, jk)
        jax.F32 = True
        res = sd.execute_sparse(lhs, rhs, jk, ks, ak)
        jax.F32 = False
        cs.put(name, {"kind": "execute_cfg", "join_keys": [list(k) for k in jk], "kernel": ks,
                      "agg_keys": [list(k) for k in ak], "res_shape": list(res.shape),
                      "res_tile": list(res.tile_shape)},
               **extra_inputs, li=np.asarray(li, np.int64), ri=np.asarray(ri, np.int64),
               res_coords=res.coords, res_values=res.values.astype(np.float32))

    w = wl.c1_block_sparse(seed=0, scale=8)
    lhs = STR(w.lhs.coords, w.lhs.values.astype(np.float64), w.lhs.shape, w.lhs.tile_shape)
    rhs = STR(w.rhs.coords, w.rhs.values.astype(np.float64), w.rhs.shape, w.rhs.tile_shape)
    run_exec("C1_small", lhs, rhs, w.join_keys, w.kernel_string, w.agg_keys,
             {**rel_arrays("lhs", lhs, np.float32), **rel_arrays("rhs", rhs, np.float32)})

    w = wl.c2_spmm(seed=0, scale=128, n_cols=64)
    coo = ssp.coo_matrix((w.lhs.values.astype(np.float64), (w.lhs.indices[:, 0], w.lhs.indices[:, 1])),
                         shape=w.lhs.shape)
    lhs = sp_mod.SparseTensor("A", coo).to_relation(w.lhs_tile)
    rhs = sp_mod.SparseTensor("B", w.rhs.astype(np.float64)).to_relation(w.rhs_tile)
    run_exec("C2_small", lhs, rhs, w.join_keys, w.kernel_string, w.agg_keys,
             {"a_indices": w.lhs.indices, "a_values": w.lhs.values, "a_shape": np.array(w.lhs.shape),
              "b_dense": w.rhs, "lhs_coords": lhs.coords, "rhs_coords": rhs.coords})

    w = wl.c3_batched_bf16(seed=0, scale=16, batch=2)
    lhs = STR(w.lhs.coords, w.lhs.values.astype(np.float64), w.lhs.shape, w.lhs.tile_shape)
    rhs = STR(w.rhs.coords, w.rhs.values.astype(np.float64), w.rhs.shape, w.rhs.tile_shape)
    run_exec("C3_small", lhs, rhs, w.join_keys, w.kernel_string, w.agg_keys,
             {**rel_arrays("lhs", lhs, np.float32), **rel_arrays("rhs", rhs, np.float32)})

    ch = wl.c4_chain(seed=0, scale=32)
    rels = {k: STR(ch[k].coords, ch[k].values.astype(np.float64), ch[k].shape, ch[k].tile_shape) for k in "ABC"}
    jax.F32 = True
    ab = sd.execute_sparse(rels["A"], rels["B"], [(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
    abc = sd.execute_sparse(ab, rels["C"], [(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
    jax.F32 = False
    l1, r1 = sd.coordinate_join(rels["A"], rels["B"], [(1, 0)])
    cs.put("C4_small", {"kind": "chain"}, **rel_arrays("A", rels["A"], np.float32),
           **rel_arrays("B", rels["B"], np.float32), **rel_arrays("C", rels["C"], np.float32), ab_coords=ab.coords, ab_values=ab.values.astype(np.float32),
           abc_coords=abc.coords, abc_values=abc.values.astype(np.float32), l1=l1, r1=r1)

    w = wl.c5_order3(seed=0, scale=32, n_out=32)
    dense = np.zeros(w.lhs.shape)
    dense[tuple(w.lhs.indices.T)] = w.lhs.values
    lhs = sp_mod.SparseTensor("X", dense).to_relation(w.lhs_tile)
    rhs = sp_mod.SparseTensor("W", w.rhs.astype(np.float64)).to_relation(w.rhs_tile)
    run_exec("C5_small", lhs, rhs, w.join_keys, w.kernel_string, w.agg_keys,
             {"x_indices": w.lhs.indices, "x_values": w.lhs.values, "x_shape": np.array(w.lhs.shape),
              "w_dense": w.rhs, "lhs_coords": lhs.coords, "rhs_coords": rhs.coords})
    cs.save(os.path.join(HERE, "golden_configs.npz"))
    print("wrote", len(st.arrays), "+", len(cs.arrays), "arrays")


if __name__ == "__main__":
    main()
