"""GPU parity of the sparse plan executor (``execute_sparse_plan``): multi-step
plans against the reference's own plan results (golden vectors from
``ExecutionEngine.execute_plan`` over the dense operands and from its sparse
``execute_sparse`` chained in plan order), against the oracle's plan walk on
larger random chains, and gradients through a plan against a float64 dense
autograd reference.

Tolerances: output tile coordinates bit-exact and in order; fp32 values within
|got - ref| <= 1e-5 * (|ref| + mag) per element, mag being the same plan over
absolute values; bf16 operands within 2e-2 of the same bound.
"""

import numpy as np
import pytest
import torch

import einjax_b200 as E
import oracle as O
from golden_io import cases_of_kind, load_cases

pytestmark = pytest.mark.gpu

PLAN = load_cases("golden_plan.npz")
RTOL32 = 1e-5
RTOL_BF16 = 2e-2


def _ops(c):
    return [O.Relation(c[f"op{i}_coords"], c[f"op{i}_values"].astype(np.float64),
                       tuple(int(v) for v in c[f"op{i}_shape"]), tuple(int(v) for v in c[f"op{i}_tile"]))
            for i in range(c.meta["n_ops"])]


def _abs(ops):
    return [O.Relation(r.coords, np.abs(r.values), r.shape, r.tile_shape) for r in ops]


def _dev(r, dtype=None):
    return E.SparseTensorRelation.from_arrays(r.coords, r.values, r.shape, r.tile_shape, dtype=dtype)


def _check(res, ref, mag, rtol):
    c, v = res.to_numpy()
    ok, msg = O.relation_allclose(c, v, ref, rtol=rtol, mag=mag)
    assert ok, msg


@pytest.mark.parametrize("form", ["tuples", "steps", "path"])
@pytest.mark.parametrize("name", sorted(cases_of_kind("plan", "golden_plan.npz")))
def test_plan_golden(name, form):
    c = PLAN[name]
    m = c.meta
    if form == "tuples":
        steps = [(s["formula"], tuple(s["input_indices"])) for s in m["steps"]]
    elif form == "steps":
        steps = [E.PlanStep(s["formula"], tuple(s["input_indices"])) for s in m["steps"]]
    else:
        steps = E.plan_from_path(m["einsum"], m["path"])
    ops = _ops(c)
    res = E.execute_sparse_plan(steps, [_dev(r) for r in ops])
    assert list(res.shape) == m["res_shape"] and list(res.tile_shape) == m["res_tile"]
    osteps = [(s["formula"], tuple(s["input_indices"])) for s in m["steps"]]
    mag = O.execute_plan(osteps, _abs(ops)).values
    ref = O.Relation(c["res_coords"], c["res_values"], tuple(m["res_shape"]), tuple(m["res_tile"]))
    _check(res, ref, mag, RTOL32)
    got = res.to_dense().cpu().numpy().astype(np.float64)
    magd = O.execute_plan(osteps, _abs(ops)).to_dense()
    assert np.all(np.abs(got - c["out_dense"]) <= RTOL32 * (np.abs(c["out_dense"]) + magd) + 1e-12)


def _random_rel(rng, shape, tile, tile_density, elem_density=1.0):
    grid = [s // t for s, t in zip(shape, tile)]
    n = int(np.prod(grid))
    keep = np.flatnonzero(rng.random(n) < tile_density)
    coords = np.stack(np.unravel_index(keep, grid), 1).astype(np.int32)
    vals = rng.standard_normal((len(keep), *tile)) * (rng.random((len(keep), *tile)) < elem_density)
    return O.Relation(coords, vals, tuple(shape), tuple(tile))


CHAINS = {
    # einsum, path, operand shapes, tile shapes, tile density
    "chain4_t32": ("ij,jk,kl,lm->im", [(1, 2), (0, 2), (0, 1)],
                   [(512, 384), (384, 640), (640, 256), (256, 320)], [(32, 32)] * 4, 0.25),
    "mixed_t64_t32": ("ij,jk,kl->il", [(0, 1), (0, 1)], [(512, 512), (512, 256), (256, 384)],
                      [(64, 64), (64, 32), (32, 32)], 0.3),
    "batched_order3": ("bij,bjk,kl->bil", [(0, 1), (0, 1)], [(4, 128, 96), (4, 96, 64), (64, 80)],
                       [(1, 32, 32), (1, 32, 32), (32, 16)], 0.4),
}


@pytest.mark.parametrize("name", sorted(CHAINS))
def test_plan_random_chain_vs_oracle(name):
    es, path, shapes, tiles, dens = CHAINS[name]
    rng = np.random.default_rng(len(name))
    ops = [_random_rel(rng, s, t, dens) for s, t in zip(shapes, tiles)]
    steps = E.plan_from_path(es, path)
    res = E.execute_sparse_plan(steps, [_dev(r) for r in ops])
    osteps = [(s.formula, s.input_indices) for s in steps]
    ref = O.execute_plan(osteps, ops)
    _check(res, ref, O.execute_plan(osteps, _abs(ops)).values, RTOL32)


def test_plan_bf16_operands():
    es, path, shapes, tiles, dens = CHAINS["chain4_t32"]
    rng = np.random.default_rng(11)
    ops = [_random_rel(rng, s, t, dens) for s, t in zip(shapes, tiles)]
    dev = [_dev(r, torch.bfloat16) for r in ops]
    ops_b = [O.Relation(r.coords, d.values.float().cpu().numpy().astype(np.float64), r.shape, r.tile_shape)
             for r, d in zip(ops, dev)]
    steps = E.plan_from_path(es, path)
    res = E.execute_sparse_plan(steps, dev)
    osteps = [(s.formula, s.input_indices) for s in steps]
    _check(res, O.execute_plan(osteps, ops_b), O.execute_plan(osteps, _abs(ops_b)).values, RTOL_BF16)


def test_plan_empty_intermediate_and_single_step():
    a = O.relation_from_dense(np.diag(np.arange(1.0, 9.0)), (4, 4))
    b = O.relation_from_dense(np.zeros((8, 8)), (4, 4))
    c = O.relation_from_dense(np.ones((8, 8)), (4, 4))
    res = E.execute_sparse_plan([("ij,jk->ik", (0, 1)), ("ik,kl->il", (0, 1))], [_dev(a), _dev(b), _dev(c)])
    assert res.num_tuples == 0 and res.shape == (8, 8)
    one = E.execute_sparse_plan([("ij,jk->ik", (0, 1))], [_dev(a), _dev(c)])
    ref = O.execute_sparse(a, c, [(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
    _check(one, ref, O.execute_sparse(_abs([a])[0], c, [(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)]).values, RTOL32)


def _tile_mask(r):
    m = np.zeros(r.shape)
    for co in r.coords:
        m[tuple(slice(int(x) * t, (int(x) + 1) * t) for x, t in zip(co, r.tile_shape))] = 1.0
    return m


def test_plan_gradients_vs_dense_autograd():
    """sum(out * G) through a 3-step plan: gradients of every operand's tile
    values against float64 torch autograd of the dense einsum chain,
    restricted to each operand's tile support."""
    es, path, shapes, tiles, dens = CHAINS["chain4_t32"]
    rng = np.random.default_rng(3)
    ops = [_random_rel(rng, s, t, dens) for s, t in zip(shapes, tiles)]
    dev = [_dev(r) for r in ops]
    for d in dev:
        d.values.requires_grad_(True)
    steps = E.plan_from_path(es, path)
    res = E.execute_sparse_plan(steps, dev, differentiable=True)
    G = rng.standard_normal(res.shape)
    res_g = O.relation_from_dense(G, res.tile_shape)
    gt = torch.from_numpy(O.Relation(res_g.coords, res_g.values, res.shape, res.tile_shape).to_dense()).cuda()
    loss = (res.to_dense() * gt.float()).sum()
    loss.backward()

    dense = [torch.from_numpy(r.to_dense()).requires_grad_(True) for r in ops]
    torch.einsum(es, *dense).mul(torch.from_numpy(G)).sum().backward()
    dense_abs = [torch.from_numpy(np.abs(r.to_dense())).requires_grad_(True) for r in ops]
    torch.einsum(es, *dense_abs).mul(torch.from_numpy(np.abs(G))).sum().backward()
    for r, d, ref, mag in zip(ops, dev, dense, dense_abs):
        assert d.values.grad is not None
        got = E.SparseTensorRelation(d.coords, d.values.grad, r.shape, r.tile_shape).to_dense().cpu().numpy()
        mask = _tile_mask(r)
        want = ref.grad.numpy() * mask
        assert np.all(np.abs(got - want) <= RTOL32 * (np.abs(want) + mag.grad.numpy() * mask) + 1e-12)
