"""Pending value fills of the tiling calls: coordinates at once, values
launched by the next count read or the first ``values`` access; results
equal to an immediate fill."""

import numpy as np
import pytest
import torch

import einjax_b200 as E
from einjax_b200 import sparse as S
from einjax_b200 import sparse_dispatch as SD

pytestmark = pytest.mark.gpu


def _coo(seed, shape=(256, 512), nnz=3000):
    g = np.random.default_rng(seed)
    idx = np.stack([g.integers(0, s, nnz) for s in shape], 1).astype(np.int32)
    val = g.standard_normal(nnz).astype(np.float32)
    return torch.from_numpy(idx).cuda(), torch.from_numpy(val).cuda()


def test_plan_count_read_launches_pending_fills():
    idx, val = _coo(0)
    A = E.tile_coo(idx, val, (256, 512), (32, 32))
    assert A.pending
    b = torch.randn(512, 64, device="cuda")
    B = E.tile_dense(b, (32, 64))  # a tiling's count read leaves A's fill pending
    assert A.pending and B.pending
    plan = SD.plan_pairs(A, B, [(1, 0)], [(0, 0), (1, 1)])  # the plan's count read launches both
    assert not A.pending and not B.pending
    ref = E.tile_coo(idx, val, (256, 512), (32, 32), marks=[])  # filled before returning
    assert not ref.pending
    torch.testing.assert_close(A.values, ref.values, rtol=0, atol=0)
    assert torch.equal(A.coords, ref.coords)
    dense = b.reshape(16, 32, 1, 64).permute(0, 2, 1, 3).reshape(16, 32, 64)
    torch.testing.assert_close(B.values, dense, rtol=0, atol=0)
    out = SD.tile_einsum("ij,jk->ik", A.values, B.values, plan.seg_lhs, plan.seg_rhs, plan.seg_offsets)
    a = np.zeros((256, 512))
    ih, vh = idx.cpu().numpy(), val.cpu().numpy()
    a[ih[:, 0], ih[:, 1]] = vh  # the last repeated entry wins, as in the tiling
    want = torch.from_numpy(a @ b.double().cpu().numpy()).float().cuda()
    got = torch.zeros_like(want)
    for o in range(plan.num_segments):
        i, k = (int(v) for v in plan.out_coords[o])
        got[i * 32:(i + 1) * 32, k * 64:(k + 1) * 64] = out[o]
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-4)


def test_pending_fill_on_first_values_access_and_other_stream():
    idx, val = _coo(1)
    A = E.tile_coo(idx, val, (256, 512), (32, 32))
    ref = E.tile_coo(idx, val, (256, 512), (32, 32), marks=[])
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        v = A.values.clone()  # filled on the creation stream, this stream waits for it
    s.synchronize()
    torch.testing.assert_close(v, ref.values, rtol=0, atol=0)


def test_input_changed_before_fill_raises():
    idx, val = _coo(2)
    A = E.tile_coo(idx, val, (256, 512), (32, 32))
    val.mul_(2.0)
    with pytest.raises(RuntimeError, match="changed in place"):
        A.materialize()
    d = torch.randn(64, 64, device="cuda")
    B = E.tile_dense(d, (32, 32))
    d.zero_()
    with pytest.raises(RuntimeError, match="changed in place"):
        _ = B.values
    S.launch_pending_fills()


def test_unresolved_tilings_resolve_together_and_raise_late():
    idx, val = _coo(3)
    A = E.tile_coo(idx, val, (256, 512), (32, 32))
    B = E.tile_dense(torch.randn(512, 64, device="cuda"), (32, 64))
    assert A._finish is not None and B._finish is not None
    assert A.device.type == "cuda"  # known without resolving
    _ = A.num_tuples  # one wait resolves both
    assert A._finish is None and B._finish is None
    assert B.pending  # its values are still a pending fill
    S.launch_pending_fills()
    bad = torch.tensor([[0, 0], [4, 1]], dtype=torch.int32, device="cuda")
    R = E.tile_coo(bad, torch.ones(2, device="cuda"), (4, 4), (2, 2))  # no wait, no error yet
    with pytest.raises(ValueError):
        _ = R.coords
    with pytest.raises(ValueError):  # every later use raises again
        _ = R.values
    with pytest.raises(ValueError):  # the reference-facing call raises at once
        E.SparseTensor("t", (bad.cpu().numpy(), np.ones(2), (4, 4))).to_relation((2, 2))


def test_fill_overlaps_gemm_grouping_and_matches_eager():
    """execute_sparse with the tile fill on the fill stream (the GEMM waits
    for it inside the call) equals the same call on filled operands."""
    idx, val = _coo(4, shape=(512, 1024), nnz=20000)
    b = torch.randn(1024, 128, device="cuda")
    A = E.tile_coo(idx, val, (512, 1024), (32, 32))
    B = E.tile_dense(b, (32, 32))
    got = E.execute_sparse(A, B, [(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
    A2 = E.tile_coo(idx, val, (512, 1024), (32, 32)).materialize()
    B2 = E.tile_dense(b, (32, 32)).materialize()
    torch.cuda.synchronize()
    want = E.execute_sparse(A2, B2, [(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
    assert torch.equal(got.coords, want.coords)
    assert torch.equal(got.values, want.values)
    lv, ready = A.values_and_ready()
    assert ready is not None and ready[1].query() in (True, False)
