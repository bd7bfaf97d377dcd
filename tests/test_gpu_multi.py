"""Two ranks over NCCL, one GPU each: output-strip sharding (no data-path
collective, all-gather of the shards), contracted-range sharding (partial
tiles written in the order of the union of output coordinates, summed by a
reduce-scatter), each with and without the final gather, and element COO
split by rows before tiling, checked against the CPU oracle.

Skipped unless the host has at least two GPUs.
"""

import os
import socket

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
RTOL = 1e-5

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cases():
    import oracle as O
    rng = np.random.default_rng(11)
    out = []
    # C2-like: element-sparse lhs tiles (32 x 32), dense rhs row strip
    A = rng.standard_normal((512, 1024)) * (rng.random((512, 1024)) < 0.01)
    B = rng.standard_normal((1024, 256))
    out.append(("C2-like", O.relation_from_dense(A, (32, 32)), O.relation_from_dense(B, (32, 32)),
                ([(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])))
    # C1-like: block-sparse 128 x 128 tiles
    A = rng.standard_normal((1024, 1024)) * np.kron(rng.random((8, 8)) < 0.3, np.ones((128, 128)))
    B = rng.standard_normal((1024, 768)) * np.kron(rng.random((8, 6)) < 0.4, np.ones((128, 128)))
    out.append(("C1-like", O.relation_from_dense(A, (128, 128)), O.relation_from_dense(B, (128, 128)),
                ([(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])))
    return out


def _close(got, ref, mag):
    gc = got.coords.cpu().numpy()
    gv = got.values.float().cpu().numpy().astype(np.float64)
    return np.array_equal(gc, ref.coords) and gv.shape == ref.values.shape and bool(
        np.all(np.abs(gv - ref.values) <= RTOL * (np.abs(ref.values) + mag.values)))


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    results = []
    try:
        import oracle as O
        import einjax_b200 as E
        from einjax_b200 import distributed as D
        for name, lhs, rhs, (jk, ks, ak) in _cases():
            # fp32 operands (the tensor-core path); the oracle sums the same
            # fp32 values in float64
            lhs = O.Relation(lhs.coords, lhs.values.astype(np.float32).astype(np.float64), lhs.shape, lhs.tile_shape)
            rhs = O.Relation(rhs.coords, rhs.values.astype(np.float32).astype(np.float64), rhs.shape, rhs.tile_shape)
            ref = O.execute_sparse(lhs, rhs, jk, ks, ak)
            mag = O.execute_sparse(O.Relation(lhs.coords, np.abs(lhs.values), lhs.shape, lhs.tile_shape),
                                   O.Relation(rhs.coords, np.abs(rhs.values), rhs.shape, rhs.tile_shape), jk, ks, ak)
            dl = E.SparseTensorRelation.from_reference(lhs, dev, torch.float32)
            dr = E.SparseTensorRelation.from_reference(rhs, dev, torch.float32)
            for shard in ("output", "contracted"):
                got = E.execute_sharded_sparse(dl, dr, jk, ks, ak, shard=shard)
                results.append((name, shard, _close(got, ref, mag)))
                # without the gather: this rank's share, all-gathered here
                part = E.execute_sharded_sparse(dl, dr, jk, ks, ak, shard=shard, gather=False)
                gc = torch.cat(D.all_gather_rows(part.coords.contiguous()))
                gv = torch.cat(D.all_gather_rows(part.values.contiguous()))
                whole = E.SparseTensorRelation(gc, gv, part.shape, part.tile_shape)
                results.append((name, shard + "/no-gather", _close(whole, ref, mag)))
        # element COO split by rows before tiling (the benchmark's layout):
        # each rank tiles only its rows and passes lhs_sharded
        rng = np.random.default_rng(5)
        A = rng.standard_normal((1024, 2048)).astype(np.float32) * (rng.random((1024, 2048)) < 0.01)
        Bd = rng.standard_normal((2048, 256)).astype(np.float32)
        idx = np.argwhere(A != 0).astype(np.int32)
        val = A[A != 0]
        r0, r1 = D.balanced_row_ranges(idx, A.shape, (32, 32), world)[rank]
        keep = (idx[:, 0] >= r0) & (idx[:, 0] < r1)
        la = E.tile_coo(torch.from_numpy(idx[keep]).to(dev), torch.from_numpy(val[keep]).to(dev), A.shape, (32, 32))
        rb = E.tile_dense(torch.from_numpy(Bd).to(dev), (32, 32))
        mm = ([(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
        got = E.execute_sharded_sparse(la, rb, *mm, lhs_sharded=True)
        lr = O.relation_from_dense(A.astype(np.float64), (32, 32))
        rr = O.relation_from_dense(Bd.astype(np.float64), (32, 32))
        ref = O.execute_sparse(lr, rr, *mm)
        mag = O.execute_sparse(O.Relation(lr.coords, np.abs(lr.values), lr.shape, lr.tile_shape),
                               O.Relation(rr.coords, np.abs(rr.values), rr.shape, rr.tile_shape), *mm)
        results.append(("COO rows", "output/lhs_sharded", _close(got, ref, mag)))
        # order-3 contraction sharded over its contracted range (C5's layout)
        X = rng.standard_normal((64, 64, 128)).astype(np.float32) * (rng.random((64, 64, 128)) < 0.02)
        Wd = rng.standard_normal((128, 32)).astype(np.float32)
        xr = O.relation_from_dense(X.astype(np.float64), (16, 16, 16))
        wr = O.relation_from_dense(Wd.astype(np.float64), (16, 16))
        m5 = ([(2, 0)], "ijk,kl->ijl", [(0, 0), (0, 1), (1, 1)])
        ref = O.execute_sparse(xr, wr, *m5)
        mag = O.execute_sparse(O.Relation(xr.coords, np.abs(xr.values), xr.shape, xr.tile_shape),
                               O.Relation(wr.coords, np.abs(wr.values), wr.shape, wr.tile_shape), *m5)
        dx = E.SparseTensorRelation.from_reference(xr, dev, torch.float32)
        dw = E.SparseTensorRelation.from_reference(wr, dev, torch.float32)
        got = E.execute_sharded_sparse(dx, dw, *m5, shard="contracted")
        results.append(("order-3", "contracted", _close(got, ref, mag)))
        torch.cuda.synchronize()
        dist.barrier()
        q.put((rank, results))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_sharded_nccl_world2():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
    res = sorted(q.get(timeout=5) for _ in range(2))
    for p in procs:
        assert p.exitcode == 0
    for rank, results in res:
        for name, shard, ok in results:
            assert ok, f"rank {rank}: {name} sharded over {shard} differs from the oracle"
