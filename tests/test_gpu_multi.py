"""Two ranks over NCCL, one GPU each: output-tile sharding (no data-path
collective, all-gather of the shards) and contracted-range sharding (partial
tiles summed by the sparse reduce-scatter), checked against the CPU oracle.

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
                gc = got.coords.cpu().numpy()
                gv = got.values.float().cpu().numpy().astype(np.float64)
                ok = np.array_equal(gc, ref.coords) and bool(
                    np.all(np.abs(gv - ref.values) <= RTOL * (np.abs(ref.values) + mag.values)))
                results.append((name, shard, ok))
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
