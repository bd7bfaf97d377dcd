"""World-size-2 CPU (gloo) tests of the multi-GPU host logic.

The per-rank tile arithmetic is the GPU library's job and is not available on
a CPU host, so each rank here computes its share with the CPU oracle; what
is under test is the partitioning, the all-gather of shards and the sparse
reduce-scatter of partial output tiles.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(seed=3):
    import oracle as O
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((32, 48)) * (rng.random((32, 48)) < 0.15)
    B = rng.standard_normal((48, 24)) * (rng.random((48, 24)) < 0.15)
    return O.relation_from_dense(A, (4, 4)), O.relation_from_dense(B, (4, 4))


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle as O
        from einjax_b200 import distributed as D
        lhs, rhs = _case()
        mm = ([(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
        full = O.execute_sparse(lhs, rhs, *mm)

        # output-tile sharding: balanced segment ranges, shard, all-gather
        li, ri = O.coordinate_join(lhs.coords, rhs.coords, mm[0])
        oc = O.compute_output_coords(lhs.coords, rhs.coords, li, ri, mm[2])
        uc, inv = np.unique(oc, axis=0, return_inverse=True)
        order = np.argsort(inv.reshape(-1), kind="stable")
        counts = np.bincount(inv.reshape(-1))
        so = np.concatenate([[0], np.cumsum(counts)])
        s0, s1 = D.balanced_segment_ranges(so, world)[rank]
        vals = np.zeros((s1 - s0, 4, 4))
        for s in range(s0, s1):
            for p in order[so[s]:so[s + 1]]:
                vals[s - s0] += lhs.values[li[p]] @ rhs.values[ri[p]]
        gc = torch.cat(D.all_gather_rows(torch.from_numpy(uc[s0:s1].astype(np.int32))))
        gv = torch.cat(D.all_gather_rows(torch.from_numpy(vals)))
        ok1 = np.array_equal(gc.numpy(), full.coords) and np.allclose(gv.numpy(), full.values, atol=1e-12)

        # contracted sharding: key ranges over lhs column tiles, partial
        # products per rank, sparse reduce-scatter of the partials
        kcounts = np.bincount(lhs.coords[:, 1], minlength=lhs.shape[1] // lhs.tile_shape[1])
        k0, k1 = D.balanced_key_ranges(kcounts, world)[rank]
        keep = (lhs.coords[:, 1] >= k0) & (lhs.coords[:, 1] < k1)
        local = O.Relation(lhs.coords[keep], lhs.values[keep], lhs.shape, lhs.tile_shape)
        part = O.execute_sparse(local, rhs, *mm)
        c, v = D.sparse_reduce_scatter(torch.from_numpy(part.coords), torch.from_numpy(part.values))
        ok2 = np.array_equal(c.numpy(), full.coords) and np.allclose(v.numpy(), full.values, atol=1e-12)
        c2, v2 = D.sparse_reduce_scatter(torch.from_numpy(part.coords), torch.from_numpy(part.values), gather=False)
        gc2 = torch.cat(D.all_gather_rows(c2.contiguous()))
        gv2 = torch.cat(D.all_gather_rows(v2.contiguous()))
        ok3 = np.array_equal(gc2.numpy(), full.coords) and np.allclose(gv2.numpy(), full.values, atol=1e-12)
        q.put((rank, ok1, ok2, ok3))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(180)
def test_sharded_paths_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(150)
    res = sorted(q.get(timeout=5) for _ in range(2))
    for p in procs:
        assert p.exitcode == 0
    assert all(r[1] for r in res), "output-tile sharding + all-gather mismatch"
    assert all(r[2] for r in res), "contracted sharding + reduce-scatter mismatch"
    assert all(r[3] for r in res), "reduce-scatter without gather mismatch"
