"""World-size-2 CPU (gloo) tests of the multi-GPU host logic.

The per-rank tile arithmetic is the GPU library's job and is not available on
a CPU host, so each rank computes its share with the CPU oracle. Under test
are the functions of ``einjax_b200.distributed`` that decide and move the
shares: ``output_strip_ranges`` (output sharding of tile relations),
``balanced_row_ranges`` (output sharding of element COO before tiling),
``contracted_key_range`` and ``sparse_reduce_scatter`` (contracted sharding;
the coordinate union is passed in, computed here with numpy), and the
all-gather of shards.
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


def _dense(seed=3):
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((32, 48)) * (rng.random((32, 48)) < 0.15)
    B = rng.standard_normal((48, 24)) * (rng.random((48, 24)) < 0.15)
    return A, B


def _device_rel(rel):
    """The oracle relation as this package's relation of CPU tensors (what
    the sharding functions read: coords, shape, tile_shape)."""
    from einjax_b200.sparse import SparseTensorRelation
    return SparseTensorRelation(torch.from_numpy(rel.coords.astype(np.int32)), torch.from_numpy(rel.values),
                                rel.shape, rel.tile_shape)


def _oracle_union(coords, extents, group=None):
    """numpy stand-in for the library's coordinate union (all-gather, then
    np.unique with inverse)."""
    from einjax_b200 import distributed as D
    rank, n = D.world(group)
    parts = D.all_gather_rows(coords.contiguous(), group)
    off = sum(int(p.shape[0]) for p in parts[:rank])
    allc = torch.cat(parts).numpy()
    uc, inv = np.unique(allc, axis=0, return_inverse=True)
    inv = inv.reshape(-1)
    return torch.from_numpy(uc.astype(np.int32)), torch.from_numpy(inv[off:off + coords.shape[0]].astype(np.int32))


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle as O
        from einjax_b200 import distributed as D
        A, B = _dense()
        lhs, rhs = O.relation_from_dense(A, (4, 4)), O.relation_from_dense(B, (4, 4))
        mm = ([(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
        full = O.execute_sparse(lhs, rhs, *mm)
        res = {}

        # output sharding of tile relations: strip ranges balanced by pairs
        ranges = D.output_strip_ranges(_device_rel(lhs), _device_rel(rhs), mm[0], mm[2], world)
        t0, t1 = ranges[rank]
        assert ranges[0][0] == 0 and ranges[-1][1] == lhs.coords.shape[0]
        assert all(ranges[r][1] == ranges[r + 1][0] for r in range(world - 1))
        local = O.Relation(lhs.coords[t0:t1], lhs.values[t0:t1], lhs.shape, lhs.tile_shape)
        # no strip is split between ranks
        if 0 < t0 < lhs.coords.shape[0]:
            assert lhs.coords[t0 - 1, 0] != lhs.coords[t0, 0]
        part = O.execute_sparse(local, rhs, *mm)
        gc = torch.cat(D.all_gather_rows(torch.from_numpy(part.coords.astype(np.int32))))
        gv = torch.cat(D.all_gather_rows(torch.from_numpy(part.values)))
        res["strips"] = np.array_equal(gc.numpy(), full.coords) and np.allclose(gv.numpy(), full.values, atol=1e-12)
        # balance: each rank within one strip's pairs of P / world
        li, _ = O.coordinate_join(lhs.coords, rhs.coords, mm[0])
        per_tile = np.bincount(li, minlength=lhs.coords.shape[0])
        strip_pairs = np.bincount(lhs.coords[:, 0], weights=per_tile)
        mine = per_tile[t0:t1].sum()
        res["balanced"] = abs(mine - per_tile.sum() / world) <= strip_pairs.max()

        # output sharding of element COO before tiling: tile-aligned row ranges
        idx = np.argwhere(A != 0).astype(np.int32)
        val = A[A != 0]
        rr = D.balanced_row_ranges(idx, A.shape, (4, 4), world)
        r0, r1 = rr[rank]
        assert r0 % 4 == 0 and r1 % 4 == 0 and rr[-1][1] == A.shape[0]
        keep = (idx[:, 0] >= r0) & (idx[:, 0] < r1)
        mine_rel = O.to_relation(idx[keep], val[keep], A.shape, (4, 4))
        part = O.execute_sparse(mine_rel, rhs, *mm)
        gc = torch.cat(D.all_gather_rows(torch.from_numpy(part.coords.astype(np.int32))))
        gv = torch.cat(D.all_gather_rows(torch.from_numpy(part.values)))
        res["rows"] = np.array_equal(gc.numpy(), full.coords) and np.allclose(gv.numpy(), full.values, atol=1e-12)

        # contracted sharding: key ranges over lhs column tiles, partial
        # products per rank, reduce-scatter over the union of coordinates
        k0, k1 = D.contracted_key_range(_device_rel(lhs), mm[0], world, rank)
        keep = (lhs.coords[:, 1] >= k0) & (lhs.coords[:, 1] < k1)
        local = O.Relation(lhs.coords[keep], lhs.values[keep], lhs.shape, lhs.tile_shape)
        part = O.execute_sparse(local, rhs, *mm)
        ext = [A.shape[0] // 4, B.shape[1] // 4]
        pc, pv = torch.from_numpy(part.coords.astype(np.int32)), torch.from_numpy(part.values)
        c, v = D.sparse_reduce_scatter(pc, pv, extents=ext, union=_oracle_union)
        res["contracted"] = np.array_equal(c.numpy(), full.coords) and np.allclose(v.numpy(), full.values,
                                                                                  atol=1e-12)
        c2, v2 = D.sparse_reduce_scatter(pc, pv, gather=False, extents=ext, union=_oracle_union)
        gc2 = torch.cat(D.all_gather_rows(c2.contiguous()))
        gv2 = torch.cat(D.all_gather_rows(v2.contiguous()))
        res["contracted_nogather"] = np.array_equal(gc2.numpy(), full.coords) and np.allclose(
            gv2.numpy(), full.values, atol=1e-12)
        # extents found by the collective when the caller gives none
        c3, v3 = D.sparse_reduce_scatter(pc, pv, union=_oracle_union)
        res["contracted_extents"] = np.array_equal(c3.numpy(), full.coords)
        q.put((rank, res))
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
    res = sorted((q.get(timeout=5) for _ in range(2)), key=lambda x: x[0])
    for p in procs:
        assert p.exitcode == 0
    for rank, r in res:
        for name, ok in r.items():
            assert ok, f"rank {rank}: {name} mismatch"


def test_balanced_row_ranges_cover_and_balance():
    from einjax_b200 import distributed as D
    rng = np.random.default_rng(0)
    # skewed rows: most tiles in the first strips
    rows = np.minimum((rng.pareto(1.2, 20000) * 20).astype(np.int64), 1023)
    cols = rng.integers(0, 1024, 20000)
    idx = np.stack([rows, cols], 1).astype(np.int32)
    for n in (1, 2, 3, 8):
        rr = D.balanced_row_ranges(idx, (1024, 1024), (32, 32), n)
        assert rr[0][0] == 0 and rr[-1][1] == 1024 and len(rr) == n
        assert all(a % 32 == 0 and b % 32 == 0 and a <= b for a, b in rr)
        assert all(rr[i][1] == rr[i + 1][0] for i in range(n - 1))
