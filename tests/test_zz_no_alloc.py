"""The allocation-free join entry point (``es_join_static``) against the
regular join (``es_join_plan`` + ``es_join_fill``), through the C ABI.

Some callers cannot allocate device memory at the moment they join (a host
callback, an engine that reserves all memory up front, a plugin whose host
framework owns every buffer); ``es_join_static`` serves them by taking its
scratch from a fixed array inside the library. Pair indices are integers, so
the comparison is exact: same pairs, same order. Two calls in a row check
that the second call is not affected by what the first left in the shared
array. This file is collected last so a failure here does not hide others.
"""

import numpy as np
import pytest
import torch

from einjax_b200 import _lib as L
from einjax_b200.sparse import read_counts, stream_ptr, workspace

pytestmark = pytest.mark.gpu


def _regular_join(lc, rc, keys, ext):
    lib = L.lib()
    dev = lc.device
    nl, nr = lc.shape[0], rc.shape[0]
    ws = workspace(lib.es_join_workspace_size(nl, nr), dev)
    cnt = torch.zeros(2, dtype=torch.int64, device=dev)
    flat = [v for k in keys for v in k]
    L.check("es_join_plan", lib.es_join_plan(lc.data_ptr(), nl, lc.shape[1], rc.data_ptr(), nr, rc.shape[1],
                                             L.i32arr(flat), len(keys), L.i64arr(ext), ws.data_ptr(), ws.numel(),
                                             cnt.data_ptr(), cnt[1:].data_ptr(), stream_ptr(dev)))
    P, err = read_counts(cnt)
    assert err == 0
    li = torch.empty(P, dtype=torch.int64, device=dev)
    ri = torch.empty(P, dtype=torch.int64, device=dev)
    L.check("es_join_fill", lib.es_join_fill(nl, nr, len(keys), ws.data_ptr(), ws.numel(), P, li.data_ptr(),
                                             ri.data_ptr(), L.ES_I64, stream_ptr(dev)))
    return li.cpu().numpy(), ri.cpu().numpy()


def _static_join(lc, rc, keys, ext, capacity, index_dtype=torch.int64):
    lib = L.lib()
    dev = lc.device
    li = torch.full((capacity,), -1, dtype=index_dtype, device=dev)
    ri = torch.full((capacity,), -1, dtype=index_dtype, device=dev)
    cnt = torch.zeros(2, dtype=torch.int64, device=dev)
    flat = [v for k in keys for v in k]
    code = L.ES_I64 if index_dtype == torch.int64 else L.ES_I32
    L.check("es_join_static", lib.es_join_static(
        lc.data_ptr(), lc.shape[0], lc.shape[1], rc.data_ptr(), rc.shape[0], rc.shape[1], L.i32arr(flat), len(keys),
        L.i64arr(ext), li.data_ptr(), ri.data_ptr(), code, capacity, cnt.data_ptr(), cnt[1:].data_ptr(),
        stream_ptr(dev)))
    P, err = read_counts(cnt)
    return P, err, li.cpu().numpy(), ri.cpu().numpy()


def _case(seed, nl, nr, hi):
    rng = np.random.default_rng(seed)
    lc = torch.from_numpy(rng.integers(0, hi, (nl, 2)).astype(np.int32)).cuda()
    rc = torch.from_numpy(rng.integers(0, hi, (nr, 2)).astype(np.int32)).cuda()
    return lc, rc


def test_static_join_matches_regular_join_twice():
    keys = [(1, 0)]
    # first a larger join, then a smaller one reusing the same shared array
    for seed, nl, nr, hi in [(1, 60000, 50000, 700), (2, 3000, 4000, 50)]:
        lc, rc = _case(seed, nl, nr, hi)
        ext = [hi]
        want_l, want_r = _regular_join(lc, rc, keys, ext)
        P, err, got_l, got_r = _static_join(lc, rc, keys, ext, capacity=want_l.size + 16)
        assert err == 0
        assert P == want_l.size
        np.testing.assert_array_equal(got_l[:P], want_l)
        np.testing.assert_array_equal(got_r[:P], want_r)
        assert np.all(got_l[P:] == -1)


def test_static_join_limits():
    lib = L.lib()
    lc, rc = _case(3, 200, 300, 20)
    P, err, got_l, _ = _static_join(lc, rc, [(1, 0)], [20], capacity=10)
    assert err == L.ES_ERR_WORKSPACE and P > 10
    want_l, _ = _regular_join(lc, rc, [(1, 0)], [20])
    np.testing.assert_array_equal(got_l[:10], want_l[:10])
    big = torch.zeros((65537, 2), dtype=torch.int32, device="cuda")
    cnt = torch.zeros(2, dtype=torch.int64, device="cuda")
    out = torch.empty(4, dtype=torch.int64, device="cuda")
    st = lib.es_join_static(big.data_ptr(), 65537, 2, big.data_ptr(), 10, 2, L.i32arr([1, 0]), 1, L.i64arr([1]),
                            out.data_ptr(), out.data_ptr(), L.ES_I64, 4, cnt.data_ptr(), cnt[1:].data_ptr(),
                            stream_ptr(big.device))
    assert st == L.ES_ERR_UNSUPPORTED


def test_static_join_at_the_tile_limit():
    # exactly 65536 tiles per side: the largest input the fixed array serves
    lc, rc = _case(4, 65536, 65536, 4096)
    keys, ext = [(1, 0)], [4096]
    want_l, want_r = _regular_join(lc, rc, keys, ext)
    P, err, got_l, got_r = _static_join(lc, rc, keys, ext, capacity=want_l.size)
    assert err == 0 and P == want_l.size
    np.testing.assert_array_equal(got_l, want_l)
    np.testing.assert_array_equal(got_r, want_r)


def test_static_join_int32_outputs():
    lc, rc = _case(5, 5000, 7000, 300)
    keys, ext = [(1, 0), (0, 1)], [300, 300]
    want_l, want_r = _regular_join(lc, rc, keys, ext)
    P, err, got_l, got_r = _static_join(lc, rc, keys, ext, capacity=want_l.size + 8, index_dtype=torch.int32)
    assert err == 0 and P == want_l.size
    np.testing.assert_array_equal(got_l[:P].astype(np.int64), want_l)
    np.testing.assert_array_equal(got_r[:P].astype(np.int64), want_r)
    assert np.all(got_l[P:] == -1)


def test_static_join_capped_cross_product():
    # no join keys: the lhs-major cross product, cut at the capacity
    lc, rc = _case(6, 300, 200, 10)
    want_l, want_r = _regular_join(lc, rc, [], [])
    assert want_l.size == 300 * 200
    cap = 1000
    P, err, got_l, got_r = _static_join(lc, rc, [], [], capacity=cap)
    assert err == L.ES_ERR_WORKSPACE and P == 300 * 200
    np.testing.assert_array_equal(got_l, want_l[:cap])
    np.testing.assert_array_equal(got_r, want_r[:cap])
