"""The C-ABI library loads on a CPU-only host and exports what include/*.h declares.

Only host-side entry points (version, status strings, workspace-size
queries, kernel-string parsing) are called here; nothing launches a kernel.
"""

import ctypes
import glob
import os
import re

import pytest

from einjax_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        txt = open(h).read()
        names |= set(re.findall(r"^(?:int|size_t|int64_t|void|const char\*)\s+(es_\w+)\(", txt, re.M))
    return names


def test_library_exports_every_declared_symbol():
    lib = L.load()
    declared = _declared()
    assert len(declared) >= 20
    for name in declared:
        assert hasattr(lib, name), name
    assert declared == set(L.SIGNATURES), "ctypes binding and header disagree"


def test_host_entry_points():
    lib = L.load()
    assert lib.es_version() >= 100
    assert lib.es_status_string(0) == b"ok"
    assert lib.es_tile_coo_workspace_size(1000, 2, L.i64arr([64, 64]), L.i64arr([8, 8])) > 0
    assert lib.es_tile_coo_workspace_size(10, 2, L.i64arr([6, 6]), L.i64arr([4, 4])) == 0  # not divisible
    assert lib.es_join_workspace_size(100, 100) > 0
    assert lib.es_segments_workspace_size(1 << 20) > (1 << 20) * 8


@pytest.mark.parametrize("ks,lt,rt,want", [
    ("ij,jk->ik", (2, 3), (3, 4), (2, 4)),
    ("i,j->ij", (3,), (4,), (3, 4)),
    ("i,i->", (5,), (5,), ()),
    ("ii,ij->j", (3, 3), (3, 4), (4,)),
    ("ijk,kl->ijl", (16, 16, 16), (16, 16), (16, 16, 16)),
    ("bij,bjk->bik", (1, 64, 64), (1, 64, 64), (1, 64, 64)),
    ("ij,kl->ij", (2, 3), (4, 2), (2, 3)),
])
def test_out_tile_shape(ks, lt, rt, want):
    lib = L.load()
    out = L.i64arr([0] * 8)
    nd = lib.es_out_tile_shape(ks.encode(), L.i64arr(lt), len(lt), L.i64arr(rt), len(rt), out)
    assert nd == len(want)
    assert tuple(out[i] for i in range(nd)) == want


@pytest.mark.parametrize("ks,lt,rt", [
    ("ij,jk", (2, 3), (3, 4)),          # no arrow
    ("ij,jk->ik", (2, 3), (4, 4)),      # size conflict on j
    ("ij,jk->iz", (2, 3), (3, 4)),      # output label absent from inputs
    ("ij,jk->ii", (2, 3), (3, 4)),      # repeated output label
    ("ijk,jk->ik", (2, 3), (3, 4)),     # operand rank mismatch
])
def test_out_tile_shape_rejects(ks, lt, rt):
    lib = L.load()
    out = L.i64arr([0] * 8)
    assert lib.es_out_tile_shape(ks.encode(), L.i64arr(lt), len(lt), L.i64arr(rt), len(rt), out) < 0


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    monkeypatch.setattr(L, "_LIB", None)
    with pytest.raises(L.EinsparseUnavailable):
        L.load(str(tmp_path / "nope.so"))
    L._LIB = None
    L.load()
