"""Registration into the reference's own ``KernelRegistry`` (CPU).

Loads einjax's ``kernels/registry.py`` unchanged, through the numpy stand-in
for ``jax`` that the golden-vector generator uses (``tests/golden/_jaxstub``),
in a child process so the stand-in does not leak into other tests. Checks
that after ``register_b200_kernels`` the reference's own ``lookup`` returns
the B200 kernels for GPU backends (``"gpu"`` and ``"gpu:<x>"``) and still its
generic kernels for others, and that a B200 kernel hands back the reference's
``SparseTensorRelation``. The kernel's compute is replaced by the CPU oracle
here (no GPU); the adapters' conversion is what is under test.

The reference tree is found through ``EINJAX_REFERENCE`` or as ``reference``
next to this repository; the test is skipped when neither exists.
"""

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _reference_root():
    for p in (os.environ.get("EINJAX_REFERENCE"), os.path.join(os.path.dirname(ROOT), "reference")):
        if p and os.path.isfile(os.path.join(p, "kernels", "registry.py")):
            return p
    return None


CHILD = r'''
import importlib.util, json, os, sys
import numpy as np
root, ref = sys.argv[1], sys.argv[2]
sys.path.insert(0, root)
spec = importlib.util.spec_from_file_location("make_golden", os.path.join(root, "tests", "golden", "make_golden.py"))
mg = importlib.util.module_from_spec(spec)
spec.loader.exec_module(mg)
mods = mg.load_reference(ref)
R = mods["kernels.registry"]
SR = mods["tensor.sparse"].SparseTensorRelation
import einjax_b200 as E
from einjax_b200 import sparse_dispatch as SD
import oracle as O

class _Res:  # what the GPU path returns: a relation with to_numpy()
    def __init__(self, rel):
        self.rel, self.shape, self.tile_shape = rel, rel.shape, rel.tile_shape
    def to_numpy(self):
        return self.rel.coords, self.rel.values.astype(np.float32)

def fake_execute(lhs, rhs, jk, ks, ak, output_shape=None, output_tile_shape=None, **kw):
    return _Res(O.execute_sparse(O.Relation(lhs.coords, lhs.values, lhs.shape, lhs.tile_shape),
                                 O.Relation(rhs.coords, rhs.values, rhs.shape, rhs.tile_shape), jk, ks, ak))
SD.execute_sparse = fake_execute   # bound by the adapter when it is made

reg = R.KernelRegistry()
generic = reg.lookup("ij,jk->ik", backend="cpu", sparsity="sparse")
E.register_b200_kernels(reg, info_cls=R.KernelInfo)   # relation class defaults to the reference's
out = {}
out["mm_gpu"] = reg.lookup("ij,jk->ik", backend="gpu", sparsity="sparse").__name__
out["any_gpu_sub"] = reg.lookup("bij,bjk->bik", backend="gpu:triton", sparsity="sparse").__name__
out["cpu_unchanged"] = reg.lookup("ij,jk->ik", backend="cpu", sparsity="sparse") is generic
out["names"] = sorted(k.name for k in reg.list_kernels(sparsity="sparse"))
rng = np.random.default_rng(0)
A = rng.standard_normal((8, 12)) * (rng.random((8, 12)) < 0.5)
B = rng.standard_normal((12, 4))
lhs = mods["tensor.sparse"].SparseTensor("A", A).to_relation((4, 4))
rhs = mods["tensor.sparse"].SparseTensor("B", B).to_relation((4, 4))
fn = reg.lookup("bij,bjk->bik", backend="gpu", sparsity="sparse")
res = fn(lhs, rhs, [(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
out["result_is_reference_relation"] = isinstance(res, SR)
want = mods["execution.sparse_dispatch"].execute_sparse(lhs, rhs, [(1, 0)], "ij,jk->ik", [(0, 0), (1, 1)])
out["coords_equal"] = bool(np.array_equal(res.coords, want.coords))
out["values_close"] = bool(np.allclose(res.values, want.values, rtol=1e-5, atol=1e-6))
print("RESULT " + json.dumps(out))
'''


def test_register_into_reference_registry():
    ref = _reference_root()
    if ref is None:
        pytest.skip("the einjax reference tree is not available here")
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT, ref], capture_output=True, text=True, timeout=300)
    line = [x for x in r.stdout.splitlines() if x.startswith("RESULT ")]
    assert r.returncode == 0 and line, r.stderr[-3000:]
    out = json.loads(line[0][len("RESULT "):])
    assert out["mm_gpu"] == "b200_block_sparse_matmul"
    assert out["any_gpu_sub"] == "b200_sparse_einsum"
    assert out["cpu_unchanged"]
    assert {"b200_block_sparse_matmul", "b200_sparse_einsum"} <= set(out["names"])
    assert out["result_is_reference_relation"] and out["coords_equal"] and out["values_close"]
