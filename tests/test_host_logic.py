"""Host-side logic that needs no GPU: registry dispatch, partitioning helpers,
kernel-string helpers — checked against the reference's golden vectors and
against the reference tests' expectations (tests/test_pallas.py:346-525)."""

import numpy as np
import pytest

import einjax_b200 as E
from einjax_b200 import distributed as D
from golden_io import load_cases

H = load_cases()["helpers"].meta


def test_helpers_match_reference():
    for s, want in H["add_batch_dim"].items():
        assert E._add_batch_dim(s) == want
    for s, a, b, want in H["infer_tile"]:
        assert list(E._infer_output_tile_shape(s, tuple(a), tuple(b))) == want
    for s, want in H["reverse"].items():
        assert list(E._reverse_einsum_string(s)) == want
    for n, d, want in H["partition"]:
        assert [list(p) for p in E._partition_matched_pairs(n, d)] == want
    with pytest.raises(ValueError):
        E._add_batch_dim("ij,jk")


def test_partition_spec_matches_reference():
    for shape, tile, want in H["partition_spec"]:
        if want == "ValueError":
            with pytest.raises(ValueError):
                E.tile_shape_to_partition_spec(tuple(shape), tuple(tile))
        else:
            assert list(E.tile_shape_to_partition_spec(tuple(shape), tuple(tile))) == want


def test_register_into_foreign_registry():
    """The adapters register into any registry with the reference's interface."""

    class ForeignInfo:
        def __init__(self, name, pattern, backend, sparsity, priority, kernel_fn):
            self.name, self.pattern, self.backend = name, pattern, backend
            self.sparsity, self.priority, self.kernel_fn = sparsity, priority, kernel_fn

    class ForeignRegistry:
        def __init__(self):
            self.k = []

        def register(self, ki):
            self.k.append(ki)

    r = E.register_b200_kernels(ForeignRegistry(), info_cls=ForeignInfo)
    names = {k.name: k for k in r.k}
    assert set(names) == {"b200_block_sparse_matmul", "b200_sparse_einsum"}
    assert names["b200_sparse_einsum"].pattern == "*" and names["b200_sparse_einsum"].backend == "gpu"


@pytest.mark.parametrize("n_ranks", [1, 2, 3, 4, 8])
def test_balanced_segment_ranges(n_ranks):
    rng = np.random.default_rng(n_ranks)
    counts = rng.zipf(1.5, size=500).clip(max=2000)
    so = np.concatenate([[0], np.cumsum(counts)])
    parts = D.balanced_segment_ranges(so, n_ranks)
    assert parts[0][0] == 0 and parts[-1][1] == 500
    for (a, b), (c, d) in zip(parts, parts[1:]):
        assert b == c and a <= b
    loads = [so[b] - so[a] for a, b in parts]
    assert sum(loads) == so[-1]
    assert max(loads) <= so[-1] / n_ranks + counts.max()


def test_balanced_segment_ranges_edge():
    assert D.balanced_segment_ranges(np.array([0]), 4) == [(0, 0)] * 4
    parts = D.balanced_segment_ranges(np.array([0, 5]), 4)
    assert sum(b - a for a, b in parts) == 1


@pytest.mark.parametrize("n_ranks", [1, 2, 4, 8])
def test_balanced_key_ranges(n_ranks):
    rng = np.random.default_rng(0)
    counts = (1000 * np.arange(1, 257, dtype=np.float64) ** -1.2).astype(np.int64) + rng.integers(0, 3, 256)
    parts = D.balanced_key_ranges(counts, n_ranks)
    assert parts[0][0] == 0 and parts[-1][1] == 256
    loads = [counts[a:b].sum() for a, b in parts]
    assert sum(loads) == counts.sum()
    assert max(loads) <= counts.sum() / n_ranks + counts.max()


PLAN = load_cases("golden_plan.npz")


@pytest.mark.parametrize("name", sorted(k for k in PLAN if PLAN[k].meta["kind"] == "keys"))
def test_reduction_keys_match_reference(name):
    """Keys of the plan executor's steps against the reference's infer_reduction_info."""
    m = PLAN[name].meta
    jk, ks, ak = E.reduction_keys(m["formula"])
    assert [list(k) for k in jk] == m["join_keys"]
    assert [list(k) for k in ak] == m["agg_keys"]
    assert ks == m["formula"]


@pytest.mark.parametrize("name", sorted(k for k in PLAN if PLAN[k].meta["kind"] == "plan"))
def test_plan_from_path_matches_reference_steps(name):
    m = PLAN[name].meta
    steps = E.plan_from_path(m["einsum"], m["path"])
    assert [s.formula for s in steps] == [s["formula"] for s in m["steps"]]
    assert [list(s.input_indices) for s in steps] == [s["input_indices"] for s in m["steps"]]


def test_plan_helpers_reject_bad_input():
    for bad in ("ij,jk", "ij->i", "ii,ij->j", "ij,jk->iq", "ij,jk,kl->il"):
        with pytest.raises(ValueError):
            E.reduction_keys(bad)
    with pytest.raises(ValueError):
        E.plan_from_path("ij,jk,kl->il", [(0, 1)])
    with pytest.raises(ValueError):
        E.plan_from_path("ij,jk->ik", [(0, 0)])
    steps = E.plan_from_path("ij,jk->ki", [(0, 1)])
    assert steps[0].formula == "ij,jk->ki"


def test_extract_coo_input_kinds():
    """The COO boundary on the host: torch sparse tensors (uncoalesced COO and
    CSR), pydata-style COO objects, DLPack exporters, COO triples."""
    from types import SimpleNamespace

    import torch

    from einjax_b200.sparse import _extract_coo, as_device_tensor
    i = torch.tensor([[0, 2, 0], [1, 3, 1]])
    ts = torch.sparse_coo_tensor(i, torch.tensor([1.0, 2.0, 3.0]), (4, 5))
    kind, idx, val, shape = _extract_coo(ts)
    assert kind == "coo" and shape == (4, 5) and idx.tolist() == [[0, 1], [2, 3], [0, 1]]
    assert val.tolist() == [1.0, 2.0, 3.0]  # uncoalesced: repeats kept for the policy to resolve
    kind, idx, val, shape = _extract_coo(ts.coalesce().to_sparse_csr())
    assert kind == "coo" and idx.tolist() == [[0, 1], [2, 3]] and val.tolist() == [4.0, 2.0]
    pyd = SimpleNamespace(coords=np.array([[1, 2], [0, 4]]), data=np.array([5.0, 6.0]), shape=(3, 5))
    kind, idx, val, shape = _extract_coo(pyd)
    assert kind == "coo" and idx.tolist() == [[1, 0], [2, 4]] and shape == (3, 5)

    class DL:
        def __init__(self, t):
            self.t = t

        def __dlpack__(self, **kw):
            return self.t.__dlpack__(**kw)

        def __dlpack_device__(self):
            return self.t.__dlpack_device__()
    d = torch.arange(6.0).reshape(2, 3)
    kind, arr, _, shape = _extract_coo(DL(d))
    assert kind == "dense" and shape == (2, 3) and arr.data_ptr() == d.data_ptr()
    assert as_device_tensor(DL(d)).data_ptr() == d.data_ptr()
    assert as_device_tensor(np.array([1, 2])).tolist() == [1, 2]
    assert E.DUPLICATE_POLICIES == ("last", "sum", "error")


def _fake_cost_module():
    """A stand-in with the shape of einjax's optimizer/cost_model.py: a profile
    table, a CostModelConfig with from_device_type, and a detection rule that
    sends unknown GPUs to the A100 profile (optimizer/cost_model.py:291-333)."""
    import types
    from dataclasses import dataclass

    m = types.ModuleType("fake_cost_model")
    m._HARDWARE_PROFILES = {"gpu:a100": {"hbm_bandwidth": 2.0e12, "interconnect_bandwidth": 600e9,
                                         "peak_flops": 19.5e12, "launch_overhead": 5e-6}}

    @dataclass
    class CostModelConfig:
        hbm_bandwidth: float
        interconnect_bandwidth: float
        peak_flops: float
        launch_overhead: float
        num_devices: int
        device_type: str

        @classmethod
        def from_device_type(cls, device_type, num_devices=1):
            p = m._HARDWARE_PROFILES[device_type]
            return cls(num_devices=num_devices, device_type=device_type, **p)

    m.CostModelConfig = CostModelConfig
    m.detect_device_config = lambda: CostModelConfig.from_device_type("gpu:a100", 1)
    return m


def test_b200_cost_profile_detection(monkeypatch):
    from einjax_b200 import cost_model as CM
    assert CM.device_type_for("NVIDIA B200") == "gpu:b200"
    assert CM.device_type_for("NVIDIA GB200") == "gpu:b200"
    assert CM.device_type_for("", (10, 0)) == "gpu:b200"
    assert CM.device_type_for("NVIDIA H100 80GB HBM3", (9, 0)) is None
    assert CM.device_type_for("NVIDIA A100-SXM4-80GB") is None
    m = _fake_cost_module()
    CM.install_b200_profile(m)
    CM.install_b200_profile(m)  # idempotent
    assert m._HARDWARE_PROFILES["gpu:b200"] == CM.B200_PROFILE
    # a JAX GPU device reporting "NVIDIA B200" (8 of them) gets the B200 profile
    monkeypatch.setattr(CM, "_jax_device_kind", lambda: ("NVIDIA B200", 8))
    cfg = m.detect_device_config()
    assert cfg.device_type == "gpu:b200" and cfg.num_devices == 8
    assert cfg.hbm_bandwidth == CM.B200_PROFILE["hbm_bandwidth"]
    assert cfg == m.CostModelConfig(**CM.b200_config_kwargs(8))
    # other devices keep the module's own rule
    monkeypatch.setattr(CM, "_jax_device_kind", lambda: ("NVIDIA H100 80GB HBM3", 8))
    assert m.detect_device_config().device_type == "gpu:a100"
    # no JAX: the torch device decides
    monkeypatch.setattr(CM, "_jax_device_kind", lambda: (None, 0))
    monkeypatch.setattr(CM, "detect_device_type", lambda: "gpu:b200")
    monkeypatch.setattr(CM, "_torch_device_count", lambda: 2)
    cfg = m.detect_device_config()
    assert cfg.device_type == "gpu:b200" and cfg.num_devices == 2


def test_plan_operand_order_prefers_tensor_core_form():
    """A plan step whose tile product only the swapped operand order puts on the
    tensor cores runs swapped; natural orders stay (host-side path query)."""
    from types import SimpleNamespace

    import torch

    from einjax_b200.plan import _operand_order
    a = SimpleNamespace(tile_shape=(128, 128), values=torch.zeros(1))
    b = SimpleNamespace(tile_shape=(128, 64), values=torch.zeros(1))
    f, lhs, rhs = _operand_order("kl,ik->il", b, a, "auto")
    assert f == "ik,kl->il" and lhs is a and rhs is b
    f, lhs, rhs = _operand_order("ik,kl->il", a, b, "auto")
    assert f == "ik,kl->il" and lhs is a and rhs is b
    t = SimpleNamespace(tile_shape=(1, 32, 32), values=torch.zeros(1))
    assert _operand_order("bkl,bik->bil", t, t, "auto")[0] == "bik,bkl->bil"


def test_pending_fill_runs_once_in_creation_order():
    """A relation's pending value fill runs at the first ``values`` access or
    at ``launch_pending_fills`` (oldest first), once; assigning ``values``
    drops it."""
    import torch
    from einjax_b200 import sparse as S

    S.launch_pending_fills()  # nothing left from other tests
    ran = []

    def fake(tag, rel_box):
        def fill():
            ran.append(tag)
            rel_box[0]._values.fill_(1.0)
        return fill

    boxes = [[None], [None], [None]]
    rels = []
    for i, box in enumerate(boxes):
        r = S.SparseTensorRelation(torch.zeros((1, 2), dtype=torch.int32), torch.zeros((1, 2, 2)), (4, 4), (2, 2),
                                   pending=fake(i, box))
        box[0] = r
        rels.append(r)
    assert all(r.pending for r in rels)
    assert rels[1].device == torch.device("cpu")  # from the coords: no fill
    assert float(rels[1].values.sum()) == 4.0 and ran == [1]
    assert not rels[1].pending
    rels[2].values = torch.full((1, 2, 2), 7.0)  # replaced: its fill is dropped
    assert not rels[2].pending
    S.launch_pending_fills()
    assert ran == [1, 0]
    assert float(rels[0].values.sum()) == 4.0 and float(rels[2].values.sum()) == 28.0
    rels[0].materialize()
    assert ran == [1, 0]
    assert "pending=False" in repr(rels[0])
