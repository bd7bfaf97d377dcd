"""B200 hardware profile for einjax's cost model, and the detection rule that
selects it.

einjax's DP optimizer prices every candidate tiling with a ``CostModelConfig``
built from a hardware profile (``optimizer/cost_model.py:26-63``):
``hbm_bandwidth``, ``interconnect_bandwidth``, ``peak_flops`` and
``launch_overhead``. Its detection rule (``detect_device_config``,
``optimizer/cost_model.py:291-333``) maps any GPU it does not know to the A100
profile, so on a B200 the planner prices memory at a third and compute at a
tenth of what the part does. ``B200_PROFILE`` holds numbers measured on B200s
(sm_100a, 180 GB HBM3e, NVLink 5):

* ``hbm_bandwidth`` -- a device-to-device copy (read + write bytes);
* ``interconnect_bandwidth`` -- a peer copy over NVLink, one direction;
* ``peak_flops`` -- the fp32 rate ceiling of this package's tile-einsum
  kernel: fp32 tiles run on the tensor cores as three TF32 passes, so one
  sixth of the measured dense bf16 matmul rate (the role fp32 peak plays in
  the reference's GPU profiles);
* ``launch_overhead`` -- one kernel launch issued back to back on a stream.

``install_b200_profile(cost_model_module)`` adds ``"gpu:b200"`` to a cost-model
module's profile table and wraps its ``detect_device_config`` so that a B200
(JAX ``device_kind`` "NVIDIA B200", or torch's device name / compute
capability 10.x here) gets it. ``calibrate()`` re-measures the four numbers on
the current GPU, as the reference's ``calibrate`` does with JAX
(``optimizer/cost_model.py:400-478``).
"""

from __future__ import annotations

import time

B200_DEVICE_TYPE = "gpu:b200"

B200_PROFILE = {
    "hbm_bandwidth": 6.54e12,           # copy b <- a, 1 Gi bf16 elements, CUDA events
    "interconnect_bandwidth": 770e9,    # peer copy over NVLink 5, one direction
    "peak_flops": 272e12,               # fp32 as 3 TF32 passes: 1634 TFLOP/s bf16 dense / 6
    "launch_overhead": 2.5e-6,          # back-to-back launches on one stream
}


def device_type_for(name: str = "", capability=None) -> str | None:
    """``"gpu:b200"`` for a B200 (by device name, or a compute capability of
    10.x when the name says nothing), else ``None`` (leave the decision to the
    reference's own rule)."""
    n = (name or "").lower()
    if "b200" in n or "gb200" in n:
        return B200_DEVICE_TYPE
    if not n.strip() and capability is not None and int(capability[0]) == 10:
        return B200_DEVICE_TYPE
    return None


def detect_device_type() -> str | None:
    """The B200 rule applied to the current torch CUDA device (``None`` without one)."""
    import torch
    if not torch.cuda.is_available():
        return None
    i = torch.cuda.current_device()
    return device_type_for(torch.cuda.get_device_name(i), torch.cuda.get_device_capability(i))


def b200_config_kwargs(num_devices: int = 1, profile=None) -> dict:
    """Keyword arguments of a ``CostModelConfig`` for ``num_devices`` B200s."""
    p = dict(B200_PROFILE if profile is None else profile)
    return dict(hbm_bandwidth=p["hbm_bandwidth"], interconnect_bandwidth=p["interconnect_bandwidth"],
                peak_flops=p["peak_flops"], launch_overhead=p["launch_overhead"], num_devices=int(num_devices),
                device_type=B200_DEVICE_TYPE)


def install_b200_profile(cost_model_module, profile=None):
    """Add ``"gpu:b200"`` to ``cost_model_module._HARDWARE_PROFILES`` and wrap its
    ``detect_device_config`` so a B200 gets that profile; other devices keep the
    module's own rule. Idempotent. Returns the module."""
    table = getattr(cost_model_module, "_HARDWARE_PROFILES")
    table[B200_DEVICE_TYPE] = dict(B200_PROFILE if profile is None else profile)
    orig = getattr(cost_model_module, "detect_device_config")
    if getattr(orig, "_b200_wrapped", False):
        return cost_model_module
    cfg_cls = getattr(cost_model_module, "CostModelConfig")

    def detect_device_config():
        kind, n = _jax_device_kind()
        if kind is None:
            dt, n = detect_device_type(), _torch_device_count()
        else:
            dt = device_type_for(kind)
        if dt == B200_DEVICE_TYPE:
            return cfg_cls.from_device_type(B200_DEVICE_TYPE, max(n, 1))
        return orig()

    detect_device_config._b200_wrapped = True
    detect_device_config.__doc__ = orig.__doc__
    cost_model_module.detect_device_config = detect_device_config
    return cost_model_module


def _jax_device_kind():
    try:
        import jax
        devs = jax.devices()
    except (ImportError, RuntimeError):
        return None, 0
    if not devs or getattr(devs[0], "platform", "") != "gpu":
        return None, 0
    return getattr(devs[0], "device_kind", ""), len(devs)


def _torch_device_count() -> int:
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def calibrate(device=None, trials: int = 10) -> dict:
    """Measure the profile's four numbers on a GPU (CUDA events, best of
    ``trials``): a 1 GiB copy, this package's fp32 block-sparse matmul over
    fully populated 128x128 tiles, a launch of a one-element kernel repeated
    back to back, and (with two or more GPUs) a 256 MiB peer copy (wall
    clock around synchronised copies, as the reference's calibration)."""
    import torch

    from .kernels import block_sparse_matmul_generic
    from .sparse import SparseTensorRelation
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())

    def best(fn, n=trials):
        ts = []
        for _ in range(n + 1):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            e.synchronize()
            ts.append(s.elapsed_time(e) * 1e-3)
        return min(ts[1:])

    with torch.cuda.device(dev):
        a = torch.empty(1 << 28, dtype=torch.float32, device=dev)
        b = torch.empty_like(a)
        hbm = 2 * a.numel() * 4 / best(lambda: b.copy_(a))
        del a, b
        g, t = 32, 128
        ii, jj = torch.meshgrid(torch.arange(g), torch.arange(g), indexing="ij")
        coords = torch.stack([ii.reshape(-1), jj.reshape(-1)], 1).to(dev, torch.int32)
        vals = torch.randn(g * g, t, t, device=dev)
        rel = SparseTensorRelation(coords, vals, (g * t, g * t), (t, t))
        flops = 2.0 * (g * t) ** 3 / best(lambda: block_sparse_matmul_generic(rel, rel), 3)
        x = torch.zeros(1, device=dev)
        reps = 200

        def launches():
            for _ in range(reps):
                x.add_(1.0)
        launch = best(launches, 3) / reps
        inter = B200_PROFILE["interconnect_bandwidth"]
        if torch.cuda.device_count() >= 2:
            peer = torch.device("cuda", (dev.index + 1) % torch.cuda.device_count())
            src = torch.empty(1 << 26, dtype=torch.float32, device=dev)
            dst = torch.empty(1 << 26, dtype=torch.float32, device=peer)
            ts = []
            for _ in range(trials + 1):
                torch.cuda.synchronize(dev)
                torch.cuda.synchronize(peer)
                t0 = time.perf_counter()
                dst.copy_(src)
                torch.cuda.synchronize(dev)
                torch.cuda.synchronize(peer)
                ts.append(time.perf_counter() - t0)
            inter = src.numel() * 4 / min(ts[1:])
    return {"hbm_bandwidth": hbm, "interconnect_bandwidth": inter, "peak_flops": flops,
            "launch_overhead": launch}
