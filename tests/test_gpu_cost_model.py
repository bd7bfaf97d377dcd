"""The B200 cost-model profile on a B200: detection through torch, and a
calibration run whose measurements land near the profile's numbers."""

import pytest
import torch

from einjax_b200 import cost_model as CM

pytestmark = pytest.mark.gpu


def test_detect_and_calibrate():
    assert CM.detect_device_type() == "gpu:b200", torch.cuda.get_device_name(0)
    m = CM.calibrate(trials=5)
    p = CM.B200_PROFILE
    assert 0.7 * p["hbm_bandwidth"] < m["hbm_bandwidth"] < 1.3 * p["hbm_bandwidth"], m
    # the block-sparse fp32 path reaches a fraction of its 3-pass TF32 ceiling
    assert 0.05 * p["peak_flops"] < m["peak_flops"] < 1.2 * p["peak_flops"], m
    assert 0.3e-6 < m["launch_overhead"] < 20e-6, m
    print("calibrated:", {k: f"{v:.3g}" for k, v in m.items()})
