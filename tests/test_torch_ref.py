"""Pins the torch FP32 SPAN reference (tests/torch_ref.py, used by the full-size GPU tests) to the
numpy oracle and to the reference interpreter's fixtures, on the CPU."""
import numpy as np
import pytest

import torch_ref
from oracle import nets, ref_lib
from util import golden


def test_torch_span_reference_matches_the_oracle():
    rng = np.random.default_rng(4)
    x = rng.random((2, 3, 20, 36), dtype=np.float32)
    p = nets.span_init(1)
    got = torch_ref.span_forward(x, p, device="cpu")
    ref = nets.span_forward(x, p)
    assert got.shape == ref.shape
    assert float(np.max(np.abs(got - ref))) < 1e-5


def test_torch_span_reference_matches_reference_golden():
    g = golden("span_fp32_2x20x136.npz")
    got = torch_ref.span_forward(g["x"], nets.span_init(1), device="cpu")
    assert float(np.max(np.abs(got - g["out"]))) < 1e-5


def test_torch_span_reference_matches_config0_golden():
    """configs[0] (1x3x270x480, the reference interpreter's output stored in FP16)."""
    g = golden("span_config0_270x480.npz")
    x = np.random.default_rng(int(g["x_seed"])).random((1, 3, 270, 480), dtype=np.float32)
    x = x.astype(np.float16).astype(np.float32)
    got = torch_ref.span_forward(x, nets.span_init(1), device="cpu")
    ref = g["out"].astype(np.float32)
    # the fixture's FP16 rounding: half an FP16 ulp of the value
    assert float(np.max(np.abs(got - ref) - np.abs(ref) * 2.0 ** -11)) < 1e-4


def test_torch_ifnet_reference_matches_the_oracle():
    from synth import shifted_pair
    p = nets.ifnet_init(2)
    a, b = shifted_pair(64, 96, seed=8)
    got, flow, mask = torch_ref.ifnet_forward(a[None], b[None], 0.3, p, device="cpu", return_flow=True)
    ref, rflow, rmask = nets.ifnet_forward(a[None], b[None], 0.3, p, return_flow=True)
    assert float(np.max(np.abs(got - ref))) < 1e-4
    assert float(np.max(np.abs(flow - rflow))) < 1e-3
    assert float(np.max(np.abs(mask - rmask))) < 1e-4


def test_torch_ifnet_reference_matches_reference_golden():
    g = golden("ifnet_64x96_t05.npz")
    got = torch_ref.ifnet_forward(g["a"], g["b"], float(g["t"]), nets.ifnet_init(2), device="cpu")
    assert float(np.max(np.abs(got - g["out"]))) < 1e-4


@pytest.mark.skipif(not ref_lib.available(), reason="oracle/_ref not built (needs the reference sources)")
@pytest.mark.parametrize("name", ["4.25", "4.22lite"])
def test_torch_rife42_reference_matches_the_interpreter(name):
    from synth import shifted_pair
    plan = nets.RIFE_PLANS[name]
    flat = nets.rife_flat(nets.rife_init(plan), plan)
    a, b = shifted_pair(64, 128, seed=9)
    got, flow, mask = torch_ref.rife42_forward(a[None], b[None], 0.4, flat, device="cpu")
    ref, rflow, rmask = ref_lib.rife42_forward(a[None], b[None], 0.4, flat)
    assert float(np.max(np.abs(got - ref))) < 1e-4
    assert float(np.max(np.abs(flow - rflow))) < 1e-3
    assert float(np.max(np.abs(mask - rmask))) < 1e-4
