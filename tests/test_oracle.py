"""The CPU oracle (oracle/nets.py) pinned against the reference: golden fixtures made by the
reference's own FP32 interpreter, and known-answer tests restated from the reference's test suite."""
import hashlib
import math

import numpy as np
import pytest

from oracle import nets
from util import golden


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a, np.float32).tobytes()).hexdigest()


@pytest.mark.parametrize("name", ["span_fp32_16x24.npz", "span_fp32_2x20x136.npz"])
def test_span_restatement_matches_reference(name):
    g = golden(name)
    p = nets.span_init(int(g["param_seed"]))
    assert _sha(nets.span_flat(p)) == str(g["param_sha256"]), "seeded SPAN weights changed"
    out = nets.span_forward(g["x"], p)
    assert out.shape == g["out"].shape
    np.testing.assert_allclose(out, g["out"], rtol=0, atol=2e-5)


def test_span_fake_quant_restatement_matches_reference():
    """E4M3 fake-quantised block-conv inputs (the reference's FakeQuantE4M3 conv input): the
    restatement agrees with the reference except where FP32 summation order flips one rounding."""
    g = golden("span_fq_16x24.npz")
    p = nets.span_init(int(g["param_seed"]))
    out = nets.span_forward(g["x"], p, act_scales=g["act_scales"])
    assert nets.psnr(out, g["out"]) > 60.0
    assert np.mean(np.abs(out - g["out"]) < 1e-4) > 0.99


@pytest.mark.parametrize("name", ["ifnet_64x96_t05.npz", "ifnet_64x96_t03.npz"])
def test_ifnet_restatement_matches_reference(name):
    g = golden(name)
    p = nets.ifnet_init(int(g["param_seed"]))
    assert _sha(nets.ifnet_flat(p)) == str(g["param_sha256"]), "seeded IFNet weights changed"
    out = nets.ifnet_forward(g["a"], g["b"], float(g["t"]), p)
    np.testing.assert_allclose(out, g["out"], rtol=0, atol=5e-5)


def test_nearest_x2_package_is_exact():
    """Identity conv_1, zero blocks, conv_cat selecting source 0, a centre-tap upsampler: the
    network is nearest x2 exactly (the reference's hand-built 'nearest' package test,
    tests/unit/gpu_span_fp8/forward_test.cpp:32-86, restated on the canonical net)."""
    p = nearest_params()
    rng = np.random.default_rng(7)
    x = rng.random((1, 3, 5, 48), dtype=np.float32)
    out = nets.span_forward(x, p)
    np.testing.assert_array_equal(out, np.repeat(np.repeat(x, 2, axis=2), 2, axis=3))


def test_cat_upsampler_composition():
    """SPAN's conv_cat (1x1, 192 -> 48, bias) followed by its upsampler (3x3, 48 -> 12, zero padding)
    equals one 3x3 conv of the four sources with the composed weights, whose bias is the
    upsampler's plus, for each tap that reads inside the image, that tap's share of conv_cat's
    bias. This is the algebra the library's fused conv_cat + upsampler layer computes (the weights
    composed on the host, the border terms dropped in the epilogue); checked here with the oracle's
    FP32 conv on frames whose every pixel is a border pixel in some direction."""
    rng = np.random.default_rng(3)
    c = 48
    wcat = rng.standard_normal((c, 4 * c, 1, 1)) * 0.1
    bcat = rng.standard_normal(c)
    wup = rng.standard_normal((12, c, 3, 3)) * 0.1
    bup = rng.standard_normal(12)
    wc = np.einsum("omyx,mi->oiyx", wup, wcat[:, :, 0, 0])
    tap = np.einsum("omyx,m->yxo", wup, bcat)  # [ky][kx][o]
    for h, w in ((1, 1), (2, 3), (3, 2), (5, 7)):
        src = rng.standard_normal((1, 4 * c, h, w))
        ref = nets.conv2d(nets.conv2d(src, wcat, bcat, pad=0), wup, bup)
        out = nets.conv2d(src, wc, bup + tap.sum(axis=(0, 1)))
        for y in range(h):
            for x in range(w):
                for ky in range(3):
                    for kx in range(3):
                        if not (0 <= y + ky - 1 < h and 0 <= x + kx - 1 < w):
                            out[0, :, y, x] -= tap[ky, kx]
        np.testing.assert_allclose(out, ref, rtol=0, atol=2e-5 * max(1.0, float(np.abs(ref).max())))


def nearest_params():
    p = {k: np.zeros(s, np.float32) for k, s in nets.span_param_shapes()}
    for c in range(3):
        p["conv_1.w"][c, c, 1, 1] = 1.0
        p["conv_cat.w"][c, c, 0, 0] = 1.0
        for i in range(2):
            for j in range(2):
                p["upsampler.w"][4 * c + 2 * i + j, c, 1, 1] = 1.0
    return p


def test_warp_tap_known_answers():
    """tests/unit/kernels/warp_test.cpp:49-62 of the reference: a 4x2 plane holding 10y + x."""
    plane = (10 * np.arange(2)[:, None] + np.arange(4)[None, :]).astype(np.float32)

    def sample(x, y, window=(0, 0, 4, 2)):
        left, top, right, bottom = window
        fx = np.array([[x - left]], np.float32)
        fy = np.array([[y - top]], np.float32)
        x0, x1, y0, y1, wx, wy = nets.warp_taps(fx, fy, 0, 0, right - left, bottom - top)
        sub = plane[top:bottom, left:right]
        a, b, d, e = sub[y0, x0], sub[y0, x1], sub[y1, x0], sub[y1, x1]
        one = np.float32(1)
        return float(((a * (one - wx) + b * wx) * (one - wy) + (d * (one - wx) + e * wx) * wy)[0, 0])

    assert sample(2.0, 1.0) == 12.0
    assert sample(1.5, 0.0) == 1.5
    assert sample(1.5, 0.5) == 6.5
    assert sample(-3.0, 0.0) == 0.0      # clamp left
    assert sample(9.0, 5.0) == 13.0      # clamp bottom right
    assert sample(float("nan"), 1.0) == 10.0  # NaN goes to the left bound
    # inside a window: coordinates relative to its corner, clamp to its edges
    assert sample(1.0, 0.0, window=(1, 0, 3, 2)) == 1.0
    assert sample(6.0, 1.0, window=(1, 0, 3, 2)) == 12.0


def test_warp_backward_displacement():
    """warp_test.cpp:95-107: a ramp warped by f0x = +2 reads x + 2, clamped at the right edge;
    f0x = 0.5 reads halfway."""
    ramp = np.tile(np.arange(16, dtype=np.float32), (1, 3, 4, 1))
    flow = np.zeros((1, 2, 4, 16), np.float32)
    flow[:, 0] = 2.0
    out = nets.warp(ramp, flow)
    assert out[0, 0, 1, 3] == 5.0 and out[0, 0, 1, 14] == 15.0
    flow[:, 0] = 0.5
    assert nets.warp(ramp, flow)[0, 2, 0, 6] == 6.5


def test_tap_indices_fp32_rounding():
    """ix = fl32(x + fx): the sum is rounded to FP32 before truncation (warp_lib.cuh:45-47)."""
    fx = np.array([[np.float32(0.99999994), np.float32(-1e-8), np.float32(2.5)]], np.float32)
    fy = np.zeros_like(fx)
    x0, x1, y0, y1, wx, _ = nets.warp_taps(fx, fy, 0, 0, 3, 1)
    # 0 + 0.99999994 stays below 1; 1 + (-1e-8) rounds to 1.0 in FP32; 2 + 2.5 clamps to 2
    assert x0.tolist() == [[0, 1, 2]]
    assert x1.tolist() == [[1, 2, 2]]
    assert wx[0, 2] == 0.0


def test_resize_taps_half_pixel():
    lo, hi, t = nets.resize_axis_taps(64, 8)  # 1/8 down: 2x2 average at 8i + 3, 8i + 4
    assert lo.tolist() == [8 * i + 3 for i in range(8)] and hi.tolist() == [8 * i + 4 for i in range(8)]
    assert np.all(t == 0.5)
    lo, hi, t = nets.resize_axis_taps(4, 8)   # x2 up: first and last clamp
    assert lo[0] == 0 and t[0] == 0.0 and lo[-1] == 3 and hi[-1] == 3


def test_e4m3_rounding_table():
    """RNE with saturation to +-448 (span_fp8::e4m3_round, src/gpu/span_fp8/quantize.h:14-18)."""
    cases = {0.0: 0.0, 1.0: 1.0, 448.0: 448.0, 1e6: 448.0, -500.0: -448.0, 1.0625: 1.0, 1.1875: 1.25,
             1.125: 1.125, 2 ** -9: 2 ** -9, 2 ** -10: 0.0, 3 * 2 ** -10: 2 ** -8, 0.3: 0.3125, 17.0: 16.0,
             19.0: 20.0, 240.0: 240.0, 248.0: 256.0}
    for x, want in cases.items():
        assert float(nets.e4m3_round(np.float32(x))) == want, x
    assert math.isnan(float(nets.e4m3_round(np.float32("nan"))))


def test_e4m3_matches_torch_cast_in_range():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.standard_normal(20000) * s for s in (1e-3, 0.1, 1.0, 30.0, 200.0)]).astype(np.float32)
    x = x[np.abs(x) <= 448.0]
    ours = nets.e4m3_round(x)
    theirs = torch.from_numpy(x).to(torch.float8_e4m3fn).to(torch.float32).numpy()
    np.testing.assert_array_equal(ours, theirs)


def test_span_scales_refuse_zero_peaks():
    with pytest.raises(ValueError):
        nets.span_scales_from_peaks([1.0, 0.0])
    s = nets.span_scales_from_peaks([1.0, 0.0], floor=2.0 ** -14)
    assert s[0] == np.float32(1.25 / 448.0)
