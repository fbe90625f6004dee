"""SPAN x2 on the B200 through the C ABI, against the CPU oracle (pinned to the reference).

Tolerances (the contract's): FP16 max-abs <= 2/255 after clamp to [0, 1] vs the FP32 oracle;
FP8 PSNR >= 45 dB vs the FP32 oracle; structural cases bit-exact."""
import numpy as np
import pytest

import kirari_b200 as kb
from oracle import nets
from test_oracle import nearest_params
from util import ensure_built

pytestmark = pytest.mark.gpu

FP16_MAX_ABS = 2.0 / 255.0
FP8_MIN_PSNR = 45.0


@pytest.fixture(scope="module", autouse=True)
def _built():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ensure_built()


def run_span(x, params, precision=kb.PREC_FP16, act_scales=None, max_batch=None):
    import torch
    n, _, h, w = x.shape
    eng = kb.Engine(kb.MODEL_SPAN_X2, kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(params)), h, w,
                    max_batch=max_batch or n, precision=precision, act_scales=act_scales)
    xin = torch.from_numpy(np.ascontiguousarray(x, np.float16)).cuda()
    out = torch.full((n, 3, 2 * h, 2 * w), float("nan"), dtype=torch.float16, device="cuda")
    eng.enqueue([xin], [out])
    eng.check_device()
    res = out.float().cpu().numpy()
    eng.close()
    return res


def f16(x):
    return np.asarray(x, np.float16).astype(np.float32)


def test_nearest_x2_is_bit_exact():
    rng = np.random.default_rng(11)
    x = f16(rng.random((2, 3, 37, 300), dtype=np.float32))
    out = run_span(x, nearest_params())
    np.testing.assert_array_equal(out, np.repeat(np.repeat(x, 2, axis=2), 2, axis=3))


def test_zero_blocks_path():
    """Blocks with zero weights output exact zeros: checks conv_1, the 4-source conv_cat and the
    pixel-shuffle upsampler in isolation."""
    p = nets.span_init(1)
    for k in list(p):
        if k.startswith("block"):
            p[k][...] = 0.0
    rng = np.random.default_rng(12)
    x = f16(rng.random((1, 3, 24, 160), dtype=np.float32))
    out = run_span(x, p)
    ref = nets.span_forward(x, p)
    assert np.isfinite(out).all()
    assert np.max(np.abs(out - ref)) < 2e-2 * max(1.0, float(np.abs(ref).max()))


# the tiny shapes put both image borders on one output pixel (1 x 1, 2 x 3, 3 x 2), where the
# conv_cat + upsampler layer drops the bias terms of taps outside the image on both sides at once;
# 1 x 130 is one row over two strips, the second holding 4 pixels
@pytest.mark.parametrize("shape", [(1, 16, 24), (2, 20, 136), (1, 67, 300), (3, 9, 129), (1, 1, 1), (2, 2, 3),
                                   (1, 3, 2), (1, 1, 130)])
def test_span_fp16_parity(shape):
    n, h, w = shape
    rng = np.random.default_rng(h * 1000 + w)
    x = f16(rng.random((n, 3, h, w), dtype=np.float32))
    p = nets.span_init(1)
    out = run_span(x, p)
    ref = nets.span_forward(x, p)
    assert np.isfinite(out).all()
    err = nets.max_abs_clamped(out, ref)
    assert err <= FP16_MAX_ABS, f"max-abs {err * 255:.3f}/255"


def test_span_fp16_matches_golden():
    from util import golden
    g = golden("span_fp32_2x20x136.npz")
    out = run_span(f16(g["x"]), nets.span_init(1))
    assert nets.max_abs_clamped(out, g["out"]) <= FP16_MAX_ABS


def test_batch_is_independent_per_frame():
    rng = np.random.default_rng(13)
    x = f16(rng.random((3, 3, 33, 140), dtype=np.float32))
    p = nets.span_init(1)
    together = run_span(x, p)
    for i in range(3):
        alone = run_span(x[i:i + 1], p, max_batch=3)
        np.testing.assert_array_equal(together[i:i + 1], alone)


def test_fp8_calibrated_psnr():
    import torch
    from synth import anime_frames
    h, w = 48, 160
    p = nets.span_init(1)
    blob = kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(p))
    calib = anime_frames(16, h, w, seed=100)
    eng16 = kb.Engine(kb.MODEL_SPAN_X2, blob, h, w, max_batch=8)
    peaks = eng16.calibrate(torch.from_numpy(calib.astype(np.float16)).cuda())
    eng16.close()
    # the GPU FP16 peaks track the FP32 oracle's
    taps = {}
    nets.span_forward(f16(calib[:4]), p, taps=taps)
    assert peaks[0] >= 0.99 * max(taps[0])
    scales = nets.span_scales_from_peaks(peaks, floor=2.0 ** -14)
    x = f16(anime_frames(2, h, w, seed=7))
    out = run_span(x, p, precision=kb.PREC_FP8, act_scales=scales)
    ref = nets.span_forward(x, p)
    assert np.isfinite(out).all()
    db = nets.psnr(out, ref)
    assert db >= FP8_MIN_PSNR, f"FP8 PSNR {db:.2f} dB"


def live_params(gain=1.2):
    """The seeded SPAN with its block conv weights scaled by `gain`: at 1.0 the deep blocks'
    activations decay towards zero (their peaks fall below 1e-5 by block 4), so an E4M3 error there
    cannot show in the output; at 1.2 every block stays live (peaks 3-10 through block 5)."""
    p = nets.span_init(1)
    for k in p:
        if k.startswith("block") and not k.endswith(".b"):
            p[k] = p[k] * gain
    return p


def test_fp8_live_blocks_psnr():
    """FP8 bar on a network whose E4M3 blocks all carry signal, plus FP16 parity on it."""
    import torch
    from synth import anime_frames
    h, w = 48, 160
    p = live_params()
    blob = kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(p))
    calib = anime_frames(16, h, w, seed=100)
    eng16 = kb.Engine(kb.MODEL_SPAN_X2, blob, h, w, max_batch=8)
    peaks = eng16.calibrate(torch.from_numpy(calib.astype(np.float16)).cuda())
    eng16.close()
    assert min(peaks[:19]) > 1.0, "every calibrated tensor should be live"
    scales = nets.span_scales_from_peaks(peaks, floor=2.0 ** -14)
    x = f16(anime_frames(2, h, w, seed=7))
    ref = nets.span_forward(x, p)
    out8 = run_span(x, p, precision=kb.PREC_FP8, act_scales=scales)
    assert np.isfinite(out8).all()
    db = nets.psnr(out8, ref)
    assert db >= FP8_MIN_PSNR, f"FP8 PSNR {db:.2f} dB"
    out16 = run_span(x, p)
    err = nets.max_abs_clamped(out16, ref)
    assert err <= FP16_MAX_ABS, f"max-abs {err * 255:.3f}/255"


def test_enqueue_refusals():
    import torch
    p = nets.span_init(1)
    eng = kb.Engine(kb.MODEL_SPAN_X2, kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(p)), 16, 32, max_batch=2)
    good_in = torch.zeros((1, 3, 16, 32), dtype=torch.float16, device="cuda")
    good_out = torch.zeros((1, 3, 32, 64), dtype=torch.float16, device="cuda")
    cases = [
        ([torch.zeros((3, 3, 16, 32), dtype=torch.float16, device="cuda")], [torch.zeros((3, 3, 32, 64), dtype=torch.float16, device="cuda")], kb.KB2_SHAPE_INVALID),
        ([torch.zeros((1, 3, 16, 32), dtype=torch.float32, device="cuda")], [good_out], kb.KB2_INPUT_MISMATCH),
        ([good_in], [torch.zeros((1, 3, 32, 62), dtype=torch.float16, device="cuda")], kb.KB2_INPUT_MISMATCH),
        ([good_in, good_in], [good_out], kb.KB2_INPUT_MISMATCH),
    ]
    for ins, outs, status in cases:
        with pytest.raises(kb.KB2Error) as e:
            eng.enqueue(ins, outs)
        assert e.value.status == status
    eng.enqueue([good_in], [good_out])
    eng.check_device()
    eng.close()
