"""The unshuffle SPAN of a .span8 package on the B200 through the C ABI (KB2_MODEL_SPAN_UNSHUFFLE),
against the CPU oracle (oracle/nets.py span8_forward, pinned to the reference's own FP32 forward by
tests/test_span8.py) and against the reference's outputs in the golden fixtures.

Tolerances (the contract's): FP16 max-abs <= 2/255 after clamp to [0, 1] vs the FP32 oracle; E4M3
blocks PSNR >= 45 dB vs the FP32 oracle."""
import numpy as np
import pytest

import kirari_b200 as kb
from oracle import nets
from util import ensure_built, golden

pytestmark = pytest.mark.gpu

FP16_MAX_ABS = 2.0 / 255.0


@pytest.fixture(scope="module", autouse=True)
def _built():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ensure_built()


def run_span8(pkg, x, max_batch=None):
    import torch
    n, _, h, w = x.shape
    eng = kb.Engine(kb.MODEL_SPAN_UNSHUFFLE, pkg, h, w, max_batch=max_batch or n)
    tx = torch.from_numpy(np.ascontiguousarray(x, np.float16)).cuda()
    out = torch.full((n, 3, 2 * h, 2 * w), float("nan"), dtype=torch.float16, device="cuda")
    eng.enqueue([tx], [out])
    eng.check_device()
    res = out.float().cpu().numpy()
    eng.close()
    return res


def f16(x):
    return np.asarray(x, np.float16).astype(np.float32)


@pytest.mark.parametrize("name", ["span8_b2f48_20x36.npz", "span8_b3f64_16x30.npz"])
def test_span8_matches_reference_golden(name):
    g = golden(name)
    pkg = nets.span8_package(nets.span8_init(int(g["blocks"]), int(g["real"]), seed=int(g["seed"])))
    out = run_span8(pkg, g["x"])
    assert np.isfinite(out).all()
    err = nets.max_abs_clamped(out, g["out"])
    assert err <= FP16_MAX_ABS, f"max-abs {err * 255:.3f}/255"


# (blocks, real channels, frames, H, W): the working plane is H/2 x W/2; W = 540 gives 270
# columns, three 126-pixel strips, so the pair kernels run two strip pairs (one strip partly
# outside); 64 channels run rows of 12 K steps on 6-slot rings
@pytest.mark.parametrize("blocks,real,n,h,w", [(2, 48, 2, 40, 72), (5, 48, 1, 64, 540), (3, 64, 2, 36, 100),
                                               (8, 64, 1, 64, 540)])
def test_span8_fp16_parity(blocks, real, n, h, w):
    from synth import anime_frames
    pkg_p = nets.span8_init(blocks, real, seed=40 + blocks)
    pkg = nets.span8_package(pkg_p)
    x = f16(anime_frames(n, h, w, seed=7 + blocks))
    out = run_span8(pkg, x)
    ref = nets.span8_forward(x, pkg_p)
    assert np.isfinite(out).all()
    err = nets.max_abs_clamped(out, ref)
    assert err <= FP16_MAX_ABS, f"b{blocks}f{real} {h}x{w}: max-abs {err * 255:.3f}/255"


def test_span8_batch_is_independent_per_frame():
    from synth import anime_frames
    pkg = nets.span8_package(nets.span8_init(3, 64, seed=9))
    x = f16(anime_frames(3, 48, 64, seed=12))
    together = run_span8(pkg, x)
    for i in range(3):
        alone = run_span8(pkg, x[i:i + 1], max_batch=3)
        np.testing.assert_array_equal(together[i:i + 1], alone)


def test_span8_refusals():
    pkg = nets.span8_package(nets.span8_init(2, 48, seed=4))
    with pytest.raises(kb.KB2Error) as e:
        kb.Engine(kb.MODEL_SPAN_UNSHUFFLE, pkg, 33, 64)  # odd height: the 2x2 unshuffle needs even sides
    assert e.value.status == kb.KB2_SHAPE_INVALID


# E4M3 blocks of an FP8 package (scales calibrated on the frames the reference's way), against the
# FP32 oracle: the contract's FP8 bar, PSNR >= 45 dB
@pytest.mark.parametrize("blocks,real,n,h,w", [(3, 48, 2, 40, 72), (5, 48, 1, 64, 540), (3, 64, 2, 36, 100),
                                               (8, 64, 1, 64, 540)])
def test_span8_fp8_psnr(blocks, real, n, h, w):
    import torch
    from synth import anime_frames
    x = f16(anime_frames(n, h, w, seed=17 + blocks))
    p = nets.span8_fp8_package(nets.span8_init(blocks, real, seed=50 + blocks), x)
    pkg = nets.span8_package(p)
    ref = nets.span8_forward(x, p)
    eng = kb.Engine(kb.MODEL_SPAN_UNSHUFFLE, pkg, h, w, max_batch=n, precision=kb.PREC_FP8)
    tx = torch.from_numpy(np.ascontiguousarray(x, np.float16)).cuda()
    out = torch.full((n, 3, 2 * h, 2 * w), float("nan"), dtype=torch.float16, device="cuda")
    eng.enqueue([tx], [out])
    eng.check_device()
    res = out.float().cpu().numpy()
    eng.close()
    assert np.isfinite(res).all()
    db = nets.psnr(res, ref)
    assert db >= 45.0, f"b{blocks}f{real}: {db:.2f} dB"
    # the FP16 engine of the same package stays within the FP16 bar
    assert nets.max_abs_clamped(run_span8(pkg, x), ref) <= FP16_MAX_ABS


def test_span8_fp8_refuses_fp16_packages():
    pkg = nets.span8_package(nets.span8_init(2, 48, seed=4))  # the FP16 flag: unit scales
    with pytest.raises(kb.KB2Error) as e:
        kb.Engine(kb.MODEL_SPAN_UNSHUFFLE, pkg, 32, 64, precision=kb.PREC_FP8)
    assert e.value.status == kb.KB2_FORMAT_UNSUPPORTED


@pytest.mark.parametrize("blocks,real", [(2, 48), (3, 64)])
def test_span8_calibration_peaks_track_the_oracle(blocks, real):
    """kb2_span_calibrate on an unshuffle-SPAN engine: the package's 1 + 3 * blocks peaks (conv_1's
    output, per block its two ReLU outputs and its output) from the FP16 engine, against the FP32
    oracle's peaks of the same tensors (span8_forward); an FP8 package made from them runs."""
    import torch
    from synth import anime_frames
    p = nets.span8_init(blocks, real, seed=5)
    pkg = nets.span8_package(p)
    x = f16(anime_frames(3, 40, 72, seed=8))
    eng = kb.Engine(kb.MODEL_SPAN_UNSHUFFLE, pkg, 40, 72, max_batch=2)  # 3 frames: batches of 2 and 1
    try:
        got = eng.calibrate(torch.from_numpy(x.astype(np.float16)).cuda(), n_peaks=1 + 3 * blocks)
        with pytest.raises(kb.KB2Error) as e:
            eng.calibrate(torch.from_numpy(x.astype(np.float16)).cuda(), n_peaks=19 if blocks != 6 else 16)
        assert e.value.status == kb.KB2_INPUT_MISMATCH
    finally:
        eng.close()
    ref = []
    for i in range(3):
        pk = []
        nets.span8_forward(x[i:i + 1], p, peaks=pk)
        ref.append(pk)
    ref = np.max(np.asarray(ref, np.float32), axis=0)
    np.testing.assert_allclose(got, ref, rtol=1e-2)
    import seeded
    q = seeded.span8_fp8_from_peaks(p, got)
    e8 = kb.Engine(kb.MODEL_SPAN_UNSHUFFLE, seeded.span8_package(q), 40, 72, max_batch=1, precision=kb.PREC_FP8)
    try:
        out8 = torch.full((1, 3, 80, 144), float("nan"), dtype=torch.float16, device="cuda")
        e8.enqueue([torch.from_numpy(x[:1].astype(np.float16)).cuda()], [out8])
        e8.check_device()
        out8 = out8.float().cpu().numpy()
    finally:
        e8.close()
    assert nets.psnr(out8, nets.span8_forward(x[:1], q)) >= 45.0
