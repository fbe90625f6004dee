"""Parity at the contract's own shapes, on the B200 through the C ABI.

  * one 1x3x270x480 frame through the FP16 engine, against the reference interpreter's
    output (tests/golden/span_config0_270x480.npz, made by tests/golden/make_golden.py --config0);
  * a batch of 8 seeded 1920x1080 frames through the FP16 engine, the benched shape
    (8 frames x 16 strips x 1080 rows over 74 clusters: the pair kernel's row split, its 6-row slot
    mapping and its multi-unit segments all run), against the torch FP32 reference;
  * the same batch through the E4M3 engine, calibrated on 16 other frames, per-frame PSNR;
  * one 1920x1080 IFNet pair at t = 0.5 (image and motion), and one 3840-wide strip pair
    (64 rows at the 4K width), against the numpy oracle on the padded plane.

Tolerances (the contract's): FP16 max-abs <= 2/255 after clamp to [0, 1]; FP8 PSNR >= 45 dB; both
against FP32."""
import hashlib

import numpy as np
import pytest

import kirari_b200 as kb
import torch_ref
from oracle import nets
from util import ensure_built, golden

pytestmark = pytest.mark.gpu

FP16_MAX_ABS = 2.0 / 255.0
FP8_MIN_PSNR = 45.0
MOTION_FLOW_MAX_ABS = 0.02


@pytest.fixture(scope="module", autouse=True)
def _built():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ensure_built()


def f16(x):
    return np.asarray(x, np.float16).astype(np.float32)


def span_engine(p, h, w, batch, precision=kb.PREC_FP16, scales=None):
    return kb.Engine(kb.MODEL_SPAN_X2, kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(p)), h, w, max_batch=batch,
                     precision=precision, act_scales=scales)


def run(eng, x_dev, h, w):
    import torch
    n = int(x_dev.shape[0])
    out = torch.full((n, 3, 2 * h, 2 * w), float("nan"), dtype=torch.float16, device="cuda")
    eng.enqueue([x_dev], [out])
    eng.check_device()
    return out


def test_config0_matches_reference_interpreter():
    import torch
    g = golden("span_config0_270x480.npz")
    x = f16(np.random.default_rng(int(g["x_seed"])).random((1, 3, 270, 480), dtype=np.float32))
    assert hashlib.sha256(x.tobytes()).hexdigest() == str(g["x_sha256"]), "input generator changed"
    p = nets.span_init(1)
    assert hashlib.sha256(nets.span_flat(p).tobytes()).hexdigest() == str(g["param_sha256"])
    eng = span_engine(p, 270, 480, 1)
    try:
        out = run(eng, torch.from_numpy(x.astype(np.float16)).cuda(), 270, 480).float().cpu().numpy()
    finally:
        eng.close()
    assert np.isfinite(out).all()
    err = nets.max_abs_clamped(out, g["out"].astype(np.float32))
    print(f"configs[0] 270x480: max-abs {err * 255:.3f}/255 vs the reference interpreter")
    assert err <= FP16_MAX_ABS


@pytest.fixture(scope="module")
def frames_1080p():
    from synth import anime_frames
    return f16(anime_frames(8, 1080, 1920, seed=2024))


@pytest.fixture(scope="module")
def ref_1080p(frames_1080p):
    p = nets.span_init(1)
    # the torch reference is pinned to the numpy oracle on a crop of the same frames first
    crop = frames_1080p[:1, :, 500:540, 900:972]
    assert float(np.max(np.abs(torch_ref.span_forward(crop, p) - nets.span_forward(crop, p)))) < 1e-4
    return torch_ref.span_forward(frames_1080p, p)


def test_config1_fp16_batch8_1080p(frames_1080p, ref_1080p):
    import torch
    eng = span_engine(nets.span_init(1), 1080, 1920, 8)
    try:
        out = run(eng, torch.from_numpy(frames_1080p.astype(np.float16)).cuda(), 1080, 1920).float().cpu().numpy()
    finally:
        eng.close()
    assert np.isfinite(out).all()
    errs = [nets.max_abs_clamped(out[i], ref_1080p[i]) for i in range(8)]
    print("configs[1] 8 x 1080p FP16 max-abs /255: " + " ".join(f"{e * 255:.3f}" for e in errs))
    assert max(errs) <= FP16_MAX_ABS


def test_config2_fp8_batch8_1080p(frames_1080p, ref_1080p):
    import torch
    from synth import anime_frames
    p = nets.span_init(1)
    calib = torch.from_numpy(anime_frames(16, 1080, 1920, seed=1000).astype(np.float16)).cuda()
    e16 = span_engine(p, 1080, 1920, 8)
    try:
        peaks = e16.calibrate(calib)
    finally:
        e16.close()
    del calib
    scales = nets.span_scales_from_peaks(peaks, floor=2.0 ** -14)
    eng = span_engine(p, 1080, 1920, 8, precision=kb.PREC_FP8, scales=scales)
    try:
        out = run(eng, torch.from_numpy(frames_1080p.astype(np.float16)).cuda(), 1080, 1920).float().cpu().numpy()
    finally:
        eng.close()
    assert np.isfinite(out).all()
    dbs = [nets.psnr(out[i], ref_1080p[i]) for i in range(8)]
    print("configs[2] 8 x 1080p E4M3 PSNR dB: " + " ".join(f"{d:.1f}" for d in dbs))
    assert min(dbs) >= FP8_MIN_PSNR


def padded(a, b, t, p):
    n, c, h, w = a.shape
    hp, wp = -(-h // 32) * 32, -(-w // 32) * 32
    top, left = ((hp - h) // 2) & ~1, ((wp - w) // 2) & ~1

    def pad(x):
        z = np.zeros((n, c, hp, wp), np.float32)
        z[:, :, top:top + h, left:left + w] = x
        return z

    out, flow, mask = nets.ifnet_forward(pad(a), pad(b), t, p, return_flow=True)
    return out[:, :, top:top + h, left:left + w], flow, nets.sigmoid(mask)


@pytest.mark.parametrize("h,w", [(1080, 1920), (64, 3840)])
def test_config3_ifnet_full_width(h, w):
    import torch
    from synth import shifted_pair
    p = nets.ifnet_init(2)
    fa, fb = shifted_pair(h, w, seed=31)
    a, b = np.ascontiguousarray(f16(fa[None])), np.ascontiguousarray(f16(fb[None]))
    eng = kb.Engine(kb.MODEL_IFNET, kb.make_blob(kb.MODEL_IFNET, nets.ifnet_flat(p)), h, w, max_batch=1)
    try:
        eng.set_timestep(0.5)
        ta = torch.from_numpy(a.astype(np.float16)).cuda()
        tb = torch.from_numpy(b.astype(np.float16)).cuda()
        out = torch.full((1, 3, h, w), float("nan"), dtype=torch.float16, device="cuda")
        eng.enqueue([ta, tb], [out])
        flow, mask, _ = eng.motion(ta, tb)
        eng.check_device()
        out, flow, mask = out.float().cpu().numpy(), flow.cpu().numpy(), mask.cpu().numpy()
    finally:
        eng.close()
    ref, rflow, rmask = padded(a, b, 0.5, p)
    assert np.isfinite(out).all()
    err = nets.max_abs_clamped(out, ref)
    ferr = float(np.max(np.abs(flow - rflow)))
    merr = float(np.max(np.abs(mask - rmask)))
    print(f"configs[3] IFNet {w}x{h}: frame max-abs {err * 255:.3f}/255, flow {ferr:.5f} px, "
          f"mask {merr * 255:.3f}/255")
    assert err <= FP16_MAX_ABS
    assert ferr <= MOTION_FLOW_MAX_ABS
    assert merr <= FP16_MAX_ABS
