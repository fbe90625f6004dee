"""IFNet (RIFE) on the B200 through the C ABI, against the CPU oracle (pinned to the reference).

Tolerances (the contract's): FP16 path max-abs <= 2/255 after clamp to [0, 1] vs the FP32 oracle;
warp taps bit-exact against the CPU restatement of the reference's tap_at."""
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


@pytest.fixture(scope="module")
def params():
    return nets.ifnet_init(2)


def run_ifnet(a, b, t, p, max_batch=None):
    import torch
    n, _, h, w = a.shape
    eng = kb.Engine(kb.MODEL_IFNET, kb.make_blob(kb.MODEL_IFNET, nets.ifnet_flat(p)), h, w, max_batch=max_batch or n)
    eng.set_timestep(t)
    ta = torch.from_numpy(np.ascontiguousarray(a, np.float16)).cuda()
    tb = torch.from_numpy(np.ascontiguousarray(b, np.float16)).cuda()
    out = torch.full((n, 3, h, w), float("nan"), dtype=torch.float16, device="cuda")
    eng.enqueue([ta, tb], [out])
    eng.check_device()
    res = out.float().cpu().numpy()
    eng.close()
    return res


def padded_oracle(a, b, t, p):
    """The oracle on the engine's zero padded plane (multiples of 32, window of the reference's
    rife_window), cropped back to the frame."""
    n, c, h, w = a.shape
    hp, wp = -(-h // 32) * 32, -(-w // 32) * 32
    top, left = ((hp - h) // 2) & ~1, ((wp - w) // 2) & ~1

    def pad(x):
        z = np.zeros((n, c, hp, wp), np.float32)
        z[:, :, top:top + h, left:left + w] = x
        return z

    out = nets.ifnet_forward(pad(a), pad(b), t, p)
    return out[:, :, top:top + h, left:left + w]


def f16(x):
    return np.asarray(x, np.float16).astype(np.float32)


def test_warp_taps_bit_exact():
    import torch
    rng = np.random.default_rng(5)
    n, h, w = 2, 37, 53
    flow = (rng.standard_normal((n, 2, h, w)) * 6.0).astype(np.float32)
    flow[0, 0, 0, :8] = [1e9, -1e9, np.inf, -np.inf, np.nan, 0.5, -0.5, 52.9999]
    flow[1, 1, 3, :4] = [np.nan, 1e-30, -1e-30, 36.5]
    flow[1, :, 5, 5] = [0.1, 0.2]
    taps, weights = kb.warp_taps(torch.from_numpy(flow).cuda())
    taps, weights = taps.cpu().numpy(), weights.cpu().numpy()
    for i in range(n):
        x0, x1, y0, y1, wx, wy = nets.warp_taps(flow[i, 0], flow[i, 1], 0, 0, w, h)
        np.testing.assert_array_equal(taps[i, 0], x0)
        np.testing.assert_array_equal(taps[i, 1], x1)
        np.testing.assert_array_equal(taps[i, 2], y0)
        np.testing.assert_array_equal(taps[i, 3], y1)
        np.testing.assert_array_equal(weights[i, 0], wx)
        np.testing.assert_array_equal(weights[i, 1], wy)


@pytest.mark.parametrize("name", ["ifnet_64x96_t05.npz", "ifnet_64x96_t03.npz"])
def test_ifnet_matches_reference_golden(name, params):
    g = golden(name)
    out = run_ifnet(g["a"], g["b"], float(g["t"]), params)
    err = nets.max_abs_clamped(out, g["out"])
    assert err <= FP16_MAX_ABS, f"max-abs {err * 255:.3f}/255"


# (1, 256, 1056): block 3's residual level is 64 x 264, three 126-pixel strips, so the pair
# kernel of the 64-channel residual convs runs two strip pairs, one with a strip wholly outside
@pytest.mark.parametrize("shape,t", [((1, 64, 128), 0.5), ((2, 128, 192), 0.25), ((1, 72, 100), 0.5),
                                     ((1, 130, 66), 0.7), ((1, 256, 1056), 0.5)])
def test_ifnet_fp16_parity(shape, t, params):
    from synth import shifted_pair
    n, h, w = shape
    pairs = [shifted_pair(h, w, seed=30 + i) for i in range(n)]
    a = f16(np.stack([p[0] for p in pairs]))
    b = f16(np.stack([p[1] for p in pairs]))
    out = run_ifnet(a, b, t, params)
    ref = padded_oracle(a, b, t, params)
    assert np.isfinite(out).all()
    err = nets.max_abs_clamped(out, ref)
    assert err <= FP16_MAX_ABS, f"{shape} t={t}: max-abs {err * 255:.3f}/255"


def test_zero_network_is_the_plain_blend():
    """All-zero weights: zero flow, zero mask, so the output is 0.5 * img0 + 0.5 * img1 exactly
    (the reference's zero-flow identity case, tests/unit/gpu_cuda/rife_fused_test.cpp:131-179)."""
    p = {k: np.zeros(s, np.float32) for k, s in nets.ifnet_param_shapes()}
    rng = np.random.default_rng(3)
    a = f16(rng.random((1, 3, 64, 64), dtype=np.float32))
    b = f16(rng.random((1, 3, 64, 64), dtype=np.float32))
    out = run_ifnet(a, b, 0.5, p)
    np.testing.assert_array_equal(out, f16(a * np.float32(0.5) + b * np.float32(0.5)))


def test_batch_is_independent_per_pair(params):
    from synth import shifted_pair
    pairs = [shifted_pair(64, 96, seed=50 + i) for i in range(3)]
    a = f16(np.stack([p[0] for p in pairs]))
    b = f16(np.stack([p[1] for p in pairs]))
    together = run_ifnet(a, b, 0.5, params)
    for i in range(3):
        alone = run_ifnet(a[i:i + 1], b[i:i + 1], 0.5, params, max_batch=3)
        np.testing.assert_array_equal(together[i:i + 1], alone)


def test_stream_pairs_as_overlapping_views(params):
    """Consecutive pairs of one frame sequence, (f_i, f_i+1), given as two views one frame apart
    into the same device buffer (how a player streams a video; the bench's e2e leg does this),
    give the same frames as the pairs copied into separate tensors."""
    import torch
    from synth import shifted_pair
    seq = f16(np.stack([shifted_pair(64, 96, seed=70 + i)[0] for i in range(4)]))
    separate = run_ifnet(seq[:3], seq[1:], 0.5, params)
    eng = kb.Engine(kb.MODEL_IFNET, kb.make_blob(kb.MODEL_IFNET, nets.ifnet_flat(params)), 64, 96, max_batch=3)
    eng.set_timestep(0.5)
    d = torch.from_numpy(np.ascontiguousarray(seq, np.float16)).cuda()
    out = torch.full((3, 3, 64, 96), float("nan"), dtype=torch.float16, device="cuda")
    eng.enqueue([d[:3], d[1:]], [out])
    eng.check_device()
    eng.close()
    np.testing.assert_array_equal(out.float().cpu().numpy(), separate)
    np.testing.assert_array_equal(d.float().cpu().numpy(), seq)  # the inputs are only read


def test_ifnet_refusals(params):
    import torch
    blob = kb.make_blob(kb.MODEL_IFNET, nets.ifnet_flat(params))
    with pytest.raises(kb.KB2Error) as e:
        kb.Engine(kb.MODEL_IFNET, blob, 64, 64, precision=kb.PREC_FP8)
    assert e.value.status == kb.KB2_FORMAT_UNSUPPORTED
    eng = kb.Engine(kb.MODEL_IFNET, blob, 64, 64, max_batch=1)
    try:
        for bad in (0.0, 1.0, 1.5, float("nan")):
            with pytest.raises(kb.KB2Error) as e:
                eng.set_timestep(bad)
            assert e.value.status == kb.KB2_INVALID_ARGUMENT
        x = torch.zeros((1, 3, 64, 64), dtype=torch.float16, device="cuda")
        out = torch.zeros((1, 3, 64, 64), dtype=torch.float16, device="cuda")
        with pytest.raises(kb.KB2Error) as e:
            eng.enqueue([x], [out])  # one frame instead of two
        assert e.value.status == kb.KB2_INPUT_MISMATCH
        with pytest.raises(kb.KB2Error) as e:
            eng.enqueue([x, torch.zeros((1, 3, 64, 32), dtype=torch.float16, device="cuda")], [out])
        assert e.value.status == kb.KB2_INPUT_MISMATCH
        big = torch.zeros((2, 3, 64, 64), dtype=torch.float16, device="cuda")
        with pytest.raises(kb.KB2Error) as e:
            eng.enqueue([big, big], [torch.zeros_like(big)])
        assert e.value.status == kb.KB2_SHAPE_INVALID
    finally:
        eng.close()


# ------------------------------------------------------------------------------------------------
# the motion variant: flow and mask in place of the frame (the reference's run_motion,
# src/app/play/upscale_motion.cpp:71-84; finish src/gpu/cuda/backend/rife_finish.cuh:40-55)
# ------------------------------------------------------------------------------------------------
# Flow is in pixels; the FP16 network's flow error that keeps the blended frame within 2/255 at a
# sharp edge (an image gradient of ~1 a pixel) is about 0.01 px, and the measured error is below it.
MOTION_FLOW_MAX_ABS = 0.02
MOTION_MASK_MAX_ABS = 2.0 / 255.0


def padded_motion_oracle(a, b, t, p):
    """The oracle's final flow [n,4,Hp,Wp] and sigmoid(mask) [n,1,Hp,Wp] on the engine's padded plane,
    with the window (x, y, w, h) of the frames in it."""
    n, c, h, w = a.shape
    hp, wp = -(-h // 32) * 32, -(-w // 32) * 32
    top, left = ((hp - h) // 2) & ~1, ((wp - w) // 2) & ~1

    def pad(x):
        z = np.zeros((n, c, hp, wp), np.float32)
        z[:, :, top:top + h, left:left + w] = x
        return z

    _, flow, mask = nets.ifnet_forward(pad(a), pad(b), t, p, return_flow=True)
    return flow, nets.sigmoid(mask), (left, top, w, h)


def run_motion(a, b, t, p, dtype="float32"):
    import torch
    n, _, h, w = a.shape
    eng = kb.Engine(kb.MODEL_IFNET, kb.make_blob(kb.MODEL_IFNET, nets.ifnet_flat(p)), h, w, max_batch=n)
    try:
        eng.set_timestep(t)
        ta = torch.from_numpy(np.ascontiguousarray(a, np.float16)).cuda()
        tb = torch.from_numpy(np.ascontiguousarray(b, np.float16)).cuda()
        flow, mask, win = eng.motion(ta, tb, dtype=getattr(torch, dtype))
        eng.check_device()
    finally:
        eng.close()
    return flow, mask, win


@pytest.mark.parametrize("shape,t", [((1, 72, 100), 0.5), ((2, 64, 96), 0.5), ((1, 130, 66), 0.3)])
def test_motion_matches_oracle(shape, t, params):
    from synth import shifted_pair
    n, h, w = shape
    pairs = [shifted_pair(h, w, seed=90 + i) for i in range(n)]
    a = f16(np.stack([q[0] for q in pairs]))
    b = f16(np.stack([q[1] for q in pairs]))
    flow, mask, win = run_motion(a, b, t, params)
    rflow, rmask, rwin = padded_motion_oracle(a, b, t, params)
    assert win == rwin
    flow, mask = flow.cpu().numpy(), mask.cpu().numpy()
    assert flow.shape == rflow.shape and mask.shape == rmask.shape
    assert np.isfinite(flow).all() and np.isfinite(mask).all()
    ferr = float(np.max(np.abs(flow - rflow)))
    merr = float(np.max(np.abs(mask - rmask)))
    print(f"motion {shape} t={t}: flow max-abs {ferr:.5f} px (|flow| up to {np.abs(rflow).max():.2f}), "
          f"mask max-abs {merr * 255:.3f}/255")
    assert ferr <= MOTION_FLOW_MAX_ABS, f"flow max-abs {ferr:.5f} px"
    assert merr <= MOTION_MASK_MAX_ABS, f"mask max-abs {merr * 255:.3f}/255"


def test_motion_f16_is_the_f32_motion_rounded(params):
    from synth import shifted_pair
    a, b = (np.ascontiguousarray(f16(x[None])) for x in shifted_pair(64, 96, seed=95))
    flow32, mask32, _ = run_motion(a, b, 0.5, params)
    flow16, mask16, _ = run_motion(a, b, 0.5, params, dtype="float16")
    np.testing.assert_array_equal(flow16.cpu().numpy(), flow32.half().cpu().numpy())
    np.testing.assert_array_equal(mask16.cpu().numpy(), mask32.half().cpu().numpy())


@pytest.mark.parametrize("t", [1.0 / 3.0, 0.5])
def test_motion_feeds_warp_blend_at(t, params):
    """The library's interpolator feeding its own warp: IFNet motion at the middle of the pair, then
    kb2_warp_blend_at at t, against the oracle's motion through the reference's CPU warp_blend_at
    (src/kernels/ref/warp.cpp:261; the numpy restatement where the reference build is absent)."""
    import torch
    from oracle import ref_lib
    from synth import shifted_pair
    a, b = (np.ascontiguousarray(f16(x[None])) for x in shifted_pair(72, 100, seed=97))
    flow, mask, win = run_motion(a, b, 0.5, params)
    ta = torch.from_numpy(a.astype(np.float16)).cuda()
    tb = torch.from_numpy(b.astype(np.float16)).cuda()
    got = kb.warp_blend_at(ta, tb, flow, mask, win, t)
    torch.cuda.synchronize()
    got = got.float().cpu().numpy()[0]
    rflow, rmask, rwin = padded_motion_oracle(a, b, 0.5, params)
    warp = ref_lib.warp_blend_at if ref_lib.available() else nets.warp_blend_at
    ref = warp(a[0], b[0], rflow[0], rmask[0, 0], rwin, t)
    err = nets.max_abs_clamped(got, ref)
    print(f"motion -> warp_blend_at t={t:.3f}: max-abs {err * 255:.3f}/255")
    assert err <= FP16_MAX_ABS, f"t={t}: max-abs {err * 255:.3f}/255"


def test_motion_refusals(params):
    import torch
    blob = kb.make_blob(kb.MODEL_IFNET, nets.ifnet_flat(params))
    eng = kb.Engine(kb.MODEL_IFNET, blob, 72, 100, max_batch=1)
    try:
        assert eng.rife_geometry() == (96, 128, 14, 12)
        x = torch.zeros((1, 3, 72, 100), dtype=torch.float16, device="cuda")
        flow = torch.zeros((1, 4, 96, 128), dtype=torch.float32, device="cuda")
        mask = torch.zeros((1, 1, 96, 128), dtype=torch.float32, device="cuda")
        for bad in ([flow, mask.half()],  # types differ
                    [torch.zeros((1, 4, 72, 100), device="cuda"), mask],  # the window, not the plane
                    [flow, torch.zeros((1, 2, 96, 128), device="cuda")],
                    [flow.to(torch.uint8), mask.to(torch.uint8)]):
            with pytest.raises(kb.KB2Error) as e:
                eng.enqueue([x, x], bad)
            assert e.value.status == kb.KB2_INPUT_MISMATCH
    finally:
        eng.close()
