"""RIFE 4.2x (KB2_MODEL_RIFE_FUSED: 4.25, 4.26, 4.25 lite, 4.22 lite plans) on the B200 through the
C ABI, against the reference's own FP32 interpreter running the same network (oracle/ref_graphs.cpp
kref_rife42_forward, whose glue is pinned to the reference's fused-RIFE statement by
tests/test_rife42_oracle.py).

Tolerances (the contract's FP16 bar): image max-abs <= 2/255 after clamp to [0, 1] vs FP32; the
motion variant's flow within 0.05 px and its mask within 2/255 (FP16 activations and Z)."""
import numpy as np
import pytest

import kirari_b200 as kb
from oracle import nets
from util import ensure_built

pytestmark = pytest.mark.gpu

FP16_MAX_ABS = 2.0 / 255.0
FLOW_MAX_ABS = 0.05
MASK_MAX_ABS = 2.0 / 255.0


@pytest.fixture(scope="module", autouse=True)
def _built():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ensure_built()


def f16(x):
    return np.asarray(x, np.float16).astype(np.float32)


def flat_of(name, seed=3, **kw):
    plan = nets.RIFE_PLANS[name]
    return nets.rife_flat(nets.rife_init(plan, seed=seed, **kw), plan)


def align_of(flat):
    blocks = int(flat[0])
    return max(64, 4 * max(int(d) for d in flat[1:1 + blocks]))


def pad_window(h, w, align):
    hp, wp = -(-h // align) * align, -(-w // align) * align
    return hp, wp, ((hp - h) // 2) & ~1, ((wp - w) // 2) & ~1


def padded_oracle(a, b, t, flat):
    """The reference interpreter on the engine's zero padded plane (the window of rife_window):
    (image cropped to the frame, flow and mask over the plane)."""
    from oracle import ref_lib
    n, c, h, w = a.shape
    hp, wp, top, left = pad_window(h, w, align_of(flat))

    def pad(x):
        z = np.zeros((n, c, hp, wp), np.float32)
        z[:, :, top:top + h, left:left + w] = x
        return z

    img, flow, mask = ref_lib.rife42_forward(pad(a), pad(b), t, flat)
    return img[:, :, top:top + h, left:left + w], flow, mask, (left, top)


def engine(flat, h, w, n):
    return kb.Engine(kb.MODEL_RIFE_FUSED, kb.make_blob(kb.MODEL_RIFE_FUSED, flat), h, w, max_batch=n)


def run(flat, a, b, t, max_batch=None):
    import torch
    n, _, h, w = a.shape
    eng = engine(flat, h, w, max_batch or n)
    try:
        eng.set_timestep(t)
        ta = torch.from_numpy(np.ascontiguousarray(a, np.float16)).cuda()
        tb = torch.from_numpy(np.ascontiguousarray(b, np.float16)).cuda()
        out = torch.full((n, 3, h, w), float("nan"), dtype=torch.float16, device="cuda")
        eng.enqueue([ta, tb], [out])
        eng.check_device()
        return out.float().cpu().numpy()
    finally:
        eng.close()


def pairs(n, h, w, seed):
    from synth import shifted_pair
    ps = [shifted_pair(h, w, seed=seed + i) for i in range(n)]
    return (np.ascontiguousarray(f16(np.stack([p[0] for p in ps]))),
            np.ascontiguousarray(f16(np.stack([p[1] for p in ps]))))


@pytest.mark.parametrize("name,shape,t", [
    ("4.25", (1, 128, 192), 0.5),
    ("4.25", (2, 100, 150), 0.3),    # window inside a 128 x 192 plane, two pairs
    ("4.22lite", (1, 64, 128), 0.5),
    ("4.26", (1, 128, 128), 0.7),
    ("4.25lite", (1, 128, 256), 0.5),
])
def test_rife42_matches_reference(name, shape, t):
    n, h, w = shape
    flat = flat_of(name)
    a, b = pairs(n, h, w, 40)
    out = run(flat, a, b, t)
    ref, _, _, _ = padded_oracle(a, b, t, flat)
    assert np.isfinite(out).all()
    err = nets.max_abs_clamped(out, ref)
    print(f"RIFE {name} {shape} t={t}: max-abs {err * 255:.3f}/255")
    assert err <= FP16_MAX_ABS


def test_rife42_motion_matches_reference():
    import torch
    flat = flat_of("4.25")
    a, b = pairs(2, 72, 100, 60)
    eng = engine(flat, 72, 100, 2)
    try:
        eng.set_timestep(0.5)
        ta = torch.from_numpy(a.astype(np.float16)).cuda()
        tb = torch.from_numpy(b.astype(np.float16)).cuda()
        flow, mask, win = eng.motion(ta, tb)
        flow16, mask16, _ = eng.motion(ta, tb, dtype=torch.float16)
        eng.check_device()
    finally:
        eng.close()
    _, rflow, rmask, (left, top) = padded_oracle(a, b, 0.5, flat)
    assert win == (left, top, 100, 72)
    flow, mask = flow.cpu().numpy(), mask.cpu().numpy()
    assert flow.shape == rflow.shape and mask.shape == rmask.shape
    ferr = float(np.max(np.abs(flow - rflow)))
    merr = float(np.max(np.abs(mask - rmask)))
    print(f"RIFE 4.25 motion: flow max-abs {ferr:.4f} px (|flow| up to {np.abs(rflow).max():.2f}), mask {merr:.5f}")
    assert ferr <= FLOW_MAX_ABS and merr <= MASK_MAX_ABS
    np.testing.assert_array_equal(flow16.cpu().numpy(), flow.astype(np.float16))
    np.testing.assert_array_equal(mask16.cpu().numpy(), mask.astype(np.float16))


def test_rife42_batch_independence():
    """A pair's output does not depend on the other pairs of the batch or on max_batch."""
    flat = flat_of("4.25")
    a, b = pairs(3, 64, 128, 70)
    whole = run(flat, a, b, 0.5)
    alone = run(flat, a[1:2], b[1:2], 0.5, max_batch=3)
    np.testing.assert_array_equal(whole[1:2], alone)


def test_rife42_zero_network_is_the_plain_blend():
    """All-zero weights: zero flow and mask logit, so the output is 0.5 A + 0.5 B exactly (the
    reference's zero-flow case, tests/unit/gpu_cuda/rife_fused_test.cpp:131-179)."""
    plan = nets.RIFE_PLANS["4.25"]
    p = {k: np.zeros(s, np.float32) for k, s in nets.rife_param_shapes(plan)}
    flat = nets.rife_flat(p, plan)
    rng = np.random.default_rng(4)
    a = f16(rng.random((1, 3, 64, 64), dtype=np.float32))
    b = f16(rng.random((1, 3, 64, 64), dtype=np.float32))
    out = run(flat, a, b, 0.5)
    np.testing.assert_array_equal(out, f16(a * np.float32(0.5) + b * np.float32(0.5)))


def test_rife42_geometry_and_refusals():
    import torch
    flat = flat_of("4.25")
    eng = engine(flat, 72, 100, 1)
    try:
        assert eng.rife_geometry() == (128, 128, 14, 28)
        with pytest.raises(kb.KB2Error) as e:
            eng.set_timestep(1.0)
        assert e.value.status == kb.KB2_INVALID_ARGUMENT
        x = torch.zeros((1, 3, 72, 100), dtype=torch.float16, device="cuda")
        wrong = torch.zeros((1, 3, 72, 98), dtype=torch.float16, device="cuda")
        with pytest.raises(kb.KB2Error):
            eng.enqueue([x, x], [wrong])
        with pytest.raises(kb.KB2Error):
            eng.enqueue([torch.zeros((2, 3, 72, 100), dtype=torch.float16, device="cuda")] * 2,
                        [torch.zeros((2, 3, 72, 100), dtype=torch.float16, device="cuda")])
    finally:
        eng.close()
    with pytest.raises(kb.KB2Error) as e:
        kb.Engine(kb.MODEL_RIFE_FUSED, kb.make_blob(kb.MODEL_RIFE_FUSED, flat), 72, 100, max_batch=1,
                  precision=kb.PREC_FP8)
    assert e.value.status == kb.KB2_FORMAT_UNSUPPORTED
