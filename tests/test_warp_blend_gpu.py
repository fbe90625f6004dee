"""kb2_warp_blend_at and kb2_flow_max on the B200, against the reference's own CPU warp_blend_at /
flow_max (golden fixtures) and the numpy restatement (oracle/nets.py, pinned by
tests/test_warp_blend.py).

Bars: at t = 1/2 (flow and mask read as they are; no ln / exp) the FP16 output equals the FP16
rounding of the reference's and the restatement's FP32 result, bit for bit (both frame filters); at other t CUDA's logf / expf stand for the
host's, and the output stays within 2e-3 of the FP32 result (FP16 rounding of values up to 1 plus
that); flow_max is exact."""
import numpy as np
import pytest

import kirari_b200 as kb
from oracle import nets
from util import ensure_built, golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _built():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ensure_built()


def _dev(x, dtype):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).to(dtype).cuda()


def _run(a, b, flow, mask, win, t, warp=0):
    import torch
    out = kb.warp_blend_at(_dev(a, torch.float16), _dev(b, torch.float16), _dev(flow, torch.float32),
                           _dev(mask, torch.float32), win, t, warp=warp)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


@pytest.mark.parametrize("name", ["warp_blend_36x52_win.npz", "warp_blend_64x96_full.npz"])
def test_warp_blend_matches_reference_golden(name):
    g = golden(name)
    win = tuple(int(v) for v in g["window"])
    for warp in (0, 1):
        for i, t in enumerate(g["times"]):
            out = _run(g["a"][None], g["b"][None], g["flow"][None], g["mask"][None], win, float(t), warp)[0]
            if t == 0.5:
                np.testing.assert_array_equal(out, g["out"][warp, i].astype(np.float16).astype(np.float32))
            else:
                assert np.abs(out - g["out"][warp, i]).max() <= 2e-3, f"t={t} warp={warp}"
    import torch
    got = kb.flow_max(_dev(g["flow"][None], torch.float32), _dev(g["mask"][None], torch.float32), win)
    assert got == [float(g["flow_max"])]


def test_warp_blend_batch_against_restatement():
    import torch
    rng = np.random.default_rng(7)
    n, h, w, ph, pw = 3, 70, 130, 48, 80
    win = (5, 3, 66, 40)
    a = rng.random((n, 3, h, w), dtype=np.float32).astype(np.float16).astype(np.float32)
    b = rng.random((n, 3, h, w), dtype=np.float32).astype(np.float16).astype(np.float32)
    flow = (rng.standard_normal((n, 4, ph, pw)) * 5.0).astype(np.float32)
    flow[1, 0, 4, 9] = np.nan  # NaN reads as 0 in the clamp, as fmaxf
    mask = rng.random((n, ph, pw), dtype=np.float32)
    for t, warp in ((0.5, 0), (0.3, 0), (0.5, 1), (0.7, 1)):
        out = _run(a, b, flow, mask, win, t, warp)
        for i in range(n):
            ref = nets.warp_blend_at(a[i], b[i], flow[i], mask[i], win, t, warp)
            if t == 0.5:
                np.testing.assert_array_equal(out[i], ref.astype(np.float16).astype(np.float32))
            else:
                assert np.abs(out[i] - ref).max() <= 2e-3
    got = kb.flow_max(_dev(flow, torch.float32), _dev(mask, torch.float32), win)
    assert got == [nets.flow_max(flow[i], win) for i in range(n)]


def test_warp_blend_refusals():
    import torch
    a = torch.zeros((1, 3, 8, 8), dtype=torch.float16, device="cuda")
    flow = torch.zeros((1, 4, 8, 8), dtype=torch.float32, device="cuda")
    mask = torch.zeros((1, 8, 8), dtype=torch.float32, device="cuda")
    for t in (0.0, 1.0, float("nan")):
        with pytest.raises(kb.KB2Error) as e:
            kb.warp_blend_at(a, a, flow, mask, (0, 0, 8, 8), t)
        assert e.value.status == kb.KB2_INVALID_ARGUMENT
    with pytest.raises(kb.KB2Error) as e:
        kb.warp_blend_at(a, a, flow, mask, (2, 0, 8, 8), 0.5)  # window past the planes
    assert e.value.status == kb.KB2_SHAPE_INVALID


def test_keep_poses_matches_reference_golden():
    import torch
    g = golden("warp_poses_40x60.npz")
    win = tuple(int(v) for v in g["window"])
    k = 0
    for warp in (0, 1):
        for t in g["times"]:
            for prev in (True, False):
                out = kb.warp_blend_poses(_dev(g["a"][None], torch.float16), _dev(g["b"][None], torch.float16),
                                          _dev(g["flow"][None], torch.float32), _dev(g["mask"][None], torch.float32),
                                          _dev(g["prev_flow"][None], torch.float32) if prev else None,
                                          _dev(g["prev_mask"][None], torch.float32) if prev else None, win, float(t),
                                          warp=warp)
                torch.cuda.synchronize()
                err = np.abs(out.float().cpu().numpy()[0] - g["out"][k]).max()
                assert err <= 2e-3, f"t={t} prev={prev} warp={warp}"
                k += 1


def test_pan_lock_matches_reference_golden():
    import torch
    g = golden("warp_pan_64x96.npz")
    win = tuple(int(v) for v in g["window"])
    for i, t in enumerate(g["times"]):
        out = kb.warp_blend_at(_dev(g["a"][None], torch.float16), _dev(g["b"][None], torch.float16),
                               _dev(g["flow"][None], torch.float32), _dev(g["mask"][None], torch.float32), win,
                               float(t), pan_lock=1)
        torch.cuda.synchronize()
        assert np.abs(out.float().cpu().numpy()[0] - g["out"][i]).max() <= 2e-3, f"t={t}"
    for lock in (0, 1):  # a motion estimated at the output instant, read as it is
        out = kb.warp_blend_at(_dev(g["a"][None], torch.float16), _dev(g["b"][None], torch.float16),
                               _dev(g["flow"][None], torch.float32), _dev(g["mask"][None], torch.float32), win, 0.3,
                               pan_lock=lock, at_instant=1)
        torch.cuda.synchronize()
        assert np.abs(out.float().cpu().numpy()[0] - g["out_instant"][lock]).max() <= 2e-3, f"instant lock={lock}"
    # the lock changes the result here (a sure pan and sub-2-px flow)
    plain = _run(g["a"][None], g["b"][None], g["flow"][None], g["mask"][None], win, 0.3)[0]
    assert np.abs(plain - g["out"][1]).max() > 1e-2
