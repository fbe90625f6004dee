"""Frames at any instant from one mid-pair motion (warp_blend_at) and the motion's 99.9th percentile
(flow_max), CPU side: the numpy restatement (oracle/nets.py) against the reference's own CPU
implementation (src/kernels/ref/warp.cpp, golden fixtures from tests/golden/make_warp_golden.py)."""
import numpy as np
import pytest

from oracle import nets
from util import golden


@pytest.mark.parametrize("name", ["warp_blend_36x52_win.npz", "warp_blend_64x96_full.npz"])
def test_warp_blend_restatement_matches_reference(name):
    g = golden(name)
    win = tuple(int(v) for v in g["window"])
    for warp in (0, 1):
        for i, t in enumerate(g["times"]):
            out = nets.warp_blend_at(g["a"], g["b"], g["flow"], g["mask"], win, float(t), warp)
            if t == 0.5:  # no ln / exp: the same FP32 operations in the same order
                np.testing.assert_array_equal(out, g["out"][warp, i])
            else:  # numpy's ln / exp against the C library's
                np.testing.assert_allclose(out, g["out"][warp, i], rtol=0, atol=2e-6)
    assert nets.flow_max(g["flow"], win) == float(g["flow_max"])


def test_flow_max_edges():
    win = (0, 0, 40, 25)
    flow = np.zeros((4, 25, 40), np.float32)
    assert nets.flow_max(flow, win) == 0.0  # no motion: bin 0
    flow[2] = 1000.0  # beyond the last bin: the last bin's edge
    assert nets.flow_max(flow, win) == 255 * 0.25
    flow[2] = 0.0
    flow[0, 0, 0] = 50.0  # one point of 1,000 does not move the 99.9th percentile
    assert nets.flow_max(flow, win) == 0.0
    flow[0, 0, :2] = 50.0  # two points of 1,000 do: rank 999 of 1,000
    assert nets.flow_max(flow, win) == 50.0


def test_keep_poses_restatement_matches_reference():
    g = golden("warp_poses_40x60.npz")
    win = tuple(int(v) for v in g["window"])
    k = 0
    for warp in (0, 1):
        for t in g["times"]:
            for pf, pm in ((g["prev_flow"], g["prev_mask"]), (None, None)):
                out = nets.warp_blend_poses(g["a"], g["b"], g["flow"], g["mask"], pf, pm, win, float(t), warp)
                np.testing.assert_allclose(out, g["out"][k], rtol=0, atol=1e-5)
                k += 1


def test_pan_lock_restatement_matches_reference():
    g = golden("warp_pan_64x96.npz")
    win = tuple(int(v) for v in g["window"])
    dx, dy, sure = nets.pan_estimate(g["a"], g["b"])
    np.testing.assert_array_equal(np.array([dx, dy, float(sure)], np.float32), g["pan"])
    for i, t in enumerate(g["times"]):
        out = nets.warp_blend_at(g["a"], g["b"], g["flow"], g["mask"], win, float(t), 0, 1)
        np.testing.assert_allclose(out, g["out"][i], rtol=0, atol=2e-6)
    for lock in (0, 1):  # a motion estimated at the output instant
        out = nets.warp_blend_at(g["a"], g["b"], g["flow"], g["mask"], win, 0.3, 0, lock, 1)
        np.testing.assert_allclose(out, g["out_instant"][lock], rtol=0, atol=2e-6)
