"""Generates tests/golden/warp_*.npz from the reference's own CPU warp_blend_at, warp_blend_poses and
flow_max (src/kernels/ref/warp.cpp:261, :270, :290), built into oracle/_ref/libkirari_ref.so by oracle/Makefile.

    make -C oracle REF=<reference checkout>
    python tests/golden/make_warp_golden.py

Frames are rounded to FP16 first (the library's frame format), so the GPU path reads the same values.
Outputs cover both frame filters (bilinear, Catmull-Rom); the reference's kernels/ sources are built
without multiply-add contraction, as the reference builds them.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import ref_lib  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
TIMES = (0.5, 0.25, 0.7)

# (name, frame h, w, plane h, w, window (x, y, w, h), flow scale, seed)
CASES = [
    ("warp_blend_36x52_win", 36, 52, 24, 40, (3, 2, 30, 20), 3.0, 1),
    ("warp_blend_64x96_full", 64, 96, 64, 96, (0, 0, 96, 64), 6.0, 2),
]


def main():
    for name, h, w, ph, pw, win, scale, seed in CASES:
        rng = np.random.default_rng(seed)
        a = rng.random((3, h, w), dtype=np.float32).astype(np.float16).astype(np.float32)
        b = rng.random((3, h, w), dtype=np.float32).astype(np.float16).astype(np.float32)
        flow = (rng.standard_normal((4, ph, pw)) * scale).astype(np.float32)
        mask = rng.random((ph, pw), dtype=np.float32)
        # [filter][t]: bilinear, then Catmull-Rom frame reads
        outs = np.stack([np.stack([ref_lib.warp_blend_at(a, b, flow, mask, win, t, warp) for t in TIMES])
                         for warp in (0, 1)])
        fmax = ref_lib.flow_max(flow, mask, win)
        np.savez_compressed(os.path.join(OUT, name + ".npz"), a=a, b=b, flow=flow, mask=mask,
                            window=np.array(win, np.int32), times=np.array(TIMES, np.float32), out=outs,
                            flow_max=np.float32(fmax))
        print(name, outs.shape, fmax)


def smooth_motion(ph, pw, amp, phase):
    """A smooth flow (4 planes) and mask: keeping the poses iterates q = pa - f1'(q), which amplifies
    rounding differences (the reference build's multiply-add contraction) on rough random fields."""
    yy, xx = np.meshgrid(np.linspace(0, 3, ph, dtype=np.float32), np.linspace(0, 3, pw, dtype=np.float32),
                         indexing="ij")
    flow = np.stack([np.sin(xx + phase) * amp, np.cos(yy) * 0.75 * amp, -np.sin(xx + 1 + phase) * amp,
                     np.cos(yy + 0.5) * 0.5 * amp]).astype(np.float32)
    mask = (0.5 + 0.4 * np.sin(xx + yy + phase)).astype(np.float32)
    return flow, mask


def poses():
    h, w, ph, pw, win = 40, 60, 32, 48, (4, 3, 40, 26)
    rng = np.random.default_rng(3)
    a = rng.random((3, h, w), dtype=np.float32).astype(np.float16).astype(np.float32)
    b = rng.random((3, h, w), dtype=np.float32).astype(np.float16).astype(np.float32)
    flow, mask = smooth_motion(ph, pw, 2.5, 0.0)
    pflow, pmask = smooth_motion(ph, pw, 1.0, 0.7)
    outs = np.stack([ref_lib.warp_blend_poses(a, b, flow, mask, pf, pm, win, t, warp)
                     for warp in (0, 1) for t in TIMES for pf, pm in ((pflow, pmask), (None, None))])
    np.savez_compressed(os.path.join(OUT, "warp_poses_40x60.npz"), a=a, b=b, flow=flow, mask=mask, prev_flow=pflow,
                        prev_mask=pmask, window=np.array(win, np.int32), times=np.array(TIMES, np.float32), out=outs)
    print("warp_poses_40x60", outs.shape)


def pan():
    """A pair that moves as a whole by (2, 1) px, RIFE-like flow near it with a smooth error, the pan
    lock on."""
    sys.path.insert(0, os.path.join(ROOT, "ultimate-anime-videoplayer_b200"))
    from synth import anime_frames
    h, w = 64, 96
    a = anime_frames(1, h, w, seed=3)[0].astype(np.float16).astype(np.float32)
    b = np.roll(a, (1, 2), axis=(1, 2))
    yy, xx = np.meshgrid(np.linspace(0, 3, h, dtype=np.float32), np.linspace(0, 3, w, dtype=np.float32),
                         indexing="ij")
    flow = np.stack([-1.0 + 0.3 * np.sin(xx), np.full_like(xx, -0.5), np.full_like(xx, 1.0) + 0.1 * np.sin(yy),
                     0.5 + 0.2 * np.cos(yy)]).astype(np.float32)
    flow[:, 40:, 60:] *= 4.0  # a region that moves on its own: its flow stays RIFE's
    mask = (0.5 + 0.3 * np.sin(xx + yy)).astype(np.float32)
    win = (0, 0, w, h)
    times = (0.5, 0.3)
    outs = np.stack([ref_lib.warp_blend_at(a, b, flow, mask, win, t, 0, 1) for t in times])
    # the same motion taken as estimated at the output instant (read as it is), without and with the lock
    instant = np.stack([ref_lib.warp_blend_at(a, b, flow, mask, win, 0.3, 0, lock, 1) for lock in (0, 1)])
    np.savez_compressed(os.path.join(OUT, "warp_pan_64x96.npz"), a=a, b=b, flow=flow, mask=mask,
                        window=np.array(win, np.int32), times=np.array(times, np.float32), out=outs,
                        out_instant=instant,
                        pan=np.array(ref_lib.pan_estimate(a, b), np.float32))
    print("warp_pan_64x96", outs.shape, ref_lib.pan_estimate(a, b))


if __name__ == "__main__":
    main()
    poses()
    pan()
