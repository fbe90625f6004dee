"""Generates tests/golden/warp_blend_*.npz from the reference's own CPU warp_blend_at and flow_max
(src/kernels/ref/warp.cpp:261, :290), built into oracle/_ref/libkirari_ref.so by oracle/Makefile.

    make -C oracle
    python tests/golden/make_warp_golden.py

Frames are rounded to FP16 first (the library's frame format), so the GPU path reads the same values.
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
        outs = np.stack([ref_lib.warp_blend_at(a, b, flow, mask, win, t) for t in TIMES])
        fmax = ref_lib.flow_max(flow, mask, win)
        np.savez_compressed(os.path.join(OUT, name + ".npz"), a=a, b=b, flow=flow, mask=mask,
                            window=np.array(win, np.int32), times=np.array(TIMES, np.float32), out=outs,
                            flow_max=np.float32(fmax))
        print(name, outs.shape, fmax)


if __name__ == "__main__":
    main()
