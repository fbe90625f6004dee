"""Generates tests/golden/display_pack.npz from the reference's display-ring packing
(src/kernels/spec/ring_pack.h, color.h unorm16), built into oracle/_ref/libkirari_ref.so by
oracle/Makefile (without multiply-add contraction, as the reference compiles it).

    make -C oracle REF=<reference checkout>
    python tests/golden/make_pack_golden.py

The frame holds FP16 values (the engines' output format): a ramp over [-0.1, 1.1], the code
boundaries of both depths, NaN and infinities.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import ref_lib  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def frame():
    h, w = 24, 70
    rng = np.random.default_rng(4)
    x = rng.uniform(-0.1, 1.1, (3, h, w)).astype(np.float32)
    specials = np.array([0.0, 1.0, -0.0, np.nan, np.inf, -np.inf, 0.5, 0.25, 65504.0, -65504.0,
                         0.5 / 1023, 1.5 / 1023, 0.5 / 65535, 1022.5 / 1023, 6e-8], np.float32)
    x[0, 0, :specials.size] = specials
    x[1, 1, :specials.size] = specials[::-1]
    x[2, 2, :specials.size] = specials
    return x.astype(np.float16).astype(np.float32)


def main():
    x = frame()
    outs = {f"fmt{f}": ref_lib.pack_display(x, f) for f in (1, 2, 3)}
    np.savez_compressed(os.path.join(OUT, "display_pack.npz"), x=x, **outs)
    print({k: v.shape for k, v in outs.items()})


if __name__ == "__main__":
    main()
