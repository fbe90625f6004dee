"""Generates tests/golden/span8_*.npz from the reference's own .span8 reader and FP32 CPU forward of
the unshuffle SPAN (src/gpu/span_fp8/package.cpp:143, forward.cpp:144), built into
oracle/_ref/libkirari_ref.so by oracle/Makefile.

    make -C oracle REF=<reference checkout>
    python tests/golden/make_span8_golden.py

The packages are regenerated from their seeds by oracle/nets.py (span8_init, span8_package); each
fixture stores the package's SHA-256 so that a change of the generator is caught instead of silently
compared, plus the frames and the reference's output.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import nets, ref_lib  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))

# (name, blocks, real channels, package seed, frames, height, width, frame seed)
CASES = [
    ("span8_b2f48_20x36", 2, 48, 21, 1, 20, 36, 5),
    ("span8_b3f64_16x30", 3, 64, 22, 2, 16, 30, 6),
]


def main():
    for name, blocks, real, seed, n, h, w, xseed in CASES:
        pkg = nets.span8_package(nets.span8_init(blocks, real, seed=seed))
        assert ref_lib.span8_parse(pkg)[0] == 0
        x = np.random.default_rng(xseed).random((n, 3, h, w), dtype=np.float32)
        out = ref_lib.span8_forward(pkg, x)
        np.savez_compressed(os.path.join(OUT, name + ".npz"), x=x, out=out, blocks=blocks, real=real, seed=seed,
                            package_sha256=hashlib.sha256(pkg).hexdigest())
        print(name, out.shape, float(out.min()), float(out.max()))


if __name__ == "__main__":
    main()
