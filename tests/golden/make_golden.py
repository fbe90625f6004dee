"""Generates tests/golden/*.npz from the reference's own FP32 CPU interpreter.

    make -C oracle REF=<reference checkout>     # builds oracle/_ref/libkirari_ref.so from the reference sources
    python tests/golden/make_golden.py [--config0]      (--config0: only the ~60 s configs[0] frame)

The fixtures pin the numpy restatement (oracle/nets.py) and, through it, the CUDA path. Weights are
regenerated from their seeds by oracle/nets.py; each fixture stores a SHA-256 of the flat float32
parameters so that a change of the generator is caught instead of silently compared.
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


def digest(a):
    return hashlib.sha256(np.ascontiguousarray(a, np.float32).tobytes()).hexdigest()


def span_case(name, n, h, w, seed, fq=False):
    rng = np.random.default_rng(seed)
    x = rng.random((n, 3, h, w), dtype=np.float32)
    flat = nets.span_flat(nets.span_init(1))
    scales = None
    if fq:
        taps = {}
        nets.span_forward(x, nets.span_init(1), taps=taps)
        scales = nets.span_scales_from_peaks([max(taps[i]) for i in range(19)], floor=2.0 ** -14)
    out = ref_lib.span_forward(x, flat, scales)
    extra = {} if scales is None else {"act_scales": scales}
    np.savez_compressed(os.path.join(OUT, name), x=x, out=out, param_seed=1, param_sha256=digest(flat), **extra)
    print(name, out.shape)


def ifnet_case(name, n, h, w, seed, shift, t):
    rng = np.random.default_rng(seed)
    a = rng.random((n, 3, h, w), dtype=np.float32)
    b = np.roll(a, shift, axis=3).copy()
    flat = nets.ifnet_flat(nets.ifnet_init(2))
    out = ref_lib.ifnet_forward(a, b, t, flat)
    np.savez_compressed(os.path.join(OUT, name), a=a, b=b, t=np.float32(t), out=out, param_seed=2,
                        param_sha256=digest(flat))
    print(name, out.shape)


def span_config0(name):
    """one 1x3x270x480 frame, uniform [0, 1] FP32 from seed 0, through the reference's
    interpreter after rounding to FP16 (the engines take FP16 frames). The 540x960 output is stored
    in FP16 (an error of at most 2^-12 below 1, against a 2/255 bar) to keep the fixture small; the
    input is regenerated from its seed by the test and checked against the stored digest."""
    x = np.random.default_rng(0).random((1, 3, 270, 480), dtype=np.float32)
    x = x.astype(np.float16).astype(np.float32)
    flat = nets.span_flat(nets.span_init(1))
    out = ref_lib.span_forward(x, flat)
    np.savez_compressed(os.path.join(OUT, name), out=out.astype(np.float16), x_seed=0, x_sha256=digest(x),
                        param_seed=1, param_sha256=digest(flat))
    print(name, out.shape)


if __name__ == "__main__":
    if "--config0" in sys.argv:
        span_config0("span_config0_270x480.npz")
        sys.exit(0)
    span_case("span_fp32_16x24.npz", 1, 16, 24, seed=0)
    span_case("span_fp32_2x20x136.npz", 2, 20, 136, seed=5)
    span_case("span_fq_16x24.npz", 1, 16, 24, seed=0, fq=True)
    ifnet_case("ifnet_64x96_t05.npz", 1, 64, 96, seed=3, shift=3, t=0.5)
    ifnet_case("ifnet_64x96_t03.npz", 1, 64, 96, seed=4, shift=-2, t=0.3)
