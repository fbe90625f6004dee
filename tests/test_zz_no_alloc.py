"""kb2_span_calibrate_static: the calibration entry point that allocates nothing, checked against
kb2_span_calibrate on the same engine and frames.

It exists for callers that cannot allocate device memory once they are running: a player that has
handed the rest of the GPU to its decoder and display ring, or a process under a hard memory cap.
Its scratch is a fixed 64 MiB device array compiled into the library, looked up in the current
context on every call. The file name sorts last so that the test also runs after every other GPU
test in one session (the static array is then first used late); the last test runs the same check
in a fresh process, where the static path is the first thing the library does on the device."""
import os
import subprocess
import sys

import numpy as np
import pytest

import kirari_b200 as kb
from oracle import nets
from util import ROOT, ensure_built


@pytest.fixture(scope="module", autouse=True)
def built():
    ensure_built()


def _static_matches_allocating(h, w, n, max_batch):
    """Peaks of the static path, called twice in a row, against kb2_span_calibrate's (bit-exact)."""
    import torch
    from synth import anime_frames
    blob = kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(nets.span_init(1)))
    frames = torch.from_numpy(anime_frames(n, h, w, seed=21).astype(np.float16)).cuda()
    eng = kb.Engine(kb.MODEL_SPAN_X2, blob, h, w, max_batch=max_batch)
    try:
        ref = eng.calibrate(frames)
        first = eng.calibrate_static(frames)
        second = eng.calibrate_static(frames)
        eng.check_device()
    finally:
        eng.close()
    assert (ref > 0).any()
    np.testing.assert_array_equal(first, ref)
    np.testing.assert_array_equal(second, ref)


@pytest.mark.gpu
def test_static_calibration_matches_allocating_entry_point():
    _static_matches_allocating(40, 136, 5, 2)  # 5 frames: chunks of max_batch = 2, 2, then 1


@pytest.mark.gpu
def test_static_calibration_chunks_by_what_fits_the_array():
    # one x2 output frame of 720x1280 is 22.1 MB, so 3 fit in the 64 MiB array, fewer than
    # max_batch = 4: the 5 frames run as chunks of 3 and 2, set by the array's size
    _static_matches_allocating(720, 1280, 5, 4)


@pytest.mark.gpu
def test_static_calibration_refuses_frames_beyond_the_array():
    import torch
    h, w = 1440, 2048  # 24 * H * W = 70.8 MB > 64 MiB
    blob = kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(nets.span_init(1)))
    eng = kb.Engine(kb.MODEL_SPAN_X2, blob, h, w, max_batch=1)
    try:
        frames = torch.zeros((1, 3, h, w), dtype=torch.float16, device="cuda")
        with pytest.raises(kb.KB2Error) as e:
            eng.calibrate_static(frames)
        assert e.value.status == kb.KB2_SHAPE_INVALID
        assert "static scratch holds 67108864" in str(e.value)
    finally:
        eng.close()


@pytest.mark.gpu
def test_static_calibration_in_a_fresh_process():
    code = ("import sys; sys.path[:0] = [sys.argv[1], sys.argv[2], sys.argv[3]]\n"
            "import test_zz_no_alloc as t\n"
            "t._static_matches_allocating(40, 136, 5, 2)\n"
            "print('fresh-process static calibration ok')\n")
    pkg = os.path.join(ROOT, "ultimate-anime-videoplayer_b200")
    r = subprocess.run([sys.executable, "-c", code, os.path.join(ROOT, "tests"), ROOT, pkg],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "fresh-process static calibration ok" in r.stdout
