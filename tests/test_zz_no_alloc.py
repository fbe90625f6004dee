"""kb2_span_calibrate_static: the calibration entry point that allocates nothing, checked against
kb2_span_calibrate on the same engine and frames. The file name sorts last so that the test also
runs after every other GPU test in one session (the static array is then first used late)."""
import numpy as np
import pytest

import kirari_b200 as kb
from oracle import nets
from util import ensure_built


@pytest.fixture(scope="module", autouse=True)
def built():
    ensure_built()


@pytest.mark.gpu
def test_static_calibration_matches_allocating_entry_point():
    import torch
    from synth import anime_frames
    h, w = 40, 136
    blob = kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(nets.span_init(1)))
    frames = torch.from_numpy(anime_frames(5, h, w, seed=21).astype(np.float16)).cuda()
    eng = kb.Engine(kb.MODEL_SPAN_X2, blob, h, w, max_batch=2)  # 5 frames: chunks of 2, 2, 1
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
