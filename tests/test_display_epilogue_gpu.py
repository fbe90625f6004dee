"""SPAN x2 writing display pixels from its upsampler's epilogue (kb2_set_output_format), the way the
reference's last layer writes its ring (store_pixel, src/gpu/cuda/backend/span_native16_kernels.cuh:325):
bit for bit the pixels kb2_pack_display makes of the F16 frame the same engine writes (that pass is
itself pinned bit-exact to the reference's packing by tests/test_display_pack_gpu.py)."""
import numpy as np
import pytest

import kirari_b200 as kb
from oracle import nets
from util import ensure_built

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _built():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ensure_built()


def _frames_and_pixels(eng, x, fmt):
    import torch
    n, _, h, w = x.shape
    xin = torch.from_numpy(np.ascontiguousarray(x, np.float16)).cuda()
    eng.set_output_format(0)
    frame = torch.full((n, 3, 2 * h, 2 * w), float("nan"), dtype=torch.float16, device="cuda")
    eng.enqueue([xin], [frame])
    packed = kb.pack_display(frame, fmt)
    bpp = 8 if fmt == kb.DISPLAY_RGBA16 else 4
    eng.set_output_format(fmt)
    direct = torch.full((n, bpp, 2 * h, 2 * w), 0xAB, dtype=torch.uint8, device="cuda")
    eng.enqueue([xin], [direct])
    eng.check_device()
    return packed.cpu().numpy().view(np.uint8).reshape(-1), direct.cpu().numpy().reshape(-1)


@pytest.mark.parametrize("fmt", [kb.DISPLAY_RGBA16, kb.DISPLAY_RGB10A2, kb.DISPLAY_RGB10A2_DITHER])
@pytest.mark.parametrize("shape", [(2, 37, 300), (1, 20, 136)])
def test_display_epilogue_equals_packed_frame(fmt, shape):
    from synth import anime_frames
    n, h, w = shape
    x = anime_frames(n, h, w, seed=h + w).astype(np.float16)
    x[0, :, 0, :4] = [[-0.5, 2.0, np.nan, 1.0]] * 3  # out-of-range and NaN inputs reach the codes
    p = nets.span_init(1)
    eng = kb.Engine(kb.MODEL_SPAN_X2, kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(p)), h, w, max_batch=n)
    try:
        packed, direct = _frames_and_pixels(eng, x, fmt)
    finally:
        eng.close()
    np.testing.assert_array_equal(direct, packed)


def test_display_epilogue_fp8_engine():
    import torch
    from synth import anime_frames
    h, w = 48, 160
    p = nets.span_init(1)
    blob = kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(p))
    e16 = kb.Engine(kb.MODEL_SPAN_X2, blob, h, w, max_batch=4)
    e16.set_output_format(kb.DISPLAY_RGB10A2)  # calibration ignores it: its passes write F16 frames
    peaks = e16.calibrate(torch.from_numpy(anime_frames(4, h, w, seed=100).astype(np.float16)).cuda())
    e16.close()
    scales = nets.span_scales_from_peaks(peaks, floor=2.0 ** -14)
    eng = kb.Engine(kb.MODEL_SPAN_X2, blob, h, w, max_batch=2, precision=kb.PREC_FP8, act_scales=scales)
    try:
        packed, direct = _frames_and_pixels(eng, anime_frames(2, h, w, seed=5).astype(np.float16),
                                            kb.DISPLAY_RGB10A2)
    finally:
        eng.close()
    np.testing.assert_array_equal(direct, packed)


def test_output_format_refusals():
    import torch
    p = nets.span_init(1)
    eng = kb.Engine(kb.MODEL_SPAN_X2, kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(p)), 16, 32, max_batch=1)
    try:
        with pytest.raises(kb.KB2Error) as e:
            eng.set_output_format(7)
        assert e.value.status == kb.KB2_FORMAT_UNSUPPORTED
        eng.set_output_format(kb.DISPLAY_RGB10A2)
        x = torch.zeros((1, 3, 16, 32), dtype=torch.float16, device="cuda")
        for bad in (torch.zeros((1, 3, 32, 64), dtype=torch.float16, device="cuda"),  # the F16 frame
                    torch.zeros((1, 8, 32, 64), dtype=torch.uint8, device="cuda")):  # RGBA16's size
            with pytest.raises(kb.KB2Error) as e:
                eng.enqueue([x], [bad])
            assert e.value.status == kb.KB2_INPUT_MISMATCH
        eng.enqueue([x], [torch.zeros((1, 4, 32, 64), dtype=torch.uint8, device="cuda")])
        eng.check_device()
    finally:
        eng.close()
    ifn = kb.Engine(kb.MODEL_IFNET, kb.make_blob(kb.MODEL_IFNET, nets.ifnet_flat(nets.ifnet_init(2))), 64, 64)
    try:
        with pytest.raises(kb.KB2Error) as e:
            ifn.set_output_format(kb.DISPLAY_RGB10A2)
        assert e.value.status == kb.KB2_FORMAT_UNSUPPORTED
    finally:
        ifn.close()
