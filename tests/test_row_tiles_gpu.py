"""SPAN x2 run as row tiles with a halo and stitched (kb2_set_row_tiles; configs[2] of the contract:
8 row tiles with an 8-pixel halo), on the B200 through the C ABI.

The network's receptive radius is 20 input rows, so a 20-row halo reproduces the whole-frame result
(up to the order of FP32 sums: a tile's rows map onto the pair kernel's accumulator slots with
another offset), while the contract's 8-row halo changes the rows near the seams. The 8-row case is
measured against the FP32 whole-frame reference: PSNR over the frame, and over the seam bands
(output rows within 2 x 20 of a seam) and the interior separately."""
import numpy as np
import pytest

import kirari_b200 as kb
import torch_ref
from oracle import nets
from util import ensure_built

pytestmark = pytest.mark.gpu

FP8_MIN_PSNR = 45.0


@pytest.fixture(scope="module", autouse=True)
def _built():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ensure_built()


def _run(eng, x, fmt=0):
    import torch
    n, _, h, w = x.shape
    eng.set_output_format(fmt)
    if fmt == 0:
        out = torch.full((n, 3, 2 * h, 2 * w), float("nan"), dtype=torch.float16, device="cuda")
    else:
        out = torch.zeros((n, 4, 2 * h, 2 * w), dtype=torch.uint8, device="cuda")
    eng.enqueue([torch.from_numpy(np.ascontiguousarray(x, np.float16)).cuda()], [out])
    eng.check_device()
    return out.cpu().numpy()


def _seam_rows(h, tiles, band=20):
    core = -(-h // tiles)
    rows = np.zeros(2 * h, bool)
    for t in range(1, tiles):
        c = 2 * t * core
        rows[max(0, c - 2 * band):min(2 * h, c + 2 * band)] = True
    return rows


def test_halo_at_the_receptive_radius_gives_the_whole_frame():
    from synth import anime_frames
    n, h, w = 2, 200, 264
    x = anime_frames(n, h, w, seed=77).astype(np.float16)
    p = nets.span_init(1)
    eng = kb.Engine(kb.MODEL_SPAN_X2, kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(p)), h, w, max_batch=n)
    try:
        whole = _run(eng, x).astype(np.float32)
        eng.set_row_tiles(5, 20)
        tiled = _run(eng, x).astype(np.float32)
        pix_whole = _run(eng, x, kb.DISPLAY_RGB10A2)  # stitched display pixels: the tiled frame's
        eng.set_row_tiles(1, 0)
        again = _run(eng, x).astype(np.float32)
    finally:
        eng.close()
    np.testing.assert_array_equal(again, whole)
    assert np.isfinite(tiled).all()
    diff = float(np.max(np.abs(tiled - whole)))
    print(f"5 tiles, halo 20: max |tiled - whole| = {diff:.2e}")
    assert diff <= 4e-3
    import torch
    packed = kb.pack_display(torch.from_numpy(tiled.astype(np.float16)).cuda(), kb.DISPLAY_RGB10A2)
    np.testing.assert_array_equal(pix_whole.reshape(-1), packed.cpu().numpy().view(np.uint8).reshape(-1))


def test_config2_eight_tiles_halo_8_fp8_1080p():
    """configs[2] as stated: 1080p, E4M3, 8 row tiles with an 8-pixel halo, stitched; PSNR against the
    FP32 whole frame, seams included, and its seam bands reported apart."""
    import torch
    from synth import anime_frames
    h, w, n = 1080, 1920, 2
    p = nets.span_init(1)
    blob = kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(p))
    e16 = kb.Engine(kb.MODEL_SPAN_X2, blob, h, w, max_batch=8)
    try:
        peaks = e16.calibrate(torch.from_numpy(anime_frames(16, h, w, seed=1000).astype(np.float16)).cuda())
    finally:
        e16.close()
    scales = nets.span_scales_from_peaks(peaks, floor=2.0 ** -14)
    x = anime_frames(n, h, w, seed=2024).astype(np.float16)
    eng = kb.Engine(kb.MODEL_SPAN_X2, blob, h, w, max_batch=n, precision=kb.PREC_FP8, act_scales=scales)
    try:
        whole = _run(eng, x).astype(np.float32)
        eng.set_row_tiles(8, 8)
        tiled = _run(eng, x).astype(np.float32)
    finally:
        eng.close()
    ref = torch_ref.span_forward(x.astype(np.float32), p)
    seam = _seam_rows(h, 8)
    for i in range(n):
        full = nets.psnr(tiled[i], ref[i])
        at_seams = nets.psnr(tiled[i][:, seam], ref[i][:, seam])
        inside = nets.psnr(tiled[i][:, ~seam], ref[i][:, ~seam])
        untiled = nets.psnr(whole[i], ref[i])
        print(f"frame {i}: 8 tiles halo 8 PSNR {full:.1f} dB (seam bands {at_seams:.1f}, interior {inside:.1f}); "
              f"whole frame {untiled:.1f} dB")
        assert full >= FP8_MIN_PSNR


def test_row_tile_refusals():
    p = nets.span_init(1)
    eng = kb.Engine(kb.MODEL_SPAN_X2, kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(p)), 16, 32, max_batch=1)
    try:
        for tiles, halo in ((9, 4), (2, 65), (-1, 0), (2, -1)):
            with pytest.raises(kb.KB2Error) as e:
                eng.set_row_tiles(tiles, halo)
            assert e.value.status == kb.KB2_SHAPE_INVALID
    finally:
        eng.close()
    ifn = kb.Engine(kb.MODEL_IFNET, kb.make_blob(kb.MODEL_IFNET, nets.ifnet_flat(nets.ifnet_init(2))), 64, 64)
    try:
        with pytest.raises(kb.KB2Error) as e:
            ifn.set_row_tiles(2, 8)
        assert e.value.status == kb.KB2_FORMAT_UNSUPPORTED
    finally:
        ifn.close()
