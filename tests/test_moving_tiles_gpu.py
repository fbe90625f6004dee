"""Moving tiles of SPAN x2 (kb2_span_tile_grid / kb2_next_span_tiles; the reference's
src/kernels/spec/span_tiles.h and Engine::next_span_tiles, src/gpu/backend.h:401-412), on the B200
through the C ABI.

The contract: the next enqueue computes only what the core tiles need and writes only them; the other
tiles keep the previous output (moved by the pan when one is given). Checks: the core tiles equal
the whole-frame result of the new frame (up to the order of FP32 sums) and the FP32 reference within
the FP16 bar; every other tile is bit-identical to the previous output, shifted or not."""
import numpy as np
import pytest

import kirari_b200 as kb
import torch_ref
from oracle import nets
from util import ensure_built

pytestmark = pytest.mark.gpu

FP16_MAX_ABS = 2.0 / 255.0
SUM_ORDER_MAX_ABS = 4e-3  # FP32 sum order (window rows map onto other accumulator slots), then FP16


@pytest.fixture(scope="module", autouse=True)
def _built():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ensure_built()


def dilate(core, reach):
    """kernels::dilate_span_tiles: every tile within `reach` tiles of a marked one."""
    rows, cols = core.shape
    out = np.zeros_like(core)
    for r, c in zip(*np.nonzero(core)):
        out[max(0, r - reach):min(rows, r + reach + 1), max(0, c - reach):min(cols, c + reach + 1)] = 1
    return out


def tiles_of(rect_y0, rect_y1, rect_x0, rect_x1, grid):
    """Tiles touched by the input rectangle [y0, y1) x [x0, x1)."""
    core = np.zeros((grid["rows"], grid["cols"]), np.uint8)
    t = grid["tile_w"]
    core[rect_y0 // t:(rect_y1 - 1) // t + 1, rect_x0 // t:(rect_x1 - 1) // t + 1] = 1
    return core


def run(eng, x, out=None, fmt=0):
    import torch
    n, _, h, w = x.shape
    if out is None:
        out = torch.full((n, 3, 2 * h, 2 * w), float("nan"), dtype=torch.float16, device="cuda")
    eng.enqueue([torch.from_numpy(np.ascontiguousarray(x, np.float16)).cuda()], [out])
    eng.check_device()
    return out


def mask_px(core, grid, scale=2):
    """Output-pixel mask of the core tiles."""
    t = grid["tile_w"] * scale
    return np.repeat(np.repeat(core, t, 0), t, 1)


@pytest.fixture(scope="module")
def setup():
    from synth import anime_frames
    # 9 x 6 tiles of 64 (the last row and column cut); a window is 64 + 2 x 20 = 104 rows, so up to
    # 4 dirty tile rows take the window path and more the whole-frame one
    h, w = 520, 328
    a = anime_frames(2, h, w, seed=41).astype(np.float16)
    b = a.copy()
    b[:, :, 70:110, 150:200] = anime_frames(2, 40, 50, seed=42).astype(np.float16)  # a moving character
    p = nets.span_init(1)
    return h, w, a, b, p


def test_grid(setup):
    h, w, a, b, p = setup
    eng = kb.Engine(kb.MODEL_SPAN_X2, kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(p)), h, w, max_batch=2)
    try:
        g = eng.span_tile_grid()
    finally:
        eng.close()
    assert g == {"tile_w": 64, "tile_h": 64, "cols": 6, "rows": 9, "reach_cols": 1, "reach_rows": 1,
                 "shift_step": 1, "scale": 2}


@pytest.mark.parametrize("in_place", [False, True])
def test_changed_tiles_only(setup, in_place):
    import torch
    h, w, a, b, p = setup
    eng = kb.Engine(kb.MODEL_SPAN_X2, kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(p)), h, w, max_batch=2)
    try:
        g = eng.span_tile_grid()
        out_a = run(eng, a)
        whole_b = run(eng, b).float().cpu().numpy()
        core = dilate(tiles_of(70, 110, 150, 200, g), g["reach_cols"])
        if in_place:
            out = out_a.clone()
            eng.next_span_tiles(core)  # the output buffer already holds the previous output
        else:
            out = torch.full_like(out_a, float("nan"))
            eng.next_span_tiles(core, previous=out_a)
        run(eng, b, out)
        got = out.float().cpu().numpy()
        again = run(eng, b).float().cpu().numpy()  # one call only: the next one is whole again
    finally:
        eng.close()
    np.testing.assert_array_equal(again, whole_b)
    m = mask_px(core, g)[:2 * h, :2 * w].astype(bool)
    prev = out_a.float().cpu().numpy()
    np.testing.assert_array_equal(got[:, :, ~m], prev[:, :, ~m])
    diff = float(np.max(np.abs(got[:, :, m] - whole_b[:, :, m])))
    ref = torch_ref.span_forward(b.astype(np.float32), p)
    err = nets.max_abs_clamped(got[:, :, m], ref[:, :, m])
    print(f"core {int(core.sum())} of {core.size} tiles: max |tiles - whole| {diff:.2e}, vs FP32 {err * 255:.3f}/255")
    assert diff <= SUM_ORDER_MAX_ABS
    assert err <= FP16_MAX_ABS


def test_pan_shifts_the_previous_output(setup):
    """A pan of 8 input pixels to the right: the previous output moves by 16 output pixels; the strip
    that enters on the left and the tiles within reach of either side border are core."""
    import torch
    h, w, a, b, p = setup
    s = 8
    b2 = np.zeros_like(a)
    b2[:, :, :, s:] = a[:, :, :, :w - s]
    b2[:, :, :, :s] = np.flip(a[:, :, :, :s], axis=3)
    eng = kb.Engine(kb.MODEL_SPAN_X2, kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(p)), h, w, max_batch=2)
    try:
        g = eng.span_tile_grid()
        out_a = run(eng, a)
        whole_b = run(eng, b2).float().cpu().numpy()
        core = np.zeros((g["rows"], g["cols"]), np.uint8)
        core[:, 0] = 1
        core[:, -1] = 1
        core = dilate(core, 0)
        out = torch.full_like(out_a, float("nan"))
        eng.next_span_tiles(core, s, 0, previous=out_a)
        run(eng, b2, out)
        got = out.float().cpu().numpy()
    finally:
        eng.close()
    m = mask_px(core, g)[:2 * h, :2 * w].astype(bool)
    prev = out_a.float().cpu().numpy()
    shifted = np.full_like(prev, np.nan)
    shifted[:, :, :, 2 * s:] = prev[:, :, :, :2 * w - 2 * s]
    np.testing.assert_array_equal(got[:, :, ~m], shifted[:, :, ~m])
    assert float(np.max(np.abs(got[:, :, m] - whole_b[:, :, m]))) <= SUM_ORDER_MAX_ABS


def test_most_tiles_take_the_whole_frame_path(setup):
    """With every tile row dirty the engine computes whole frames; it still writes the core only."""
    import torch
    h, w, a, b, p = setup
    eng = kb.Engine(kb.MODEL_SPAN_X2, kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(p)), h, w, max_batch=2)
    try:
        g = eng.span_tile_grid()
        out_a = run(eng, a)
        whole_b = run(eng, b).float().cpu().numpy()
        core = np.zeros((g["rows"], g["cols"]), np.uint8)
        core[:, 1::2] = 1  # every row dirty, half the tiles core
        out = out_a.clone()
        eng.next_span_tiles(core)
        run(eng, b, out)
        got = out.float().cpu().numpy()
    finally:
        eng.close()
    m = mask_px(core, g)[:2 * h, :2 * w].astype(bool)
    np.testing.assert_array_equal(got[:, :, m], whole_b[:, :, m])  # the very same whole-frame launch
    np.testing.assert_array_equal(got[:, :, ~m], out_a.float().cpu().numpy()[:, :, ~m])


def test_display_pixels(setup):
    """The same with display pixels (RGB10A2): core tiles equal the packed whole frame's up to one
    code of sum-order difference, the rest is the previous output's bytes."""
    import torch
    h, w, a, b, p = setup
    eng = kb.Engine(kb.MODEL_SPAN_X2, kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(p)), h, w, max_batch=2)
    try:
        eng.set_output_format(kb.DISPLAY_RGB10A2)
        g = eng.span_tile_grid()
        pix = lambda: torch.zeros((2, 4, 2 * h, 2 * w), dtype=torch.uint8, device="cuda")  # noqa: E731
        out_a = run(eng, a, pix())
        whole_b = run(eng, b, pix()).cpu().numpy().view(np.uint32)
        core = dilate(tiles_of(70, 110, 150, 200, g), 1)
        out = out_a.clone()
        eng.next_span_tiles(core)
        run(eng, b, out)
        got = out.cpu().numpy().view(np.uint32)
    finally:
        eng.close()
    # [n, 4, 2h, 2w] bytes viewed as uint32 along the last axis: pixels are rows of 2w words
    got = got.reshape(2, 2 * h, 2 * w)
    whole_b = whole_b.reshape(2, 2 * h, 2 * w)
    prev = out_a.cpu().numpy().view(np.uint32).reshape(2, 2 * h, 2 * w)
    m = mask_px(core, g)[:2 * h, :2 * w].astype(bool)
    np.testing.assert_array_equal(got[:, ~m], prev[:, ~m])
    for sh in (0, 10, 20):
        d = np.abs(((got[:, m] >> sh) & 1023).astype(np.int64) - ((whole_b[:, m] >> sh) & 1023).astype(np.int64))
        assert d.max() <= 2


def test_refusals(setup):
    import torch
    h, w, a, b, p = setup
    eng = kb.Engine(kb.MODEL_SPAN_X2, kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(p)), h, w, max_batch=2)
    try:
        g = eng.span_tile_grid()
        core = np.ones((g["rows"], g["cols"]), np.uint8)
        with pytest.raises(kb.KB2Error) as e:
            eng.next_span_tiles(core[:, :-1])
        assert e.value.status == kb.KB2_INPUT_MISMATCH
        with pytest.raises(kb.KB2Error) as e:
            eng.next_span_tiles(core, 2, 0)  # a shift needs the previous output
        assert e.value.status == kb.KB2_FORMAT_UNSUPPORTED
        with pytest.raises(kb.KB2Error) as e:
            eng.next_span_tiles(np.zeros_like(core))  # empty: cancels, the next call is whole
        assert e.value.status == kb.KB2_FORMAT_UNSUPPORTED
        eng.set_row_tiles(2, 8)
        with pytest.raises(kb.KB2Error) as e:
            eng.next_span_tiles(core)
        assert e.value.status == kb.KB2_FORMAT_UNSUPPORTED
        eng.set_row_tiles(1, 0)
        out = run(eng, a)
        wrong = torch.zeros((2, 3, 2 * h, 2 * w - 2), dtype=torch.float16, device="cuda")
        eng.next_span_tiles(core, previous=wrong)
        with pytest.raises(kb.KB2Error) as e:
            run(eng, a, out)
        assert e.value.status == kb.KB2_INPUT_MISMATCH
    finally:
        eng.close()
    ifn = kb.Engine(kb.MODEL_IFNET, kb.make_blob(kb.MODEL_IFNET, nets.ifnet_flat(nets.ifnet_init(2))), 64, 64)
    try:
        with pytest.raises(kb.KB2Error) as e:
            ifn.span_tile_grid()
        assert e.value.status == kb.KB2_FORMAT_UNSUPPORTED
    finally:
        ifn.close()
