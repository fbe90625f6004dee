"""Display-ring pixels (RGBA16, RGB10A2, dithered RGB10A2), CPU side: the numpy restatement
(oracle/nets.py pack_display) against the reference's own packing (src/kernels/spec/ring_pack.h,
golden fixture from tests/golden/make_pack_golden.py), bit for bit."""
import numpy as np
import pytest

from oracle import nets
from util import golden


@pytest.mark.parametrize("fmt", [1, 2, 3])
def test_pack_restatement_matches_reference(fmt):
    g = golden("display_pack.npz")
    np.testing.assert_array_equal(nets.pack_display(g["x"], fmt), g[f"fmt{fmt}"])


def test_pack_known_codes():
    x = np.zeros((3, 1, 4), np.float32)
    x[:, 0, :] = [[0.0, 1.0, np.nan, 0.5]] * 3
    rgba = nets.pack_display(x, 1)
    assert rgba[0, :, 0].tolist() == [0, 65535, 0, 32768]
    assert (rgba[0, :, 3] == 65535).all()
    p = nets.pack_display(x, 2)[0]
    assert [(int(v) & 1023) for v in p] == [0, 1023, 0, 512] and all(int(v) >> 30 == 3 for v in p)
