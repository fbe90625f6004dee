"""kb2_pack_display on the B200, bit for bit against the reference's packing (golden fixture) and the
numpy restatement, on frames of FP16 values."""
import numpy as np
import pytest

import kirari_b200 as kb
from oracle import nets
from util import ensure_built, golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _built():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ensure_built()


def _pack(x, fmt):
    import torch
    out = kb.pack_display(torch.from_numpy(np.ascontiguousarray(x)).to(torch.float16).cuda(), fmt)
    torch.cuda.synchronize()
    o = out.cpu().numpy()
    return o.view(np.uint16) if fmt == 1 else o.view(np.uint32)


@pytest.mark.parametrize("fmt", [1, 2, 3])
def test_pack_matches_reference_golden(fmt):
    g = golden("display_pack.npz")
    np.testing.assert_array_equal(_pack(g["x"][None], fmt)[0], g[f"fmt{fmt}"])


@pytest.mark.parametrize("fmt", [1, 2, 3])
def test_pack_batch_against_restatement(fmt):
    rng = np.random.default_rng(9)
    x = rng.uniform(-0.2, 1.2, (2, 3, 37, 301)).astype(np.float16).astype(np.float32)
    got = _pack(x, fmt)
    for i in range(2):
        np.testing.assert_array_equal(got[i], nets.pack_display(x[i], fmt))


def test_pack_refusals():
    import torch
    x = torch.zeros((1, 3, 4, 4), dtype=torch.float16, device="cuda")
    out = torch.zeros(64, dtype=torch.int32, device="cuda")
    t = kb.to_kb2_tensor(x)
    lib = kb.lib()
    assert lib.kb2_pack_display(None, kb.ctypes.byref(t), 7, kb.ctypes.c_void_p(out.data_ptr()), 16) == \
        kb.KB2_FORMAT_UNSUPPORTED
    assert lib.kb2_pack_display(None, kb.ctypes.byref(t), 2, kb.ctypes.c_void_p(out.data_ptr()), 12) == \
        kb.KB2_INPUT_MISMATCH  # a row of 4 pixels needs 16 bytes
