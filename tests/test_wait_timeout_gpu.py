"""The bounded device wait behind KB2_KERNEL_TIMEOUT, exercised on the GPU without a fault: a wait on
a barrier that nothing completes (kb2_selftest_bounded_wait) gives up after its time limit, reports
its code, and leaves the device usable for the next engine."""
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


def test_bounded_wait_gives_up_and_the_device_stays_usable():
    import torch
    from synth import anime_frames
    rc, code, waited = kb.selftest_bounded_wait(0)
    assert rc == kb.KB2_KERNEL_TIMEOUT
    assert code == 0x500
    assert 1.9 <= waited <= 10.0, waited
    # the same process then runs an engine as usual: its output matches the oracle
    x = anime_frames(1, 16, 24, seed=3).astype(np.float16)
    p = nets.span_init(1)
    eng = kb.Engine(kb.MODEL_SPAN_X2, kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(p)), 16, 24)
    out = torch.empty((1, 3, 32, 48), dtype=torch.float16, device="cuda")
    eng.enqueue([torch.from_numpy(x).cuda()], [out])
    eng.check_device()
    eng.close()
    ref = nets.span_forward(x.astype(np.float32), p)
    assert nets.max_abs_clamped(out.float().cpu().numpy(), ref) <= 2.0 / 255.0


def test_bounded_wait_refuses_a_missing_device():
    import torch
    rc, _, _ = kb.selftest_bounded_wait(torch.cuda.device_count() + 3)
    assert rc == kb.KB2_INPUT_MISMATCH
