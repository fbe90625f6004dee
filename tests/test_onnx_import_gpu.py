"""RIFE 4.2x from ONNX pieces through to the B200: a model exported with FP16 initializers and PRelu
activations, cut into the pieces the reference's splitter hands its native reader, imported by
kb2_rife_blob_from_onnx, run by the KB2_MODEL_RIFE_FUSED engine and compared with the reference's
FP32 interpreter on the weights the pieces hold (the FP16-rounded values).

Tolerance: the FP16 bar, image max-abs <= 2/255 after clamp to [0, 1] vs FP32."""
import numpy as np
import pytest

import kirari_b200 as kb
import onnx_pieces as op
import seeded
from oracle import nets
from test_rife42_gpu import FP16_MAX_ABS, f16, padded_oracle, run
from util import ensure_built

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _built():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ensure_built()


def test_onnx_pieces_run_on_the_engine():
    plan = seeded.RIFE_PLANS["4.22lite"]
    blocks, reduce, _ = plan
    p = seeded.rife_init(plan, seed=5)
    opts = dict(dtype=op.FLOAT16, act="prelu")
    pieces = [op.encoder_piece(p, **opts)] + [op.block_piece(p, k, **opts) for k in range(blocks)]
    blob = kb.rife_blob_from_onnx(pieces, list(reduce))
    flat = np.frombuffer(blob, "<f4", offset=32).copy()
    # the weights the pieces hold: FP16-rounded weights and biases, FP32 slopes and betas
    want = {n: (v if n.endswith(".slope") or n.endswith(".beta") else op.representable(v, op.FLOAT16))
            for n, v in p.items()}
    assert np.array_equal(flat, seeded.rife_flat(want, plan))
    rng = np.random.default_rng(11)
    a = f16(rng.random((1, 3, 64, 128), dtype=np.float32))
    b = f16(np.roll(a, 3, axis=3))
    import torch
    n, _, h, w = a.shape
    eng = kb.Engine(kb.MODEL_RIFE_FUSED, blob, h, w, max_batch=n)
    try:
        eng.set_timestep(0.5)
        ta = torch.from_numpy(np.ascontiguousarray(a, np.float16)).cuda()
        tb = torch.from_numpy(np.ascontiguousarray(b, np.float16)).cuda()
        out = torch.full((n, 3, h, w), float("nan"), dtype=torch.float16, device="cuda")
        eng.enqueue([ta, tb], [out])
        eng.check_device()
        got = out.float().cpu().numpy()
    finally:
        eng.close()
    ref, _, _, _ = padded_oracle(a, b, 0.5, flat)
    err = nets.max_abs_clamped(got, ref)
    print(f"RIFE 4.22 lite from ONNX pieces (FP16, PRelu): max-abs {err * 255:.3f}/255")
    assert np.isfinite(got).all() and err <= FP16_MAX_ABS
    # the same blob as the seeded path's run of those weights
    assert np.array_equal(got, run(flat, a, b, 0.5))
