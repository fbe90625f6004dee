"""RIFE 4.2x without a GPU: the oracle's graph pinned to the reference's own statement of the fused
RIFE glue, and the C ABI's plan checks, which refuse a bad blob before touching a device.

The pin: oracle/ref_graphs.cpp builds RIFE 4.2x from the reference's IR operators; its block
inputs X_k, final image, flow and mask are compared with src/kernels/ref/rife_fused.cpp
(rife_fused_block_input / rife_fused_finish, double precision), fed the graph's own encodings and
block outputs Y_k. Agreement to FP32 rounding shows the graph wires the channels, resizes, flow
sums and warps the way the reference's fused RIFE does."""
import numpy as np
import pytest

import kirari_b200 as kb
from oracle import nets, ref_lib
from util import ensure_built

GLUE_MAX_ABS = 1e-3  # FP32 graph vs double glue statement


def flat_of(name, seed=3):
    plan = nets.RIFE_PLANS[name]
    return nets.rife_flat(nets.rife_init(plan, seed=seed), plan)


@pytest.mark.skipif(not ref_lib.available(), reason="oracle/_ref not built (needs the reference sources)")
@pytest.mark.parametrize("name,h,w", [("4.25", 64, 128), ("4.26", 64, 64), ("4.22lite", 64, 96),
                                      ("4.25lite", 128, 128)])
def test_graph_glue_matches_reference_statement(name, h, w):
    from synth import shifted_pair
    a, b = shifted_pair(h, w, seed=12)
    flat = flat_of(name)
    err = ref_lib.rife42_glue_check(a[None], b[None], 0.5, flat)
    blocks = int(flat[0])
    print(name, "X_k:", ["%.1e" % e for e in err[:blocks]], "image %.1e flow %.1e mask %.1e" % tuple(err[blocks:]))
    assert max(err) <= GLUE_MAX_ABS


def test_param_counts_match_the_header():
    """12 plan floats + the parameters of include/kirari_b200.h's KB2_MODEL_RIFE_FUSED order."""
    for name, (blocks, reduce, channels) in nets.RIFE_PLANS.items():
        n = 16 * 27 + 32 + 2 * (16 * 16 * 9 + 32) + 16 * 4 * 16 + 4
        for k in range(blocks):
            c, cin = channels[k], 15 if k == 0 else 28
            n += (c // 2) * cin * 9 + c + c * (c // 2) * 9 + 2 * c + 8 * (c * c * 9 + 3 * c) + c * 52 * 16 + 52
        assert nets.rife_flat(nets.rife_init((blocks, reduce, channels)), (blocks, reduce, channels)).size == 12 + n


def _status(flat, h=64, w=64):
    try:
        kb.Engine(kb.MODEL_RIFE_FUSED, kb.make_blob(kb.MODEL_RIFE_FUSED, flat), h, w, max_batch=1)
    except kb.KB2Error as e:
        return e.status
    return kb.KB2_OK


def test_plan_refusals_before_device():
    ensure_built()
    good = flat_of("4.25")
    # a valid blob gets past every weight check (on a machine without the GPU it then fails at
    # the device, with another status)
    assert _status(good) != kb.KB2_WEIGHTS_INVALID

    def bad(i, v):
        f = good.copy()
        f[i] = v
        return f

    assert _status(bad(0, 6)) == kb.KB2_WEIGHTS_INVALID        # 6 blocks
    assert _status(bad(0, 4.5)) == kb.KB2_WEIGHTS_INVALID      # not an integer
    assert _status(bad(1, 3)) == kb.KB2_WEIGHTS_INVALID        # d_0 not a power of two
    assert _status(bad(1, 1)) == kb.KB2_WEIGHTS_INVALID        # d_0 < 2
    assert _status(bad(5, 2)) == kb.KB2_WEIGHTS_INVALID        # last d != 1
    assert _status(bad(11, 32)) == kb.KB2_WEIGHTS_INVALID      # encoder width
    assert _status(bad(6, 80)) == kb.KB2_FORMAT_UNSUPPORTED    # a block width the kernels do not have
    assert _status(good[:-1]) == kb.KB2_WEIGHTS_INVALID        # parameter count
    lite = flat_of("4.22lite")
    assert _status(lite) != kb.KB2_WEIGHTS_INVALID
    assert _status(np.concatenate([lite[:5], [4.0], lite[6:]])) == kb.KB2_WEIGHTS_INVALID  # d past the last block
    assert _status(good[:8]) == kb.KB2_WEIGHTS_INVALID         # no room for the plan
