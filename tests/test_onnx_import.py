"""kb2_rife_blob_from_onnx: the KB2_MODEL_RIFE_FUSED weight blob from the ONNX pieces of a split
RIFE 4.2x model, checked on the CPU (the importer is host code; nothing runs on a GPU).

- Against the seeded parameters: pieces written from them give exactly the blob kb.make_blob writes.
- Against the reference's own reader (src/prepare/rife_native.cpp rife_native_layers, compiled into
  oracle/_ref): every piece's layers, under each encoding a real export may use, bit-exact; a
  separable conv folded the reference's way; the same pieces refused.
"""
from __future__ import annotations

import numpy as np
import pytest

import kirari_b200 as kb
import onnx_pieces as op
import seeded
from oracle import ref_lib

PLAN = seeded.RIFE_PLANS["4.25"]
BLOCKS, REDUCE, CHANNELS = PLAN

needs_ref = pytest.mark.skipif(not ref_lib.available(), reason="oracle/_ref not built")


@pytest.fixture(scope="module")
def params():
    return seeded.rife_init(PLAN)


@pytest.fixture(scope="module")
def pieces(params):
    return [op.encoder_piece(params)] + [op.block_piece(params, k) for k in range(BLOCKS)]


def blob_floats(blob: bytes) -> np.ndarray:
    return np.frombuffer(blob, "<f4", offset=32)


def rounded(params, dtype):
    """The parameters as a reader returns them from weights stored in `dtype`: weights and biases
    rounded, slopes and betas (stored as FLOAT) as they are."""
    out = {}
    for name, v in params.items():
        keep = name.endswith(".slope") or name.endswith(".beta")
        out[name] = v if keep else op.representable(v, dtype)
    return out


def test_blob_from_pieces_is_the_seeded_blob(params, pieces):
    got = kb.rife_blob_from_onnx(pieces, list(REDUCE))
    want = kb.make_blob(kb.MODEL_RIFE_FUSED, seeded.rife_flat(params, PLAN))
    assert got == want


ENCODINGS = {
    "f32-typed": dict(storage="typed"),
    "f16-raw": dict(dtype=op.FLOAT16),
    "f16-int32-words": dict(dtype=op.FLOAT16, storage="typed"),
    "prelu": dict(act="prelu"),
    "constant-nodes": dict(constant_nodes=True),
    "identity-and-cast": dict(passthrough=True),
}


@pytest.mark.parametrize("enc", sorted(ENCODINGS))
def test_encodings_give_the_same_blob(params, enc):
    opts = ENCODINGS[enc]
    pieces = [op.encoder_piece(params, **opts)] + [op.block_piece(params, k, **opts) for k in range(2)]
    plan2 = (2, REDUCE[:2], CHANNELS[:2])
    want_params = rounded(params, opts.get("dtype", op.FLOAT))
    names = [n for n, _ in seeded.rife_param_shapes(plan2)]
    want = kb.make_blob(kb.MODEL_RIFE_FUSED, seeded.rife_flat({n: want_params[n] for n in names}, plan2))
    assert kb.rife_blob_from_onnx(pieces, list(REDUCE[:2])) == want


def ref_flat(layers) -> np.ndarray:
    """The reference reader's layers in the weight blob's order: w, b, [scale], [slope] per layer."""
    parts = []
    for l in layers:
        parts += [l["w"].reshape(-1), l["b"]]
        if l["scale"].size:
            parts.append(l["scale"])
        if l["slope"].size:
            parts.append(l["slope"])
    return np.concatenate(parts)


@needs_ref
@pytest.mark.parametrize("enc", sorted(ENCODINGS) + ["f32-raw"])
def test_layers_match_the_reference_reader(params, enc):
    opts = ENCODINGS.get(enc, {})
    pieces = [op.encoder_piece(params, **opts)] + [op.block_piece(params, k, **opts) for k in range(2)]
    got = blob_floats(kb.rife_blob_from_onnx(pieces, list(REDUCE[:2])))[12:]
    want = np.concatenate([ref_flat(ref_lib.rife_native_layers(p)) for p in pieces])
    assert got.shape == want.shape
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@needs_ref
def test_separable_conv_folds_like_the_reference(params):
    rng = np.random.default_rng(7)
    cin, mid = 15, CHANNELS[0] // 2
    dw = (rng.standard_normal((cin, 1, 3, 3)) * 0.3).astype(np.float32)
    db = (rng.standard_normal(cin) * 0.05).astype(np.float32)
    pw = (rng.standard_normal((mid, cin, 1, 1)) * 0.2).astype(np.float32)
    pb = (rng.standard_normal(mid) * 0.05).astype(np.float32)
    block = op.separable_block_piece(params, 0, dw, db, pw, pb)
    pieces = [op.encoder_piece(params), block, op.block_piece(params, 1)]
    got = blob_floats(kb.rife_blob_from_onnx(pieces, list(REDUCE[:2])))[12:]
    ref = [ref_lib.rife_native_layers(p) for p in pieces]
    assert ref[1][0]["cin"] == cin and ref[1][0]["cout"] == mid and ref[1][0]["stride"] == 2
    want = np.concatenate([ref_flat(layers) for layers in ref])
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # the fold is the composition: W'[o] = sum_m P[o][m] diag(dw)[m]
    w0 = got[ref_flat(ref[0]).size:][:mid * cin * 9].reshape(mid, cin, 3, 3)
    comp = np.einsum("om,mkl->omkl", pw[:, :, 0, 0].astype(np.float64), dw[:, 0].astype(np.float64))
    assert np.allclose(w0, comp, rtol=1e-6, atol=1e-7)


def _refusal(pieces, reduce):
    with pytest.raises(kb.KB2Error) as e:
        kb.rife_blob_from_onnx(pieces, reduce)
    return e.value


def _ref_refuses(piece):
    if not ref_lib.available():
        return
    with pytest.raises(ref_lib.RefRefusal):
        ref_lib.rife_native_layers(piece)


def _enc_with(params, replace_cnn1=None, **kw):
    c = op.Piece(**kw)
    c.conv(params["enc.cnn0.w"], params["enc.cnn0.b"], 2)
    c.activation(params["enc.cnn0.slope"])
    if replace_cnn1 is not None:
        replace_cnn1(c)
    else:
        c.conv(params["enc.cnn1.w"], params["enc.cnn1.b"], 1)
        c.activation(params["enc.cnn1.slope"])
    c.conv(params["enc.cnn2.w"], params["enc.cnn2.b"], 1)
    c.activation(params["enc.cnn2.slope"])
    c.conv(params["enc.cnn3.w"], params["enc.cnn3.b"], 2, transposed=True)
    return c.bytes()


def test_refuses_external_weights(params, pieces):
    c = op.Piece()
    c.inits.append(op.tensor("w_ext", params["enc.cnn0.w"], external=True))
    c.op("Conv", [c.cur, "w_ext", c.const("b", params["enc.cnn0.b"])],
         [op.attr("strides", ints=[2, 2]), op.attr("pads", ints=[1, 1, 1, 1])])
    piece = c.bytes()
    err = _refusal([piece] + pieces[1:3], list(REDUCE[:2]))
    assert err.status == kb.KB2_FORMAT_UNSUPPORTED and "outside" in err.message
    _ref_refuses(piece)


@pytest.mark.parametrize("dtype", [op.BFLOAT16, op.DOUBLE])
def test_refuses_element_types_the_reference_refuses(params, pieces, dtype):
    piece = op.encoder_piece(params, dtype=dtype)
    err = _refusal([piece] + pieces[1:3], list(REDUCE[:2]))
    assert err.status == kb.KB2_FORMAT_UNSUPPORTED and "data type" in err.message
    _ref_refuses(piece)


def test_refuses_truncated_bytes(pieces):
    piece = pieces[0][:len(pieces[0]) // 2]
    err = _refusal([piece] + pieces[1:3], list(REDUCE[:2]))
    assert err.status == kb.KB2_WEIGHTS_INVALID
    _ref_refuses(piece)


def test_refuses_an_unknown_operator(params, pieces):
    def sigmoid(c):
        c.conv(params["enc.cnn1.w"], params["enc.cnn1.b"], 1)
        c.op("Sigmoid", [c.cur])
    piece = _enc_with(params, sigmoid)
    err = _refusal([piece] + pieces[1:3], list(REDUCE[:2]))
    assert err.status == kb.KB2_WEIGHTS_INVALID and "Sigmoid" in err.message
    _ref_refuses(piece)


def test_refuses_a_branch(params, pieces):
    def branch(c):
        x = c.cur
        c.conv(params["enc.cnn1.w"], params["enc.cnn1.b"], 1)
        c.activation(params["enc.cnn1.slope"])
        c.nodes.append(op.node("Relu", [x], ["side"], "side_node"))  # a second reader of x
    piece = _enc_with(params, branch)
    err = _refusal([piece] + pieces[1:3], list(REDUCE[:2]))
    assert err.status == kb.KB2_WEIGHTS_INVALID and "branch" in err.message
    _ref_refuses(piece)


def test_refuses_a_residual_without_activation(params, pieces):
    def bare_residual(c):
        x = c.cur
        c.conv(params["enc.cnn1.w"], params["enc.cnn1.b"], 1)
        c.op("Add", [c.cur, x])
    piece = _enc_with(params, bare_residual)
    err = _refusal([piece] + pieces[1:3], list(REDUCE[:2]))
    assert err.status == kb.KB2_WEIGHTS_INVALID
    _ref_refuses(piece)


def test_refuses_a_block_off_the_topology(params, pieces):
    """Seven ResConv instead of eight: the reference's reader reads the layers, the RIFE 4.2x plan
    (two stride-2 convs, eight residual convs, the transposed conv to 52 channels) refuses them."""
    piece = op.block_piece(params, 1, res=7)
    err = _refusal(pieces[:2] + [piece], list(REDUCE[:2]))
    assert err.status == kb.KB2_WEIGHTS_INVALID and "11 layers" in err.message
    if ref_lib.available():
        assert len(ref_lib.rife_native_layers(piece)) == 10


def test_refuses_bad_arguments(pieces):
    with pytest.raises(kb.KB2Error) as e:
        kb.rife_blob_from_onnx(pieces[:1], [])
    assert e.value.status == kb.KB2_INVALID_ARGUMENT
    for bad in ([8, 3], [0, 8], [64, 8]):
        with pytest.raises(kb.KB2Error) as e:
            kb.rife_blob_from_onnx(pieces[:3], bad)
        assert e.value.status == kb.KB2_INVALID_ARGUMENT and "reductions" in e.value.message


def test_blob_creates_an_engine_shape_check(pieces):
    """The blob passes the library's own blob check (header, CRC, plan) without a GPU: the parameter
    count matches the plan the blob declares."""
    blob = kb.rife_blob_from_onnx(pieces, list(REDUCE))
    flat = blob_floats(blob)
    assert int(flat[0]) == BLOCKS and list(flat[1:1 + BLOCKS]) == list(REDUCE)
    assert list(flat[6:6 + BLOCKS]) == list(CHANNELS)
    assert flat.size == 12 + sum(int(np.prod(s)) for _, s in seeded.rife_param_shapes(PLAN))
