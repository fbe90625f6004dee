"""The unshuffle SPAN of a .span8 package, CPU side: the numpy restatement (oracle/nets.py
span8_forward) against the reference's own FP32 forward (golden fixtures), and the library's package
reader (kb2_create with KB2_MODEL_SPAN_UNSHUFFLE, which reads the package before any device call)
against the reference's reader, span_fp8::parse (src/gpu/span_fp8/package.cpp:143), on valid and
damaged packages."""
import hashlib
import struct
import zlib

import numpy as np
import pytest

import kirari_b200 as kb
from oracle import nets, ref_lib
from util import ensure_built, golden

# The reference's refusal codes as its parser reports them through oracle/ref_span8.cpp (code + 1),
# by their order in KIRARI_REFUSAL_CODES (src/core/types.h:23-70).
REF_FILE_UNREADABLE = 7 + 1
REF_FORMAT_UNSUPPORTED = 20 + 1
# the library's status for each
OURS = {REF_FILE_UNREADABLE: kb.KB2_WEIGHTS_INVALID, REF_FORMAT_UNSUPPORTED: kb.KB2_FORMAT_UNSUPPORTED}


@pytest.mark.parametrize("name", ["span8_b2f48_20x36.npz", "span8_b3f64_16x30.npz"])
def test_span8_restatement_matches_reference(name):
    g = golden(name)
    pkg = nets.span8_package(nets.span8_init(int(g["blocks"]), int(g["real"]), seed=int(g["seed"])))
    assert hashlib.sha256(pkg).hexdigest() == str(g["package_sha256"]), "seeded package changed"
    out = nets.span8_forward(g["x"], nets.span8_init(int(g["blocks"]), int(g["real"]), seed=int(g["seed"])))
    assert out.shape == g["out"].shape
    np.testing.assert_allclose(out, g["out"], rtol=0, atol=2e-5)


def _reheader(body, version=2, blocks=2, stored=64, real=48, flags=2, payload=None, crc=None):
    payload = len(body) if payload is None else payload
    crc = zlib.crc32(body) & 0xFFFFFFFF if crc is None else crc
    return b"AJPSPAN8" + struct.pack("<IIIIQII", version, blocks, stored, real, payload, crc, flags) + body


def _damaged():
    """(label, bytes) of valid and damaged packages, each damage a way the reader must refuse."""
    good = nets.span8_package(nets.span8_init(2, 48, seed=4))
    body = good[40:]
    cases = [("valid b2f48", good),
             ("valid b3f64", nets.span8_package(nets.span8_init(3, 64, seed=4))),
             ("bad magic", b"AJPSPAN9" + good[8:]),
             ("version 3", _reheader(body, version=3)),
             ("one block", _reheader(body, blocks=1)),
             ("nine blocks", _reheader(body, blocks=9)),
             ("stored 48", _reheader(body, stored=48)),
             ("32 real channels", _reheader(body, real=32)),
             ("unknown flag", _reheader(body, flags=2 | 8)),
             ("f32 sums without FP16", _reheader(body, flags=4)),
             ("version 1 with flags", _reheader(body, version=1, blocks=8, flags=2)),
             ("wrong payload size", _reheader(body, payload=len(body) + 4)),
             ("truncated", good[:-6]),
             ("CRC flipped", _reheader(body, crc=(zlib.crc32(body) ^ 1) & 0xFFFFFFFF)),
             ("short header", good[:30]),
             ("trailing bytes", _reheader(body + b"\0\0\0\0")),
             ("block count disagrees with payload", _reheader(body, blocks=3))]
    nan_w = bytearray(body)
    at = 4 * 7  # first conv_1 weight after the 7 scales of 2 blocks
    nan_w[at:at + 2] = struct.pack("<H", 0x7E00)
    cases.append(("NaN weight", _reheader(bytes(nan_w))))
    zero_scale = bytearray(body)
    zero_scale[0:4] = struct.pack("<f", 0.0)
    cases.append(("zero scale", _reheader(bytes(zero_scale))))
    inf_bias = bytearray(body)
    at = 4 * 7 + 2 * 64 * 9 * 16  # first conv_1 bias
    inf_bias[at:at + 4] = struct.pack("<f", float("inf"))
    cases.append(("infinite bias", _reheader(bytes(inf_bias))))
    return cases


def _ours(pkg):
    try:
        kb.Engine(kb.MODEL_SPAN_UNSHUFFLE, pkg, 32, 32, max_batch=1)
    except kb.KB2Error as e:
        return e.status, str(e)
    return kb.KB2_OK, ""


@pytest.fixture(scope="module")
def _lib():
    ensure_built()
    return kb.lib()


@pytest.mark.parametrize("label,pkg", _damaged(), ids=[c[0] for c in _damaged()])
def test_span8_reader_agrees_with_reference(_lib, label, pkg):
    status, msg = _ours(pkg)
    if label.startswith("valid"):
        # accepted by the reader: whatever follows (no device here, or an engine) is not a package refusal
        assert ".span8 package" not in msg, msg
    else:
        assert status in (kb.KB2_WEIGHTS_INVALID, kb.KB2_FORMAT_UNSUPPORTED) and ".span8 package" in msg, (status, msg)
    if not ref_lib.available():
        pytest.skip("oracle/_ref not built: reader checked against the format only")
    ref = ref_lib.span8_parse(pkg)
    if label.startswith("valid"):
        assert ref[0] == 0
    else:
        assert ref[0] in OURS, ref
        assert OURS[ref[0]] == status, (label, ref, status, msg)
