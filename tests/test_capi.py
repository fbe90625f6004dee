"""The C-ABI library without a GPU: it builds for sm_100a, loads, exports every entry point of
include/kirari_b200.h, and refuses bad weight blobs and shapes before touching a device."""
import os
import re

import numpy as np
import pytest

import kirari_b200 as kb
from oracle import nets
from util import ROOT, ensure_built


@pytest.fixture(scope="module")
def lib():
    ensure_built()
    return kb.lib()


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "kirari_b200.h")).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(kb2_\w+)\s*\(", text, re.M)))


def test_header_and_binding_agree():
    assert declared_symbols() == sorted(kb.EXPORTS)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.kb2_abi_version() == 1


def _create_status(blob, model=kb.MODEL_SPAN_X2, h=32, w=32, batch=1):
    try:
        kb.Engine(model, blob, h, w, max_batch=batch)
    except kb.KB2Error as e:
        return e.status, e.message
    return kb.KB2_OK, ""


def test_blob_refusals(lib):
    blob = kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(nets.span_init(1)))
    bad_crc = bytearray(blob)
    bad_crc[200] ^= 0x40
    assert _create_status(bytes(bad_crc))[0] == kb.KB2_WEIGHTS_INVALID
    bad_magic = b"XB2WGT01" + blob[8:]
    assert _create_status(bad_magic)[0] == kb.KB2_WEIGHTS_INVALID
    assert _create_status(blob[:-4])[0] == kb.KB2_WEIGHTS_INVALID
    assert _create_status(blob[:16])[0] == kb.KB2_WEIGHTS_INVALID
    wrong_model = kb.make_blob(kb.MODEL_IFNET, nets.span_flat(nets.span_init(1)))
    assert _create_status(wrong_model)[0] == kb.KB2_WEIGHTS_INVALID
    nan = nets.span_flat(nets.span_init(1)).copy()
    nan[5] = np.nan
    assert _create_status(kb.make_blob(kb.MODEL_SPAN_X2, nan))[0] == kb.KB2_WEIGHTS_INVALID


def test_shape_refusals_before_device(lib):
    blob = kb.make_blob(kb.MODEL_SPAN_X2, nets.span_flat(nets.span_init(1)))
    assert _create_status(blob, batch=0)[0] == kb.KB2_SHAPE_INVALID
    assert _create_status(blob, h=0)[0] == kb.KB2_SHAPE_INVALID
    assert _create_status(blob, w=100000)[0] == kb.KB2_SHAPE_INVALID


def test_null_arguments(lib):
    assert lib.kb2_create(None, None) == kb.KB2_INVALID_ARGUMENT
    assert lib.kb2_destroy(None) == kb.KB2_INVALID_ARGUMENT
    assert lib.kb2_enqueue(None, None, None, 0, None, 0) == kb.KB2_INVALID_ARGUMENT
    assert lib.kb2_last_error(None) == b""
