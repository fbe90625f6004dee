"""ctypes binding of oracle/_ref/libkirari_ref.so — TEST INFRASTRUCTURE ONLY.

The library is the reference's own FP32 CPU interpreter (Ta2b/Ultimate-Anime-VideoPlayer
``src/gpu/ir``, compiled in place by ``oracle/Makefile``) driving the in-code graphs of
``oracle/ref_graphs.cpp``. It is used to pin the numpy restatement (``oracle/nets.py``) and as the
timed reference CPU implementation in ``bench.py``. Nothing in the product path loads it.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_ref", "libkirari_ref.so")
_lib = None
_fp = ctypes.POINTER(ctypes.c_float)


def available() -> bool:
    return os.path.exists(LIB_PATH)


def lib():
    global _lib
    if _lib is None:
        if not available():
            raise FileNotFoundError(f"{LIB_PATH} missing: run `make -C oracle` where the reference exists")
        L = ctypes.CDLL(LIB_PATH)
        L.kref_last_error.restype = ctypes.c_char_p
        L.kref_span_forward.argtypes = [_fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _fp, ctypes.c_long,
                                        _fp, _fp]
        L.kref_span_forward.restype = ctypes.c_int
        L.kref_ifnet_forward.argtypes = [_fp, _fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                         _fp, ctypes.c_long, _fp]
        L.kref_ifnet_forward.restype = ctypes.c_int
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(_fp)


def span_forward(x, flat_params, act_scales=None):
    """Reference FP32 SPAN x2 on x [n,3,h,w]; act_scales (19) selects the E4M3 fake-quant graph."""
    x = np.ascontiguousarray(x, np.float32)
    flat = np.ascontiguousarray(flat_params, np.float32)
    n, _, h, w = x.shape
    out = np.zeros((n, 3, 2 * h, 2 * w), np.float32)
    sc = None if act_scales is None else np.ascontiguousarray(act_scales, np.float32)
    rc = lib().kref_span_forward(_ptr(x), n, h, w, _ptr(flat), flat.size,
                                 None if sc is None else _ptr(sc), _ptr(out))
    if rc != 0:
        raise RuntimeError(f"kref_span_forward: {rc} {lib().kref_last_error().decode(errors='replace')}")
    return out


def ifnet_forward(img0, img1, timestep, flat_params):
    """Reference FP32 classic IFNet on img0, img1 [n,3,h,w] (h, w multiples of 32)."""
    a = np.ascontiguousarray(img0, np.float32)
    b = np.ascontiguousarray(img1, np.float32)
    flat = np.ascontiguousarray(flat_params, np.float32)
    n, _, h, w = a.shape
    out = np.zeros((n, 3, h, w), np.float32)
    rc = lib().kref_ifnet_forward(_ptr(a), _ptr(b), n, h, w, float(timestep), _ptr(flat), flat.size, _ptr(out))
    if rc != 0:
        raise RuntimeError(f"kref_ifnet_forward: {rc} {lib().kref_last_error().decode(errors='replace')}")
    return out


def _rife42_bind(L):
    if not hasattr(L, "_rife42"):
        i = ctypes.c_int
        L.kref_rife42_forward.argtypes = [_fp, _fp, i, i, i, ctypes.c_float, _fp, ctypes.c_long, _fp, _fp, _fp]
        L.kref_rife42_glue_check.argtypes = [_fp, _fp, i, i, ctypes.c_float, _fp, ctypes.c_long,
                                             ctypes.POINTER(ctypes.c_double)]
        L._rife42 = True
    return L


def rife42_forward(img0, img1, timestep, flat_params):
    """RIFE 4.2x through the reference's interpreter: (image [n,3,h,w], flow [n,4,h,w], sigmoid(mask)
    [n,1,h,w]); flat_params starts with the 12 plan floats."""
    L = _rife42_bind(lib())
    a = np.ascontiguousarray(img0, np.float32)
    b = np.ascontiguousarray(img1, np.float32)
    p = np.ascontiguousarray(flat_params, np.float32)
    n, _, h, w = a.shape
    out = np.empty((n, 3, h, w), np.float32)
    flow = np.empty((n, 4, h, w), np.float32)
    mask = np.empty((n, 1, h, w), np.float32)
    rc = L.kref_rife42_forward(_ptr(a), _ptr(b), n, h, w, timestep, _ptr(p), p.size, _ptr(out), _ptr(flow),
                               _ptr(mask))
    if rc != 0:
        raise RuntimeError(f"kref_rife42_forward: {rc} {L.kref_last_error().decode()}")
    return out, flow, mask


def rife42_glue_check(img0, img1, timestep, flat_params):
    """Max differences between the graph's X_k / image / flow / mask and the reference's own
    double-precision fused-RIFE glue (src/kernels/ref/rife_fused.cpp), on the first frame pair."""
    L = _rife42_bind(lib())
    a = np.ascontiguousarray(img0[0], np.float32)
    b = np.ascontiguousarray(img1[0], np.float32)
    p = np.ascontiguousarray(flat_params, np.float32)
    _, h, w = a.shape
    blocks = int(p[0])
    err = (ctypes.c_double * (blocks + 3))()
    rc = L.kref_rife42_glue_check(_ptr(a), _ptr(b), h, w, timestep, _ptr(p), p.size, err)
    if rc != 0:
        raise RuntimeError(f"kref_rife42_glue_check: {rc} {L.kref_last_error().decode()}")
    return list(err)


def _span8_bind(L):
    if getattr(L, "_span8_bound", False):
        return L
    _u8 = ctypes.POINTER(ctypes.c_ubyte)
    L.kref_span8_last_error.restype = ctypes.c_char_p
    L.kref_span8_parse.argtypes = [_u8, ctypes.c_long, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                                   ctypes.POINTER(ctypes.c_int)]
    L.kref_span8_parse.restype = ctypes.c_int
    L.kref_span8_forward.argtypes = [_u8, ctypes.c_long, _fp, ctypes.c_int, ctypes.c_int, _fp]
    L.kref_span8_forward.restype = ctypes.c_int
    L._span8_bound = True
    return L


def span8_parse(package: bytes):
    """The reference's .span8 reader (package.cpp:143): (0, blocks, real, fp16) when it accepts the
    bytes, else (its refusal code + 1, message)."""
    L = _span8_bind(lib())
    buf = (ctypes.c_ubyte * len(package)).from_buffer_copy(package)
    b, r, f = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    rc = L.kref_span8_parse(buf, len(package), ctypes.byref(b), ctypes.byref(r), ctypes.byref(f))
    if rc != 0:
        return rc, L.kref_span8_last_error().decode(errors="replace")
    return 0, b.value, r.value, f.value


def span8_forward(package: bytes, x):
    """The reference's FP32 unshuffle-SPAN forward (forward.cpp:144) of x [n,3,h,w]."""
    L = _span8_bind(lib())
    x = np.ascontiguousarray(x, np.float32)
    n, _, h, w = x.shape
    buf = (ctypes.c_ubyte * len(package)).from_buffer_copy(package)
    out = np.zeros((n, 3, 2 * h, 2 * w), np.float32)
    for i in range(n):
        xi = np.ascontiguousarray(x[i])
        oi = np.zeros((3, 2 * h, 2 * w), np.float32)
        rc = L.kref_span8_forward(buf, len(package), _ptr(xi), h, w, _ptr(oi))
        if rc != 0:
            raise RuntimeError(f"kref_span8_forward: {rc} {L.kref_span8_last_error().decode(errors='replace')}")
        out[i] = oi
    return out


def _warp_bind(L):
    if getattr(L, "_warp_bound", False):
        return L
    i = ctypes.c_int
    L.kref_warp_last_error.restype = ctypes.c_char_p
    L.kref_warp_blend_at.argtypes = [_fp, _fp, i, i, _fp, _fp, i, i, i, i, i, i, ctypes.c_float, i, i, i, _fp]
    L.kref_pan_estimate.argtypes = [_fp, _fp, i, i, _fp]
    L.kref_pan_estimate.restype = i
    L.kref_warp_blend_at.restype = i
    L.kref_flow_max.argtypes = [_fp, _fp, i, i, i, i, i, i, _fp]
    L.kref_warp_blend_poses.argtypes = [_fp, _fp, i, i, _fp, _fp, _fp, _fp, i, i, i, i, i, i, ctypes.c_float, i,
                                        _fp]
    L.kref_warp_blend_poses.restype = i
    L.kref_flow_max.restype = i
    L._warp_bound = True
    return L


def warp_blend_at(a, b, flow, mask, window, t, warp=0, pan_lock=0, at_instant=0):
    """The reference's CPU warp_blend_at (src/kernels/ref/warp.cpp:261): a, b [3,h,w], flow
    [4,ph,pw], mask [ph,pw], window (x, y, w, h); returns [3,h,w]."""
    L = _warp_bind(lib())
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    flow = np.ascontiguousarray(flow, np.float32)
    mask = np.ascontiguousarray(mask, np.float32)
    _, h, w = a.shape
    ph, pw = mask.shape
    out = np.zeros_like(a)
    rc = L.kref_warp_blend_at(_ptr(a), _ptr(b), h, w, _ptr(flow), _ptr(mask), ph, pw, *window, float(t), int(warp),
                              int(pan_lock), int(at_instant), _ptr(out))
    if rc != 0:
        raise RuntimeError(f"kref_warp_blend_at: {L.kref_warp_last_error().decode(errors='replace')}")
    return out


def flow_max(flow, mask, window):
    """The reference's CPU flow_max (src/kernels/ref/warp.cpp:290)."""
    L = _warp_bind(lib())
    flow = np.ascontiguousarray(flow, np.float32)
    mask = np.ascontiguousarray(mask, np.float32)
    ph, pw = mask.shape
    out = np.zeros(1, np.float32)
    rc = L.kref_flow_max(_ptr(flow), _ptr(mask), ph, pw, *window, _ptr(out))
    if rc != 0:
        raise RuntimeError(f"kref_flow_max: {L.kref_warp_last_error().decode(errors='replace')}")
    return float(out[0])


def warp_blend_poses(a, b, flow, mask, prev_flow, prev_mask, window, t, warp=0):
    """The reference's CPU warp_blend_poses (src/kernels/ref/warp.cpp:270): keep the poses, with the
    previous pair's motion (or None for a held previous pair)."""
    L = _warp_bind(lib())
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    flow = np.ascontiguousarray(flow, np.float32)
    mask = np.ascontiguousarray(mask, np.float32)
    pf = None if prev_flow is None else np.ascontiguousarray(prev_flow, np.float32)
    pm = None if prev_mask is None else np.ascontiguousarray(prev_mask, np.float32)
    _, h, w = a.shape
    ph, pw = mask.shape
    out = np.zeros_like(a)
    rc = L.kref_warp_blend_poses(_ptr(a), _ptr(b), h, w, _ptr(flow), _ptr(mask), None if pf is None else _ptr(pf),
                                 None if pm is None else _ptr(pm), ph, pw, *window, float(t), int(warp), _ptr(out))
    if rc != 0:
        raise RuntimeError(f"kref_warp_blend_poses: {L.kref_warp_last_error().decode(errors='replace')}")
    return out


def pack_display(rgb, fmt):
    """The reference's display-ring packing (src/kernels/spec/ring_pack.h) of one frame [3,h,w]."""
    L = lib()
    if not getattr(L, "_pack_bound", False):
        L.kref_pack_display.argtypes = [_fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        L.kref_pack_display.restype = ctypes.c_int
        L._pack_bound = True
    rgb = np.ascontiguousarray(rgb, np.float32)
    _, h, w = rgb.shape
    out = np.zeros((h, w, 4), np.uint16) if fmt == 1 else np.zeros((h, w), np.uint32)
    rc = L.kref_pack_display(_ptr(rgb), h, w, int(fmt), out.ctypes.data_as(ctypes.c_void_p))
    if rc != 0:
        raise RuntimeError("kref_pack_display: unknown format")
    return out


def pan_estimate(a, b):
    """The reference's pan estimate (src/kernels/ref/warp_pan.cpp) of frames [3,h,w]: (dx, dy, sure)."""
    L = _warp_bind(lib())
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    _, h, w = a.shape
    out = np.zeros(3, np.float32)
    L.kref_pan_estimate(_ptr(a), _ptr(b), h, w, _ptr(out))
    return float(out[0]), float(out[1]), bool(out[2] != 0)


class RefRefusal(RuntimeError):
    """The reference's reader refused a piece; the message is its refusal detail."""


def rife_native_layers(piece: bytes):
    """The reference's reader of one RIFE ONNX piece (src/prepare/rife_native.cpp
    rife_native_layers): a list of layers, each a dict with transposed, cin, cout, kernel, stride and
    the float arrays w (OIHW for a conv, [cin][cout][4][4] for the transposed conv: the ONNX and
    weight-blob layouts, rearranged from the reference's [cout][k^2][cin]), b, slope and scale
    (empty when absent). Raises RefRefusal when the reference refuses the piece."""
    L = lib()
    if not getattr(L, "_onnx_bound", False):
        L.kref_rife_native_layers.argtypes = [ctypes.c_char_p, ctypes.c_uint64, ctypes.POINTER(ctypes.c_int32),
                                              ctypes.c_int, _fp, ctypes.c_uint64, ctypes.c_char_p, ctypes.c_int]
        L.kref_rife_native_layers.restype = ctypes.c_int
        L._onnx_bound = True
    max_layers = 64
    meta = np.zeros((max_layers, 9), np.int32)
    vals = np.zeros(len(piece) + 4096, np.float32)  # a piece holds at least a byte per value
    err = ctypes.create_string_buffer(512)
    n = L.kref_rife_native_layers(piece, len(piece), meta.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                  max_layers, _ptr(vals), vals.size, err, 512)
    if n == -1:
        raise RefRefusal(err.value.decode(errors="replace"))
    if n < 0:
        raise RuntimeError("kref_rife_native_layers: buffer too small")
    out, at = [], 0
    for m in meta[:n]:
        tr, cin, cout, k, stride, nw, nb, ns, nsc = (int(v) for v in m)
        w = vals[at:at + nw].reshape(cout, k * k, cin)
        at += nw
        if tr:
            w = w.transpose(2, 0, 1).reshape(cin, cout, k, k)
        else:
            w = w.transpose(0, 2, 1).reshape(cout, cin, k, k)
        layer = {"transposed": bool(tr), "cin": cin, "cout": cout, "kernel": k, "stride": stride,
                 "w": np.ascontiguousarray(w)}
        for key, cnt in (("b", nb), ("slope", ns), ("scale", nsc)):
            layer[key] = vals[at:at + cnt].copy()
            at += cnt
        out.append(layer)
    return out
