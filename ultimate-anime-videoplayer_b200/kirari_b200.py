"""Python mirror of the C ABI in include/kirari_b200.h (ctypes), with torch for device memory.

This is the host-side interface the tests and the benchmark use: the same calls a C++ player makes
through the header (create with a weight blob, enqueue device frames on a stream, read refusals).
The library it loads is the in-tree libkirari_b200.so; there is no other backend and no CPU
fallback: if the library is missing, every call raises.
"""
from __future__ import annotations

import ctypes
import os
import struct
import zlib

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkirari_b200.so")

KB2_OK = 0
KB2_SHAPE_INVALID = 1
KB2_INPUT_MISMATCH = 2
KB2_FORMAT_UNSUPPORTED = 3
KB2_GPU_MEMORY_EXHAUSTED = 4
KB2_VENDOR_CALL_FAILED = 5
KB2_WEIGHTS_INVALID = 6
KB2_KERNEL_TIMEOUT = 7
KB2_INVALID_ARGUMENT = 8

KB2_F32, KB2_F16, KB2_U8, KB2_I8 = 0, 1, 2, 3
MODEL_SPAN_X2 = 1
MODEL_IFNET = 2
MODEL_SPAN_UNSHUFFLE = 3  # weights: the bytes of a .span8 package
MODEL_RIFE_FUSED = 4  # RIFE 4.2x: 12 plan floats, then the parameters
DISPLAY_RGBA16, DISPLAY_RGB10A2, DISPLAY_RGB10A2_DITHER = 1, 2, 3
PREC_FP16 = 1
PREC_FP8 = 2

# every entry point of include/kirari_b200.h
EXPORTS = ("kb2_abi_version", "kb2_create", "kb2_create_error", "kb2_destroy", "kb2_last_error",
           "kb2_workspace_bytes", "kb2_enqueue", "kb2_set_timestep", "kb2_check_device", "kb2_span_calibrate",
           "kb2_set_profiling", "kb2_read_profile", "kb2_launches_per_enqueue", "kb2_span_calibrate_static",
           "kb2_warp_taps", "kb2_selftest_bounded_wait", "kb2_warp_blend_at", "kb2_flow_max",
           "kb2_warp_blend_poses", "kb2_pack_display", "kb2_rife_geometry", "kb2_set_output_format",
           "kb2_set_row_tiles", "kb2_span_tile_grid", "kb2_next_span_tiles", "kb2_rife_blob_from_onnx")


class KB2Error(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"kb2 status {status}: {message}")
        self.status = status
        self.message = message


class Tensor(ctypes.Structure):
    _fields_ = [("type", ctypes.c_int32), ("dims", ctypes.c_int64 * 4), ("handle", ctypes.c_uint64),
                ("offset", ctypes.c_uint64)]


class EngineDesc(ctypes.Structure):
    _fields_ = [("model", ctypes.c_int32), ("precision", ctypes.c_int32), ("max_batch", ctypes.c_int32),
                ("height", ctypes.c_int32), ("width", ctypes.c_int32), ("device", ctypes.c_int32),
                ("weights", ctypes.c_void_p), ("weights_bytes", ctypes.c_uint64),
                ("act_scales", ctypes.POINTER(ctypes.c_float)), ("act_scale_count", ctypes.c_int32)]


class Motion(ctypes.Structure):
    _fields_ = [("flow", ctypes.c_void_p), ("mask", ctypes.c_void_p), ("plane_h", ctypes.c_int32),
                ("plane_w", ctypes.c_int32), ("x", ctypes.c_int32), ("y", ctypes.c_int32),
                ("width", ctypes.c_int32), ("height", ctypes.c_int32), ("warp", ctypes.c_int32),
                ("pan_lock", ctypes.c_int32), ("at_instant", ctypes.c_int32)]


class SpanTileGrid(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("tile_w", "tile_h", "cols", "rows", "reach_cols", "reach_rows",
                                             "shift_step", "scale")]


class LayerProfile(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 48), ("launches", ctypes.c_uint64), ("total_ms", ctypes.c_double),
                ("flops", ctypes.c_double), ("bytes", ctypes.c_double)]


_lib = None


def lib():
    """Loads libkirari_b200.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(f"{LIB_PATH} not built: run `python ultimate-anime-videoplayer_b200/build.py`")
        L = ctypes.CDLL(LIB_PATH)
        L.kb2_abi_version.restype = ctypes.c_int
        L.kb2_create.argtypes = [ctypes.POINTER(EngineDesc), ctypes.POINTER(ctypes.c_void_p)]
        L.kb2_create_error.restype = ctypes.c_char_p
        L.kb2_rife_blob_from_onnx.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_uint64),
                                              ctypes.c_int32, ctypes.POINTER(ctypes.c_int32), ctypes.c_void_p,
                                              ctypes.POINTER(ctypes.c_uint64)]
        L.kb2_destroy.argtypes = [ctypes.c_void_p]
        L.kb2_last_error.argtypes = [ctypes.c_void_p]
        L.kb2_last_error.restype = ctypes.c_char_p
        L.kb2_workspace_bytes.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64)]
        L.kb2_enqueue.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(Tensor), ctypes.c_int32,
                                  ctypes.POINTER(Tensor), ctypes.c_int32]
        L.kb2_set_timestep.argtypes = [ctypes.c_void_p, ctypes.c_float]
        L.kb2_check_device.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32)]
        L.kb2_span_calibrate.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(Tensor),
                                         ctypes.POINTER(ctypes.c_float), ctypes.c_int32]
        L.kb2_span_calibrate_static.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(Tensor),
                                                ctypes.POINTER(ctypes.c_float), ctypes.c_int32]
        L.kb2_warp_blend_at.argtypes = [ctypes.c_void_p, ctypes.POINTER(Tensor), ctypes.POINTER(Tensor),
                                        ctypes.POINTER(Motion), ctypes.c_float, ctypes.POINTER(Tensor)]
        L.kb2_warp_blend_poses.argtypes = [ctypes.c_void_p, ctypes.POINTER(Tensor), ctypes.POINTER(Tensor),
                                           ctypes.POINTER(Motion), ctypes.POINTER(Motion), ctypes.c_float,
                                           ctypes.POINTER(Tensor)]
        L.kb2_pack_display.argtypes = [ctypes.c_void_p, ctypes.POINTER(Tensor), ctypes.c_int32, ctypes.c_void_p,
                                       ctypes.c_int64]
        L.kb2_flow_max.argtypes = [ctypes.c_void_p, ctypes.POINTER(Motion), ctypes.c_int32, ctypes.c_void_p,
                                   ctypes.POINTER(ctypes.c_float)]
        L.kb2_selftest_bounded_wait.argtypes = [ctypes.c_int32, ctypes.POINTER(ctypes.c_int32),
                                                ctypes.POINTER(ctypes.c_double)]
        L.kb2_warp_taps.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                    ctypes.c_void_p, ctypes.c_void_p]
        L.kb2_set_profiling.argtypes = [ctypes.c_void_p, ctypes.c_int32]
        L.kb2_read_profile.argtypes = [ctypes.c_void_p, ctypes.POINTER(LayerProfile), ctypes.c_int32,
                                       ctypes.POINTER(ctypes.c_int32)]
        L.kb2_launches_per_enqueue.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32)]
        L.kb2_rife_geometry.argtypes = [ctypes.c_void_p] + [ctypes.POINTER(ctypes.c_int32)] * 4
        L.kb2_set_output_format.argtypes = [ctypes.c_void_p, ctypes.c_int32]
        L.kb2_set_row_tiles.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32]
        L.kb2_span_tile_grid.argtypes = [ctypes.c_void_p, ctypes.POINTER(SpanTileGrid)]
        L.kb2_next_span_tiles.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                          ctypes.c_int32, ctypes.POINTER(Tensor)]
        _lib = L
    return _lib


def make_blob(model: int, flat_params) -> bytes:
    """Weight blob v1: 'KB2WGT01', u32 version 1, u32 model, u64 count, u32 CRC-32, u32 0, floats."""
    payload = np.ascontiguousarray(flat_params, dtype="<f4").tobytes()
    header = b"KB2WGT01" + struct.pack("<IIQII", 1, model, len(payload) // 4, zlib.crc32(payload) & 0xFFFFFFFF, 0)
    return header + payload


def to_kb2_tensor(t) -> Tensor:
    """torch CUDA tensor -> kb2_tensor (NCHW, contiguous)."""
    import torch
    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    dtype = {torch.float16: KB2_F16, torch.float32: KB2_F32, torch.uint8: KB2_U8, torch.int8: KB2_I8}[t.dtype]
    dims = list(t.shape) + [1] * (4 - t.dim())
    return Tensor(dtype, (ctypes.c_int64 * 4)(*dims), t.data_ptr(), 0)


def _stream_handle(stream):
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


def rife_blob_from_onnx(pieces, reduce) -> bytes:
    """kb2_rife_blob_from_onnx: the KB2_MODEL_RIFE_FUSED weight blob from ONNX pieces (bytes: the
    encoder, then one per block) and the plan's input reductions."""
    n = len(pieces)
    bufs = [ctypes.create_string_buffer(bytes(p), len(p)) for p in pieces]
    ptrs = (ctypes.c_void_p * n)(*[ctypes.cast(b, ctypes.c_void_p) for b in bufs])
    sizes = (ctypes.c_uint64 * n)(*[len(p) for p in pieces])
    red = (ctypes.c_int32 * max(1, len(reduce)))(*reduce)
    size = ctypes.c_uint64(0)
    L = lib()
    rc = L.kb2_rife_blob_from_onnx(ptrs, sizes, n - 1, red, None, ctypes.byref(size))
    if rc != KB2_OK:
        raise KB2Error(rc, L.kb2_create_error().decode(errors="replace"))
    out = ctypes.create_string_buffer(size.value)
    rc = L.kb2_rife_blob_from_onnx(ptrs, sizes, n - 1, red, out, ctypes.byref(size))
    if rc != KB2_OK:
        raise KB2Error(rc, L.kb2_create_error().decode(errors="replace"))
    return out.raw[:size.value]


class Engine:
    """An engine of the C ABI (SPAN x2 or IFNet)."""

    def __init__(self, model, blob: bytes, height, width, max_batch=1, precision=PREC_FP16, act_scales=None,
                 device=0):
        self._blob = ctypes.create_string_buffer(blob, len(blob))
        self._scales = None
        n_scales = 0
        if act_scales is not None:
            arr = np.ascontiguousarray(act_scales, np.float32)
            self._scales = (ctypes.c_float * arr.size)(*arr.tolist())
            n_scales = arr.size
        desc = EngineDesc(model, precision, max_batch, height, width, device,
                          ctypes.cast(self._blob, ctypes.c_void_p), len(blob),
                          ctypes.cast(self._scales, ctypes.POINTER(ctypes.c_float)) if self._scales else None,
                          n_scales)
        h = ctypes.c_void_p()
        rc = lib().kb2_create(ctypes.byref(desc), ctypes.byref(h))
        if rc != KB2_OK:
            raise KB2Error(rc, lib().kb2_create_error().decode(errors="replace"))
        self.h = h
        self.height, self.width, self.max_batch = height, width, max_batch

    def _check(self, rc):
        if rc != KB2_OK:
            raise KB2Error(rc, lib().kb2_last_error(self.h).decode(errors="replace"))

    def enqueue(self, inputs, outputs, stream=None):
        ins = (Tensor * len(inputs))(*[to_kb2_tensor(t) for t in inputs])
        outs = (Tensor * len(outputs))(*[to_kb2_tensor(t) for t in outputs])
        self._check(lib().kb2_enqueue(self.h, _stream_handle(stream), ins, len(inputs), outs, len(outputs)))

    def enqueue_raw(self, ins, outs, stream_handle):
        """Pre-built kb2_tensor arrays (no per-call marshalling), for timing loops."""
        self._check(lib().kb2_enqueue(self.h, stream_handle, ins, len(ins), outs, len(outs)))

    def set_output_format(self, fmt):
        """SPAN x2: 0 = F16 frames, or a DISPLAY_* format (outputs U8 [n, 8 or 4, 2H, 2W], packed pixels)."""
        self._check(lib().kb2_set_output_format(self.h, int(fmt)))

    def set_row_tiles(self, tiles, halo):
        """SPAN x2: run frames as `tiles` row tiles with `halo` rows of context, stitched (1: whole frames)."""
        self._check(lib().kb2_set_row_tiles(self.h, int(tiles), int(halo)))

    def span_tile_grid(self):
        """SPAN x2 moving tiles: dict(tile_w, tile_h, cols, rows, reach_cols, reach_rows, shift_step, scale)."""
        g = SpanTileGrid()
        self._check(lib().kb2_span_tile_grid(self.h, ctypes.byref(g)))
        return {n: getattr(g, n) for n, _ in SpanTileGrid._fields_}

    def next_span_tiles(self, core, shift_x=0, shift_y=0, previous=None):
        """Requests that the next enqueue recompute only the core tiles (uint8 [rows, cols]); raises
        KB2Error (KB2_FORMAT_UNSUPPORTED: the next call computes the whole frame) when refused."""
        c = np.ascontiguousarray(core, np.uint8)
        self._core_keep = c
        prev = None if previous is None else to_kb2_tensor(previous)
        self._check(lib().kb2_next_span_tiles(self.h, c.ctypes.data_as(ctypes.c_void_p), int(c.size), int(shift_x),
                                              int(shift_y), None if prev is None else ctypes.byref(prev)))

    def rife_geometry(self):
        """IFNet: (plane_h, plane_w, window_x, window_y) of the motion outputs."""
        v = [ctypes.c_int32(0) for _ in range(4)]
        self._check(lib().kb2_rife_geometry(self.h, *[ctypes.byref(x) for x in v]))
        return tuple(x.value for x in v)

    def motion(self, a, b, dtype=None, stream=None):
        """IFNet motion variant on torch device frames a, b F16 [n,3,H,W]: returns (flow [n,4,Hp,Wp],
        mask [n,1,Hp,Wp], window (x, y, W, H)) as torch tensors of `dtype` (float32 by default)."""
        import torch
        dtype = dtype or torch.float32
        ph, pw, x, y = self.rife_geometry()
        n = int(a.shape[0])
        flow = torch.full((n, 4, ph, pw), float("nan"), dtype=dtype, device=a.device)
        mask = torch.full((n, 1, ph, pw), float("nan"), dtype=dtype, device=a.device)
        self.enqueue([a, b], [flow, mask], stream)
        return flow, mask, (x, y, self.width, self.height)

    def set_timestep(self, t):
        self._check(lib().kb2_set_timestep(self.h, float(t)))

    def check_device(self, stream=None):
        code = ctypes.c_int32(0)
        rc = lib().kb2_check_device(self.h, _stream_handle(stream), ctypes.byref(code))
        if rc != KB2_OK:
            raise KB2Error(rc, f"device error word {code.value:#x}")

    def workspace_bytes(self):
        v = ctypes.c_uint64(0)
        self._check(lib().kb2_workspace_bytes(self.h, ctypes.byref(v)))
        return v.value

    def calibrate(self, frames, stream=None, n_peaks=19):
        """kb2_span_calibrate: 19 peaks (canonical SPAN) or 1 + 3 * blocks (a .span8 package's engine)."""
        peaks = (ctypes.c_float * n_peaks)()
        t = to_kb2_tensor(frames)
        self._check(lib().kb2_span_calibrate(self.h, _stream_handle(stream), ctypes.byref(t), peaks, n_peaks))
        return np.array(peaks[:], np.float32)

    def calibrate_static(self, frames, stream=None):
        """calibrate() with its scratch in the library's static device array: no device allocation."""
        peaks = (ctypes.c_float * 19)()
        t = to_kb2_tensor(frames)
        self._check(lib().kb2_span_calibrate_static(self.h, _stream_handle(stream), ctypes.byref(t), peaks, 19))
        return np.array(peaks[:], np.float32)

    def set_profiling(self, on=True):
        self._check(lib().kb2_set_profiling(self.h, 1 if on else 0))

    def read_profile(self):
        """{name: dict(launches, total_ms, flops, bytes)} since profiling was enabled / last read."""
        recs = (LayerProfile * 64)()
        n = ctypes.c_int32(0)
        self._check(lib().kb2_read_profile(self.h, recs, 64, ctypes.byref(n)))
        return {recs[i].name.decode(): dict(launches=recs[i].launches, total_ms=recs[i].total_ms,
                                            flops=recs[i].flops, bytes=recs[i].bytes) for i in range(min(n.value, 64))}

    def launches_per_enqueue(self):
        n = ctypes.c_int32(0)
        self._check(lib().kb2_launches_per_enqueue(self.h, ctypes.byref(n)))
        return n.value

    def close(self):
        if getattr(self, "h", None):
            lib().kb2_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def warp_taps(flow, stream=None):
    """Device warp taps of a flow field (torch float32 CUDA tensor [n, 2, h, w]):
    returns (taps int32 [n, 4, h, w] = x0, x1, y0, y1; weights float32 [n, 2, h, w] = wx, wy)."""
    import torch
    n, two, h, w = flow.shape
    assert two == 2 and flow.dtype == torch.float32 and flow.is_cuda and flow.is_contiguous()
    taps = torch.empty((n, 4, h, w), dtype=torch.int32, device=flow.device)
    weights = torch.empty((n, 2, h, w), dtype=torch.float32, device=flow.device)
    rc = lib().kb2_warp_taps(_stream_handle(stream), ctypes.c_void_p(flow.data_ptr()), n, h, w,
                             ctypes.c_void_p(taps.data_ptr()), ctypes.c_void_p(weights.data_ptr()))
    if rc != KB2_OK:
        raise KB2Error(rc, "kb2_warp_taps")
    return taps, weights


def selftest_bounded_wait(device=0):
    """kb2_selftest_bounded_wait: (status, error code, seconds the device waited)."""
    code = ctypes.c_int32(0)
    waited = ctypes.c_double(0.0)
    rc = lib().kb2_selftest_bounded_wait(device, ctypes.byref(code), ctypes.byref(waited))
    return rc, code.value, waited.value


def _motion(flow, mask, window, warp=0, pan_lock=0, at_instant=0):
    """kb2_motion over torch device tensors flow [n,4,ph,pw] and mask [n,ph,pw] (FP32, contiguous);
    warp: the frames' filter, 0 bilinear, 1 Catmull-Rom; pan_lock: the pair's global translation."""
    ph, pw = int(mask.shape[-2]), int(mask.shape[-1])
    return Motion(flow.data_ptr(), mask.data_ptr(), ph, pw, *[int(v) for v in window], int(warp), int(pan_lock),
                  int(at_instant))


def warp_blend_at(a, b, flow, mask, window, t, stream=None, warp=0, pan_lock=0, at_instant=0):
    """kb2_warp_blend_at on torch device tensors: a, b F16 [n,3,H,W]; returns F16 [n,3,H,W]."""
    import torch
    out = torch.empty_like(a)
    m = _motion(flow, mask, window, warp, pan_lock, at_instant)
    ta, tb, to = to_kb2_tensor(a), to_kb2_tensor(b), to_kb2_tensor(out)
    rc = lib().kb2_warp_blend_at(_stream_handle(stream), ctypes.byref(ta), ctypes.byref(tb), ctypes.byref(m),
                                 float(t), ctypes.byref(to))
    if rc != KB2_OK:
        raise KB2Error(rc, "kb2_warp_blend_at")
    return out


def warp_blend_poses(a, b, flow, mask, prev_flow, prev_mask, window, t, stream=None, warp=0):
    """kb2_warp_blend_poses on torch device tensors (prev_flow None: a held previous pair)."""
    import torch
    out = torch.empty_like(a)
    m = _motion(flow, mask, window, warp)
    pm = None if prev_flow is None else _motion(prev_flow, prev_mask, window)
    ta, tb, to = to_kb2_tensor(a), to_kb2_tensor(b), to_kb2_tensor(out)
    rc = lib().kb2_warp_blend_poses(_stream_handle(stream), ctypes.byref(ta), ctypes.byref(tb), ctypes.byref(m),
                                    None if pm is None else ctypes.byref(pm), float(t), ctypes.byref(to))
    if rc != KB2_OK:
        raise KB2Error(rc, "kb2_warp_blend_poses")
    return out


def flow_max(flow, mask, window, stream=None):
    """kb2_flow_max on torch device tensors: one value (pixels of the window) per pair."""
    import torch
    n = int(flow.shape[0])
    bins = torch.empty((n, 256), dtype=torch.int32, device=flow.device)
    out = (ctypes.c_float * n)()
    m = _motion(flow, mask, window)
    rc = lib().kb2_flow_max(_stream_handle(stream), ctypes.byref(m), n, ctypes.c_void_p(bins.data_ptr()), out)
    if rc != KB2_OK:
        raise KB2Error(rc, "kb2_flow_max")
    return list(out)


def pack_display(frames, fmt, stream=None):
    """kb2_pack_display on an F16 [n,3,H,W] device tensor: uint16 [n,H,W,4] (RGBA16) or uint32
    [n,H,W] (RGB10A2 forms) as an int32 / int16 torch tensor of the same bytes, rows packed."""
    import torch
    n, _, h, w = frames.shape
    if fmt == DISPLAY_RGBA16:
        out = torch.empty((n, h, w, 4), dtype=torch.int16, device=frames.device)
        pitch = w * 8
    else:
        out = torch.empty((n, h, w), dtype=torch.int32, device=frames.device)
        pitch = w * 4
    t = to_kb2_tensor(frames)
    rc = lib().kb2_pack_display(_stream_handle(stream), ctypes.byref(t), int(fmt), ctypes.c_void_p(out.data_ptr()),
                                pitch)
    if rc != KB2_OK:
        raise KB2Error(rc, "kb2_pack_display")
    return out
