"""CPU restatement (numpy, float32) of the frame path's two networks — TEST INFRASTRUCTURE ONLY.

This module is the parity checker. Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline leg may import it; the product path (the CUDA library behind ``include/kirari_b200.h``)
never does. Its results are pinned against the reference's own FP32 interpreter (``oracle/_ref``,
built by ``oracle/Makefile`` from Ta2b/Ultimate-Anime-VideoPlayer's ``src/gpu/ir``) by the committed
fixtures in ``tests/golden/`` (``tests/golden/make_golden.py``).

Operator semantics follow the reference file by file:

* Conv, zero padding, FP32 sums: ``src/gpu/ir/op_window.cpp:227-288``.
* ConvTranspose, scatter form: ``src/gpu/ir/op_window.cpp:309-335``.
* Resize linear / half-pixel, clamp then lerp: ``src/gpu/ir/op_sample.cpp:88-170``.
* DepthToSpace CRD (PyTorch pixel_shuffle order): ``src/gpu/ir/op_pixel.cpp:78``.
* Backward warp: the tap of ``src/gpu/cuda/backend/warp_lib.cuh:45-58`` (``ix = x + fx`` rounded
  to FP32, clamped to the window, truncated, right/bottom neighbour clamped) and the bilinear
  blend of ``warp_lib.cuh:61-69`` / ``src/kernels/spec/warp.h:44-49``.
* E4M3 rounding (RNE, saturate to +-448): ``src/gpu/span_fp8/quantize.h:14-18``.
* FP8 scales ``max * 1.25 / 448``: ``src/gpu/span_fp8/derive.h:42-46``.

The network definitions are the contract's canonical SPAN x2 and classic IFNet 4.x; the concat
order of SPAN's conv_cat follows the reference's ``span_fp8::forward``
(``src/gpu/span_fp8/forward.cpp:158-160``: conv_1 output, last block output, first block output,
the last block's first activation).
"""
from __future__ import annotations

import math
import os
import sys

import numpy as np

# the seeded weights and the weight formats are inputs shared with the benchmark (package module)
_PKG = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "ultimate-anime-videoplayer_b200")
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)
from seeded import (E4M3_MAX, IFNET_CHANNELS, IFNET_RES, IFNET_SCALES, RIFE_PLANS, SCALE_HEADROOM,  # noqa: E402,F401
                    SPAN8_HEADER, SPAN8_IN, SPAN8_PIXEL, SPAN8_STORED, SPAN_BLOCKS, SPAN_C, _crc32, _flat,
                    ifnet_flat, ifnet_init, ifnet_param_shapes, kaiming, rife_flat, rife_init, rife_param_shapes,
                    span8_init, span8_package, span_flat, span_init, span_param_shapes, unflatten)


# --------------------------------------------------------------------------------------------
# Parameter layouts (flat float32, the order oracle/ref_graphs.cpp and the C ABI read)
# --------------------------------------------------------------------------------------------


















# --------------------------------------------------------------------------------------------
# Operators
# --------------------------------------------------------------------------------------------
def conv2d(x, w, b=None, stride=1, pad=1):
    """Cross-correlation with zero padding, FP32 (op_window.cpp:227-288 semantics)."""
    x = np.asarray(x, np.float32)
    n, c, h, wd = x.shape
    o, ci, kh, kw = w.shape
    assert ci == c
    xp = np.pad(x, ((0, 0), (0, 0), (pad, pad), (pad, pad)))
    ho = (h + 2 * pad - kh) // stride + 1
    wo = (wd + 2 * pad - kw) // stride + 1
    out = np.zeros((n, o, ho, wo), np.float32)
    wm = w.reshape(o, c * kh * kw).T.astype(np.float32)
    # rows of output at a time keep the im2col buffer bounded
    rows = max(1, int(2 ** 25 // max(1, wo * c * kh * kw)))
    for i in range(n):
        for y0 in range(0, ho, rows):
            y1 = min(ho, y0 + rows)
            win = np.lib.stride_tricks.sliding_window_view(
                xp[i, :, y0 * stride:(y1 - 1) * stride + kh, :], (kh, kw), axis=(1, 2))
            win = win[:, ::stride, ::stride]  # c, rows, wo, kh, kw
            cols = win.transpose(1, 2, 0, 3, 4).reshape((y1 - y0) * wo, c * kh * kw)
            out[i, :, y0:y1, :] = (cols @ wm).reshape(y1 - y0, wo, o).transpose(2, 0, 1)
    if b is not None:
        out += np.asarray(b, np.float32)[None, :, None, None]
    return out


def conv_transpose_4x4s2(x, w, b):
    """ConvTranspose kernel 4, stride 2, pad 1 (op_window.cpp:309-335, scatter form)."""
    n, c, h, wd = x.shape
    co = w.shape[1]
    out = np.zeros((n, co, 2 * h + 2, 2 * wd + 2), np.float32)  # 1-px margin each side
    for ky in range(4):
        for kx in range(4):
            contrib = np.einsum("nchw,co->nohw", x, w[:, :, ky, kx], optimize=True).astype(np.float32)
            out[:, :, ky:ky + 2 * h:2, kx:kx + 2 * wd:2] += contrib
    out = out[:, :, 1:2 * h + 1, 1:2 * wd + 1]
    return out + np.asarray(b, np.float32)[None, :, None, None]


def sigmoid(x):
    x = np.asarray(x, np.float32)
    return (1.0 / (1.0 + np.exp(-x))).astype(np.float32)


def silu(x):
    return (x * sigmoid(x)).astype(np.float32)


def prelu(x, slope):
    s = np.asarray(slope, np.float32)[None, :, None, None]
    return np.where(x >= 0, x, x * s).astype(np.float32)


def pixel_shuffle(x, r=2):
    """DepthToSpace CRD: channel c*r*r + i*r + j goes to pixel (r*y + i, r*x + j) of plane c."""
    n, c, h, w = x.shape
    oc = c // (r * r)
    return x.reshape(n, oc, r, r, h, w).transpose(0, 1, 4, 2, 5, 3).reshape(n, oc, h * r, w * r)


def resize_axis_taps(n_in, n_out):
    """Half-pixel linear taps of the reference Resize (op_sample.cpp:88-170): float32 position
    (o + 0.5) / scale - 0.5 with scale = n_out / n_in, clamped to [0, n_in - 1], truncated."""
    scale = np.float32(n_out) / np.float32(n_in)
    o = np.arange(n_out, dtype=np.float32)
    pos = (o + np.float32(0.5)) / scale - np.float32(0.5)
    pos = np.clip(pos, np.float32(0.0), np.float32(n_in - 1)).astype(np.float32)
    lo = pos.astype(np.int64)
    hi = np.minimum(lo + 1, n_in - 1)
    t = (pos - lo.astype(np.float32)).astype(np.float32)
    return lo, hi, t


def resize_bilinear(x, h_out, w_out):
    n, c, h, w = x.shape
    ylo, yhi, ty = resize_axis_taps(h, h_out)
    xlo, xhi, tx = resize_axis_taps(w, w_out)
    tx = tx[None, None, None, :]
    ty = ty[None, None, :, None]
    one = np.float32(1.0)
    top = (one - tx) * x[:, :, ylo][:, :, :, xlo] + tx * x[:, :, ylo][:, :, :, xhi]
    bot = (one - tx) * x[:, :, yhi][:, :, :, xlo] + tx * x[:, :, yhi][:, :, :, xhi]
    return ((one - ty) * top + ty * bot).astype(np.float32)


def warp_taps(fx, fy, left, top, right, bottom):
    """Bilinear tap of warp_lib.cuh:45-58 for every pixel of a flow plane pair [h, w]:
    ix = fl32(x + fx), clamped to [left, right - 1], x0 = trunc(ix), x1 = min(x0 + 1, right - 1).
    Returns (x0, x1, y0, y1, wx, wy)."""
    h, w = fx.shape
    xs = np.arange(w, dtype=np.float32)[None, :]
    ys = np.arange(h, dtype=np.float32)[:, None]
    ix = (xs + fx.astype(np.float32)).astype(np.float32)
    iy = (ys + fy.astype(np.float32)).astype(np.float32)
    # fmaxf/fminf: a NaN position goes to the lower bound (fmaxf(NaN, lo) = lo)
    ix = np.where(np.isnan(ix), np.float32(left), ix)
    iy = np.where(np.isnan(iy), np.float32(top), iy)
    ix = np.minimum(np.maximum(ix, np.float32(left)), np.float32(right - 1))
    iy = np.minimum(np.maximum(iy, np.float32(top)), np.float32(bottom - 1))
    x0 = ix.astype(np.int32)
    y0 = iy.astype(np.int32)
    x1 = np.minimum(x0 + 1, right - 1)
    y1 = np.minimum(y0 + 1, bottom - 1)
    wx = (ix - x0.astype(np.float32)).astype(np.float32)
    wy = (iy - y0.astype(np.float32)).astype(np.float32)
    return x0, x1, y0, y1, wx, wy


def warp(img, flow2, window=None):
    """Backward warp of img [n,c,h,w] by flow2 [n,2,h,w] (bilinear, border clamp to the window,
    by default the whole plane)."""
    n, c, h, w = img.shape
    left, top, right, bottom = window if window is not None else (0, 0, w, h)
    out = np.empty_like(img, dtype=np.float32)
    one = np.float32(1.0)
    for i in range(n):
        x0, x1, y0, y1, wx, wy = warp_taps(flow2[i, 0], flow2[i, 1], left, top, right, bottom)
        for ch in range(c):
            p = img[i, ch].astype(np.float32)
            a, b_, d, e = p[y0, x0], p[y0, x1], p[y1, x0], p[y1, x1]
            out[i, ch] = (a * (one - wx) + b_ * wx) * (one - wy) + (d * (one - wx) + e * wx) * wy
    return out


# --------------------------------------------------------------------------------------------
# FP8 E4M3 (host rounding of the reference, quantize.h:14-18)
# --------------------------------------------------------------------------------------------
def _e4m3_grid():
    vals = [0.0]
    for e in range(16):
        for m in range(8):
            if e == 15 and m == 7:
                continue  # NaN encoding
            v = (m / 8.0) * 2.0 ** -6 if e == 0 else (1.0 + m / 8.0) * 2.0 ** (e - 7)
            vals.append(v)
    return np.array(sorted(set(vals)), np.float64)


_E4M3 = _e4m3_grid()


def e4m3_round(x):
    """Round to nearest E4M3, ties to even mantissa, saturating to +-448 (NaN -> NaN)."""
    x = np.asarray(x, np.float32)
    a = np.abs(x.astype(np.float64))
    a = np.minimum(a, E4M3_MAX)
    idx = np.searchsorted(_E4M3, a)
    idx = np.clip(idx, 1, _E4M3.size - 1)
    lo, hi = _E4M3[idx - 1], _E4M3[idx]
    dlo, dhi = a - lo, hi - a
    # ties: pick the even mantissa (codes alternate even/odd along the sorted grid)
    pick_hi = (dhi < dlo) | ((dhi == dlo) & ((idx % 2) == 0))
    r = np.where(pick_hi, hi, lo)
    r = np.where(a >= _E4M3[-1], E4M3_MAX, r)
    out = (np.sign(x) * r).astype(np.float32)
    return np.where(np.isnan(x), np.float32(np.nan), out)


def fake_quant(x, scale):
    return (e4m3_round(np.asarray(x, np.float32) / np.float32(scale)) * np.float32(scale)).astype(np.float32)


# --------------------------------------------------------------------------------------------
# Networks
# --------------------------------------------------------------------------------------------
def span_forward(x, p, act_scales=None, store=None, taps=None):
    """Canonical SPAN x2: x [n,3,h,w] -> [n,3,2h,2w].

    act_scales: 19 per-tensor E4M3 scales of the block conv inputs ([3b] c1, [1+3b] c2, [2+3b] c3;
      [18] the last block output), the fake-quantised FP8 network (block conv inputs rounded to E4M3).
    store: optional rounding applied to every stored activation (e.g. FP16 storage emulation).
    taps: optional dict that receives the block conv inputs (calibration peaks)."""
    st = store if store is not None else (lambda v: v)
    q = (lambda v, i: fake_quant(v, act_scales[i])) if act_scales is not None else (lambda v, i: v)
    s0 = st(conv2d(x, p["conv_1.w"], p["conv_1.b"]))
    xb = s0
    first_block = last_act = None
    for b in range(SPAN_BLOCKS):
        if taps is not None:
            taps.setdefault(3 * b, []).append(float(np.abs(xb).max()))
        a1 = st(silu(conv2d(q(xb, 3 * b), p[f"block{b}.c1.w"], p[f"block{b}.c1.b"])))
        if taps is not None:
            taps.setdefault(3 * b + 1, []).append(float(np.abs(a1).max()))
        a2 = st(silu(conv2d(q(a1, 3 * b + 1), p[f"block{b}.c2.w"], p[f"block{b}.c2.b"])))
        if taps is not None:
            taps.setdefault(3 * b + 2, []).append(float(np.abs(a2).max()))
        c3 = conv2d(q(a2, 3 * b + 2), p[f"block{b}.c3.w"], p[f"block{b}.c3.b"])
        xb = st(((c3 + xb) * (sigmoid(c3) - np.float32(0.5))).astype(np.float32))
        if b == 0:
            first_block = xb
        if b == SPAN_BLOCKS - 1:
            last_act = a1
    if taps is not None:
        taps.setdefault(3 * SPAN_BLOCKS, []).append(float(np.abs(xb).max()))
    cat = np.concatenate([s0, xb, first_block, last_act], axis=1)
    fused = st(conv2d(cat, p["conv_cat.w"], p["conv_cat.b"], pad=0))
    up = conv2d(fused, p["upsampler.w"], p["upsampler.b"])
    return pixel_shuffle(up, 2)


def quantize_weights_per_channel(w, in_scale=None):
    """E4M3 weights at one scale per output channel (max |w| / 448, quantize.h:1-5), with the input
    activation scale folded in first; returns the dequantised weights the kernel effectively uses."""
    w = np.asarray(w, np.float32)
    if in_scale is not None:
        w = (w * np.asarray(in_scale, np.float32)).astype(np.float32)
    flat = w.reshape(w.shape[0], -1)
    mx = np.abs(flat).max(axis=1)
    ws = np.where(mx > 0, mx / np.float32(E4M3_MAX), np.float32(1.0)).astype(np.float32)
    q = (e4m3_round(flat / ws[:, None]) * ws[:, None]).reshape(w.shape)
    if in_scale is not None:
        q = q / np.asarray(in_scale, np.float32)
    return q.astype(np.float32)


def span_forward_fp8_pipeline(x, p, scales):
    """Emulation of this library's FP8 SPAN data path (test aid): conv_1, block 0, conv_cat and the
    upsampler in FP16 (FP16 storage); blocks 1..5 with E4M3 per-output-channel weights on E4M3
    activations, the SPAN gate reading the E4M3 block input; every conv_cat source in FP16."""
    f16 = lambda v: np.asarray(v, np.float16).astype(np.float32)  # noqa: E731
    q = lambda v, i: fake_quant(v, scales[i])  # noqa: E731
    s0 = f16(conv2d(f16(x), f16(p["conv_1.w"]), p["conv_1.b"]))
    xb16, first_block, last_act = s0, None, None
    for b in range(SPAN_BLOCKS):
        if b == 0:
            a1 = f16(silu(conv2d(s0, f16(p["block0.c1.w"]), p["block0.c1.b"])))
            a2 = f16(silu(conv2d(a1, f16(p["block0.c2.w"]), p["block0.c2.b"])))
            c3 = conv2d(a2, f16(p["block0.c3.w"]), p["block0.c3.b"])
            xr = (c3 + s0) * (sigmoid(c3) - np.float32(0.5))
            xb16, xq = f16(xr), q(xr, 3)
            first_block = xb16
            continue
        w = [quantize_weights_per_channel(p[f"block{b}.c{k + 1}.w"]) for k in range(3)]
        a1r = silu(conv2d(xq, w[0], p[f"block{b}.c1.b"]))
        a1 = q(a1r, 3 * b + 1)
        a2 = q(silu(conv2d(a1, w[1], p[f"block{b}.c2.b"])), 3 * b + 2)
        c3 = conv2d(a2, w[2], p[f"block{b}.c3.b"])
        xr = ((c3 + xq) * (sigmoid(c3) - np.float32(0.5))).astype(np.float32)
        if b == SPAN_BLOCKS - 1:
            last_act = f16(a1r)
            xb16 = f16(xr)
        else:
            xq = q(xr, 3 * b + 3)
    cat = np.concatenate([s0, xb16, first_block, last_act], axis=1)
    fused = f16(conv2d(cat, f16(p["conv_cat.w"]), p["conv_cat.b"], pad=0))
    up = conv2d(fused, f16(p["upsampler.w"]), p["upsampler.b"])
    return pixel_shuffle(up, 2)


def span_scales_from_peaks(peaks, floor=None):
    """max * 1.25 / 448 per tensor (derive.h:42-46): seeded.scales_from_peaks."""
    from seeded import scales_from_peaks
    return scales_from_peaks(peaks, floor)


def ifnet_block(x, flow, scale, p, k):
    c = IFNET_CHANNELS[k]
    n, _, h, w = x.shape
    if scale != 1:
        x = resize_bilinear(x, h // scale, w // scale)
    if flow is not None:
        f = flow
        if scale != 1:
            f = resize_bilinear(flow, h // scale, w // scale)
        f = (f * np.float32(1.0 / scale)).astype(np.float32)
        x = np.concatenate([x, f], axis=1)
    hdn = prelu(conv2d(x, p[f"b{k}.conv0a.w"], p[f"b{k}.conv0a.b"], stride=2), p[f"b{k}.conv0a.slope"])
    hdn = prelu(conv2d(hdn, p[f"b{k}.conv0b.w"], p[f"b{k}.conv0b.b"], stride=2), p[f"b{k}.conv0b.slope"])
    for j in range(IFNET_RES):
        r = conv2d(hdn, p[f"b{k}.res{j}.w"], p[f"b{k}.res{j}.b"])
        hdn = prelu((r + hdn).astype(np.float32), p[f"b{k}.res{j}.slope"])
    tmp = conv_transpose_4x4s2(hdn, p[f"b{k}.last.w"], p[f"b{k}.last.b"])
    tmp = resize_bilinear(tmp, h, w)
    fd = (tmp[:, :4] * np.float32(scale * 2)).astype(np.float32)
    md = tmp[:, 4:5]
    del c
    return fd, md


def ifnet_forward(img0, img1, timestep, p, return_flow=False):
    """Classic IFNet 4.x on img0, img1 [n,3,h,w] (h, w multiples of 32) -> [n,3,h,w]."""
    n, _, h, w = img0.shape
    t = np.full((n, 1, h, w), np.float32(timestep), np.float32)
    flow = mask = None
    w0, w1 = img0, img1
    for k, s in enumerate(IFNET_SCALES):
        if k == 0:
            xin = np.concatenate([img0, img1, t], axis=1)
            flow, mask = ifnet_block(xin, None, s, p, k)
        else:
            xin = np.concatenate([w0, w1, t, mask], axis=1)
            fd, md = ifnet_block(xin, flow, s, p, k)
            flow = (flow + fd).astype(np.float32)
            mask = (mask + md).astype(np.float32)
        w0 = warp(img0, flow[:, 0:2])
        w1 = warp(img1, flow[:, 2:4])
    m = sigmoid(mask)
    out = (w0 * m + w1 * (np.float32(1.0) - m)).astype(np.float32)
    if return_flow:
        return out, flow, mask
    return out


# --------------------------------------------------------------------------------------------
# Metrics (span_fp8/metrics.cpp semantics: PSNR over [0, 1] after clamp)
# --------------------------------------------------------------------------------------------
def clamp01(x):
    return np.clip(np.asarray(x, np.float32), 0.0, 1.0)


def psnr(a, b):
    a = clamp01(a).astype(np.float64)
    b = clamp01(b).astype(np.float64)
    mse = float(np.mean((a - b) ** 2))
    return float("inf") if mse == 0 else 10.0 * math.log10(1.0 / mse)


def max_abs_clamped(a, b):
    return float(np.max(np.abs(clamp01(a) - clamp01(b))))


# --------------------------------------------------------------------------------------------
# AnimeJaNai "unshuffle" SPAN and its .span8 package (the reference's span_fp8 format)
# --------------------------------------------------------------------------------------------
# (the package layout and the seeded contents: seeded.py)


def span8_fp8_package(p, frames, floor=2.0 ** -14):
    """An FP8 package (no FP16 flag) of contents `p` whose activation scales are calibrated on
    `frames` the reference's way: scale = max(peak, floor) * 1.25 / 448 (derive.h:42-62)."""
    peaks = []
    span8_forward(frames, p, peaks=peaks)
    q = dict(p)
    q["flags"] = 0
    q["scales"] = (np.maximum(np.asarray(peaks, np.float32), np.float32(floor)) * np.float32(SCALE_HEADROOM)
                   / np.float32(E4M3_MAX)).astype(np.float32)
    return q






def _span8_conv(x, c, real_in, real_out, side, groups=1, stored=SPAN8_STORED):
    """One package conv on the real channels: weights [out][ky*kx][groups*stored] -> OIHW."""
    w = np.asarray(c["w"], np.float32).reshape(c["w"].shape[0], side * side, groups, stored)
    w = w[:real_out, :, :, :real_in].reshape(real_out, side, side, groups * real_in).transpose(0, 3, 1, 2)
    return conv2d(x, np.ascontiguousarray(w), c["b"][:real_out], pad=side // 2)


def span8_forward(x, p, peaks=None):
    """FP32 forward of the unshuffle SPAN (src/gpu/span_fp8/forward.cpp:144-166): 2x2 unshuffle
    (channel c*4 + dy*2 + dx), conv_1, blocks (c1, ReLU, c2, ReLU, c3; out (x + c3) * tanh(att(c3))),
    conv_cat over (conv_1 out, last block out, first block out, the last block's first ReLU),
    to_pixel, DepthToSpace(4). x: [n,3,h,w], h and w even; returns [n,3,2h,2w]. `peaks`, a list,
    receives max |v| of the package's 1 + 3 * blocks scaled tensors in their order (package.h:15-17:
    conv_1 output, then per block its two ReLU outputs and its output)."""
    def peak(t):
        if peaks is not None:
            peaks.append(float(np.max(np.abs(t))))
    x = np.asarray(x, np.float32)
    n, _, h, w = x.shape
    ch = p["real"]
    u = x.reshape(n, 3, h // 2, 2, w // 2, 2).transpose(0, 1, 3, 5, 2, 4).reshape(n, 12, h // 2, w // 2)
    first = _span8_conv(u, p["first"], 12, ch, 3, stored=SPAN8_IN)
    peak(first)
    cur = first
    first_block = last_relu = None
    for b, blk in enumerate(p["block"]):
        r1 = np.maximum(_span8_conv(cur, blk["c1"], ch, ch, 3), 0.0).astype(np.float32)
        r2 = np.maximum(_span8_conv(r1, blk["c2"], ch, ch, 3), 0.0).astype(np.float32)
        c3 = _span8_conv(r2, blk["c3"], ch, ch, 3)
        att = _span8_conv(c3, blk["att"], ch, ch, 1)
        cur = ((cur + c3) * np.tanh(att)).astype(np.float32)
        peak(r1)
        peak(r2)
        peak(cur)
        if b == 0:
            first_block = cur
        if b + 1 == len(p["block"]):
            last_relu = r1
    cat = _span8_conv(np.concatenate([first, cur, first_block, last_relu], axis=1), p["concat"], ch, ch, 1, groups=4)
    pix = _span8_conv(cat, p["pixel"], ch, SPAN8_PIXEL, 3)
    return pixel_shuffle(pix, 4)


# --------------------------------------------------------------------------------------------
# Frame synthesis at any instant from one mid-pair motion (the reference's warp_blend_at and
# flow_max, src/kernels/ref/warp.cpp; law and constants of src/kernels/spec/warp.h:50-110)
# --------------------------------------------------------------------------------------------
BLEND_LAW_A, BLEND_LAW_B, BLEND_LAW_C = np.float32(1.0), np.float32(2.591), np.float32(0.0)
MASK_EPSILON = np.float32(1e-4)
FLOW_BINS, FLOW_BIN_STEP, FLOW_PERCENTILE = 256, np.float32(0.25), 0.999


def _bilinear_window(p, win, x, y):
    """Bilinear read relative to the corner of window win = (x, y, w, h) of plane p (warp.cpp:18-34):
    clamp to the window (NaN goes to 0, as fmaxf), truncate, right / bottom neighbour clamped; FP32
    operations in the reference's order, no contraction."""
    wx, wy, ww, wh = win
    f32 = np.float32
    x = np.fmin(np.fmax(np.asarray(x, f32), f32(0)), f32(ww - 1)).astype(f32)
    y = np.fmin(np.fmax(np.asarray(y, f32), f32(0)), f32(wh - 1)).astype(f32)
    x0 = x.astype(np.int32)
    y0 = y.astype(np.int32)
    x1 = np.minimum(x0 + 1, ww - 1)
    y1 = np.minimum(y0 + 1, wh - 1)
    fx = (x - x0.astype(f32)).astype(f32)
    fy = (y - y0.astype(f32)).astype(f32)
    one = f32(1)
    top = (p[wy + y0, wx + x0] * (one - fx) + p[wy + y0, wx + x1] * fx).astype(f32)
    bot = (p[wy + y1, wx + x0] * (one - fx) + p[wy + y1, wx + x1] * fx).astype(f32)
    return (top * (one - fy) + bot * fy).astype(f32)


def _cr_weights(t):
    """Catmull-Rom weights of points -1, 0, 1, 2 for fractions t (spec/warp.h:28-34), FP32."""
    f32 = np.float32
    t = np.asarray(t, f32)
    t2 = (t * t).astype(f32)
    t3 = (t2 * t).astype(f32)
    return [((f32(-0.5) * t3 + t2) - f32(0.5) * t).astype(f32),
            ((f32(1.5) * t3 - f32(2.5) * t2) + f32(1)).astype(f32),
            ((f32(-1.5) * t3 + f32(2) * t2) + f32(0.5) * t).astype(f32),
            (f32(0.5) * t3 - f32(0.5) * t2).astype(f32)]


def _catmull_rom(p, x, y):
    """Catmull-Rom read of plane p [h,w] (ref/warp.cpp catmull_rom_at): clamped position, clamped
    indices, rows then columns, the result clamped to the range of the four central samples."""
    f32 = np.float32
    h, w = p.shape
    x = np.fmin(np.fmax(np.asarray(x, f32), f32(0)), f32(w - 1)).astype(f32)
    y = np.fmin(np.fmax(np.asarray(y, f32), f32(0)), f32(h - 1)).astype(f32)
    x0 = x.astype(np.int32)
    y0 = y.astype(np.int32)
    wx = _cr_weights((x - x0.astype(f32)).astype(f32))
    wy = _cr_weights((y - y0.astype(f32)).astype(f32))
    total = np.zeros(x.shape, f32)
    lo = np.full(x.shape, np.inf, f32)
    hi = np.full(x.shape, -np.inf, f32)
    for j in range(4):
        yy = np.clip(y0 - 1 + j, 0, h - 1)
        row = np.zeros(x.shape, f32)
        for i in range(4):
            v = p[yy, np.clip(x0 - 1 + i, 0, w - 1)]
            row = (row + v * wx[i]).astype(f32)
            if i in (1, 2) and j in (1, 2):
                lo = np.fmin(lo, v)
                hi = np.fmax(hi, v)
        total = (total + row * wy[j]).astype(f32)
    return np.fmin(np.fmax(total, lo), hi).astype(f32)


def _frame_read(p, x, y, warp):
    h, w = p.shape
    return _catmull_rom(p, x, y) if warp == 1 else _bilinear_window(p, (0, 0, w, h), x, y)


def warp_blend_at(a, b, flow, mask, window, t, warp=0, pan_lock=0, at_instant=0):
    """One frame [3,h,w] at instant t in (0, 1) from frames a, b [3,h,w] and the mid-pair motion:
    flow [4,ph,pw] (f0x, f0y, f1x, f1y), mask [ph,pw], the frame's window (x, y, w, h) in those planes
    (warp.cpp warp_blend_at:261 with the bilinear filter, no pan lock, the motion estimated at the
    middle). t = 1/2: flow and mask as they are; else straight-line motion from the middle and the
    blend law logit(m) = A logit(mm) + B ln((1 - t) / t) + C. warp: the frames' filter, 0 bilinear,
    1 Catmull-Rom."""
    f32 = np.float32
    a = np.asarray(a, f32)
    b = np.asarray(b, f32)
    flow = np.asarray(flow, f32)
    mask = np.asarray(mask, f32)
    _, h, w = a.shape
    ww, wh = window[2], window[3]
    sx = f32(w) / f32(ww)
    sy = f32(h) / f32(wh)
    fy, fx = np.meshgrid(np.arange(h, dtype=f32), np.arange(w, dtype=f32), indexing="ij")
    u = ((fx + f32(0.5)) / sx - f32(0.5)).astype(f32)
    v = ((fy + f32(0.5)) / sy - f32(0.5)).astype(f32)
    t = f32(t)
    one = f32(1)
    f = [_bilinear_window(flow[c], window, u, v) for c in range(4)]
    g_pan = None
    if pan_lock:
        dx, dy, sure = pan_estimate(a, b)
        sm = t if at_instant else f32(0.5)
        g_pan = [f32(f32(-sm * f32(dx)) / sx), f32(f32(-sm * f32(dy)) / sy), f32(f32((one - sm) * f32(dx)) / sx),
                 f32(f32((one - sm) * f32(dy)) / sy)]
        if sure:
            f = _pan_substitute(f, g_pan)
    if t == f32(0.5) or at_instant:
        ax, ay, bx, by = f
        wgt = _bilinear_window(mask, window, u, v)
        if pan_lock:
            mm = np.fmin(np.fmax(wgt, MASK_EPSILON), one - MASK_EPSILON).astype(f32)
            w = _slow_fade_weight(np.hypot((f[2] - f[0]).astype(f32), (f[3] - f[1]).astype(f32)).astype(f32))
            z = (w * np.log(mm / (one - mm)) + (one - w) * np.log((one - t) / t)).astype(f32)
            wgt = (one / (one + np.exp(-z))).astype(f32)
    else:
        u2 = (u - ((one - t) * f[0] + t * f[2])).astype(f32)
        v2 = (v - ((one - t) * f[1] + t * f[3])).astype(f32)
        g = [_bilinear_window(flow[c], window, u2, v2) for c in range(4)]
        if pan_lock and pan_estimate(a, b)[2]:
            g = _pan_substitute(g, g_pan)
        tx = (g[2] - g[0]).astype(f32)
        ty = (g[3] - g[1]).astype(f32)
        mm = np.fmin(np.fmax(_bilinear_window(mask, window, u2, v2), MASK_EPSILON), one - MASK_EPSILON).astype(f32)
        z = (BLEND_LAW_A * np.log(mm / (one - mm)) + BLEND_LAW_B * np.log((one - t) / t) + BLEND_LAW_C).astype(f32)
        if pan_lock:
            w = _slow_fade_weight(np.hypot(tx, ty).astype(f32))
            z = (w * z + (one - w) * np.log((one - t) / t)).astype(f32)
        wgt = (one / (one + np.exp(-z))).astype(f32)
        ax, ay = (-t * tx).astype(f32), (-t * ty).astype(f32)
        bx, by = ((one - t) * tx).astype(f32), ((one - t) * ty).astype(f32)
    out = np.empty_like(a)
    for c in range(3):
        va = _frame_read(a[c], (fx + sx * ax).astype(f32), (fy + sy * ay).astype(f32), warp)
        vb = _frame_read(b[c], (fx + sx * bx).astype(f32), (fy + sy * by).astype(f32), warp)
        out[c] = (va * wgt + vb * (one - wgt)).astype(f32)
    return out


PAN_GRID, PAN_ITERATIONS = 32, 3
PAN_LUMA = (np.float32(0.2126), np.float32(0.7152), np.float32(0.0722))
PAN_DET_RATIO, PAN_MAX_SHIFT, PAN_FLOW_LIMIT, PAN_AGREEMENT = 1e-6, np.float32(8), np.float32(2), np.float32(1)
SLOW_FADE_LO, SLOW_FADE_HI = np.float32(0.5), np.float32(2.0)


def _luma(img):
    return ((PAN_LUMA[0] * img[0] + PAN_LUMA[1] * img[1]).astype(np.float32) + PAN_LUMA[2] * img[2]).astype(np.float32)


def pan_estimate(a, b):
    """The pair's global translation (ref/warp_pan.cpp pan_estimate): Lucas-Kanade on the luma at a
    32 x 32 grid, 3 iterations, double sums in point order; returns (dx, dy, sure)."""
    f32 = np.float32
    a = np.asarray(a, f32)
    b = np.asarray(b, f32)
    _, h, w = a.shape
    if w < 16 or h < 16:
        return 0.0, 0.0, False
    la_img, lb_img = _luma(a), _luma(b)

    def point(i, n):
        m = n // 12 if n // 12 > 4 else 4
        return m + (i * (n - 2 * m)) // PAN_GRID

    q = np.arange(PAN_GRID * PAN_GRID)
    px = np.array([point(i % PAN_GRID, w) for i in q])
    py = np.array([point(i // PAN_GRID, h) for i in q])
    la = la_img[py, px]
    gx = (f32(0.5) * (la_img[py, px + 1] - la_img[py, px - 1])).astype(f32)
    gy = (f32(0.5) * (la_img[py + 1, px] - la_img[py - 1, px])).astype(f32)
    dx = dy = f32(0)
    valid = False
    for _ in range(PAN_ITERATIONS):
        r = (_bilinear_window(lb_img, (0, 0, w, h), px.astype(f32) + dx, py.astype(f32) + dy) - la).astype(f32)
        sxx = sxy = syy = sxr = syr = 0.0
        for k in range(q.size):  # the reference's order
            sxx += float(f32(gx[k] * gx[k]))
            sxy += float(f32(gx[k] * gy[k]))
            syy += float(f32(gy[k] * gy[k]))
            sxr += float(f32(gx[k] * r[k]))
            syr += float(f32(gy[k] * r[k]))
        det = sxx * syy - sxy * sxy
        valid = det > PAN_DET_RATIO * (sxx + syy) * (sxx + syy) and det > 0.0
        if not valid:
            break
        dx = f32(dx - f32((syy * sxr - sxy * syr) / det))
        dy = f32(dy - f32((sxx * syr - sxy * sxr) / det))
    sure = valid and float(np.hypot(dx, dy)) < float(PAN_MAX_SHIFT)
    return float(dx), float(dy), bool(sure)


def _slow_fade_weight(d):
    f32 = np.float32
    s = ((np.asarray(d, f32) - SLOW_FADE_LO) / (SLOW_FADE_HI - SLOW_FADE_LO)).astype(f32)
    s = np.where(s < 0, f32(0), np.where(s > 1, f32(1), s)).astype(f32)
    return ((s * s).astype(f32) * (f32(3) - f32(2) * s)).astype(f32)


def _pan_substitute(f, g):
    m = np.max(np.abs(np.stack(f)), axis=0)
    e = np.max(np.abs(np.stack([f[c] - g[c] for c in range(4)])), axis=0)
    use = (m < PAN_FLOW_LIMIT) & (e < PAN_AGREEMENT)
    return [np.where(use, np.float32(g[c]), f[c]).astype(np.float32) for c in range(4)]


POSE_ITERATIONS, POSE_EPSILON, POSE_TIME_LIMIT = 2, np.float32(0.01), np.float32(1e-3)


def warp_blend_poses(a, b, flow, mask, prev_flow, prev_mask, window, t, warp=0):
    """Keep the poses (warp.cpp keeping_poses / warp_blend_poses, spec/poses.h): each pixel's instant
    tp is adjusted by the ratio of the distance its point moved in the previous pair (prev_flow /
    prev_mask, None for a held pair) to the one it moves now, two iterations, then warp_blend_at at
    tp for that pixel."""
    f32 = np.float32
    a = np.asarray(a, f32)
    b = np.asarray(b, f32)
    flow = np.asarray(flow, f32)
    mask = np.asarray(mask, f32)
    _, h, w = a.shape
    ww, wh = window[2], window[3]
    sx = f32(w) / f32(ww)
    sy = f32(h) / f32(wh)
    fy, fx = np.meshgrid(np.arange(h, dtype=f32), np.arange(w, dtype=f32), indexing="ij")
    u = ((fx + f32(0.5)) / sx - f32(0.5)).astype(f32)
    v = ((fy + f32(0.5)) / sy - f32(0.5)).astype(f32)
    one = f32(1)
    t = f32(t)
    tp = np.full(u.shape, t, f32)
    B = lambda pl, x, y: _bilinear_window(pl, window, x, y)  # noqa: E731
    for _ in range(POSE_ITERATIONS):
        u2 = (u - ((one - tp) * B(flow[0], u, v) + tp * B(flow[2], u, v))).astype(f32)
        v2 = (v - ((one - tp) * B(flow[1], u, v) + tp * B(flow[3], u, v))).astype(f32)
        dx = (B(flow[2], u2, v2) - B(flow[0], u2, v2)).astype(f32)
        dy = (B(flow[3], u2, v2) - B(flow[1], u2, v2)).astype(f32)
        before = np.zeros_like(u)
        if prev_flow is not None:
            pf = np.asarray(prev_flow, f32)
            ax = (u - tp * dx).astype(f32)
            ay = (v - tp * dy).astype(f32)
            qx, qy = ax, ay
            for _step in range(2):
                nx = (ax - B(pf[2], qx, qy)).astype(f32)
                ny = (ay - B(pf[3], qx, qy)).astype(f32)
                qx, qy = nx, ny
            before = np.hypot((B(pf[2], qx, qy) - B(pf[0], qx, qy)).astype(f32),
                              (B(pf[3], qx, qy) - B(pf[1], qx, qy)).astype(f32)).astype(f32)
        now = np.hypot(dx, dy).astype(f32)
        r = ((before + POSE_EPSILON) / (before + now + f32(2) * POSE_EPSILON)).astype(f32)
        pt = np.where(t < f32(0.5), f32(2) * t * r, one - f32(2) * (one - t) * r).astype(f32)
        tp = np.fmin(np.fmax(pt, POSE_TIME_LIMIT), one - POSE_TIME_LIMIT).astype(f32)
    # from_middle at the per-pixel tp
    f = [B(flow[c], u, v) for c in range(4)]
    u2 = (u - ((one - tp) * f[0] + tp * f[2])).astype(f32)
    v2 = (v - ((one - tp) * f[1] + tp * f[3])).astype(f32)
    g = [B(flow[c], u2, v2) for c in range(4)]
    tx = (g[2] - g[0]).astype(f32)
    ty = (g[3] - g[1]).astype(f32)
    mm = np.fmin(np.fmax(B(mask, u2, v2), MASK_EPSILON), one - MASK_EPSILON).astype(f32)
    z = (BLEND_LAW_A * np.log(mm / (one - mm)) + BLEND_LAW_B * np.log((one - tp) / tp) + BLEND_LAW_C).astype(f32)
    wgt = (one / (one + np.exp(-z))).astype(f32)
    ax, ay = (-tp * tx).astype(f32), (-tp * ty).astype(f32)
    bx, by = ((one - tp) * tx).astype(f32), ((one - tp) * ty).astype(f32)
    out = np.empty_like(a)
    for c in range(3):
        va = _frame_read(a[c], (fx + sx * ax).astype(f32), (fy + sy * ay).astype(f32), warp)
        vb = _frame_read(b[c], (fx + sx * bx).astype(f32), (fy + sy * by).astype(f32), warp)
        out[c] = (va * wgt + vb * (one - wgt)).astype(f32)
    return out


def flow_max(flow, window):
    """The 99.9th percentile of max |f| over the 4 flow planes inside the window, as the lower edge
    of its histogram bin (256 bins of 0.25 px, the last taking the rest; warp.cpp flow_max:290,
    spec/warp.h:91-110)."""
    wx, wy, ww, wh = window
    m = np.max(np.abs(np.asarray(flow, np.float32)[:, wy:wy + wh, wx:wx + ww]), axis=0)
    m = np.where(np.isnan(m), np.float32(0), m)
    scaled = (m / FLOW_BIN_STEP).astype(np.float32)
    bins = np.where(~(m > 0), 0, np.where(scaled >= FLOW_BINS - 1, FLOW_BINS - 1,
                                          np.minimum(scaled, FLOW_BINS - 1).astype(np.int64)))
    hist = np.bincount(bins.ravel(), minlength=FLOW_BINS)
    points = int(ww) * int(wh)
    rank = int(float(points) * FLOW_PERCENTILE)
    if float(rank) < float(points) * FLOW_PERCENTILE:
        rank += 1
    rank = max(rank, 1)
    seen = np.cumsum(hist)
    i = int(np.argmax(seen >= rank))
    return float(np.float32(i) * FLOW_BIN_STEP)


# --------------------------------------------------------------------------------------------
# Display-ring pixels (src/kernels/spec/ring_pack.h, color.h unorm16; no contraction)
# --------------------------------------------------------------------------------------------
def _clamp_unit(v):
    v = np.asarray(v, np.float32)
    return np.where(np.isnan(v), np.float32(0), np.fmin(np.fmax(v, np.float32(0)), np.float32(1))).astype(np.float32)


def _ring_hash(x, y, salt):
    with np.errstate(over="ignore"):
        x = np.asarray(x, np.uint32)
        y = np.asarray(y, np.uint32)
        v = (x * np.uint32(0x9E3779B1)) ^ (y * np.uint32(0x85EBCA77)) ^ np.uint32((salt * 0xC2B2AE3D) & 0xFFFFFFFF)
        v = (v * np.uint32(747796405) + np.uint32(2891336453)).astype(np.uint32)
        v = (((v >> ((v >> np.uint32(28)) + np.uint32(4))) ^ v) * np.uint32(277803737)).astype(np.uint32)
        return ((v >> np.uint32(22)) ^ v).astype(np.uint32)


def pack_display(rgb, fmt):
    """Display pixels of one frame rgb [3,h,w]: fmt 1 RGBA16 -> uint16 [h,w,4]; 2 RGB10A2, 3 RGB10A2
    with the pixel's TPDF dither -> uint32 [h,w] (r | g << 10 | b << 20 | 3 << 30)."""
    f32 = np.float32
    rgb = np.asarray(rgb, f32)
    _, h, w = rgb.shape
    c = _clamp_unit(rgb)
    if fmt == 1:
        q = (c * f32(65535) + f32(0.5)).astype(f32).astype(np.uint16)
        return np.concatenate([q.transpose(1, 2, 0), np.full((h, w, 1), 65535, np.uint16)], axis=2)
    if fmt == 2:
        q = (c * f32(1023) + f32(0.5)).astype(f32).astype(np.uint32)
    else:
        yy, xx = np.meshgrid(np.arange(h, dtype=np.uint32), np.arange(w, dtype=np.uint32), indexing="ij")
        u5 = ((_ring_hash(xx, yy, 5) >> np.uint32(8)).astype(f32) * f32(1.0 / 16777216.0)).astype(f32)
        u6 = ((_ring_hash(xx, yy, 6) >> np.uint32(8)).astype(f32) * f32(1.0 / 16777216.0)).astype(f32)
        noise = ((u5 + u6).astype(f32) - f32(1)).astype(f32)
        biased = ((c * f32(1023) + f32(0.5)).astype(f32) + noise[None]).astype(f32)
        q = np.where(~(biased > 0), 0, np.where(biased >= f32(1023), 1023, np.maximum(biased, 0).astype(np.uint32)))
        q = q.astype(np.uint32)
    return (q[0] | (q[1] << np.uint32(10)) | (q[2] << np.uint32(20)) | np.uint32(3 << 30)).astype(np.uint32)
