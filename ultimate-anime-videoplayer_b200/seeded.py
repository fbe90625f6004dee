"""Seeded synthetic weights of the frame path's networks, and the weight formats they travel in.

The contract measures and tests the networks on seeded weights (there are no trained checkpoints):
canonical SPAN x2 and classic IFNet as flat float32 arrays in the order of the C ABI's weight blob
(include/kirari_b200.h, above KB2_SPAN_X2_PARAMS), and the AnimeJaNai unshuffle SPAN as the contents
of a .span8 package (the reference's span_fp8 package format, src/gpu/span_fp8/package.h:1-17,
written as package.cpp:200-215 writes it). Used by the benchmark, the tests and the CPU oracle alike:
weights are inputs, not the checker.
"""
from __future__ import annotations

import math

import numpy as np

SPAN_C = 48
SPAN_BLOCKS = 6
IFNET_CHANNELS = (192, 128, 96, 64)
IFNET_SCALES = (8, 4, 2, 1)
IFNET_RES = 8
# RIFE 4.2x plans (the reference's fused RIFE, src/kernels/spec/rife_fused.h:7-12): blocks, the input
# reduction d_k of each block and its width C_k. The widths are the models' own (4.25: 192 .. 32);
# the lite models' widths are read from their weights by the importer, these are stand-ins.
RIFE_PLANS = {
    "4.25": (5, (8, 8, 4, 2, 1), (192, 128, 96, 64, 32)),
    "4.26": (5, (16, 8, 4, 2, 1), (192, 128, 96, 64, 32)),
    "4.25lite": (5, (32, 16, 8, 4, 1), (128, 96, 64, 32, 32)),
    "4.22lite": (4, (8, 4, 2, 1), (128, 96, 64, 32)),
}
RIFE_ENC = 16        # encoder width (cnn0..cnn2), 4 planes out per frame
RIFE_Y = 52          # Y_k channels (13 after DepthToSpace(2): flow 4, mask 1, attributes 8)
RIFE_PLAN_FLOATS = 12
E4M3_MAX = 448.0
SCALE_HEADROOM = 1.25

# .span8 package layout (src/gpu/span_fp8/package.h:1-17, package.cpp:143-198), little-endian:
#   header 40 bytes: "AJPSPAN8", version u32 (2), blocks u32 (2..8), stored channels u32 (64),
#   real channels u32 (48 or 64), payload bytes u64, CRC-32 of the payload u32, flags u32
#   (bit 0 f16 accumulators outside the blocks, bit 1 FP16 blocks, bit 2 f32 sums with bit 1);
#   payload: 1 + 3 * blocks f32 activation scales, then conv_1 [64][3][3][16], per block c1, c2,
#   c3 [64][3][3][64] and the 1x1 attention [64][64], conv_cat [64][256], to_pixel [48][3][3][64];
#   each conv's FP16 weights ([out][ky][kx][in]) followed by its f32 biases.
SPAN8_STORED = 64
SPAN8_IN = 16       # conv_1 reads the 12 unshuffled channels padded to 16
SPAN8_PIXEL = 48    # 3 planes x 4 x 4 before DepthToSpace(4)
SPAN8_HEADER = 40


def span_param_shapes():
    """[(name, shape)] of canonical SPAN: OIHW weights, then bias, per conv."""
    c = SPAN_C
    out = [("conv_1.w", (c, 3, 3, 3)), ("conv_1.b", (c,))]
    for b in range(SPAN_BLOCKS):
        for k in range(3):
            out += [(f"block{b}.c{k + 1}.w", (c, c, 3, 3)), (f"block{b}.c{k + 1}.b", (c,))]
    out += [("conv_cat.w", (c, 4 * c, 1, 1)), ("conv_cat.b", (c,))]
    out += [("upsampler.w", (12, c, 3, 3)), ("upsampler.b", (12,))]
    return out


def ifnet_param_shapes():
    """[(name, shape)] of classic IFNet: per block conv0a/conv0b (+PReLU), 8 residual convs,
    the 4x4 stride-2 transposed conv (ConvTranspose weights are [Cin, Cout, kh, kw])."""
    out = []
    for k, c in enumerate(IFNET_CHANNELS):
        cin = 7 if k == 0 else 12
        out += [(f"b{k}.conv0a.w", (c // 2, cin, 3, 3)), (f"b{k}.conv0a.b", (c // 2,)),
                (f"b{k}.conv0a.slope", (c // 2,))]
        out += [(f"b{k}.conv0b.w", (c, c // 2, 3, 3)), (f"b{k}.conv0b.b", (c,)),
                (f"b{k}.conv0b.slope", (c,))]
        for j in range(IFNET_RES):
            out += [(f"b{k}.res{j}.w", (c, c, 3, 3)), (f"b{k}.res{j}.b", (c,)),
                    (f"b{k}.res{j}.slope", (c,))]
        out += [(f"b{k}.last.w", (c, 5, 4, 4)), (f"b{k}.last.b", (5,))]
    return out


def rife_plan_floats(plan):
    """The 12 leading floats of a RIFE 4.2x parameter array: blocks, d_0..d_4, C_0..C_4, 16."""
    blocks, reduce, channels = plan
    v = np.zeros(RIFE_PLAN_FLOATS, np.float32)
    v[0] = blocks
    v[1:1 + blocks] = reduce
    v[6:6 + blocks] = channels
    v[11] = RIFE_ENC
    return v


def rife_param_shapes(plan):
    """[(name, shape)] of RIFE 4.2x after its plan floats: the encoder cnn0..cnn2 (3x3, + slopes) and
    cnn3 (4x4 stride-2 transposed, [Cin, Cout, kh, kw]); per block conv0a / conv0b (3x3 stride 2, +
    slopes), 8 ResConv (W, b, beta, slopes: act(beta * (conv + b) + x)) and the transposed conv to
    52 channels."""
    blocks, reduce, channels = plan
    e = RIFE_ENC
    out = [("enc.cnn0.w", (e, 3, 3, 3)), ("enc.cnn0.b", (e,)), ("enc.cnn0.slope", (e,))]
    for j in (1, 2):
        out += [(f"enc.cnn{j}.w", (e, e, 3, 3)), (f"enc.cnn{j}.b", (e,)), (f"enc.cnn{j}.slope", (e,))]
    out += [("enc.cnn3.w", (e, 4, 4, 4)), ("enc.cnn3.b", (4,))]
    for k in range(blocks):
        c = channels[k]
        cin = 15 if k == 0 else 28
        out += [(f"b{k}.conv0a.w", (c // 2, cin, 3, 3)), (f"b{k}.conv0a.b", (c // 2,)),
                (f"b{k}.conv0a.slope", (c // 2,))]
        out += [(f"b{k}.conv0b.w", (c, c // 2, 3, 3)), (f"b{k}.conv0b.b", (c,)), (f"b{k}.conv0b.slope", (c,))]
        for j in range(IFNET_RES):
            out += [(f"b{k}.res{j}.w", (c, c, 3, 3)), (f"b{k}.res{j}.b", (c,)), (f"b{k}.res{j}.beta", (c,)),
                    (f"b{k}.res{j}.slope", (c,))]
        out += [(f"b{k}.last.w", (c, RIFE_Y, 4, 4)), (f"b{k}.last.b", (RIFE_Y,))]
    return out


def rife_flat(params, plan):
    """The C ABI's parameter array of KB2_MODEL_RIFE_FUSED: plan floats, then the parameters."""
    return np.concatenate([rife_plan_floats(plan), _flat(params, rife_param_shapes(plan))])


def rife_init(plan, seed=3, res_gain=1.0, last_gain=0.3, bias_std=0.02):
    """Seeded RIFE 4.2x weights: Kaiming-normal convs, LeakyReLU slopes 0.2 (the models'
    activation), ResConv betas drawn in [0.1, 0.3] (so the residual stack neither vanishes nor
    explodes), a small gain on the transposed convs (flows of a few pixels), small biases."""
    rng = np.random.default_rng(seed)
    p = {}
    for name, shape in rife_param_shapes(plan):
        if name.endswith(".slope"):
            p[name] = np.full(shape, 0.2, np.float32)
        elif name.endswith(".beta"):
            p[name] = rng.uniform(0.1, 0.3, shape).astype(np.float32)
        elif name.endswith(".b"):
            p[name] = (rng.standard_normal(shape) * bias_std).astype(np.float32)
        elif ".last." in name:
            p[name] = kaiming(rng, shape, shape[0] * 4, gain=last_gain)
        elif name == "enc.cnn3.w":
            p[name] = kaiming(rng, shape, shape[0] * 4, gain=1.0)
        elif ".res" in name:
            p[name] = kaiming(rng, shape, int(np.prod(shape[1:])), gain=res_gain)
        else:
            p[name] = kaiming(rng, shape, int(np.prod(shape[1:])))
    return p


def _flat(params, shapes):
    return np.concatenate([np.asarray(params[n], np.float32).reshape(-1) for n, _ in shapes])


def span_flat(params):
    return _flat(params, span_param_shapes())


def ifnet_flat(params):
    return _flat(params, ifnet_param_shapes())


def unflatten(flat, shapes):
    out, at = {}, 0
    for n, s in shapes:
        k = int(np.prod(s))
        out[n] = np.asarray(flat[at:at + k], np.float32).reshape(s)
        at += k
    assert at == flat.size, "parameter count mismatch"
    return out


def kaiming(rng, shape, fan_in, gain=math.sqrt(2.0)):
    return (rng.standard_normal(shape) * (gain / math.sqrt(fan_in))).astype(np.float32)


def span_init(seed=1):
    """Kaiming-normal weights (fan_in, gain sqrt 2), zero biases (the contract's config 1)."""
    rng = np.random.default_rng(seed)
    p = {}
    for name, shape in span_param_shapes():
        if name.endswith(".b"):
            p[name] = np.zeros(shape, np.float32)
        else:
            p[name] = kaiming(rng, shape, int(np.prod(shape[1:])))
    return p


def ifnet_init(seed=2, res_gain=0.2, last_gain=0.05):
    """Seeded IFNet weights: Kaiming-normal for the entry convs, a damped Kaiming for the eight
    residual convs (x + res_gain * conv, so the residual stack neither vanishes nor explodes),
    a small gain on the transposed conv (flows of a few pixels), zero biases, PReLU slopes 0.25."""
    rng = np.random.default_rng(seed)
    p = {}
    for name, shape in ifnet_param_shapes():
        if name.endswith(".b"):
            p[name] = np.zeros(shape, np.float32)
        elif name.endswith(".slope"):
            p[name] = np.full(shape, 0.25, np.float32)
        elif ".last." in name:
            p[name] = kaiming(rng, shape, shape[0] * 4, gain=last_gain)
        elif ".res" in name:
            p[name] = kaiming(rng, shape, int(np.prod(shape[1:])), gain=res_gain)
        else:
            p[name] = kaiming(rng, shape, int(np.prod(shape[1:])))
    return p


def span8_init(blocks=5, real=48, seed=11, gain=0.7, bias_std=0.02, pixel_gain=0.2, pixel_bias=0.5):
    """Seeded package contents in the stored layout (channels beyond `real` zero, as the
    reference stores a b5f48 in 64 channels, package.h:11-13): Kaiming-normal weights (damped by
    `gain`) rounded to FP16, small normal biases, unit scales, the FP16 flag set. to_pixel is scaled
    by `pixel_gain` around `pixel_bias`, so that most output values fall inside [0, 1] as an
    image's do and the clamped comparison sees them."""
    rng = np.random.default_rng(seed)

    def conv(outs, taps, ins_real, ins_stored, groups=1, out_real=None):
        out_real = outs if out_real is None else out_real
        w = np.zeros((outs, taps, groups, ins_stored), np.float32)
        fan = taps * groups * ins_real
        w[:out_real, :, :, :ins_real] = kaiming(rng, (out_real, taps, groups, ins_real), fan, gain=gain * math.sqrt(2.0))
        b = np.zeros(outs, np.float32)
        b[:out_real] = (rng.standard_normal(out_real) * bias_std).astype(np.float32)
        return {"w": w.reshape(outs, taps, groups * ins_stored).astype(np.float16).astype(np.float32), "b": b}

    p = {"blocks": blocks, "real": real, "flags": 2, "scales": np.ones(1 + 3 * blocks, np.float32)}
    p["first"] = conv(SPAN8_STORED, 9, 12, SPAN8_IN, out_real=real)
    p["block"] = []
    for _ in range(blocks):
        blk = {k: conv(SPAN8_STORED, 9, real, SPAN8_STORED, out_real=real) for k in ("c1", "c2", "c3")}
        blk["att"] = conv(SPAN8_STORED, 1, real, SPAN8_STORED, out_real=real)
        p["block"].append(blk)
    p["concat"] = conv(SPAN8_STORED, 1, real, SPAN8_STORED, groups=4, out_real=real)
    p["pixel"] = conv(SPAN8_PIXEL, 9, real, SPAN8_STORED)
    p["pixel"]["w"] = (p["pixel"]["w"] * np.float32(pixel_gain)).astype(np.float16).astype(np.float32)
    p["pixel"]["b"] = (p["pixel"]["b"] + np.float32(pixel_bias)).astype(np.float32)
    return p


def _crc32(payload):
    import zlib
    return zlib.crc32(payload) & 0xFFFFFFFF


def span8_package(p, version=2):
    """The .span8 bytes of package contents `p` (the writer of package.cpp:200-215)."""
    import struct
    body = bytearray()
    body += np.asarray(p["scales"], "<f4").tobytes()

    def put(c):
        body.extend(np.asarray(c["w"], np.float32).astype("<f2").tobytes())
        body.extend(np.asarray(c["b"], "<f4").tobytes())

    put(p["first"])
    for blk in p["block"]:
        for k in ("c1", "c2", "c3", "att"):
            put(blk[k])
    put(p["concat"])
    put(p["pixel"])
    head = b"AJPSPAN8" + struct.pack("<IIIIQII", version, p["blocks"], SPAN8_STORED, p["real"], len(body),
                                     _crc32(bytes(body)), p["flags"])
    return bytes(head) + bytes(body)


def scales_from_peaks(peaks, floor=None):
    """E4M3 activation scales from calibration peaks: max * 1.25 / 448 per tensor (the reference's
    span_fp8::scales_from_peaks, src/gpu/span_fp8/derive.h:42-62); a non-finite peak is refused,
    and so is a zero peak unless ``floor`` is given (the seeded canonical SPAN's deep blocks decay
    to exact zeros in FP32, so its calibration floors their peaks instead of refusing them)."""
    peaks = np.asarray(peaks, np.float64)
    if floor is not None:
        peaks = np.maximum(peaks, floor)
    if not np.all(np.isfinite(peaks)) or np.any(peaks <= 0):
        raise ValueError("unusable calibration peak")
    return (peaks * SCALE_HEADROOM / E4M3_MAX).astype(np.float32)


def span8_fp8_from_peaks(p, peaks, floor=2.0 ** -14):
    """An FP8 package (no FP16 flag) of contents `p` with activation scales derived from calibration
    peaks in the package's order (conv_1's output, per block its two ReLU outputs and its output):
    scale = max(peak, floor) * 1.25 / 448, as the reference's derive writes them (derive.h:42-62)."""
    q = dict(p)
    q["flags"] = 0
    q["scales"] = scales_from_peaks(peaks, floor)
    return q
