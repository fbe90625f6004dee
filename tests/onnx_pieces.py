"""ONNX pieces of a split RIFE 4.2x model, written from seeded parameters (test infrastructure).

The `onnx` package is not installed here, so this module writes the protobuf wire format of the few
messages a piece uses (ModelProto, GraphProto, NodeProto, AttributeProto, TensorProto,
ValueInfoProto; field numbers from onnx.proto). A piece is what the reference's RIFE splitter hands
its native reader (src/prepare/rife_split.h, src/prepare/rife_native.h): the encoder (cnn0..cnn3) or
one IFBlock (conv0, 8 ResConv with beta, lastconv), one input, one output. The options vary the
encodings a real export may use: element type, raw or typed storage, constants as initializers or
Constant nodes, LeakyRelu or PRelu, Identity / Cast nodes on the chain, a separable conv0a.
"""
from __future__ import annotations

import struct

import numpy as np

FLOAT, INT8, INT32, INT64, FLOAT16, DOUBLE, BFLOAT16, E4M3 = 1, 3, 6, 7, 10, 11, 16, 17


# ---------------------------------------------------------------------------- wire format
def _varint(v: int) -> bytes:
    v &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field: int, wire: int) -> bytes:
    return _varint((field << 3) | wire)


def f_varint(field: int, v: int) -> bytes:
    return _key(field, 0) + _varint(v)


def f_bytes(field: int, payload: bytes) -> bytes:
    return _key(field, 2) + _varint(len(payload)) + payload


def f_str(field: int, s: str) -> bytes:
    return f_bytes(field, s.encode())


def f_float(field: int, v: float) -> bytes:
    return _key(field, 5) + struct.pack("<f", v)


def f_packed_ints(field: int, vals) -> bytes:
    return f_bytes(field, b"".join(_varint(int(v)) for v in vals))


# ---------------------------------------------------------------------------- messages
def tensor(name: str, arr, dtype: int = FLOAT, storage: str = "raw", external: bool = False) -> bytes:
    """TensorProto of `arr` (float32 values, already representable in `dtype`)."""
    a = np.asarray(arr, np.float32)
    out = f_packed_ints(1, a.shape) if a.ndim else b""
    out += f_varint(2, dtype) + f_str(8, name)
    if external:
        return out + f_bytes(13, f_str(1, "location") + f_str(2, name + ".bin")) + f_varint(14, 1)
    flat = a.reshape(-1)
    if dtype == FLOAT:
        if storage == "raw":
            out += f_bytes(9, flat.astype("<f4").tobytes())
        else:
            out += f_bytes(4, flat.astype("<f4").tobytes())
    elif dtype == FLOAT16:
        bits = flat.astype("<f2")
        if storage == "raw":
            out += f_bytes(9, bits.tobytes())
        else:
            out += f_packed_ints(5, bits.view("<u2"))
    elif dtype == BFLOAT16:
        out += f_bytes(9, (flat.astype("<f4").view("<u4") >> 16).astype("<u2").tobytes())
    elif dtype == DOUBLE:
        out += f_bytes(9, flat.astype("<f8").tobytes())
    else:
        raise ValueError(dtype)
    return out


def attr(name: str, *, i=None, f=None, s=None, ints=None, t=None) -> bytes:
    out = f_str(1, name)
    if f is not None:
        out += f_float(2, f) + f_varint(20, 1)
    if i is not None:
        out += f_varint(3, i) + f_varint(20, 2)
    if s is not None:
        out += f_bytes(4, s.encode()) + f_varint(20, 3)
    if t is not None:
        out += f_bytes(5, t) + f_varint(20, 4)
    if ints is not None:
        out += f_packed_ints(8, ints) + f_varint(20, 7)
    return out


def node(op: str, inputs, outputs, name: str, attrs=(), domain=None) -> bytes:
    out = b"".join(f_str(1, x) for x in inputs) + b"".join(f_str(2, x) for x in outputs)
    out += f_str(3, name) + f_str(4, op)
    out += b"".join(f_bytes(5, a) for a in attrs)
    if domain is not None:
        out += f_str(7, domain)
    return out


def value_info(name: str) -> bytes:
    # tensor type FLOAT, rank 4 with symbolic dimensions
    dims = b"".join(f_bytes(1, f_str(2, d)) for d in ("n", "c", "h", "w"))
    ttype = f_varint(1, FLOAT) + f_bytes(2, dims)
    return f_str(1, name) + f_bytes(2, f_bytes(1, ttype))


def model(nodes, inits, inputs, outputs) -> bytes:
    g = b"".join(f_bytes(1, n) for n in nodes) + f_str(2, "piece")
    g += b"".join(f_bytes(5, t) for t in inits)
    g += b"".join(f_bytes(11, value_info(x)) for x in inputs) + b"".join(f_bytes(12, value_info(x)) for x in outputs)
    opset = f_str(1, "") + f_varint(2, 17)
    return f_varint(1, 8) + f_str(2, "kb2-tests") + f_bytes(7, g) + f_bytes(8, opset)


# ---------------------------------------------------------------------------- pieces
def representable(a, dtype: int) -> np.ndarray:
    """`a` rounded to what `dtype` holds, as float32 (the values a reader must return)."""
    a = np.asarray(a, np.float32)
    return a.astype(np.float16).astype(np.float32) if dtype == FLOAT16 else a


class Piece:
    """A chain under construction: constants, nodes and the current tensor."""

    def __init__(self, dtype=FLOAT, storage="raw", constant_nodes=False, act="leaky", passthrough=False):
        self.dtype, self.storage, self.constant_nodes = dtype, storage, constant_nodes
        self.act, self.passthrough = act, passthrough
        self.nodes, self.inits = [], []
        self.cur, self.n = "input", 0

    def _name(self, stem):
        self.n += 1
        return f"{stem}_{self.n}"

    def const(self, stem, arr, dtype=None):
        name = self._name(stem)
        t = tensor(name, representable(arr, dtype or self.dtype), dtype or self.dtype, self.storage)
        if self.constant_nodes:
            self.nodes.append(node("Constant", [], [name], name + "_node", [attr("value", t=t)]))
        else:
            self.inits.append(t)
        return name

    def op(self, op, inputs, attrs=()):
        out = self._name(op.lower())
        self.nodes.append(node(op, inputs, [out], out + "_node", attrs))
        self.cur = out
        if self.passthrough and op in ("Conv", "LeakyRelu"):
            self.op("Identity", [out])
        return self.cur

    def conv(self, w, b, stride, transposed=False):
        attrs = [attr("strides", ints=[stride, stride]), attr("pads", ints=[1, 1, 1, 1])]
        kshape = 4 if transposed else 3
        attrs.append(attr("kernel_shape", ints=[kshape, kshape]))
        return self.op("ConvTranspose" if transposed else "Conv",
                       [self.cur, self.const("w", w), self.const("b", b)], attrs)

    def activation(self, slope):
        slope = np.asarray(slope, np.float32)
        if self.act == "leaky":
            assert np.all(slope == slope[0])
            return self.op("LeakyRelu", [self.cur], [attr("alpha", f=float(slope[0]))])
        if self.act == "relu":
            return self.op("Relu", [self.cur])
        return self.op("PRelu", [self.cur, self.const("slope", slope.reshape(-1, 1, 1), FLOAT)])

    def resconv(self, w, b, beta, slope):
        x = self.cur
        self.conv(w, b, 1)
        self.op("Mul", [self.cur, self.const("beta", np.asarray(beta).reshape(1, -1, 1, 1), FLOAT)])
        self.op("Add", [self.cur, x])
        return self.activation(slope)

    def bytes(self):
        if self.passthrough:
            self.op("Cast", [self.cur], [attr("to", i=FLOAT)])
        return model(self.nodes, self.inits, ["input"], [self.cur])


def encoder_piece(p, **opts) -> bytes:
    c = Piece(**opts)
    c.conv(p["enc.cnn0.w"], p["enc.cnn0.b"], 2)
    c.activation(p["enc.cnn0.slope"])
    for j in (1, 2):
        c.conv(p[f"enc.cnn{j}.w"], p[f"enc.cnn{j}.b"], 1)
        c.activation(p[f"enc.cnn{j}.slope"])
    c.conv(p["enc.cnn3.w"], p["enc.cnn3.b"], 2, transposed=True)
    return c.bytes()


def block_piece(p, k, res=8, **opts) -> bytes:
    c = Piece(**opts)
    c.conv(p[f"b{k}.conv0a.w"], p[f"b{k}.conv0a.b"], 2)
    c.activation(p[f"b{k}.conv0a.slope"])
    c.conv(p[f"b{k}.conv0b.w"], p[f"b{k}.conv0b.b"], 2)
    c.activation(p[f"b{k}.conv0b.slope"])
    for j in range(res):
        c.resconv(p[f"b{k}.res{j}.w"], p[f"b{k}.res{j}.b"], p[f"b{k}.res{j}.beta"], p[f"b{k}.res{j}.slope"])
    c.conv(p[f"b{k}.last.w"], p[f"b{k}.last.b"], 2, transposed=True)
    return c.bytes()


def separable_block_piece(p, k, depthwise_w, depthwise_b, pointwise_w, pointwise_b) -> bytes:
    """Block k with conv0a written as a depthwise 3x3 (stride 2, one group per input channel) then a
    1x1 (the reader folds the pair into one 3x3); the other layers as in block_piece."""
    c = Piece()
    cin = depthwise_w.shape[0]
    c.op("Conv", [c.cur, c.const("dw", depthwise_w), c.const("db", depthwise_b)],
         [attr("strides", ints=[2, 2]), attr("pads", ints=[1, 1, 1, 1]), attr("group", i=cin)])
    c.op("Conv", [c.cur, c.const("pw", pointwise_w), c.const("pb", pointwise_b)],
         [attr("strides", ints=[1, 1]), attr("pads", ints=[0, 0, 0, 0])])
    c.activation(p[f"b{k}.conv0a.slope"])
    c.conv(p[f"b{k}.conv0b.w"], p[f"b{k}.conv0b.b"], 2)
    c.activation(p[f"b{k}.conv0b.slope"])
    for j in range(8):
        c.resconv(p[f"b{k}.res{j}.w"], p[f"b{k}.res{j}.b"], p[f"b{k}.res{j}.beta"], p[f"b{k}.res{j}.slope"])
    c.conv(p[f"b{k}.last.w"], p[f"b{k}.last.b"], 2, transposed=True)
    return c.bytes()
