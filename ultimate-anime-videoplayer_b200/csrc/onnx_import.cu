// RIFE 4.2x weights from ONNX pieces (onnx_import.h). The reader decodes the protobuf wire format of
// the few ONNX messages a piece needs (ModelProto.graph; GraphProto nodes, initializers, inputs and
// outputs; NodeProto; AttributeProto; TensorProto with float, float16, bfloat16 or double data,
// inline); the walk follows the piece's chain from its input to its output the way the reference's
// native RIFE reader does (src/prepare/rife_native.cpp: a Conv, then optionally a per-channel Mul and
// the Add of the conv's input, then the activation; a ConvTranspose last).
#include <cuda_fp16.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <string>

#include "onnx_import.h"

namespace kb2 {

namespace {

// ------------------------------------------------------------------ protobuf wire format
struct Pb {
  const uint8_t* p = nullptr;
  const uint8_t* end = nullptr;
  bool ok = true;

  bool more() const { return ok && p < end; }
  uint64_t varint() {
    uint64_t v = 0;
    for (int s = 0; s < 64; s += 7) {
      if (p >= end) break;
      const uint8_t b = *p++;
      v |= static_cast<uint64_t>(b & 0x7Fu) << s;
      if ((b & 0x80u) == 0) return v;
    }
    ok = false;
    return 0;
  }
  uint32_t fixed32() {
    if (end - p < 4) {
      ok = false;
      return 0;
    }
    uint32_t v;
    std::memcpy(&v, p, 4);
    p += 4;
    return v;
  }
  uint64_t fixed64() {
    if (end - p < 8) {
      ok = false;
      return 0;
    }
    uint64_t v;
    std::memcpy(&v, p, 8);
    p += 8;
    return v;
  }
  Pb sub() {
    const uint64_t n = varint();
    if (!ok || n > static_cast<uint64_t>(end - p)) {
      ok = false;
      return Pb{end, end, false};
    }
    Pb s{p, p + n, true};
    p += n;
    return s;
  }
  std::string str() {
    const Pb s = sub();
    return ok ? std::string(reinterpret_cast<const char*>(s.p), static_cast<size_t>(s.end - s.p)) : std::string();
  }
  bool key(uint32_t& num, uint32_t& wire) {
    const uint64_t k = varint();
    num = static_cast<uint32_t>(k >> 3);
    wire = static_cast<uint32_t>(k & 7u);
    return ok && num != 0;
  }
  void skip(uint32_t wire) {
    switch (wire) {
      case 0: varint(); break;
      case 1: fixed64(); break;
      case 2: sub(); break;
      case 5: fixed32(); break;
      default: ok = false; break;
    }
  }
  // a repeated int64 field, packed (wire 2) or one element (wire 0)
  void ints(uint32_t wire, std::vector<int64_t>& out) {
    if (wire == 2) {
      Pb s = sub();
      while (s.more()) out.push_back(static_cast<int64_t>(s.varint()));
      ok = ok && s.ok;
    } else if (wire == 0) {
      out.push_back(static_cast<int64_t>(varint()));
    } else {
      ok = false;
    }
  }
  // a repeated float field, packed (wire 2) or one element (wire 5)
  void floats(uint32_t wire, std::vector<float>& out) {
    auto one = [&](uint32_t bits) {
      float f;
      std::memcpy(&f, &bits, 4);
      out.push_back(f);
    };
    if (wire == 2) {
      Pb s = sub();
      while (s.more()) one(s.fixed32());
      ok = ok && s.ok;
    } else if (wire == 5) {
      one(fixed32());
    } else {
      ok = false;
    }
  }
};

// ------------------------------------------------------------------ the ONNX messages a piece uses
// TensorProto.data_type values a piece may hold (onnx.proto's DataType), with their element sizes.
// The float types (FLOAT, FLOAT16, FLOAT8E4M3FN, INT8) are decoded to floats; INT32 and INT64 only
// sized (a shape constant may be one; a weight must be a float type). Every other type refuses the
// piece, as the reference's tensor reader does (src/gpu/ir/onnx_tensor.cpp:29-44).
enum OnnxType : int32_t {
  kOnnxFloat = 1,
  kOnnxInt8 = 3,
  kOnnxInt32 = 6,
  kOnnxInt64 = 7,
  kOnnxFloat16 = 10,
  kOnnxE4M3 = 17
};

size_t element_bytes(int32_t type) {
  switch (type) {
    case kOnnxFloat:
    case kOnnxInt32: return 4;
    case kOnnxInt64: return 8;
    case kOnnxFloat16: return 2;
    case kOnnxE4M3:
    case kOnnxInt8: return 1;
    default: return 0;
  }
}

// Why a piece was not read: KB2_WEIGHTS_INVALID (malformed bytes) or KB2_FORMAT_UNSUPPORTED (data
// outside the file, segments, sparse initializers, a data type outside the list above). The first
// failure is kept.
struct Fail {
  int code = KB2_OK;
  std::string why;
  bool set(int c, std::string w) {
    if (code == KB2_OK) {
      code = c;
      why = std::move(w);
    }
    return false;
  }
  bool malformed(std::string w) { return set(KB2_WEIGHTS_INVALID, "ONNX: " + std::move(w)); }
  bool unsupported(std::string w) { return set(KB2_FORMAT_UNSUPPORTED, "ONNX: " + std::move(w)); }
};

struct Tensor {
  std::string name;
  std::vector<int64_t> dims;
  std::vector<float> f;  // the values, when the type is a float type
  bool floats = false;
};

struct Attr {
  std::string name;
  float f = 0.0f;
  int64_t i = 0;
  std::string s;
  std::vector<int64_t> ints;
  std::vector<float> fl;
  std::vector<Tensor> t;  // `t`: one tensor, the last one read wins
};

struct Node {
  std::string name, op, domain;
  std::vector<std::string> in, out;
  std::vector<Attr> attrs;
  const Attr* attr(const char* n) const {
    for (const Attr& a : attrs)
      if (a.name == n) return &a;
    return nullptr;
  }
};

struct Graph {
  std::vector<Node> nodes;
  std::vector<Tensor> inits;
  std::vector<std::string> inputs, outputs;
};

float half_bits(uint16_t b) {
  __half_raw r;
  r.x = b;
  return __half2float(__half(r));
}

// An E4M3 (FN) code as a float: the codes with every exponent and mantissa bit set are NaN.
float e4m3_bits(uint8_t b) { return (b & 0x7Fu) == 0x7Fu ? NAN : e4m3_decode(b); }

// The values of a float tensor whose elements come as raw little-endian bytes.
void decode_raw(const uint8_t* r, size_t count, int32_t type, std::vector<float>& out) {
  out.resize(count);
  for (size_t i = 0; i < count; ++i) {
    switch (type) {
      case kOnnxFloat: std::memcpy(&out[i], r + 4 * i, 4); break;
      case kOnnxFloat16: out[i] = half_bits(static_cast<uint16_t>(r[2 * i] | (r[2 * i + 1] << 8))); break;
      case kOnnxE4M3: out[i] = e4m3_bits(r[i]); break;
      default: out[i] = static_cast<float>(static_cast<int8_t>(r[i])); break;  // INT8
    }
  }
}

// The values of a float tensor held in int32_data: FLOAT16 and E4M3 bit patterns, INT8 values.
bool decode_words(const std::vector<int64_t>& words, int32_t type, const std::string& name, std::vector<float>& out,
                  Fail& fail) {
  for (int64_t w : words) {
    if (type == kOnnxFloat16) {
      if (w < 0 || w > 0xFFFF) return fail.malformed("tensor " + name + ": FLOAT16 pattern out of 16 bits");
      out.push_back(half_bits(static_cast<uint16_t>(w)));
    } else if (type == kOnnxE4M3) {
      if (w < 0 || w > 0xFF) return fail.malformed("tensor " + name + ": FLOAT8E4M3FN pattern out of 8 bits");
      out.push_back(e4m3_bits(static_cast<uint8_t>(w)));
    } else if (type == kOnnxInt8) {
      if (w < -128 || w > 127) return fail.malformed("tensor " + name + ": INT8 value out of range");
      out.push_back(static_cast<float>(w));
    } else if (w < INT32_MIN || w > INT32_MAX) {
      return fail.malformed("tensor " + name + ": INT32 value out of range");
    }
  }
  return true;
}

bool read_tensor(Pb in, Tensor& t, Fail& fail) {
  int32_t type = 0;
  bool has_raw = false, external = false, segmented = false;
  std::string raw;
  std::vector<int64_t> i32, i64;
  std::vector<float> fdata;
  uint32_t num, wire;
  while (in.more() && in.key(num, wire)) {
    switch (num) {
      case 1: in.ints(wire, t.dims); break;
      case 2: type = static_cast<int32_t>(in.varint()); break;
      case 3: segmented = true; in.skip(wire); break;
      case 4: in.floats(wire, fdata); break;
      case 5: in.ints(wire, i32); break;
      case 7: in.ints(wire, i64); break;
      case 8: t.name = in.str(); break;
      case 9: raw = in.str(); has_raw = true; break;
      case 13: external = true; in.skip(wire); break;
      case 14: external = (in.varint() == 1) || external; break;
      default: in.skip(wire); break;
    }
  }
  if (!in.ok) return fail.malformed("unreadable tensor");
  if (external) return fail.unsupported("tensor " + t.name + ": weights outside the ONNX file");
  if (segmented) return fail.unsupported("tensor " + t.name + ": segments");
  const size_t size = element_bytes(type);
  if (size == 0) return fail.unsupported("tensor " + t.name + ": data type " + std::to_string(type));
  if (t.dims.size() > 8) return fail.malformed("tensor " + t.name + ": too many dimensions");
  size_t count = 1;
  for (int64_t d : t.dims) {
    if (d < 0) return fail.malformed("tensor " + t.name + ": negative dimension");
    if (d != 0 && count > UINT32_MAX / static_cast<uint64_t>(d))
      return fail.malformed("tensor " + t.name + ": too many elements");
    count *= static_cast<size_t>(d);
  }
  const bool is_float = type == kOnnxFloat || type == kOnnxFloat16 || type == kOnnxE4M3 || type == kOnnxInt8;
  const bool typed = !fdata.empty() || !i32.empty() || !i64.empty();
  if (has_raw && typed) return fail.malformed("tensor " + t.name + ": raw and typed data at once");
  if (has_raw) {
    if (raw.size() % size != 0 || raw.size() / size != count)
      return fail.malformed("tensor " + t.name + ": raw bytes do not match the shape");
    if (is_float) decode_raw(reinterpret_cast<const uint8_t*>(raw.data()), count, type, t.f);
    t.floats = is_float;
    return true;
  }
  // each type has its own typed field: float_data, int32_data (INT32 and the 8/16-bit types), int64_data
  const bool placed = type == kOnnxFloat ? (i32.empty() && i64.empty())
                      : type == kOnnxInt64 ? (fdata.empty() && i32.empty())
                                           : (fdata.empty() && i64.empty());
  if (!placed) return fail.malformed("tensor " + t.name + ": values in another type's field");
  if (type == kOnnxFloat) t.f = std::move(fdata);
  if (!decode_words(i32, type, t.name, t.f, fail)) return false;
  const size_t present = type == kOnnxFloat || is_float ? t.f.size() : type == kOnnxInt64 ? i64.size() : i32.size();
  if (present != count) return fail.malformed("tensor " + t.name + ": value count does not match the shape");
  t.floats = is_float;
  return true;
}

bool read_attr(Pb in, Attr& a, Fail& fail) {
  uint32_t num, wire;
  while (in.more() && in.key(num, wire)) {
    switch (num) {
      case 1: a.name = in.str(); break;
      case 2: {
        const uint32_t b = in.fixed32();
        std::memcpy(&a.f, &b, 4);
        break;
      }
      case 3: a.i = static_cast<int64_t>(in.varint()); break;
      case 4: a.s = in.str(); break;
      case 5: {
        Tensor t;
        if (!read_tensor(in.sub(), t, fail)) return false;
        a.t.assign(1, std::move(t));
        break;
      }
      case 7: in.floats(wire, a.fl); break;
      case 8: in.ints(wire, a.ints); break;
      default: in.skip(wire); break;
    }
  }
  return in.ok || fail.malformed("unreadable attribute");
}

bool read_node(Pb in, Node& n, Fail& fail) {
  uint32_t num, wire;
  while (in.more() && in.key(num, wire)) {
    switch (num) {
      case 1: n.in.push_back(in.str()); break;
      case 2: n.out.push_back(in.str()); break;
      case 3: n.name = in.str(); break;
      case 4: n.op = in.str(); break;
      case 5: {
        n.attrs.emplace_back();
        if (!read_attr(in.sub(), n.attrs.back(), fail)) return false;
        break;
      }
      case 7: n.domain = in.str(); break;
      default: in.skip(wire); break;
    }
  }
  return in.ok || fail.malformed("unreadable node");
}

std::string value_info_name(Pb in) {
  uint32_t num, wire;
  std::string name;
  while (in.more() && in.key(num, wire)) {
    if (num == 1)
      name = in.str();
    else
      in.skip(wire);
  }
  return name;
}

bool read_graph(Pb in, Graph& g, Fail& fail) {
  uint32_t num, wire;
  while (in.more() && in.key(num, wire)) {
    switch (num) {
      case 1: {
        g.nodes.emplace_back();
        if (wire != 2 || !read_node(in.sub(), g.nodes.back(), fail)) return fail.malformed("unreadable node");
        break;
      }
      case 5: {
        g.inits.emplace_back();
        if (wire != 2 || !read_tensor(in.sub(), g.inits.back(), fail)) return fail.malformed("unreadable tensor");
        break;
      }
      case 11: g.inputs.push_back(value_info_name(in.sub())); break;
      case 12: g.outputs.push_back(value_info_name(in.sub())); break;
      case 15: return fail.unsupported("sparse initializers");
      default: in.skip(wire); break;
    }
  }
  return in.ok || fail.malformed("unreadable graph");
}

Status read_model(const uint8_t* p, size_t n, Graph& g) {
  Pb in{p, p + n, true};
  Fail fail;
  uint32_t num, wire;
  bool found = false;
  while (in.more() && in.key(num, wire)) {
    if (num == 7) {
      if (wire != 2 || found) {
        fail.malformed(found ? "several graphs" : "unreadable graph");
        break;
      }
      if (!read_graph(in.sub(), g, fail)) break;
      found = true;
    } else {
      in.skip(wire);
    }
  }
  if (fail.code != KB2_OK) return refuse(fail.code, fail.why);
  if (!in.ok) return refuse(KB2_WEIGHTS_INVALID, "ONNX: unreadable model");
  if (!found) return refuse(KB2_WEIGHTS_INVALID, "ONNX: no graph");
  return Status::Ok();
}

// ------------------------------------------------------------------ the chain of a piece
// Where the last layer stands: its conv alone, scaled by a per-channel Mul, its residual added, or
// activated (a new conv may follow only a conv or an activation).
enum class Stage { Conv, Scaled, Added, Activated };

struct Walk {
  std::map<std::string, const Tensor*> constants;
  std::map<std::string, std::vector<const Node*>> readers;
  std::vector<OnnxLayer> layers;
  std::vector<std::string> layer_input;  // each layer's input tensor (its residual reads it)
  Stage stage = Stage::Activated;
  const Tensor* constant(const std::string& n) const {
    const auto it = constants.find(n);
    return it == constants.end() ? nullptr : it->second;
  }
};

Status unknown(const std::string& what) { return refuse(KB2_WEIGHTS_INVALID, "ONNX piece: " + what); }

std::vector<int64_t> ints_or(const Node& n, const char* name, std::vector<int64_t> fallback) {
  const Attr* a = n.attr(name);
  return a != nullptr ? a->ints : fallback;
}

bool all_are(const std::vector<int64_t>& v, int64_t want, size_t count) {
  return v.size() == count && std::all_of(v.begin(), v.end(), [want](int64_t x) { return x == want; });
}

// cout values of a constant applied per channel to an N x C x H x W activation: one value (every
// dimension 1), or C values shaped C x 1 x 1 or 1 x C x 1 x 1. Empty when it is neither.
std::vector<float> per_channel(const Tensor& t, int cout) {
  const std::vector<int64_t>& d = t.dims;
  if (!t.floats || d.size() > 4) return {};
  if (t.f.size() == 1 && std::all_of(d.begin(), d.end(), [](int64_t v) { return v == 1; }))
    return std::vector<float>(static_cast<size_t>(cout), t.f[0]);
  const bool chw = (d.size() == 3 && d[0] == cout && d[1] == 1 && d[2] == 1) ||
                   (d.size() == 4 && d[0] == 1 && d[1] == cout && d[2] == 1 && d[3] == 1);
  return chw && t.f.size() == static_cast<size_t>(cout) ? t.f : std::vector<float>{};
}

// A 1x1 Conv that directly follows a convolution (a separable conv's pointwise half) folded into
// that layer: W'[o] = sum_m P[o][m] W[m], b'[o] = c[o] + sum_m P[o][m] b[m], summed in double in the
// order of m (the reference's fold, src/prepare/rife_native.cpp:122-147).
Status fold_pointwise(Walk& w, const Node& n, const Tensor& wt, const std::vector<float>& bias) {
  OnnxLayer& last = w.layers.back();
  const size_t mid = static_cast<size_t>(last.cout), cout = static_cast<size_t>(wt.dims[0]);
  if (last.transposed || static_cast<size_t>(wt.dims[1]) != mid)
    return unknown(n.name + ": a 1x1 conv that does not follow a 3x3 conv");
  const size_t row = static_cast<size_t>(last.cin) * 9;  // one output channel's weights, [cin][3][3]
  std::vector<float> folded(cout * row), folded_bias(cout);
  for (size_t o = 0; o < cout; ++o) {
    double b = bias[o];
    for (size_t m = 0; m < mid; ++m) b += static_cast<double>(wt.f[o * mid + m]) * last.b[m];
    folded_bias[o] = static_cast<float>(b);
    for (size_t i = 0; i < row; ++i) {
      double sum = 0.0;
      for (size_t m = 0; m < mid; ++m) sum += static_cast<double>(wt.f[o * mid + m]) * last.w[m * row + i];
      folded[o * row + i] = static_cast<float>(sum);
    }
  }
  last.cout = static_cast<int>(cout);
  last.w = std::move(folded);
  last.b = std::move(folded_bias);
  return Status::Ok();  // the stage stays Conv: scale, residual and activation may follow
}

// Conv 3x3 (pad 1, stride 1 or 2; one group, or one per channel: a depthwise conv, stored as a
// diagonal 3x3), Conv 1x1 (pad 0, stride 1: folded into a conv it follows, else stored as a 3x3 with
// its centre tap alone) or ConvTranspose 4x4 (pad 1, stride 2), the attribute checks of the
// reference's conv_shape / conv_stride (src/prepare/rife_native.cpp:76-100, 159-193).
Status add_conv(Walk& w, const Node& n, const std::string& input) {
  OnnxLayer l;
  l.transposed = n.op == "ConvTranspose";
  const int full = l.transposed ? 4 : 3;
  const Tensor* wt = n.in.size() >= 2 ? w.constant(n.in[1]) : nullptr;
  const std::string shape_msg = n.name + ": constant " + std::to_string(full) + "x" + std::to_string(full) +
                                " weights expected";
  if (wt == nullptr || wt->dims.size() != 4) return unknown(shape_msg);
  const std::vector<int64_t>& d = wt->dims;
  const bool pointwise = !l.transposed && d[2] == 1 && d[3] == 1;
  const int k = pointwise ? 1 : full;
  if (d[2] != k || d[3] != k) return unknown(shape_msg);
  const Attr* group = n.attr("group");
  const bool depthwise = !l.transposed && !pointwise && d[1] == 1 && d[0] > 1 && group != nullptr && group->i == d[0];
  const int64_t g = group != nullptr ? group->i : 1;
  const Attr* auto_pad = n.attr("auto_pad");
  if ((g != 1 && (!depthwise || g != d[0])) || (auto_pad != nullptr && auto_pad->s != "NOTSET"))
    return unknown(n.name + ": groups or auto_pad");
  const std::vector<int64_t> strides = ints_or(n, "strides", {1, 1});
  if (!all_are(ints_or(n, "pads", {0, 0, 0, 0}), k == 1 ? 0 : 1, 4) || !all_are(ints_or(n, "dilations", {1, 1}), 1, 2) ||
      strides.size() != 2 || strides[0] != strides[1])
    return unknown(n.name + ": pads, dilations or strides");
  l.stride = static_cast<int>(strides[0]);
  if (l.transposed) {
    if (l.stride != 2 || !all_are(ints_or(n, "output_padding", {0, 0}), 0, 2) || n.attr("output_shape") != nullptr)
      return unknown(n.name + ": a 4x4 transposed conv of stride 2 expected");
  } else if (k == 1 ? l.stride != 1 : (l.stride != 1 && l.stride != 2)) {
    return unknown(n.name + ": stride");
  }
  l.cout = static_cast<int>(l.transposed ? d[1] : d[0]);
  l.cin = static_cast<int>(depthwise || l.transposed ? d[0] : d[1]);
  const size_t per_out = depthwise ? 1 : static_cast<size_t>(l.transposed ? d[0] : d[1]);
  if (l.cin < 1 || l.cout < 1 || !wt->floats ||
      wt->f.size() != per_out * static_cast<size_t>(l.cout) * static_cast<size_t>(k * k))
    return unknown(n.name + ": weight size");
  std::vector<float> bias;
  if (n.in.size() >= 3 && !n.in[2].empty()) {
    const Tensor* b = w.constant(n.in[2]);
    if (b == nullptr || !b->floats || b->f.size() != static_cast<size_t>(l.cout)) return unknown(n.name + ": bias");
    bias = b->f;
  } else {
    bias.assign(static_cast<size_t>(l.cout), 0.0f);
  }
  if (k == 1 && w.stage == Stage::Conv && !w.layers.empty()) return fold_pointwise(w, n, *wt, bias);
  if (pointwise || depthwise) {  // stored as a 3x3, OIHW
    const size_t cin = static_cast<size_t>(l.cin), cout = static_cast<size_t>(l.cout);
    l.w.assign(cout * cin * 9, 0.0f);
    for (size_t o = 0; o < cout; ++o) {
      if (depthwise) {
        for (size_t t = 0; t < 9; ++t) l.w[(o * cin + o) * 9 + t] = wt->f[o * 9 + t];
      } else {
        for (size_t c = 0; c < cin; ++c) l.w[(o * cin + c) * 9 + 4] = wt->f[o * cin + c];
      }
    }
  } else {
    l.w = wt->f;
  }
  l.b = std::move(bias);
  w.layers.push_back(std::move(l));
  w.layer_input.push_back(input);
  w.stage = Stage::Conv;
  return Status::Ok();
}

Status add_activation(Walk& w, const Node& n) {
  OnnxLayer& l = w.layers.back();
  if (w.stage != Stage::Conv && w.stage != Stage::Added) return unknown(n.name + ": activation out of place");
  if (n.op == "LeakyRelu") {
    const Attr* alpha = n.attr("alpha");
    l.slope.assign(static_cast<size_t>(l.cout), alpha != nullptr ? alpha->f : 0.01f);
  } else if (n.op == "Relu") {
    l.slope.assign(static_cast<size_t>(l.cout), 0.0f);
  } else {  // PRelu
    const Tensor* s = n.in.size() == 2 ? w.constant(n.in[1]) : nullptr;
    l.slope = s != nullptr ? per_channel(*s, l.cout) : std::vector<float>{};
    if (l.slope.empty()) return unknown(n.name + ": PRelu slope");
  }
  w.stage = Stage::Activated;
  return Status::Ok();
}

Status add_residual_part(Walk& w, const Node& n, const std::string& current) {
  OnnxLayer& l = w.layers.back();
  if (n.in.size() != 2) return unknown(n.name + ": two inputs expected");
  const std::string& other = n.in[0] == current ? n.in[1] : n.in[0];
  if (n.op == "Mul") {
    const Tensor* f = w.constant(other);
    if (w.stage != Stage::Conv || f == nullptr) return unknown(n.name + ": Mul out of place");
    l.scale = per_channel(*f, l.cout);
    if (l.scale.empty()) return unknown(n.name + ": Mul factor");
    w.stage = Stage::Scaled;
    return Status::Ok();
  }
  if ((w.stage != Stage::Conv && w.stage != Stage::Scaled) || other != w.layer_input.back() || l.cin != l.cout ||
      l.transposed)
    return unknown(n.name + ": an Add that is not the conv's residual");
  if (l.scale.empty()) l.scale.assign(static_cast<size_t>(l.cout), 1.0f);
  w.stage = Stage::Added;
  return Status::Ok();
}

// The node after `current` on the chain: its only reader, or the Conv of a residual conv whose Add
// is the other reader.
const Node* next_node(const Walk& w, const std::string& current) {
  const auto it = w.readers.find(current);
  if (it == w.readers.end()) return nullptr;
  const std::vector<const Node*>& r = it->second;
  if (r.size() == 1) return r[0];
  if (r.size() != 2) return nullptr;
  if (r[0]->op == "Conv" && r[1]->op == "Add") return r[0];
  if (r[1]->op == "Conv" && r[0]->op == "Add") return r[1];
  return nullptr;
}

}  // namespace

Status onnx_piece_layers(const uint8_t* model, size_t bytes, std::vector<OnnxLayer>& layers) {
  if (model == nullptr || bytes == 0) return refuse(KB2_INVALID_ARGUMENT, "ONNX piece: no bytes");
  Graph g;
  KB2_TRY(read_model(model, bytes, g));
  Walk w;
  for (const Tensor& t : g.inits) w.constants.emplace(t.name, &t);
  for (const Node& n : g.nodes) {
    if (n.op == "Constant" && n.out.size() == 1) {
      const Attr* v = n.attr("value");
      if (v != nullptr && v->t.size() == 1) w.constants.emplace(n.out[0], &v->t[0]);
      continue;
    }
    for (const std::string& in : n.in)
      if (!in.empty() && w.constant(in) == nullptr) w.readers[in].push_back(&n);
  }
  std::vector<std::string> inputs;
  for (const std::string& in : g.inputs)
    if (w.constant(in) == nullptr) inputs.push_back(in);
  if (inputs.size() != 1 || g.outputs.size() != 1) return unknown("one input and one output expected");
  std::string current = inputs[0];
  for (size_t steps = 0; current != g.outputs[0]; ++steps) {
    const Node* n = next_node(w, current);
    if (n == nullptr || n->out.size() != 1 || steps > g.nodes.size())
      return unknown("the chain breaks or branches after " + current);
    if (!n->domain.empty() && n->domain != "ai.onnx") return unknown(n->name + ": domain " + n->domain);
    const std::string& op = n->op;
    if (op == "Conv" || op == "ConvTranspose") {
      if (w.stage == Stage::Scaled || w.stage == Stage::Added) return unknown(n->name + ": residual without activation");
      KB2_TRY(add_conv(w, *n, current));
    } else if (op == "Cast" || op == "Identity") {
      // passes through
    } else if (w.layers.empty()) {
      return unknown(n->name + ": " + op + " before the first convolution");
    } else if (op == "LeakyRelu" || op == "Relu" || op == "PRelu") {
      KB2_TRY(add_activation(w, *n));
    } else if (op == "Mul" || op == "Add") {
      KB2_TRY(add_residual_part(w, *n, current));
    } else {
      return unknown(n->name + ": operator " + op);
    }
    current = n->out[0];
  }
  if (w.stage == Stage::Scaled || w.stage == Stage::Added) return unknown("unfinished residual at the end");
  layers = std::move(w.layers);
  return Status::Ok();
}

namespace {

Status expect(const OnnxLayer& l, const std::string& what, bool transposed, int cin, int cout, int stride, bool act,
              bool residual) {
  if (l.transposed != transposed || l.cin != cin || l.cout != cout || l.stride != stride || l.slope.empty() == act ||
      l.scale.empty() == residual)
    return refuse(KB2_WEIGHTS_INVALID,
                  "ONNX " + what + ": layer " + std::to_string(l.cin) + " -> " + std::to_string(l.cout) + " does not "
                  "fit the RIFE 4.2x topology");
  return Status::Ok();
}

void put(std::vector<float>& out, const std::vector<float>& v) { out.insert(out.end(), v.begin(), v.end()); }

}  // namespace

Status rife_blob_from_onnx(const uint8_t* const* pieces, const uint64_t* sizes, int blocks, const int32_t* reduce,
                           std::vector<uint8_t>& blob) {
  if (pieces == nullptr || sizes == nullptr || reduce == nullptr) return refuse(KB2_INVALID_ARGUMENT, "null argument");
  if (blocks < 2 || blocks > 5) return refuse(KB2_INVALID_ARGUMENT, "RIFE 4.2x: 2 to 5 blocks");
  for (int k = 0; k < blocks; ++k)
    if (reduce[k] < 1 || reduce[k] > 32 || (reduce[k] & (reduce[k] - 1)) != 0)
      return refuse(KB2_INVALID_ARGUMENT, "RIFE 4.2x: block input reductions are powers of two, 1 to 32");
  std::vector<float> plan(12, 0.0f), params;
  plan[0] = static_cast<float>(blocks);
  plan[11] = 16.0f;
  // the encoder: cnn0 3 -> 16 stride 2, cnn1 and cnn2 16 -> 16, cnn3 transposed 16 -> 4
  std::vector<OnnxLayer> enc;
  KB2_TRY(onnx_piece_layers(pieces[0], sizes[0], enc));
  if (enc.size() != 4) return refuse(KB2_WEIGHTS_INVALID, "ONNX encoder: 4 layers expected");
  KB2_TRY(expect(enc[0], "encoder", false, 3, 16, 2, true, false));
  KB2_TRY(expect(enc[1], "encoder", false, 16, 16, 1, true, false));
  KB2_TRY(expect(enc[2], "encoder", false, 16, 16, 1, true, false));
  KB2_TRY(expect(enc[3], "encoder", true, 16, 4, 2, false, false));
  for (int j = 0; j < 3; ++j) {
    put(params, enc[j].w);
    put(params, enc[j].b);
    put(params, enc[j].slope);
  }
  put(params, enc[3].w);
  put(params, enc[3].b);
  for (int k = 0; k < blocks; ++k) {
    std::vector<OnnxLayer> L;
    const std::string what = "block " + std::to_string(k);
    KB2_TRY(onnx_piece_layers(pieces[1 + k], sizes[1 + k], L));
    if (L.size() != 11) return refuse(KB2_WEIGHTS_INVALID, "ONNX " + what + ": 11 layers expected");
    const int c = L[1].cout, cin = k == 0 ? 15 : 28;
    if (c % 2 != 0) return refuse(KB2_WEIGHTS_INVALID, "ONNX " + what + ": odd width");
    KB2_TRY(expect(L[0], what, false, cin, c / 2, 2, true, false));
    KB2_TRY(expect(L[1], what, false, c / 2, c, 2, true, false));
    for (int j = 2; j < 10; ++j) KB2_TRY(expect(L[j], what, false, c, c, 1, true, true));
    KB2_TRY(expect(L[10], what, true, c, 52, 2, false, false));
    plan[1 + k] = static_cast<float>(reduce[k]);
    plan[6 + k] = static_cast<float>(c);
    for (int j = 0; j < 2; ++j) {
      put(params, L[j].w);
      put(params, L[j].b);
      put(params, L[j].slope);
    }
    for (int j = 2; j < 10; ++j) {
      put(params, L[j].w);
      put(params, L[j].b);
      put(params, L[j].scale);
      put(params, L[j].slope);
    }
    put(params, L[10].w);
    put(params, L[10].b);
  }
  std::vector<float> all = plan;
  put(all, params);
  for (float v : all)
    if (!std::isfinite(v)) return refuse(KB2_WEIGHTS_INVALID, "ONNX: non-finite weight");
  const uint64_t count = all.size();
  blob.assign(kBlobHeader + count * 4, 0);
  uint8_t* p = blob.data();
  std::memcpy(p, "KB2WGT01", 8);
  const uint32_t version = kBlobVersion, model = KB2_MODEL_RIFE_FUSED, zero = 0;
  std::memcpy(p + 8, &version, 4);
  std::memcpy(p + 12, &model, 4);
  std::memcpy(p + 16, &count, 8);
  std::memcpy(p + kBlobHeader, all.data(), count * 4);
  const uint32_t crc = crc32(p + kBlobHeader, count * 4);
  std::memcpy(p + 24, &crc, 4);
  std::memcpy(p + 28, &zero, 4);
  return Status::Ok();
}

}  // namespace kb2
