// Test infrastructure only: the reference's own FP32 CPU path for the frame networks.
//
// This file is compiled together with the reference's IR interpreter sources
// (src/gpu/ir/{graph,interpreter,ops,op_*,shape}.cpp and src/kernels/ref/half.cpp of
// Ta2b/Ultimate-Anime-VideoPlayer, read in place, never copied) into oracle/_ref/libkirari_ref.so by
// oracle/Makefile. It builds the two networks of the frame path as in-code `ir::Graph`s made only of
// the reference's own operators and runs them with `ir::run` (src/gpu/ir/interpreter.h:25):
//
//  * canonical SPAN x2: Conv (src/gpu/ir/op_window.cpp:227), Sigmoid/Mul/Add/Sub
//    (op_elementwise.cpp), Concat, DepthToSpace CRD (op_pixel.cpp:78);
//  * classic IFNet 4.x: Conv stride 2, PRelu, ConvTranspose (op_window.cpp:309), Resize linear
//    half-pixel (op_sample.cpp:139), Slice, GridSample bilinear/border/align-corners
//    (op_sample.cpp:200);
//  * RIFE 4.2x (4.25, 4.26, 4.25 lite, 4.22 lite): the same operators plus DepthToSpace CRD, with the
//    encoder (cnn0..cnn3) and the IFBlocks of 52-channel Y as the reference's fused RIFE describes them
//    (src/kernels/spec/rife_fused.h:1-19, src/kernels/ref/rife_fused.cpp).
//
// Only tests/, the package's smoke check and bench.py's CPU-baseline leg call it, as the checker or
// as the timed reference CPU implementation. The parameter order is the weight blob's, as the
// product's C header defines it (include/kirari_b200.h).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "gpu/ir/graph.h"
#include "gpu/ir/interpreter.h"
#include "gpu/ir/ir.h"
#include "kernels/ref/rife_fused.h"

namespace ir = kirari::gpu::ir;

namespace {

thread_local std::string g_error;

struct Builder {
  ir::Graph g;
  int counter = 0;

  ir::TensorId input(const std::string& name, ir::Dims dims) {
    ir::Tensor t;
    t.name = name;
    t.kind = ir::TensorKind::Input;
    t.type = ir::DataType::F32;
    t.dims = std::move(dims);
    t.known = true;
    const ir::TensorId id = ir::add_tensor(g, std::move(t));
    g.inputs.push_back(id);
    return id;
  }
  ir::TensorId constant(ir::Dims dims, std::vector<float> values) {
    ir::Tensor t;
    t.name = "c" + std::to_string(counter++);
    t.kind = ir::TensorKind::Constant;
    t.type = ir::DataType::F32;
    t.dims = dims;
    t.known = true;
    t.value = ir::Value{.type = ir::DataType::F32, .dims = std::move(dims), .f = std::move(values)};
    return ir::add_tensor(g, std::move(t));
  }
  ir::TensorId constant_i64(ir::Dims dims, std::vector<std::int64_t> values) {
    ir::Tensor t;
    t.name = "c" + std::to_string(counter++);
    t.kind = ir::TensorKind::Constant;
    t.type = ir::DataType::I64;
    t.dims = dims;
    t.known = true;
    t.value = ir::Value{.type = ir::DataType::I64, .dims = std::move(dims), .i = std::move(values)};
    return ir::add_tensor(g, std::move(t));
  }
  ir::TensorId activation() {
    ir::Tensor t;
    t.name = "a" + std::to_string(counter++);
    t.kind = ir::TensorKind::Activation;
    t.type = ir::DataType::F32;
    return ir::add_tensor(g, std::move(t));
  }
  ir::TensorId node(ir::OpKind op, std::vector<ir::TensorId> inputs, ir::Attrs attrs = ir::NoAttrs{}) {
    const ir::TensorId out = activation();
    ir::Node n;
    n.name = "n" + std::to_string(counter++);
    n.op = op;
    n.attrs = std::move(attrs);
    n.inputs = std::move(inputs);
    n.outputs = {out};
    g.nodes.push_back(std::move(n));
    return out;
  }
  ir::TensorId scalar(float v) { return constant({1}, {v}); }
};

// Reads `count` floats from the flat parameter array.
struct Params {
  const float* p;
  long left;
  bool ok = true;
  std::vector<float> take(long count) {
    if (count > left) {
      ok = false;
      return std::vector<float>(static_cast<std::size_t>(count), 0.0F);
    }
    std::vector<float> v(p, p + count);
    p += count;
    left -= count;
    return v;
  }
};

ir::TensorId conv(Builder& b, Params& pr, ir::TensorId x, int cin, int cout, int k, int stride, int pad) {
  ir::ConvAttrs a;
  a.strides = {stride, stride};
  a.pads = {pad, pad, pad, pad};
  const ir::TensorId w = b.constant({cout, cin, k, k}, pr.take(static_cast<long>(cout) * cin * k * k));
  const ir::TensorId bias = b.constant({cout}, pr.take(cout));
  return b.node(ir::OpKind::Conv, {x, w, bias}, a);
}

ir::TensorId prelu(Builder& b, Params& pr, ir::TensorId x, int c) {
  const ir::TensorId slope = b.constant({c, 1, 1}, pr.take(c));
  return b.node(ir::OpKind::PRelu, {x, slope});
}

ir::TensorId silu(Builder& b, ir::TensorId x) {
  return b.node(ir::OpKind::Mul, {x, b.node(ir::OpKind::Sigmoid, {x})});
}

ir::TensorId resize(Builder& b, ir::TensorId x, float scale) {
  ir::ResizeAttrs a;
  a.mode = ir::ResizeMode::Linear;
  a.coord = ir::CoordMode::HalfPixel;
  const ir::TensorId scales = b.constant({4}, {1.0F, 1.0F, scale, scale});
  return b.node(ir::OpKind::Resize, {x, ir::kNoTensor, scales}, a);
}

ir::TensorId slice_channels(Builder& b, ir::TensorId x, std::int64_t lo, std::int64_t hi) {
  return b.node(ir::OpKind::Slice, {x, b.constant_i64({1}, {lo}), b.constant_i64({1}, {hi}),
                                    b.constant_i64({1}, {1})});
}

// warp(img, flow2): GridSample bilinear, border padding, align_corners, on the grid
// mesh + flow * 2 / (size - 1) (the normalised form of "sample at (x + fx, y + fy)").
ir::TensorId warp(Builder& b, ir::TensorId img, ir::TensorId flow2, int n, int h, int w) {
  std::vector<float> mesh(static_cast<std::size_t>(n) * 2 * h * w);
  for (int i = 0; i < n; ++i)
    for (int y = 0; y < h; ++y)
      for (int x = 0; x < w; ++x) {
        const std::size_t base = static_cast<std::size_t>(i) * 2 * h * w;
        mesh[base + static_cast<std::size_t>(y) * w + x] =
            w > 1 ? -1.0F + 2.0F * static_cast<float>(x) / static_cast<float>(w - 1) : 0.0F;
        mesh[base + static_cast<std::size_t>(h) * w + static_cast<std::size_t>(y) * w + x] =
            h > 1 ? -1.0F + 2.0F * static_cast<float>(y) / static_cast<float>(h - 1) : 0.0F;
      }
  const ir::TensorId mesh_t = b.constant({n, 2, h, w}, std::move(mesh));
  const ir::TensorId norm = b.constant({1, 2, 1, 1}, {w > 1 ? 2.0F / static_cast<float>(w - 1) : 0.0F,
                                                      h > 1 ? 2.0F / static_cast<float>(h - 1) : 0.0F});
  const ir::TensorId grid = b.node(ir::OpKind::Add, {mesh_t, b.node(ir::OpKind::Mul, {flow2, norm})});
  ir::GridSampleAttrs a;
  a.mode = ir::GridMode::Bilinear;
  a.padding = ir::GridPadding::Border;
  a.align_corners = true;
  a.grid_nchw = true;
  return b.node(ir::OpKind::GridSample, {img, grid}, a);
}

int finish(Builder& b, ir::TensorId out, const std::vector<ir::NamedValue>& inputs, float* dst,
           std::size_t expected) {
  b.g.outputs.push_back(out);
  auto result = ir::run(b.g, inputs);
  if (!result) {
    g_error = result.error().detail;
    return 2;
  }
  const ir::Value& v = (*result)[0].value;
  if (v.f.size() != expected) {
    g_error = "unexpected output size";
    return 3;
  }
  std::memcpy(dst, v.f.data(), expected * sizeof(float));
  return 0;
}


// The RIFE 4.2x graph and the tensors the checks read.
struct Rife42Graph {
  Builder b;
  int blocks = 0;
  int reduce[5] = {};
  int channels[5] = {};
  ir::TensorId f0 = ir::kNoTensor, f1 = ir::kNoTensor;  // encodings [n,4,h,w]
  ir::TensorId x[5] = {};                               // block inputs X_k [n,15|28,h/d,w/d]
  ir::TensorId y[5] = {};                               // block outputs Y_k [n,52,h/2d,w/2d]
  ir::TensorId image = ir::kNoTensor, flow = ir::kNoTensor, mask = ir::kNoTensor;
};

bool build_rife42(Rife42Graph& r, int n, int h, int w, float timestep, const float* params, long n_params) {
  if (n_params < 12) {
    g_error = "no plan";
    return false;
  }
  r.blocks = static_cast<int>(params[0]);
  if (r.blocks < 2 || r.blocks > 5 || params[11] != 16.0F) {
    g_error = "plan";
    return false;
  }
  for (int k = 0; k < r.blocks; ++k) {
    r.reduce[k] = static_cast<int>(params[1 + k]);
    r.channels[k] = static_cast<int>(params[6 + k]);
  }
  Builder& b = r.b;
  Params pr{params + 12, n_params - 12};
  const ir::TensorId i0 = b.input("img0", {n, 3, h, w});
  const ir::TensorId i1 = b.input("img1", {n, 3, h, w});
  const ir::TensorId tplane =
      b.constant({n, 1, h, w}, std::vector<float>(static_cast<std::size_t>(n) * h * w, timestep));
  ir::AxisAttrs cat_axis;
  cat_axis.axis = 1;
  // the encoder (cnn0..cnn3) of both frames: its weights are read once, applied to each frame
  const long enc_count[4] = {16L * 3 * 9 + 32, 16L * 16 * 9 + 32, 16L * 16 * 9 + 32, 16L * 4 * 16 + 4};
  std::vector<float> enc_params;
  for (long c : enc_count) {
    const std::vector<float> v = pr.take(c);
    enc_params.insert(enc_params.end(), v.begin(), v.end());
  }
  auto encode = [&](ir::TensorId img) {
    Params ep{enc_params.data(), static_cast<long>(enc_params.size())};
    ir::TensorId e = prelu(b, ep, conv(b, ep, img, 3, 16, 3, 2, 1), 16);
    e = prelu(b, ep, conv(b, ep, e, 16, 16, 3, 1, 1), 16);
    e = prelu(b, ep, conv(b, ep, e, 16, 16, 3, 1, 1), 16);
    ir::ConvTransposeAttrs ta;
    ta.strides = {2, 2};
    ta.pads = {1, 1, 1, 1};
    const ir::TensorId tw = b.constant({16, 4, 4, 4}, ep.take(16L * 4 * 16));
    const ir::TensorId tb = b.constant({4}, ep.take(4));
    return b.node(ir::OpKind::ConvTranspose, {e, tw, tb}, ta);
  };
  r.f0 = encode(i0);
  r.f1 = encode(i1);
  ir::TensorId flow = ir::kNoTensor;
  ir::TensorId mask = ir::kNoTensor;
  ir::TensorId feat = ir::kNoTensor;
  ir::TensorId w0 = i0;
  ir::TensorId w1 = i1;
  ir::TensorId wf0 = r.f0;
  ir::TensorId wf1 = r.f1;
  for (int k = 0; k < r.blocks; ++k) {
    const int c = r.channels[k];
    const auto d = static_cast<float>(r.reduce[k]);
    // X_k: 0-2 A, 3-5 B, 6-9 encoding of A, 10-13 of B, 14 timestep (k = 0: unwarped, 15 channels);
    // k >= 1 warped, then 15 mask, 16-23 attributes of block k-1, 24-27 flow / d
    ir::TensorId xin = k == 0 ? b.node(ir::OpKind::Concat, {i0, i1, r.f0, r.f1, tplane}, cat_axis)
                              : b.node(ir::OpKind::Concat, {w0, w1, wf0, wf1, tplane, mask, feat}, cat_axis);
    const int in_ch = k == 0 ? 15 : 28;
    if (d != 1.0F) xin = resize(b, xin, 1.0F / d);
    if (k > 0) {
      ir::TensorId f = flow;
      if (d != 1.0F) f = resize(b, f, 1.0F / d);
      f = b.node(ir::OpKind::Mul, {f, b.scalar(1.0F / d)});
      xin = b.node(ir::OpKind::Concat, {xin, f}, cat_axis);
    }
    r.x[k] = xin;
    ir::TensorId hdn = prelu(b, pr, conv(b, pr, xin, in_ch, c / 2, 3, 2, 1), c / 2);
    hdn = prelu(b, pr, conv(b, pr, hdn, c / 2, c, 3, 2, 1), c);
    for (int j = 0; j < 8; ++j) {  // ResConv: act(conv(x) * beta + x)
      const ir::TensorId rc = conv(b, pr, hdn, c, c, 3, 1, 1);
      const ir::TensorId beta = b.constant({1, c, 1, 1}, pr.take(c));
      hdn = prelu(b, pr, b.node(ir::OpKind::Add, {b.node(ir::OpKind::Mul, {rc, beta}), hdn}), c);
    }
    ir::ConvTransposeAttrs ta;
    ta.strides = {2, 2};
    ta.pads = {1, 1, 1, 1};
    const ir::TensorId tw = b.constant({c, 52, 4, 4}, pr.take(static_cast<long>(c) * 52 * 16));
    const ir::TensorId tb = b.constant({52}, pr.take(52));
    r.y[k] = b.node(ir::OpKind::ConvTranspose, {hdn, tw, tb}, ta);
    ir::BlockAttrs d2s;
    d2s.blocksize = 2;
    d2s.mode = ir::BlockMode::Crd;
    ir::TensorId tmp = b.node(ir::OpKind::DepthToSpace, {r.y[k]}, d2s);
    if (d != 1.0F) tmp = resize(b, tmp, d);
    const ir::TensorId fd = b.node(ir::OpKind::Mul, {slice_channels(b, tmp, 0, 4), b.scalar(d)});
    mask = slice_channels(b, tmp, 4, 5);
    feat = slice_channels(b, tmp, 5, 13);
    flow = k == 0 ? fd : b.node(ir::OpKind::Add, {flow, fd});
    const ir::TensorId fa = slice_channels(b, flow, 0, 2);
    const ir::TensorId fb = slice_channels(b, flow, 2, 4);
    w0 = warp(b, i0, fa, n, h, w);
    w1 = warp(b, i1, fb, n, h, w);
    if (k + 1 < r.blocks) {
      wf0 = warp(b, r.f0, fa, n, h, w);
      wf1 = warp(b, r.f1, fb, n, h, w);
    }
  }
  r.mask = b.node(ir::OpKind::Sigmoid, {mask});
  const ir::TensorId one_minus = b.node(ir::OpKind::Sub, {b.scalar(1.0F), r.mask});
  r.image = b.node(ir::OpKind::Add, {b.node(ir::OpKind::Mul, {w0, r.mask}),
                                     b.node(ir::OpKind::Mul, {w1, one_minus})});
  r.flow = flow;
  if (!pr.ok || pr.left != 0) {
    g_error = "parameter count mismatch";
    return false;
  }
  return true;
}

std::vector<ir::NamedValue> rife42_inputs(const float* img0, const float* img1, int n, int h, int w) {
  const std::size_t count = static_cast<std::size_t>(n) * 3 * h * w;
  std::vector<ir::NamedValue> inputs;
  inputs.push_back(
      {"img0", ir::Value{.type = ir::DataType::F32, .dims = {n, 3, h, w}, .f = {img0, img0 + count}}});
  inputs.push_back(
      {"img1", ir::Value{.type = ir::DataType::F32, .dims = {n, 3, h, w}, .f = {img1, img1 + count}}});
  return inputs;
}

}  // namespace

extern "C" {

const char* kref_last_error(void) { return g_error.c_str(); }

// Canonical SPAN x2 (48 channels, 6 SPAB blocks): x [n,3,h,w] -> out [n,3,2h,2w].
// When act_scales is not null, every block convolution reads its input rounded to E4M3 at the
// given per-tensor scale (the reference's FakeQuantE4M3 conv input, ir.h ConvAttrs::in_quant):
// act_scales[0] for block inputs of block 0 ... following the order [1+3b] c2 input, [2+3b] c3 input,
// [3b] c1 input, as the reference's .span8 scale table (src/gpu/span_fp8/package.h:17-19).
int kref_span_forward(const float* x, int n, int h, int w, const float* params, long n_params,
                      const float* act_scales, float* out) {
  try {
    Builder b;
    Params pr{params, n_params};
    const ir::TensorId in = b.input("x", {n, 3, h, w});
    const int c = 48;
    auto qconv = [&](ir::TensorId v, int scale_index) {
      ir::ConvAttrs a;
      a.pads = {1, 1, 1, 1};
      if (act_scales != nullptr) a.in_quant = act_scales[scale_index];
      const ir::TensorId wt = b.constant({c, c, 3, 3}, pr.take(static_cast<long>(c) * c * 9));
      const ir::TensorId bias = b.constant({c}, pr.take(c));
      return b.node(ir::OpKind::Conv, {v, wt, bias}, a);
    };
    const ir::TensorId s0 = conv(b, pr, in, 3, c, 3, 1, 1);
    ir::TensorId xb = s0;
    ir::TensorId first_block = ir::kNoTensor;
    ir::TensorId last_act = ir::kNoTensor;
    const ir::TensorId half = b.scalar(0.5F);
    for (int blk = 0; blk < 6; ++blk) {
      const ir::TensorId a1 = silu(b, qconv(xb, 3 * blk));
      const ir::TensorId a2 = silu(b, qconv(a1, 3 * blk + 1));
      const ir::TensorId c3 = qconv(a2, 3 * blk + 2);
      const ir::TensorId att = b.node(ir::OpKind::Sub, {b.node(ir::OpKind::Sigmoid, {c3}), half});
      xb = b.node(ir::OpKind::Mul, {b.node(ir::OpKind::Add, {c3, xb}), att});
      if (blk == 0) first_block = xb;
      if (blk == 5) last_act = a1;
    }
    ir::AxisAttrs cat_axis;
    cat_axis.axis = 1;
    const ir::TensorId cat = b.node(ir::OpKind::Concat, {s0, xb, first_block, last_act}, cat_axis);
    const ir::TensorId fused = conv(b, pr, cat, 4 * c, c, 1, 1, 0);
    const ir::TensorId up = conv(b, pr, fused, c, 12, 3, 1, 1);
    ir::BlockAttrs d2s;
    d2s.blocksize = 2;
    d2s.mode = ir::BlockMode::Crd;
    const ir::TensorId y = b.node(ir::OpKind::DepthToSpace, {up}, d2s);
    if (!pr.ok || pr.left != 0) {
      g_error = "parameter count mismatch";
      return 1;
    }
    std::vector<ir::NamedValue> inputs;
    const std::size_t count = static_cast<std::size_t>(n) * 3 * h * w;
    inputs.push_back({"x", ir::Value{.type = ir::DataType::F32, .dims = {n, 3, h, w}, .f = {x, x + count}}});
    return finish(b, y, inputs, out, count * 4);
  } catch (const std::exception& e) {
    g_error = e.what();
    return 4;
  }
}

// Classic IFNet 4.x: 4 IFBlocks at scales 8/4/2/1 with 192/128/96/64 channels.
// img0, img1 [n,3,h,w] (h, w multiples of 32) -> out [n,3,h,w].
int kref_ifnet_forward(const float* img0, const float* img1, int n, int h, int w, float timestep,
                       const float* params, long n_params, float* out) {
  try {
    Builder b;
    Params pr{params, n_params};
    const ir::TensorId i0 = b.input("img0", {n, 3, h, w});
    const ir::TensorId i1 = b.input("img1", {n, 3, h, w});
    const ir::TensorId tplane =
        b.constant({n, 1, h, w}, std::vector<float>(static_cast<std::size_t>(n) * h * w, timestep));
    ir::AxisAttrs cat_axis;
    cat_axis.axis = 1;
    const int channels[4] = {192, 128, 96, 64};
    const float scales[4] = {8.0F, 4.0F, 2.0F, 1.0F};
    ir::TensorId flow = ir::kNoTensor;
    ir::TensorId mask = ir::kNoTensor;
    ir::TensorId w0 = i0;
    ir::TensorId w1 = i1;
    for (int k = 0; k < 4; ++k) {
      const int c = channels[k];
      const float s = scales[k];
      ir::TensorId xin = k == 0 ? b.node(ir::OpKind::Concat, {i0, i1, tplane}, cat_axis)
                                : b.node(ir::OpKind::Concat, {w0, w1, tplane, mask}, cat_axis);
      const int in_ch = k == 0 ? 7 : 12;
      if (s != 1.0F) xin = resize(b, xin, 1.0F / s);
      if (k > 0) {
        ir::TensorId f = flow;
        if (s != 1.0F) f = resize(b, f, 1.0F / s);
        f = b.node(ir::OpKind::Mul, {f, b.scalar(1.0F / s)});
        xin = b.node(ir::OpKind::Concat, {xin, f}, cat_axis);
      }
      ir::TensorId hdn = prelu(b, pr, conv(b, pr, xin, in_ch, c / 2, 3, 2, 1), c / 2);
      hdn = prelu(b, pr, conv(b, pr, hdn, c / 2, c, 3, 2, 1), c);
      for (int j = 0; j < 8; ++j) {
        const ir::TensorId r = conv(b, pr, hdn, c, c, 3, 1, 1);
        hdn = prelu(b, pr, b.node(ir::OpKind::Add, {r, hdn}), c);
      }
      ir::ConvTransposeAttrs ta;
      ta.strides = {2, 2};
      ta.pads = {1, 1, 1, 1};
      const ir::TensorId tw = b.constant({c, 5, 4, 4}, pr.take(static_cast<long>(c) * 5 * 16));
      const ir::TensorId tb = b.constant({5}, pr.take(5));
      ir::TensorId tmp = b.node(ir::OpKind::ConvTranspose, {hdn, tw, tb}, ta);
      tmp = resize(b, tmp, s * 2.0F);
      const ir::TensorId fd = b.node(ir::OpKind::Mul, {slice_channels(b, tmp, 0, 4), b.scalar(s * 2.0F)});
      const ir::TensorId md = slice_channels(b, tmp, 4, 5);
      if (k == 0) {
        flow = fd;
        mask = md;
      } else {
        flow = b.node(ir::OpKind::Add, {flow, fd});
        mask = b.node(ir::OpKind::Add, {mask, md});
      }
      w0 = warp(b, i0, slice_channels(b, flow, 0, 2), n, h, w);
      w1 = warp(b, i1, slice_channels(b, flow, 2, 4), n, h, w);
    }
    const ir::TensorId m = b.node(ir::OpKind::Sigmoid, {mask});
    const ir::TensorId one_minus = b.node(ir::OpKind::Sub, {b.scalar(1.0F), m});
    const ir::TensorId y = b.node(ir::OpKind::Add, {b.node(ir::OpKind::Mul, {w0, m}),
                                                    b.node(ir::OpKind::Mul, {w1, one_minus})});
    if (!pr.ok || pr.left != 0) {
      g_error = "parameter count mismatch";
      return 1;
    }
    const std::size_t count = static_cast<std::size_t>(n) * 3 * h * w;
    std::vector<ir::NamedValue> inputs;
    inputs.push_back(
        {"img0", ir::Value{.type = ir::DataType::F32, .dims = {n, 3, h, w}, .f = {img0, img0 + count}}});
    inputs.push_back(
        {"img1", ir::Value{.type = ir::DataType::F32, .dims = {n, 3, h, w}, .f = {img1, img1 + count}}});
    return finish(b, y, inputs, out, count);
  } catch (const std::exception& e) {
    g_error = e.what();
    return 4;
  }
}

// RIFE 4.2x: the plan (blocks, input reduction d_k and width C_k of each block) is the parameter
// array's first 12 floats [blocks, d_0..d_4, C_0..C_4, 16], then the encoder and the blocks in the
// order of include/kirari_b200.h (KB2_MODEL_RIFE_FUSED). img0, img1 [n,3,h,w] with h and w multiples
// of 4 * max d -> out [n,3,h,w]; flow_out [n,4,h,w] and mask_out [n,1,h,w] (after the sigmoid) when
// not null.
int kref_rife42_forward(const float* img0, const float* img1, int n, int h, int w, float timestep,
                        const float* params, long n_params, float* out, float* flow_out, float* mask_out) {
  try {
    Rife42Graph r;
    if (!build_rife42(r, n, h, w, timestep, params, n_params)) return 1;
    r.b.g.outputs = {r.image, r.flow, r.mask};
    auto result = ir::run(r.b.g, rife42_inputs(img0, img1, n, h, w));
    if (!result) {
      g_error = result.error().detail;
      return 2;
    }
    const std::size_t plane = static_cast<std::size_t>(n) * h * w;
    const std::size_t sizes[3] = {3 * plane, 4 * plane, plane};
    float* dst[3] = {out, flow_out, mask_out};
    for (int i = 0; i < 3; ++i) {
      const ir::Value& v = (*result)[static_cast<std::size_t>(i)].value;
      if (v.f.size() != sizes[i]) {
        g_error = "unexpected output size";
        return 3;
      }
      if (dst[i] != nullptr) std::memcpy(dst[i], v.f.data(), sizes[i] * sizeof(float));
    }
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 4;
  }
}

// Pins the graph above against the reference's own double-precision statement of the fused RIFE
// glue (src/kernels/ref/rife_fused.cpp: rife_fused_block_input, rife_fused_finish): one frame pair
// runs through the graph, its encodings and Y_k are handed to the reference's glue, and
// err[k] (k < blocks) = max |X_k graph - X_k reference|, err[blocks .. blocks + 2] = the same for the
// final image, flow and mask.
int kref_rife42_glue_check(const float* img0, const float* img1, int h, int w, float timestep, const float* params,
                           long n_params, double* err) {
  try {
    Rife42Graph r;
    if (!build_rife42(r, 1, h, w, timestep, params, n_params)) return 1;
    const int blocks = r.blocks;
    r.b.g.outputs = {r.f0, r.f1, r.image, r.flow, r.mask};
    for (int k = 0; k < blocks; ++k) r.b.g.outputs.push_back(r.y[k]);
    for (int k = 0; k < blocks; ++k) r.b.g.outputs.push_back(r.x[k]);
    auto result = ir::run(r.b.g, rife42_inputs(img0, img1, 1, h, w));
    if (!result) {
      g_error = result.error().detail;
      return 2;
    }
    auto value = [&](std::size_t i) -> const std::vector<float>& { return (*result)[i].value.f; };
    namespace kr = kirari::kernels::ref;
    kr::RifeFusedState st;
    st.plan.blocks = blocks;
    for (int k = 0; k < blocks; ++k) st.plan.reduce[static_cast<std::size_t>(k)] = r.reduce[k];
    st.height = h;
    st.width = w;
    const std::size_t area = static_cast<std::size_t>(h) * w;
    st.input.assign(11 * area, 0.0);
    for (std::size_t i = 0; i < 3 * area; ++i) {
      st.input[i] = img0[i];
      st.input[3 * area + i] = img1[i];
    }
    for (std::size_t i = 0; i < area; ++i) st.input[6 * area + i] = timestep;
    st.encode.assign(value(0).begin(), value(0).end());
    st.encode.insert(st.encode.end(), value(1).begin(), value(1).end());
    for (int k = 0; k < blocks; ++k)
      st.y.emplace_back(value(5 + static_cast<std::size_t>(k)).begin(), value(5 + static_cast<std::size_t>(k)).end());
    auto max_diff = [](const std::vector<double>& a, const std::vector<float>& b) {
      if (a.size() != b.size()) return 1e30;
      double m = 0.0;
      for (std::size_t i = 0; i < a.size(); ++i) m = std::max(m, std::fabs(a[i] - static_cast<double>(b[i])));
      return m;
    };
    for (int k = 0; k < blocks; ++k)
      err[k] = max_diff(kr::rife_fused_block_input(st, k), value(5 + static_cast<std::size_t>(blocks + k)));
    const kr::RifeFusedResult fin = kr::rife_fused_finish(st);
    err[blocks] = max_diff(fin.image, value(2));
    err[blocks + 1] = max_diff(fin.flow, value(3));
    err[blocks + 2] = max_diff(fin.mask, value(4));
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 4;
  }
}

}  // extern "C"
