// RIFE 4.2x on B200: the encoder (cnn0..cnn3) of both frames on the tensor cores (the two frames
// of every pair as one batch), then per block a glue kernel that builds X_k from the frames, the
// encodings and the Z of the blocks before it (rife_glue.cuh), two stride-2 convs, eight ResConv
// and the transposed conv to Y_k with DepthToSpace(2) folded into its store (Z_k), all on the
// tensor-core interpolator convs (ifnet_conv.cuh, if_layer.h); a last kernel warps both frames by
// the final flow and blends them, or writes the flow and mask (the motion variant). This is the
// reference's fused RIFE chain (RifeFusedEngine::enqueue, src/gpu/cuda/backend/
// rife_fused_engine.cpp:390: entry -> encoder -> (glue -> block) x k -> finish) with its native
// block kernels (src/prepare/rife_native.h: Conv 3x3 stride 1 or 2 + LeakyReLU / PReLU, ResConv with
// a per-channel beta, ConvTranspose 4x4 stride 2).
//
// The ResConv's beta is folded into its conv: act(beta (W x + b) + x) = act((beta W) x + beta b + x),
// exact in real arithmetic; the product is rounded to FP16 with the weights.
//
// Frames of any size are placed in a zero padded plane of multiples of max(64, 4 max d) at the
// window of rife_window (src/kernels/spec/rife.h:47-57: left / top = half the padding, rounded down
// to even), and the output is read back from that window.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>

#include "if_layer.h"
#include "rife_glue.cuh"
#include "rife_net.h"

namespace kb2 {

namespace {

constexpr int kRifeRes = 8;
constexpr int kRifeEnc = 16;
constexpr int kRifeY = 52;
constexpr size_t kRifePlanFloats = 12;

// The motion kernel of a plan whose last block is `last`.
template <typename T, class Finish>
Status launch_motion(dim3 g, cudaStream_t stream, const IfFrames& F, const RifeZ& Z, int last, int batch,
                     const Finish& f) {
  T* flow = static_cast<T*>(f.flow);
  T* mask = static_cast<T*>(f.mask);
  switch (last) {
    case 1: rife_motion_kernel<1, T><<<g, kGlueThreads, 0, stream>>>(F, Z, batch, flow, mask); break;
    case 2: rife_motion_kernel<2, T><<<g, kGlueThreads, 0, stream>>>(F, Z, batch, flow, mask); break;
    case 3: rife_motion_kernel<3, T><<<g, kGlueThreads, 0, stream>>>(F, Z, batch, flow, mask); break;
    default: rife_motion_kernel<4, T><<<g, kGlueThreads, 0, stream>>>(F, Z, batch, flow, mask); break;
  }
  return cuda_status(cudaGetLastError(), "RIFE motion launch");
}

bool block_width_ok(int c) { return c == 32 || c == 64 || c == 96 || c == 128 || c == 192; }

// A float that holds exactly the integer v.
bool int_float(float f, int* v) {
  if (!(f >= 0.0f && f <= 4096.0f) || std::floor(f) != f) return false;
  *v = static_cast<int>(f);
  return true;
}

}  // namespace

size_t rife_param_count(const RifePlan& plan) {
  const size_t e = kRifeEnc;
  size_t n = e * 3 * 9 + 2 * e + 2 * (e * e * 9 + 2 * e) + e * 4 * 16 + 4;
  for (int k = 0; k < plan.blocks; ++k) {
    const size_t c = static_cast<size_t>(plan.channels[k]);
    const size_t cin = k == 0 ? 15 : 28;
    n += (c / 2) * cin * 9 + c;                   // conv0a: W, b, slopes
    n += c * (c / 2) * 9 + 2 * c;                 // conv0b
    n += kRifeRes * (c * c * 9 + 3 * c);          // ResConv: W, b, beta, slopes
    n += c * kRifeY * 16 + kRifeY;                // transposed conv: W [c][52][4][4], b
  }
  return n;
}

Status rife_read_plan(const std::vector<float>& params, RifePlan& plan) {
  if (params.size() < kRifePlanFloats) return refuse(KB2_WEIGHTS_INVALID, "RIFE 4.2x: no plan");
  int blocks = 0, enc = 0;
  if (!int_float(params[0], &blocks) || blocks < 2 || blocks > kRifeMaxBlocks)
    return refuse(KB2_WEIGHTS_INVALID, "RIFE 4.2x plan: 2 to 5 blocks");
  if (!int_float(params[11], &enc) || enc != kRifeEnc)
    return refuse(KB2_WEIGHTS_INVALID, "RIFE 4.2x plan: encoder width 16");
  plan = RifePlan{};
  plan.blocks = blocks;
  for (int k = 0; k < kRifeMaxBlocks; ++k) {
    int d = 0, c = 0;
    if (!int_float(params[1 + k], &d) || !int_float(params[6 + k], &c))
      return refuse(KB2_WEIGHTS_INVALID, "RIFE 4.2x plan: non-integer field");
    if (k >= blocks) {
      if (d != 0 || c != 0) return refuse(KB2_WEIGHTS_INVALID, "RIFE 4.2x plan: fields past the last block");
      continue;
    }
    // the reference's rife_fused_plan_valid (src/kernels/spec/rife_fused.h:50-58)
    if (d < 1 || d > 32 || (d & (d - 1)) != 0) return refuse(KB2_WEIGHTS_INVALID, "RIFE 4.2x plan: reduction");
    if (!block_width_ok(c)) return refuse(KB2_FORMAT_UNSUPPORTED, "RIFE 4.2x plan: block width");
    plan.reduce[k] = d;
    plan.channels[k] = c;
  }
  if (plan.reduce[0] < 2 || plan.reduce[blocks - 1] != 1)
    return refuse(KB2_WEIGHTS_INVALID, "RIFE 4.2x plan: the first reduction >= 2, the last 1");
  if (params.size() != kRifePlanFloats + rife_param_count(plan))
    return refuse(KB2_WEIGHTS_INVALID, "RIFE 4.2x: parameter count mismatch");
  return Status::Ok();
}

RifeNet::RifeNet() = default;
RifeNet::~RifeNet() = default;

Status RifeNet::buffer(DeviceBuffer& b, size_t bytes) {
  KB2_TRY(b.alloc(bytes));
  return cuda_status(cudaMemset(b.ptr, 0, bytes), "cudaMemset");
}

Status RifeNet::create(const std::vector<float>& params, int max_batch, int H, int W) {
  KB2_TRY(rife_read_plan(params, plan_));
  max_batch_ = max_batch;
  H_ = H;
  W_ = W;
  int dmax = 1;
  for (int k = 0; k < plan_.blocks; ++k) dmax = std::max(dmax, plan_.reduce[k]);
  const int align = std::max(64, 4 * dmax);
  Hp_ = (H + align - 1) / align * align;
  Wp_ = (W + align - 1) / align * align;
  top_ = ((Hp_ - H) / 2) & ~1;
  left_ = ((Wp_ - W) / 2) & ~1;
  KB2_TRY(err_.alloc(sizeof(int)));
  KB2_CUDA(cudaMemset(err_.ptr, 0, sizeof(int)));
  int* err = err_.as<int>();
  k_pad_ = timer_.kind("rife.pad");
  const int k_enc0 = timer_.kind("rife.enc.cnn0"), k_enc12 = timer_.kind("rife.enc.cnn12"),
            k_enc3 = timer_.kind("rife.enc.cnn3");
  for (int k = 0; k < plan_.blocks; ++k) k_glue_[k] = timer_.kind(("rife.glue.b" + std::to_string(k)).c_str());
  k_c0a_ = timer_.kind("rife.conv0a");
  k_c0b_ = timer_.kind("rife.conv0b");
  k_res_ = timer_.kind("rife.res");
  k_ct_ = timer_.kind("rife.convt");
  k_finish_ = timer_.kind("rife.finish");
  k_motion_ = timer_.kind("rife.motion");

  const size_t mb = static_cast<size_t>(max_batch_);
  const size_t plane = static_cast<size_t>(Hp_) * Wp_;
  auto take = [&](size_t bytes, uint8_t** ptr) -> Status {
    buffers_.push_back(std::make_unique<DeviceBuffer>());
    KB2_TRY(buffer(*buffers_.back(), bytes));
    *ptr = buffers_.back()->as<uint8_t>();
    return Status::Ok();
  };
  KB2_TRY(pad_.alloc(2 * mb * plane * sizeof(uint2)));
  KB2_TRY(take(2 * mb * plane * 16, &enc_in_));
  KB2_TRY(take(2 * mb * plane * 8, &enc_));
  uint8_t *e1 = nullptr, *e2 = nullptr;
  const int eh = Hp_ / 2, ew = Wp_ / 2;
  KB2_TRY(take(2 * mb * eh * ew * 2 * 16, &e1));
  KB2_TRY(take(2 * mb * eh * ew * 2 * 16, &e2));

  // the encoder, over the 2 x max_batch frames of the pairs
  const float* p = params.data() + kRifePlanFloats;
  const int nb = 2 * max_batch_;
  auto next = [&p](size_t count) {
    const float* q = p;
    p += count;
    return q;
  };
  {
    const float* w0 = next(kRifeEnc * 3 * 9);
    const float* b0 = next(kRifeEnc);
    const float* s0 = next(kRifeEnc);
    auto l0 = std::make_unique<IfLayer>();
    // cnn0 reads one stored chunk (3 channels); the tensor map fills the second with zeros
    KB2_TRY(l0->build(16, 2, kIfPrelu, dense_conv_weights(w0, 16, 3, 16), 16, 3, b0, s0, enc_in_, nb, Hp_, Wp_, 1,
                      eh, ew, e1, 2, nullptr, err, 2));
    enc_layers_.push_back(std::move(l0));
    uint8_t* src = e1;
    uint8_t* dst = e2;
    for (int j = 1; j <= 2; ++j) {
      const float* w = next(kRifeEnc * kRifeEnc * 9);
      const float* b = next(kRifeEnc);
      const float* s = next(kRifeEnc);
      auto l = std::make_unique<IfLayer>();
      KB2_TRY(l->build(16, 1, kIfPrelu, dense_conv_weights(w, 16, 16, 16), 16, 16, b, s, src, nb, eh, ew, 2, eh, ew,
                       dst, 2, nullptr, err));
      enc_layers_.push_back(std::move(l));
      std::swap(src, dst);
    }
    const float* wt = next(kRifeEnc * 4 * 16);
    const float* bt = next(4);
    float bias_t[32] = {};
    for (int n = 0; n < 32; ++n) bias_t[n] = n % 8 < 4 ? bt[n % 8] : 0.0f;
    const std::vector<float> wc = convt_phase_weights(wt, kRifeEnc, 4, 32, [](int n, int* ph, int* co) {
      *ph = n / 8;
      *co = n % 8 < 4 ? n % 8 : -1;
    });
    auto l3 = std::make_unique<IfLayer>();
    KB2_TRY(l3->build(32, 1, kIfConvTEnc, wc, 32, kRifeEnc, bias_t, nullptr, src, nb, eh, ew, 2, eh, ew, enc_, 0,
                      nullptr, err));
    enc_layers_.push_back(std::move(l3));
  }

  for (int k = 0; k < plan_.blocks; ++k) {
    const int d = plan_.reduce[k], c = plan_.channels[k];
    const int cin = k == 0 ? 15 : 28, cx = k == 0 ? 2 : 4;
    const int h0 = Hp_ / d, w0 = Wp_ / d;  // X_k and Z_k
    const int h1 = h0 / 2, w1 = w0 / 2;    // after conv0a
    const int h2 = h1 / 2, w2 = w1 / 2;    // residual level (the transposed conv's input)
    uint8_t *a0 = nullptr, *r0 = nullptr, *r1 = nullptr;
    KB2_TRY(take(mb * h0 * w0 * cx * 16, &x_[k]));
    KB2_TRY(take(mb * h1 * w1 * (c / 16) * 16, &a0));
    KB2_TRY(take(mb * h2 * w2 * (c / 8) * 16, &r0));
    KB2_TRY(take(mb * h2 * w2 * (c / 8) * 16, &r1));
    KB2_TRY(take(mb * h0 * w0 * kRifeZBytes, &z_[k]));
    std::vector<std::unique_ptr<IfLayer>>& L = layers_[k];

    const float* wa = next(static_cast<size_t>(c / 2) * cin * 9);
    const float* ba = next(c / 2);
    const float* sa = next(c / 2);
    auto la = std::make_unique<IfLayer>();
    KB2_TRY(la->build(c / 2, 2, kIfPrelu, dense_conv_weights(wa, c / 2, cin, c / 2), c / 2, cin, ba, sa, x_[k],
                      max_batch_, h0, w0, cx, h1, w1, a0, c / 16, nullptr, err));
    la->args.out_split = 1;  // conv0b reads a0 with stride 2
    la->kind = k_c0a_;
    L.push_back(std::move(la));

    const float* wb = next(static_cast<size_t>(c) * (c / 2) * 9);
    const float* bb = next(c);
    const float* sb = next(c);
    auto lb = std::make_unique<IfLayer>();
    KB2_TRY(lb->build(c, 2, kIfPrelu, dense_conv_weights(wb, c, c / 2, c), c, c / 2, bb, sb, a0, max_batch_, h1, w1,
                      c / 16, h2, w2, r0, c / 8, nullptr, err));
    lb->kind = k_c0b_;
    L.push_back(std::move(lb));

    for (int j = 0; j < kRifeRes; ++j) {
      const float* wr = next(static_cast<size_t>(c) * c * 9);
      const float* br = next(c);
      const float* beta = next(c);
      const float* sr = next(c);
      const std::vector<float> wd = dense_conv_weights(wr, c, c, c, beta);
      std::vector<float> bd(c);
      for (int n = 0; n < c; ++n) bd[n] = br[n] * beta[n];
      uint8_t* src = j % 2 == 0 ? r0 : r1;
      uint8_t* dst = j % 2 == 0 ? r1 : r0;
      auto lr = std::make_unique<IfLayer>();
      if (c == 64)
        KB2_TRY(lr->build_paired(c, wd.data(), bd.data(), sr, src, max_batch_, h2, w2, dst, err));
      else
        KB2_TRY(lr->build(c, 1, kIfResPrelu, wd, c, c, bd.data(), sr, src, max_batch_, h2, w2, c / 8, h2, w2, dst,
                          c / 8, nullptr, err));
      lr->kind = k_res_;
      L.push_back(std::move(lr));
    }

    // the transposed conv to Y (52 channels) with DepthToSpace(2) folded into the store: column
    // n = 64 phase + 16 parity + c carries Y channel 4 c + parity (c < 13), Z channel c
    const float* wt = next(static_cast<size_t>(c) * kRifeY * 16);
    const float* bt = next(kRifeY);
    auto column = [](int n, int* ph, int* co) {
      *ph = n / 64;
      const int parity = (n % 64) / 16, ch = n % 16;
      *co = ch < 13 ? 4 * ch + parity : -1;
    };
    std::vector<float> bias_t(256, 0.0f);
    for (int n = 0; n < 256; ++n) {
      int ph = 0, co = -1;
      column(n, &ph, &co);
      if (co >= 0) bias_t[n] = bt[co];
    }
    auto lt = std::make_unique<IfLayer>();
    KB2_TRY(lt->build(256, 1, kIfConvTZ, convt_phase_weights(wt, c, kRifeY, 256, column), 256, c, bias_t.data(),
                      nullptr, r0, max_batch_, h2, w2, c / 8, h2, w2, z_[k], 0, nullptr, err, 4));
    lt->kind = k_ct_;
    L.push_back(std::move(lt));
  }
  for (size_t i = 0; i < enc_layers_.size(); ++i)
    enc_layers_[i]->kind = i == 0 ? k_enc0 : i + 1 == enc_layers_.size() ? k_enc3 : k_enc12;
  if (static_cast<size_t>(p - params.data()) != params.size())
    return refuse(KB2_WEIGHTS_INVALID, "RIFE 4.2x: parameter layout mismatch");
  return Status::Ok();
}

Status RifeNet::set_timestep(float t) {
  if (!(t > 0.0f && t < 1.0f)) return refuse(KB2_INVALID_ARGUMENT, "RIFE: timestep must be in (0, 1)");
  timestep_ = t;
  return Status::Ok();
}

int RifeNet::launches_per_run() const {
  int n = 1 + static_cast<int>(enc_layers_.size()) + 1;
  for (int k = 0; k < plan_.blocks; ++k) n += 1 + static_cast<int>(layers_[k].size());
  return n;
}

size_t RifeNet::device_bytes() const {
  size_t total = err_.bytes + pad_.bytes;
  for (const auto& b : buffers_) total += b->bytes;
  auto layer_bytes = [](const IfLayer& l) {
    return l.wpack.bytes + l.bias.bytes + l.slope.bytes + l.pair.wpack.bytes + l.pair.bias.bytes +
           l.pair.slope.bytes + l.pair.scale.bytes;
  };
  for (const auto& l : enc_layers_) total += layer_bytes(*l);
  for (int k = 0; k < plan_.blocks; ++k)
    for (const auto& l : layers_[k]) total += layer_bytes(*l);
  return total;
}

Status RifeNet::run(cudaStream_t stream, const void* img0, const void* img1, void* out, int batch) {
  return run_impl(stream, img0, img1, Finish{out, nullptr, nullptr, false}, batch);
}

Status RifeNet::run_motion(cudaStream_t stream, const void* img0, const void* img1, void* flow, void* mask, bool f16,
                           int batch) {
  return run_impl(stream, img0, img1, Finish{nullptr, flow, mask, f16}, batch);
}

Status RifeNet::run_impl(cudaStream_t stream, const void* img0, const void* img1, const Finish& finish, int batch) {
  if (batch < 1 || batch > max_batch_) return refuse(KB2_SHAPE_INVALID, "RIFE: batch out of contract");
  uint2* pad0 = pad_.as<uint2>();
  const IfFrames F{static_cast<const __half*>(img0), static_cast<const __half*>(img1), H_, W_, Hp_, Wp_, top_, left_,
                   pad0, pad0 + static_cast<size_t>(max_batch_) * Hp_ * Wp_};
  const RifeEnc E{reinterpret_cast<const uint2*>(enc_)};
  RifeZ Z{};
  for (int k = 0; k < plan_.blocks; ++k) {
    const int d = plan_.reduce[k];
    Z.z[k] = z_[k];
    Z.h[k] = Hp_ / d;
    Z.w[k] = Wp_ / d;
    Z.d[k] = static_cast<float>(d);
    Z.inv[k] = 1.0f / static_cast<float>(d);
  }
  const int sms = num_sms();
  auto row_grid = [sms](int width, int rows) {
    const int bx = (width + kGlueThreads - 1) / kGlueThreads;
    const int by = std::max(1, std::min({rows, kGlueMaxRowBlocks, (16 * sms + bx - 1) / bx}));
    return dim3(static_cast<unsigned>(bx), static_cast<unsigned>(by));
  };
  auto timed = [&](IfLayer& l, int n) -> Status {
    const double opx = static_cast<double>(n) * l.args.h_out * l.args.w_out;
    KB2_TRY(timer_.begin(stream));
    KB2_TRY(l.launch(stream, n));
    return timer_.end(l.kind, l.flops_px * opx, l.bytes_px * opx, stream);
  };
  const double full_px = static_cast<double>(batch) * Hp_ * Wp_;
  KB2_TRY(timer_.begin(stream));
  rife_pad_frames_kernel<<<row_grid(Wp_, batch * Hp_), kGlueThreads, 0, stream>>>(F, batch, enc_in_);
  KB2_CUDA(cudaGetLastError());
  KB2_TRY(timer_.end(k_pad_, 0.0, full_px * (12.0 + 2 * 8.0 + 2 * 16.0), stream));
  for (auto& l : enc_layers_) KB2_TRY(timed(*l, 2 * batch));
  auto runs = [](int rows) { return (rows + kRifeRunRows - 1) / kRifeRunRows; };
  for (int k = 0; k < plan_.blocks; ++k) {
    const int d = plan_.reduce[k];
    const int ho = Hp_ / d, wo = Wp_ / d;
    const dim3 g = row_grid(d >= 2 ? 4 * wo : wo, batch * runs(ho));
    const double px = static_cast<double>(batch) * ho * wo;
    const float t = timestep_;
    KB2_TRY(timer_.begin(stream));
    switch (k) {
      case 0: rife_first_input_kernel<<<g, kGlueThreads, 0, stream>>>(F, E, d, batch, t, x_[k]); break;
      case 1: rife_block_input_kernel<1><<<g, kGlueThreads, 0, stream>>>(F, E, Z, d, batch, t, x_[k]); break;
      case 2: rife_block_input_kernel<2><<<g, kGlueThreads, 0, stream>>>(F, E, Z, d, batch, t, x_[k]); break;
      case 3: rife_block_input_kernel<3><<<g, kGlueThreads, 0, stream>>>(F, E, Z, d, batch, t, x_[k]); break;
      default: rife_block_input_kernel<4><<<g, kGlueThreads, 0, stream>>>(F, E, Z, d, batch, t, x_[k]); break;
    }
    KB2_CUDA(cudaGetLastError());
    // X written, frames and encodings read at the sample points (4 per pixel when d >= 2)
    KB2_TRY(timer_.end(k_glue_[k], 0.0, px * ((k == 0 ? 2 : 4) * 16.0 + (d >= 2 ? 4.0 : 1.0) * 32.0), stream));
    for (auto& l : layers_[k]) KB2_TRY(timed(*l, batch));
  }
  const int last = plan_.blocks - 1;
  if (finish.image == nullptr) {
    const dim3 g = row_grid(Wp_, batch * runs(Hp_));
    KB2_TRY(timer_.begin(stream));
    KB2_TRY(finish.f16 ? launch_motion<__half>(g, stream, F, Z, last, batch, finish)
                       : launch_motion<float>(g, stream, F, Z, last, batch, finish));
    KB2_TRY(timer_.end(k_motion_, 0.0, full_px * (kRifeZBytes + 5.0 * (finish.f16 ? 2.0 : 4.0)), stream));
    return Status::Ok();
  }
  const double px = static_cast<double>(batch) * H_ * W_;
  const dim3 g = row_grid(W_, batch * runs(H_));
  __half* out = static_cast<__half*>(finish.image);
  KB2_TRY(timer_.begin(stream));
  switch (last) {
    case 1: rife_finish_kernel<1><<<g, kGlueThreads, 0, stream>>>(F, Z, batch, out); break;
    case 2: rife_finish_kernel<2><<<g, kGlueThreads, 0, stream>>>(F, Z, batch, out); break;
    case 3: rife_finish_kernel<3><<<g, kGlueThreads, 0, stream>>>(F, Z, batch, out); break;
    default: rife_finish_kernel<4><<<g, kGlueThreads, 0, stream>>>(F, Z, batch, out); break;
  }
  KB2_CUDA(cudaGetLastError());
  KB2_TRY(timer_.end(k_finish_, 0.0, px * (kRifeZBytes + 16.0 + 6.0), stream));
  return Status::Ok();
}

}  // namespace kb2
