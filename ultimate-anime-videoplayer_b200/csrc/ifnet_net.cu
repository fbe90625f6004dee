// Classic IFNet on B200: per block, a glue kernel builds the block input from the frames and the
// flow so far, two stride-2 convs and eight residual convs run on the tensor cores
// (ifnet_conv.cuh), and the 4x4 stride-2 transposed conv runs as a 3x3 conv with its four output
// phases as N, leaving a small FP32 flow / mask tensor. A last glue kernel warps both frames by the
// final flow and blends them. This is the reference's fused RIFE chain (RifeFusedEngine::enqueue,
// src/gpu/cuda/backend/rife_fused_engine.cpp:390: entry -> blocks with glue between -> finish) for
// the classic IFNet topology of the reference's IR (4 blocks, channels 192 / 128 / 96 / 64).
//
// Frames of any size are placed in a zero padded plane of multiples of 32, at the window of
// rife_window (src/kernels/spec/rife.h:47-57: left / top = half the padding, rounded down to even),
// and the output is read back from that window.
#include <algorithm>
#include <cstring>

#include "if_layer.h"
#include "ifnet_glue.cuh"
#include "ifnet_net.h"

namespace kb2 {

int num_sms();  // conv_layer.cu

namespace {

constexpr int kIfChannels[kIfBlocks] = {192, 128, 96, 64};
constexpr int kIfRes = 8;
// block 3's residual convs (64 channels) on the pair kernel (IfLayer::build_paired)
constexpr bool kIfPairedRes = true;

}  // namespace

IfnetNet::IfnetNet() = default;
IfnetNet::~IfnetNet() = default;

Status IfnetNet::tensor(std::unique_ptr<Tensor>& t, int H, int W, int chunks) {
  t = std::make_unique<Tensor>();
  t->H = H;
  t->W = W;
  t->chunks = chunks;
  const size_t bytes = static_cast<size_t>(max_batch_) * H * W * chunks * 16;
  KB2_TRY(t->buf.alloc(bytes));
  KB2_CUDA(cudaMemset(t->buf.ptr, 0, bytes));
  t->ptr = t->buf.as<uint8_t>();
  return Status::Ok();
}

Status IfnetNet::create(const std::vector<float>& params, int max_batch, int H, int W) {
  if (params.size() != kIfnetParams) return refuse(KB2_WEIGHTS_INVALID, "IFNet: parameter count mismatch");
  max_batch_ = max_batch;
  H_ = H;
  W_ = W;
  Hp_ = (H + kIfnetAlign - 1) / kIfnetAlign * kIfnetAlign;
  Wp_ = (W + kIfnetAlign - 1) / kIfnetAlign * kIfnetAlign;
  top_ = ((Hp_ - H) / 2) & ~1;
  left_ = ((Wp_ - W) / 2) & ~1;
  KB2_TRY(err_.alloc(sizeof(int)));
  KB2_CUDA(cudaMemset(err_.ptr, 0, sizeof(int)));
  for (int k = 0; k < kIfBlocks; ++k) k_glue_[k] = timer_.kind(("ifnet.glue.b" + std::to_string(k)).c_str());
  const int k_c0a = timer_.kind("ifnet.conv0a"), k_c0b = timer_.kind("ifnet.conv0b");
  const int k_res = timer_.kind("ifnet.res"), k_ct = timer_.kind("ifnet.convt");
  k_blend_ = timer_.kind("ifnet.blend");
  k_motion_ = timer_.kind("ifnet.motion");
  KB2_TRY(flow_full_.alloc(static_cast<size_t>(max_batch_) * 5 * Hp_ * Wp_ * sizeof(float)));
  KB2_CUDA(cudaMemset(flow_full_.ptr, 0, flow_full_.bytes));
  KB2_TRY(pad_.alloc(static_cast<size_t>(max_batch_) * 2 * Hp_ * Wp_ * sizeof(uint2)));
  k_pad_ = timer_.kind("ifnet.pad");

  const float* p = params.data();
  for (int k = 0; k < kIfBlocks; ++k) {
    const int c = kIfChannels[k], s = if_scale(k);
    const int cin0 = k == 0 ? 7 : 12;
    const int h0 = Hp_ / s, w0 = Wp_ / s;  // block input
    const int h1 = h0 / 2, w1 = w0 / 2;    // after conv0a (also the transposed conv's output)
    const int h2 = h1 / 2, w2 = w1 / 2;    // residual level
    std::unique_ptr<Tensor> x, a0, r0, r1;
    KB2_TRY(tensor(x, h0, w0, 2));
    KB2_TRY(tensor(a0, h1, w1, c / 16));
    KB2_TRY(tensor(r0, h2, w2, c / 8));
    KB2_TRY(tensor(r1, h2, w2, c / 8));
    KB2_TRY(flows_[k].alloc(static_cast<size_t>(max_batch_) * h1 * w1 * 8 * sizeof(float)));
    KB2_CUDA(cudaMemset(flows_[k].ptr, 0, flows_[k].bytes));
    int* err = err_.as<int>();

    // conv0a
    const float* wa = p;
    p += static_cast<size_t>(c / 2) * cin0 * 9;
    const float* ba = p;
    p += c / 2;
    const float* sa = p;
    p += c / 2;
    auto la = std::make_unique<IfLayer>();
    KB2_TRY(la->build(c / 2, 2, kIfPrelu, dense_conv_weights(wa, c / 2, cin0, c / 2), c / 2, cin0, ba, sa, x->ptr, max_batch_, h0, w0, 2, h1,
                      w1, a0->ptr, c / 16, nullptr, err));
    la->args.out_split = 1;  // conv0b reads a0 with stride 2
    la->kind = k_c0a;
    layers_.push_back(std::move(la));
    // conv0b
    const float* wb = p;
    p += static_cast<size_t>(c) * (c / 2) * 9;
    const float* bb = p;
    p += c;
    const float* sb = p;
    p += c;
    auto lb = std::make_unique<IfLayer>();
    KB2_TRY(lb->build(c, 2, kIfPrelu, dense_conv_weights(wb, c, c / 2, c), c, c / 2, bb, sb, a0->ptr, max_batch_, h1, w1, c / 16, h2,
                      w2, r0->ptr, c / 8, nullptr, err));
    lb->kind = k_c0b;
    layers_.push_back(std::move(lb));
    // residual convs, ping-pong r0 <-> r1 (the input is also the residual)
    for (int j = 0; j < kIfRes; ++j) {
      const float* wr = p;
      p += static_cast<size_t>(c) * c * 9;
      const float* br = p;
      p += c;
      const float* sr = p;
      p += c;
      Tensor* src = j % 2 == 0 ? r0.get() : r1.get();
      Tensor* dst = j % 2 == 0 ? r1.get() : r0.get();
      auto lr = std::make_unique<IfLayer>();
      if (c == 64 && kIfPairedRes)
        KB2_TRY(lr->build_paired(c, wr, br, sr, src->ptr, max_batch_, h2, w2, dst->ptr, err));
      else
        KB2_TRY(lr->build(c, 1, kIfResPrelu, dense_conv_weights(wr, c, c, c), c, c, br, sr, src->ptr, max_batch_, h2, w2, c / 8, h2,
                          w2, dst->ptr, c / 8, nullptr, err));
      lr->kind = k_res;
      layers_.push_back(std::move(lr));
    }
    // transposed conv 4x4 stride 2 (pad 1) as a 3x3 conv with N = 4 phases x 8 (5 used)
    const float* wt = p;  // [cin = c][5][4][4]
    p += static_cast<size_t>(c) * 5 * 16;
    const float* bt = p;
    p += 5;
    float bias_t[32] = {};
    for (int ph = 0; ph < 4; ++ph)
      for (int co = 0; co < 5; ++co) bias_t[ph * 8 + co] = bt[co];
    const std::vector<float> wconvt = convt_phase_weights(wt, c, 5, 32, [](int n, int* ph, int* co) {
      *ph = n / 8;
      *co = n % 8 < 5 ? n % 8 : -1;
    });
    auto lt = std::make_unique<IfLayer>();
    KB2_TRY(lt->build(32, 1, kIfConvT, wconvt, 32, c, bias_t, nullptr, r0->ptr, max_batch_, h2, w2, c / 8, h2, w2,
                      nullptr, 0, flows_[k].as<float>(), err));
    lt->kind = k_ct;
    layers_.push_back(std::move(lt));
    x_[k] = x.get();
    tensors_.push_back(std::move(x));
    tensors_.push_back(std::move(a0));
    tensors_.push_back(std::move(r0));
    tensors_.push_back(std::move(r1));
  }
  if (static_cast<size_t>(p - params.data()) != kIfnetParams)
    return refuse(KB2_WEIGHTS_INVALID, "IFNet: parameter layout mismatch");
  return Status::Ok();
}

Status IfnetNet::set_timestep(float t) {
  if (!(t > 0.0f && t < 1.0f)) return refuse(KB2_INVALID_ARGUMENT, "IFNet: timestep must be in (0, 1)");
  timestep_ = t;
  return Status::Ok();
}

int IfnetNet::launches_per_run() const { return 1 + kIfBlocks + static_cast<int>(layers_.size()) + 1; }

size_t IfnetNet::device_bytes() const {
  size_t total = err_.bytes;
  for (const auto& t : tensors_) total += t->buf.bytes;
  for (const auto& f : flows_) total += f.bytes;
  total += flow_full_.bytes + pad_.bytes;
  for (const auto& l : layers_)
    total += l->wpack.bytes + l->bias.bytes + l->slope.bytes + l->pair.wpack.bytes + l->pair.bias.bytes +
             l->pair.slope.bytes + l->pair.scale.bytes;
  return total;
}

Status IfnetNet::run(cudaStream_t stream, const void* img0, const void* img1, void* out, int batch) {
  return run_impl(stream, img0, img1, Finish{out, nullptr, nullptr, false}, batch);
}

Status IfnetNet::run_motion(cudaStream_t stream, const void* img0, const void* img1, void* flow, void* mask, bool f16,
                            int batch) {
  return run_impl(stream, img0, img1, Finish{nullptr, flow, mask, f16}, batch);
}

Status IfnetNet::run_impl(cudaStream_t stream, const void* img0, const void* img1, const Finish& finish, int batch) {
  if (batch < 1 || batch > max_batch_) return refuse(KB2_SHAPE_INVALID, "IFNet: batch out of contract");
  uint2* pad0 = pad_.as<uint2>();
  const size_t pad_plane = static_cast<size_t>(Hp_) * Wp_;
  // A video stream passes pair n as frames n and n + 1 of one buffer (img1 = img0 one frame on): its
  // batch + 1 frames are then padded once each, and pad1 is pad0 one plane on (pad_ holds 2 x
  // max_batch planes, at least batch + 1).
  const bool stream_pairs =
      static_cast<const __half*>(img1) == static_cast<const __half*>(img0) + static_cast<size_t>(3) * H_ * W_;
  IfFrames F{static_cast<const __half*>(img0), static_cast<const __half*>(img1), H_, W_, Hp_, Wp_, top_, left_, pad0,
             pad0 + (stream_pairs ? pad_plane : static_cast<size_t>(max_batch_) * pad_plane)};
  // a grid of row runs for the glue kernels (ifnet_glue.cuh): about 16 blocks per SM, each walking runs
  const int sms = num_sms();
  auto row_grid = [sms](int width, int rows) {
    const int bx = (width + kGlueThreads - 1) / kGlueThreads;
    const int by = std::max(1, std::min({rows, kGlueMaxRowBlocks, (16 * sms + bx - 1) / bx}));
    return dim3(static_cast<unsigned>(bx), static_cast<unsigned>(by));
  };
  {
    const long long px = static_cast<long long>(batch) * Hp_ * Wp_;
    KB2_TRY(timer_.begin(stream));
    if (stream_pairs) {
      ifnet_pad_stream_kernel<<<row_grid(Wp_, (batch + 1) * Hp_), kGlueThreads, 0, stream>>>(F, batch + 1);
      KB2_CUDA(cudaGetLastError());
      KB2_TRY(timer_.end(k_pad_, 0.0, static_cast<double>(px + static_cast<long long>(pad_plane)) * (6.0 + 8.0), stream));
    } else {
      ifnet_pad_frames_kernel<<<row_grid(Wp_, batch * Hp_), kGlueThreads, 0, stream>>>(F, batch);
      KB2_CUDA(cudaGetLastError());
      KB2_TRY(timer_.end(k_pad_, 0.0, px * (12.0 + 16.0), stream));
    }
  }
  IfFlowLevels L{};
  for (int k = 0; k < kIfBlocks; ++k) {
    const int s = if_scale(k);
    L.t[k] = flows_[k].as<float>();
    L.h[k] = Hp_ / (2 * s);
    L.w[k] = Wp_ / (2 * s);
    L.mul[k] = static_cast<float>(2 * s);
    L.inv[k] = 1.0f / static_cast<float>(2 * s);
  }
  const IfFlowField FF{flow_full_.as<float>(), Hp_, Wp_};
  const int per_block = 2 + kIfRes + 1;
  for (int k = 0; k < kIfBlocks; ++k) {
    const int s = if_scale(k);
    const long long px = static_cast<long long>(batch) * (Hp_ / s) * (Wp_ / s);
    // s = 1: a thread per column; s > 1: two per output column (ifnet_glue.cuh); runs of rows
    const int run = k == 0 ? glue_run<0>() : k == 1 ? glue_run<1>() : k == 2 ? glue_run<2>() : glue_run<3>();
    const dim3 g = row_grid((s == 1 ? 1 : 2) * (Wp_ / s), batch * ((Hp_ / s + run - 1) / run));
    constexpr int T = kGlueThreads;
    KB2_TRY(timer_.begin(stream));
    switch (k) {
      case 0: ifnet_block_input_kernel<0><<<g, T, 0, stream>>>(F, L, FF, batch, timestep_, x_[k]->ptr); break;
      case 1: ifnet_block_input_kernel<1><<<g, T, 0, stream>>>(F, L, FF, batch, timestep_, x_[k]->ptr); break;
      case 2: ifnet_block_input_kernel<2><<<g, T, 0, stream>>>(F, L, FF, batch, timestep_, x_[k]->ptr); break;
      default: ifnet_block_input_kernel<3><<<g, T, 0, stream>>>(F, L, FF, batch, timestep_, x_[k]->ptr); break;
    }
    KB2_CUDA(cudaGetLastError());
    KB2_TRY(timer_.end(k_glue_[k], 0.0, px * 32.0, stream));
    for (int i = 0; i < per_block; ++i) {
      IfLayer& l = *layers_[k * per_block + i];
      const double opx = static_cast<double>(batch) * l.args.h_out * l.args.w_out;
      KB2_TRY(timer_.begin(stream));
      KB2_TRY(l.launch(stream, batch));
      KB2_TRY(timer_.end(l.kind, l.flops_px * opx, l.bytes_px * opx, stream));
    }
  }
  if (finish.image == nullptr) {
    // motion: read the FP32 flow field (20 B/px), write 4 flow planes and the mask
    const long long px = static_cast<long long>(batch) * Hp_ * Wp_;
    const dim3 g = row_grid(Wp_, batch * ((Hp_ + kGlueRunRows - 1) / kGlueRunRows));
    KB2_TRY(timer_.begin(stream));
    if (finish.f16)
      ifnet_motion_kernel<__half><<<g, kGlueThreads, 0, stream>>>(F, L, FF, batch, static_cast<__half*>(finish.flow),
                                                                   static_cast<__half*>(finish.mask));
    else
      ifnet_motion_kernel<float><<<g, kGlueThreads, 0, stream>>>(F, L, FF, batch, static_cast<float*>(finish.flow),
                                                                  static_cast<float*>(finish.mask));
    KB2_CUDA(cudaGetLastError());
    KB2_TRY(timer_.end(k_motion_, 0.0, px * (20.0 + 5.0 * (finish.f16 ? 2.0 : 4.0)), stream));
    return Status::Ok();
  }
  const long long px = static_cast<long long>(batch) * H_ * W_;
  KB2_TRY(timer_.begin(stream));
  ifnet_blend_kernel<<<row_grid(W_, batch * ((H_ + kGlueRunRows - 1) / kGlueRunRows)), kGlueThreads, 0, stream>>>(
      F, L, FF, batch, static_cast<__half*>(finish.image));
  KB2_CUDA(cudaGetLastError());
  KB2_TRY(timer_.end(k_blend_, 0.0, px * (20.0 + 12.0 + 6.0), stream));
  return Status::Ok();
}

Status warp_taps(cudaStream_t stream, const float* flow, int n, int h, int w, int32_t* taps, float* weights) {
  if (flow == nullptr || taps == nullptr || weights == nullptr) return refuse(KB2_INVALID_ARGUMENT, "null pointer");
  if (n < 1 || h < 1 || w < 1 || h > 16384 || w > 16384) return refuse(KB2_SHAPE_INVALID, "warp taps: size");
  const long long px = static_cast<long long>(n) * h * w;
  const int blocks = static_cast<int>(std::min<long long>((px + 255) / 256, 32LL * num_sms()));
  warp_taps_kernel<<<blocks, 256, 0, stream>>>(flow, n, h, w, taps, weights);
  return cuda_status(cudaGetLastError(), "warp taps launch");
}

}  // namespace kb2
