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

#include "conv_layer.h"
#include "ifnet_conv.cuh"
#include "ifnet_glue.cuh"
#include "ifnet_net.h"

namespace kb2 {

int num_sms();  // conv_layer.cu

namespace {

constexpr int kIfChannels[kIfBlocks] = {192, 128, 96, 64};
constexpr int kIfRes = 8;
// block 3's residual convs (64 channels) on the pair kernel (IfLayer::build_paired)
constexpr bool kIfPairedRes = true;

using IfLaunchFn = void (*)(dim3, size_t, cudaStream_t, const IfMaps&, const IfConvArgs&);

template <int N, int S, int E, int G>
void if_launch(dim3 grid, size_t smem, cudaStream_t s, const IfMaps& m, const IfConvArgs& a) {
  ifconv_kernel<N, S, E, G><<<grid, kIfThreads, smem, s>>>(m, a);
}

struct IfKernel {
  int n, stride, epi, g;
  IfLaunchFn launch;
  const void* fn;
};

#define KB2_IFK(N, S, E, G) \
  IfKernel { N, S, E, G, &if_launch<N, S, E, G>, reinterpret_cast<const void*>(&ifconv_kernel<N, S, E, G>) }

// the classic IFNet's layers: (N, stride, epilogue, input chunks per K group)
const IfKernel kIfKernels[] = {
    // conv0a: 12 (7) channels -> C/2, stride 2
    KB2_IFK(96, 2, kIfPrelu, 2), KB2_IFK(64, 2, kIfPrelu, 2), KB2_IFK(48, 2, kIfPrelu, 2), KB2_IFK(32, 2, kIfPrelu, 2),
    // conv0b: C/2 -> C, stride 2
    KB2_IFK(192, 2, kIfPrelu, 6), KB2_IFK(128, 2, kIfPrelu, 8), KB2_IFK(96, 2, kIfPrelu, 6),
    KB2_IFK(64, 2, kIfPrelu, 4),
    // residual convs: C -> C
    KB2_IFK(192, 1, kIfResPrelu, 8), KB2_IFK(128, 1, kIfResPrelu, 8), KB2_IFK(96, 1, kIfResPrelu, 6),
    KB2_IFK(64, 1, kIfResPrelu, 8),
    // transposed conv: C -> 4 phases x 8
    KB2_IFK(32, 1, kIfConvT, 8), KB2_IFK(32, 1, kIfConvT, 6),
};

const IfKernel* find_if_kernel(int n, int stride, int epi, int g) {
  for (const IfKernel& k : kIfKernels)
    if (k.n == n && k.stride == stride && k.epi == epi && k.g == g) return &k;
  return nullptr;
}

uint16_t f16_bits(float f) {
  const __half h = __float2half_rn(f);
  uint16_t b;
  std::memcpy(&b, &h, 2);
  return b;
}

// Largest even divisor of `chunks` that is at most 8: the chunks staged per K group.
int group_chunks(int chunks) {
  for (int g = 8; g >= 2; g -= 2)
    if (chunks % g == 0) return g;
  return 0;
}

}  // namespace

// One conv of the network: packed weights, constants, tensor map and launch shape.
struct IfLayer {
  IfConvArgs args{};
  IfMaps maps{};
  const IfKernel* k = nullptr;
  DeviceBuffer wpack, bias, slope;
  size_t smem = 0;
  int per_sm = 1;
  int kind = 0;
  double flops_px = 0.0, bytes_px = 0.0;  // algorithmic work per output pixel
  // 64-channel residual convs run on the paired stacked kernel (conv3p.cuh) instead: one M = 256
  // MMA for two SMs, the three kernel rows stacked in N = 192
  ConvLayer pair;
  bool paired = false;
  uint8_t* pair_out = nullptr;
  const uint8_t* pair_res = nullptr;
  int pair_res_chunks = 0;

  // The residual conv (PReLU(conv(x) + bias + x), C -> C, stride 1) of `c` = 64 channels on the pair
  // kernel: the tensors are [n][h][c / 8][w][8] FP16, the ConvLayer row layout.
  Status build_paired(int c, const float* w, const float* b, const float* prelu, uint8_t* in, int batch, int h,
                      int wd, uint8_t* out, int* err) {
    ConvSpec s;
    s.taps = 9;
    s.fp8 = false;
    s.n_sources = 1;
    s.cin = c;
    s.n_real = c;
    s.n_pad = c;
    s.epi = kEpiResPrelu;
    s.out = kOutF16Chunk;
    s.out_chunks = c / 8;
    ChunkedTensor t;
    t.ptr = in;
    t.batch = batch;
    t.H = h;
    t.W = wd;
    t.chunks = c / 8;
    t.fp8 = false;
    const ChunkedTensor* inputs[1] = {&t};
    KB2_TRY(pair.build(s, w, b, prelu, nullptr, inputs, err));
    if (pair.kind != 2) return refuse(KB2_FORMAT_UNSUPPORTED, "IFNet: residual conv did not map to the pair kernel");
    paired = true;
    pair_out = out;
    pair_res = in;
    pair_res_chunks = c / 8;
    args.h_out = h;
    args.w_out = wd;
    flops_px = 2.0 * 9.0 * c * c;
    bytes_px = 3.0 * (c / 8) * 16.0;  // input, residual and output: one FP16 pixel each
    return Status::Ok();
  }

  // w(n, ci, dy, dx): weight of output column n, input channel ci, tap (dy, dx); cout columns used.
  template <class W>
  Status build(int n_pad, int stride, int epi, W w, int cout, int cin, const float* b, const float* prelu,
               uint8_t* in, int batch, int h_in, int w_in, int in_chunks, int h_out, int w_out, uint8_t* out,
               int out_chunks, float* out_f32, int* err) {
    const int g = group_chunks(in_chunks);
    if (g == 0 || in_chunks * 8 < cin) return refuse(KB2_FORMAT_UNSUPPORTED, "IFNet: input channel layout");
    k = find_if_kernel(n_pad, stride, epi, g);
    if (k == nullptr) return refuse(KB2_FORMAT_UNSUPPORTED, "IFNet: no conv kernel for this layer shape");
    IfConvArgs& a = args;
    a.h_in = h_in;
    a.w_in = w_in;
    a.h_out = h_out;
    a.w_out = w_out;
    a.g = g;
    a.n_groups = in_chunks / g;
    a.strips = (w_out + kIfStrip - 1) / kIfStrip;
    a.a_bytes = static_cast<uint32_t>(g) * kIfChunkBytes * (stride == 2 ? 2u : 1u);
    a.b_bytes = static_cast<uint32_t>(3 * g * n_pad * 16);
    a.stage_bytes = (a.a_bytes + a.b_bytes + 1023u) & ~1023u;
    a.out = out;
    a.out_chunks = out_chunks;
    a.out_split = 0;
    a.out_f32 = out_f32;
    a.residual = epi == kIfResPrelu ? in : nullptr;
    a.err = err;

    // weights: [dy][group][dx][K step j][half][n][8 channels], FP16
    const size_t wbytes = static_cast<size_t>(3) * a.n_groups * a.b_bytes;
    std::vector<uint16_t> pack(wbytes / 2, 0);
    for (int dy = 0; dy < 3; ++dy)
      for (int grp = 0; grp < a.n_groups; ++grp)
        for (int dx = 0; dx < 3; ++dx)
          for (int j = 0; j < g / 2; ++j)
            for (int h = 0; h < 2; ++h)
              for (int n = 0; n < cout; ++n)
                for (int e = 0; e < 8; ++e) {
                  const int ci = (grp * g + 2 * j + h) * 8 + e;
                  if (ci >= cin) continue;
                  const size_t off = (static_cast<size_t>(dy * a.n_groups + grp) * a.b_bytes +
                                      static_cast<size_t>((dx * (g / 2) + j) * 2 + h) * n_pad * 16 + n * 16 + e * 2) /
                                     2;
                  pack[off] = f16_bits(w(n, ci, dy, dx));
                }
    KB2_TRY(wpack.alloc(wbytes));
    KB2_CUDA(cudaMemcpy(wpack.ptr, pack.data(), wbytes, cudaMemcpyHostToDevice));
    std::vector<float> bv(n_pad, 0.0f), sv(n_pad, 0.0f);
    for (int n = 0; n < n_pad; ++n) {
      bv[n] = b[n];
      sv[n] = prelu != nullptr ? prelu[n] : 0.0f;
    }
    KB2_TRY(bias.alloc(n_pad * sizeof(float)));
    KB2_TRY(slope.alloc(n_pad * sizeof(float)));
    KB2_CUDA(cudaMemcpy(bias.ptr, bv.data(), n_pad * sizeof(float), cudaMemcpyHostToDevice));
    KB2_CUDA(cudaMemcpy(slope.ptr, sv.data(), n_pad * sizeof(float), cudaMemcpyHostToDevice));
    a.wpack = wpack.as<uint8_t>();
    a.bias = bias.as<float>();
    a.slope = slope.as<float>();

    // tensor map of the input rows (UINT64 words: tile mode copies bytes)
    EncodeTiledFn fn = encode_tiled_fn();
    if (fn == nullptr) return refuse(KB2_VENDOR_CALL_FAILED, "cuTensorMapEncodeTiled unavailable");
    const cuuint64_t row = static_cast<cuuint64_t>(w_in) * 16;
    const cuuint64_t rows = static_cast<cuuint64_t>(batch) * h_in;
    const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r;
    if (stride == 1) {
      const cuuint64_t dims[3] = {static_cast<cuuint64_t>(w_in) * 2, static_cast<cuuint64_t>(in_chunks), rows};
      const cuuint64_t strides[2] = {row, row * in_chunks};
      const cuuint32_t box[3] = {256, static_cast<cuuint32_t>(g), 1};
      r = fn(&maps.a, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, in, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
      // parity-split rows: a chunk row is its W/2 even pixels then its W/2 odd pixels, so each
      // parity box is one contiguous 2 KB run per chunk
      if (w_in % 2 != 0) return refuse(KB2_FORMAT_UNSUPPORTED, "IFNet: stride-2 input of odd width");
      const cuuint64_t dims[4] = {static_cast<cuuint64_t>(w_in), 2, static_cast<cuuint64_t>(in_chunks), rows};
      const cuuint64_t strides[3] = {static_cast<cuuint64_t>(w_in / 2) * 16, row, row * in_chunks};
      const cuuint32_t box[4] = {256, 1, static_cast<cuuint32_t>(g), 1};
      r = fn(&maps.a, CU_TENSOR_MAP_DATA_TYPE_UINT64, 4, in, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r != CUDA_SUCCESS)
      return refuse(KB2_VENDOR_CALL_FAILED, "IFNet: cuTensorMapEncodeTiled failed: " + std::to_string(r));

    // launch shape: as many ring slots as fit (2..4), blocks per SM by shared memory and TMEM.
    // Where TMEM holds two blocks' accumulators and two ring slots fit in half the SM's shared
    // memory, the ring is cut to that half so two blocks share the SM: one block's epilogue then
    // overlaps the other's MMAs (measured faster on the 96- and 128-channel 1080p layers).
    int dev = 0, optin = 0;
    KB2_CUDA(cudaGetDevice(&dev));
    KB2_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    const size_t budget = static_cast<size_t>(optin) - kIfSmemExtra;
    a.stages = static_cast<uint32_t>(std::min<size_t>(kIfMaxStages, budget / a.stage_bytes));
    if (a.stages < 2) return refuse(KB2_FORMAT_UNSUPPORTED, "IFNet: layer stage does not fit in shared memory");
    const uint32_t tmem_cols = 2 * n_pad <= 64 ? 64 : (2 * n_pad <= 128 ? 128 : (2 * n_pad <= 256 ? 256 : 512));
    {
      const size_t half = (228u * 1024u) / 2 - 1024u - kIfSmemExtra;
      const uint32_t st2 = static_cast<uint32_t>(std::min<size_t>(kIfMaxStages, half / a.stage_bytes));
      if (512u / tmem_cols >= 2 && st2 >= 2) a.stages = std::min(a.stages, st2);
    }
    smem = static_cast<size_t>(a.stages) * a.stage_bytes + kIfSmemExtra;
    KB2_CUDA(cudaFuncSetAttribute(k->fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    const int smem_fit = static_cast<int>((228u * 1024u) / (smem + 1024u));
    per_sm = std::max(1, std::min(smem_fit, static_cast<int>(512u / tmem_cols)));
    // algorithmic work per output pixel of this conv grid (the transposed conv: 16 taps x 5 outputs
    // per input pixel, whatever the phase layout)
    flops_px = epi == kIfConvT ? 2.0 * 16.0 * cin * 5.0 : 2.0 * 9.0 * cin * cout;
    bytes_px = (epi == kIfConvT ? 4.0 * 32.0 : out_chunks * 16.0) + (epi == kIfResPrelu ? out_chunks * 16.0 : 0.0) +
               in_chunks * 16.0 * stride * stride;
    return Status::Ok();
  }

  Status launch(cudaStream_t stream, int batch) {
    if (paired) return pair.launch(stream, batch, pair_out, pair_res, 1.0f, 1.0f, nullptr, pair_res_chunks);
    IfConvArgs a = args;
    a.batch = batch;
    a.items = batch * a.h_out * a.strips;
    const int grid = std::min(a.items, num_sms() * per_sm);
    k->launch(dim3(grid), smem, stream, maps, a);
    return cuda_status(cudaGetLastError(), "IFNet conv launch");
  }
};

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

    auto conv_w = [](const float* w, int cin) {
      return [w, cin](int n, int ci, int dy, int dx) { return w[((static_cast<size_t>(n) * cin + ci) * 3 + dy) * 3 + dx]; };
    };
    // conv0a
    const float* wa = p;
    p += static_cast<size_t>(c / 2) * cin0 * 9;
    const float* ba = p;
    p += c / 2;
    const float* sa = p;
    p += c / 2;
    auto la = std::make_unique<IfLayer>();
    KB2_TRY(la->build(c / 2, 2, kIfPrelu, conv_w(wa, cin0), c / 2, cin0, ba, sa, x->ptr, max_batch_, h0, w0, 2, h1,
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
    KB2_TRY(lb->build(c, 2, kIfPrelu, conv_w(wb, c / 2), c, c / 2, bb, sb, a0->ptr, max_batch_, h1, w1, c / 16, h2,
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
        KB2_TRY(lr->build(c, 1, kIfResPrelu, conv_w(wr, c), c, c, br, sr, src->ptr, max_batch_, h2, w2, c / 8, h2,
                          w2, dst->ptr, c / 8, nullptr, err));
      lr->kind = k_res;
      layers_.push_back(std::move(lr));
    }
    // transposed conv 4x4 stride 2 (pad 1) as a 3x3 conv with N = 4 phases x 8: output phase
    // (py, px) at (2y + py, 2x + px) takes input row y + dy - 1 with kernel row kmap[py][dy]
    // (py = 0: dy 0 -> 3, dy 1 -> 1; py = 1: dy 1 -> 2, dy 2 -> 0), the same along x
    const float* wt = p;  // [cin = c][5][4][4]
    p += static_cast<size_t>(c) * 5 * 16;
    const float* bt = p;
    p += 5;
    float bias_t[32] = {};
    for (int ph = 0; ph < 4; ++ph)
      for (int co = 0; co < 5; ++co) bias_t[ph * 8 + co] = bt[co];
    auto wconvt = [wt](int n, int ci, int dy, int dx) -> float {
      static constexpr int kmap[2][3] = {{3, 1, -1}, {-1, 2, 0}};
      const int ph = n / 8, co = n % 8;
      if (co >= 5) return 0.0f;
      const int ky = kmap[ph >> 1][dy], kx = kmap[ph & 1][dx];
      if (ky < 0 || kx < 0) return 0.0f;
      return wt[((static_cast<size_t>(ci) * 5 + co) * 4 + ky) * 4 + kx];
    };
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
  IfFrames F{static_cast<const __half*>(img0), static_cast<const __half*>(img1), H_, W_, Hp_, Wp_, top_, left_, pad0,
             pad0 + static_cast<size_t>(max_batch_) * Hp_ * Wp_};
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
    ifnet_pad_frames_kernel<<<row_grid(Wp_, batch * Hp_), kGlueThreads, 0, stream>>>(F, batch);
    KB2_CUDA(cudaGetLastError());
    KB2_TRY(timer_.end(k_pad_, 0.0, px * (12.0 + 16.0), stream));
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
