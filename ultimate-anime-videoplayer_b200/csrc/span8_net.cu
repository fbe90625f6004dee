// The AnimeJaNai "unshuffle" SPAN x2 from a .span8 package, FP16 on the tensor-core conv layers. It
// replaces the reference's FP16-native path of that package (SpanFp8Net with the package's FP16
// flag, src/gpu/cuda/backend/span_fp8_net.h:107-175; the graph of span_fp8::forward,
// src/gpu/span_fp8/forward.cpp:144-166).
//
// Launch sequence (all batch-wide, at the half-resolution working plane h x w = H/2 x W/2, C = the
// package's real channels, 48 or 64):
//   unshuffle  NCHW F16 frame -> row-chunked [n][h][2][w][8], channel c*4 + dy*2 + dx (12 real)
//   conv_1     3x3 12->C                                                        -> S0
//   block b    c1 3x3 + ReLU -> R1; c2 3x3 + ReLU -> R2; c3 3x3 -> C3;
//              att 1x1 on C3, then (x + C3) * tanh(att), x the block input        -> X(b+1)
//   conv_cat   1x1 over the four sources [S0, X_last, X1, R1 of the last block], no concat buffer
//   to_pixel   3x3 C->48 + DepthToSpace(4) in the epilogue                          -> NCHW F16 [n][3][2H][2W]
// ReLU is the PReLU epilogue with zero slopes.
//
// Precision. FP16 engine: FP16 operands and activations, FP32 accumulation (any package; its weights
// are FP16 in the file). E4M3 engine (an FP8 package, without the FP16 flag): the blocks' 3x3 convs
// run E4M3 x E4M3 -> FP32 with the package's per-tensor activation scales ([0] conv_1 output, [1+3b]
// and [2+3b] block b's ReLU outputs, [3+3b] its output: span_fp8/package.h:15-17) and per-output-
// channel weight scales; conv_1 and the gates write FP16 and E4M3 copies of each block input, c3
// writes FP16, and the attention, conv_cat and to_pixel stay FP16, as the reference keeps its ends
// in FP16 (package.h:12-16).
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>

#include "span8_net.h"
#include "span_net.h"

namespace kb2 {

namespace {

constexpr size_t kSpan8Header = 40;
constexpr uint64_t kSpan8MaxBytes = uint64_t{64} << 20;
constexpr int kStored = 64;       // channels every conv is stored with
constexpr int kFirstIn = 16;      // conv_1 input channels stored (12 real)
constexpr int kPixelOut = 48;     // to_pixel outputs: 3 planes x 4 x 4
constexpr uint32_t kFlagFp16 = 2u, kFlagAcc32 = 4u, kFlagsKnown = 7u;

uint32_t le32(const uint8_t* p) {
  return static_cast<uint32_t>(p[0]) | static_cast<uint32_t>(p[1]) << 8 | static_cast<uint32_t>(p[2]) << 16 |
         static_cast<uint32_t>(p[3]) << 24;
}
uint64_t le64(const uint8_t* p) { return static_cast<uint64_t>(le32(p)) | static_cast<uint64_t>(le32(p + 4)) << 32; }

float half_bits_to_float(uint16_t h) {
  __half_raw r;
  r.x = h;
  return __half2float(__half(r));
}

// Sequential reader of the payload: every read is bounded by the payload.
struct Reader {
  const uint8_t* p;
  uint64_t left;
  bool conv(Span8Package::Conv& c, size_t n_w, size_t n_b) {
    if (n_w * 2 + n_b * 4 > left) return false;
    c.w.resize(n_w);
    c.b.resize(n_b);
    for (size_t i = 0; i < n_w; ++i) {
      const uint16_t h = static_cast<uint16_t>(p[2 * i] | p[2 * i + 1] << 8);
      if ((h & 0x7C00u) == 0x7C00u) return false;  // infinity or NaN
      c.w[i] = half_bits_to_float(h);
    }
    p += n_w * 2;
    for (size_t i = 0; i < n_b; ++i) {
      uint32_t u = le32(p + 4 * i);
      std::memcpy(&c.b[i], &u, 4);
      if (!std::isfinite(c.b[i])) return false;
    }
    p += n_b * 4;
    left -= n_w * 2 + n_b * 4;
    return true;
  }
};

// Unshuffle: NCHW half [n][3][H][W] -> [n][H/2][2][W/2][8] half, channel c*4 + dy*2 + dx.
__global__ void span8_unshuffle_kernel(const __half* __restrict__ in, uint8_t* __restrict__ out, int batch, int H,
                                       int W) {
  const int h = H / 2, w = W / 2;
  const int x = blockIdx.x * blockDim.x + threadIdx.x;
  if (x >= w) return;
  const size_t plane = static_cast<size_t>(H) * W;
  for (int r = blockIdx.y; r < batch * h; r += gridDim.y) {
    const int n = r / h;
    const int y = r - n * h;
    __half v[16];
#pragma unroll
    for (int c = 0; c < 3; ++c)
#pragma unroll
      for (int dy = 0; dy < 2; ++dy) {
        const __half2 q = *reinterpret_cast<const __half2*>(
            in + (static_cast<size_t>(n) * 3 + c) * plane + static_cast<size_t>(2 * y + dy) * W + 2 * x);
        v[c * 4 + dy * 2] = __low2half(q);
        v[c * 4 + dy * 2 + 1] = __high2half(q);
      }
#pragma unroll
    for (int c = 12; c < 16; ++c) v[c] = __float2half_rn(0.0f);
    uint8_t* row = out + static_cast<size_t>(r) * 2 * w * 16;
    *reinterpret_cast<uint4*>(row + static_cast<size_t>(x) * 16) = *reinterpret_cast<const uint4*>(v);
    *reinterpret_cast<uint4*>(row + (static_cast<size_t>(w) + x) * 16) = *reinterpret_cast<const uint4*>(v + 8);
  }
}

// OIHW float weights of a package conv on its real channels: the package stores
// [out][ky][kx][groups x in_stored]; OIHW index ((o * groups * in_real + g * in_real + i) * k + ky) * k + kx.
std::vector<float> oihw(const Span8Package::Conv& c, int outs, int k, int groups, int in_stored, int in_real) {
  std::vector<float> w(static_cast<size_t>(outs) * groups * in_real * k * k);
  for (int o = 0; o < outs; ++o)
    for (int t = 0; t < k * k; ++t)
      for (int g = 0; g < groups; ++g)
        for (int i = 0; i < in_real; ++i)
          w[((static_cast<size_t>(o) * groups * in_real + g * in_real + i) * k * k) + t] =
              c.w[(static_cast<size_t>(o) * k * k + t) * groups * in_stored + static_cast<size_t>(g) * in_stored + i];
  return w;
}

}  // namespace

Status parse_span8(const void* bytes, uint64_t n, Span8Package& out) {
  if (bytes == nullptr || n < kSpan8Header || n > kSpan8MaxBytes)
    return refuse(KB2_WEIGHTS_INVALID, ".span8 package: size out of range");
  const uint8_t* p = static_cast<const uint8_t*>(bytes);
  if (std::memcmp(p, "AJPSPAN8", 8) != 0) return refuse(KB2_FORMAT_UNSUPPORTED, ".span8 package: no signature");
  const uint8_t* head = p + 8;
  const uint32_t version = le32(head);
  if (version != 1 && version != 2) return refuse(KB2_FORMAT_UNSUPPORTED, ".span8 package: unknown version");
  const uint32_t blocks = le32(head + 4);
  const uint32_t flags = le32(head + 28);
  const uint32_t known = version == 1 ? 0u : kFlagsKnown;
  if ((flags & kFlagAcc32) != 0u && (flags & kFlagFp16) == 0u)
    return refuse(KB2_FORMAT_UNSUPPORTED, ".span8 package: f32 sums without the FP16 flag");
  if ((flags & ~known) != 0u) return refuse(KB2_FORMAT_UNSUPPORTED, ".span8 package: unknown flags");
  const uint32_t real = version == 1 ? (le32(head + 12) == 0 ? 64u : 0u) : le32(head + 12);
  const bool shape_ok = le32(head + 8) == static_cast<uint32_t>(kStored) &&
                        (version == 1 ? blocks == 8u : blocks >= 2u && blocks <= 8u) && (real == 48u || real == 64u);
  if (!shape_ok) return refuse(KB2_FORMAT_UNSUPPORTED, ".span8 package: 2..8 blocks in 64 channels (48 or 64 real)");
  const uint64_t payload = le64(head + 16);
  if (payload != n - kSpan8Header) return refuse(KB2_WEIGHTS_INVALID, ".span8 package: truncated or too long");
  if (crc32(p + kSpan8Header, payload) != le32(head + 24))
    return refuse(KB2_WEIGHTS_INVALID, ".span8 package: CRC mismatch");

  Span8Package pkg;
  pkg.version = static_cast<int>(version);
  pkg.blocks = static_cast<int>(blocks);
  pkg.real = static_cast<int>(real);
  pkg.flags = flags;
  Reader in{p + kSpan8Header, payload};
  const auto bad = [] { return refuse(KB2_FORMAT_UNSUPPORTED, ".span8 package: inconsistent contents"); };
  const size_t n_scales = 1 + 3 * static_cast<size_t>(blocks);
  if (n_scales * 4 > in.left) return bad();
  pkg.scales.resize(n_scales);
  for (size_t i = 0; i < n_scales; ++i) {
    uint32_t u = le32(in.p + 4 * i);
    std::memcpy(&pkg.scales[i], &u, 4);
    if (!(pkg.scales[i] > 0.0f) || !std::isfinite(pkg.scales[i])) return bad();
  }
  in.p += n_scales * 4;
  in.left -= n_scales * 4;
  if (!in.conv(pkg.first, static_cast<size_t>(kStored) * 9 * kFirstIn, kStored)) return bad();
  pkg.block.resize(blocks);
  for (auto& b : pkg.block) {
    for (auto& c : b.c)
      if (!in.conv(c, static_cast<size_t>(kStored) * 9 * kStored, kStored)) return bad();
    if (!in.conv(b.att, static_cast<size_t>(kStored) * kStored, kStored)) return bad();
  }
  if (!in.conv(pkg.concat, static_cast<size_t>(kStored) * 4 * kStored, kStored)) return bad();
  if (!in.conv(pkg.pixel, static_cast<size_t>(kPixelOut) * 9 * kStored, kPixelOut)) return bad();
  if (in.left != 0) return bad();
  out = std::move(pkg);
  return Status::Ok();
}

Status Span8Net::make_tensor(std::unique_ptr<Tensor>& t, int chunks, bool fp8) {
  t = std::make_unique<Tensor>();
  t->t.batch = max_batch_;
  t->t.H = h_;
  t->t.W = w_;
  t->t.chunks = chunks;
  t->t.fp8 = fp8;
  KB2_TRY(t->buf.alloc(t->t.bytes()));
  KB2_CUDA(cudaMemset(t->buf.ptr, 0, t->t.bytes()));
  t->t.ptr = t->buf.as<uint8_t>();
  return Status::Ok();
}

Status Span8Net::create(const Span8Package& pkg, bool fp8, int max_batch, int H, int W) {
  if (H % 2 != 0 || W % 2 != 0) return refuse(KB2_SHAPE_INVALID, "unshuffle SPAN: even frame height and width");
  if (H < 4 || W < 4) return refuse(KB2_SHAPE_INVALID, "unshuffle SPAN: frame too small");
  max_batch_ = max_batch;
  H_ = H;
  W_ = W;
  h_ = H / 2;
  w_ = W / 2;
  ch_ = pkg.real;
  fp8_ = fp8;
  blocks_ = pkg.blocks;
  KB2_TRY(peaks_.alloc(static_cast<size_t>(1 + 3 * blocks_) * sizeof(unsigned int)));
  const int C = ch_, cc = C / 8, cq = C / 16;  // FP16 and E4M3 chunks of a C-channel tensor
  KB2_TRY(err_.alloc(sizeof(int)));
  KB2_CUDA(cudaMemset(err_.ptr, 0, sizeof(int)));
  int* err = err_.as<int>();
  k_pack_ = timer_.kind("span8.unshuffle");
  const int k_first = timer_.kind("span8.conv_1");
  const int k_relu = timer_.kind(fp8 ? "span8.block_relu_conv.fp8" : "span8.block_relu_conv");
  const int k_c3 = timer_.kind(fp8 ? "span8.block_c3.fp8" : "span8.block_c3");
  const int k_gate = timer_.kind("span8.block_att_gate");
  const int k_cat = timer_.kind("span8.conv_cat"), k_pix = timer_.kind("span8.to_pixel");

  // FP16 tensors: the unshuffled frame, conv_1's output, the block outputs (two alternating, the
  // first block's kept), the ReLU outputs, c3 and conv_cat's output. The E4M3 engine adds E4M3
  // copies of every block-conv input: conv_1's and each block's output, the two ReLU outputs.
  std::unique_ptr<Tensor> u, s0, xa, xb, x1, r1, r1_last, r2, c3, cat, s0q, xaq, xbq, x1q;
  KB2_TRY(make_tensor(u, 2));
  KB2_TRY(make_tensor(s0, cc));
  KB2_TRY(make_tensor(xa, cc));
  KB2_TRY(make_tensor(xb, cc));
  KB2_TRY(make_tensor(x1, cc));
  KB2_TRY(make_tensor(r1_last, cc));
  KB2_TRY(make_tensor(c3, cc));
  KB2_TRY(make_tensor(cat, cc));
  KB2_TRY(make_tensor(r1, fp8 ? cq : cc, fp8));
  KB2_TRY(make_tensor(r2, fp8 ? cq : cc, fp8));
  if (fp8) {
    KB2_TRY(make_tensor(s0q, cq, true));
    KB2_TRY(make_tensor(xaq, cq, true));
    KB2_TRY(make_tensor(xbq, cq, true));
    KB2_TRY(make_tensor(x1q, cq, true));
  }
  unshuffled_ = &u->t;
  // E4M3 copy of an FP16 block input
  auto q_of = [&](const ChunkedTensor* t) -> const ChunkedTensor* {
    if (!fp8) return nullptr;
    if (t == &s0->t) return &s0q->t;
    if (t == &xa->t) return &xaq->t;
    if (t == &xb->t) return &xbq->t;
    return &x1q->t;
  };

  auto add = [&](const ConvSpec& sp, const std::vector<float>& w, const std::vector<float>& b, const float* act_scale,
                 const ChunkedTensor* const* inputs, const ChunkedTensor* out, const ChunkedTensor* out2, float out_scale,
                 const ChunkedTensor* res, const ChunkedTensor* res2, int kind, int peak = -1) -> Status {
    auto l = std::make_unique<ConvLayer>();
    KB2_TRY(l->build(sp, w.data(), b.data(), nullptr, act_scale, inputs, err));
    steps_.push_back(Step{l.get(), out, out2, out2 != nullptr ? 1.0f / out_scale : 1.0f, res, res2, kind,
                          fp8 ? -1 : peak});
    layers_.push_back(std::move(l));
    return Status::Ok();
  };
  auto spec = [&](int taps, bool q, int cin, int n_pad, int epi, int out_fmt) {
    ConvSpec sp;
    sp.taps = taps;
    sp.fp8 = q;
    sp.cin = cin;
    sp.n_real = n_pad;
    sp.n_pad = n_pad;
    sp.epi = epi;
    sp.out = out_fmt;
    sp.out_chunks = out_fmt == kOutE4m3Chunk ? cq : cc;
    sp.out2_chunks = cq;
    return sp;
  };
  auto bias = [&](const Span8Package::Conv& c, int n) { return std::vector<float>(c.b.begin(), c.b.begin() + n); };
  const std::vector<float>& sc = pkg.scales;  // [0] conv_1 out; block b: [1+3b] ReLU 1, [2+3b] ReLU 2, [3+3b] out
  {
    const ChunkedTensor* in[1] = {&u->t};
    KB2_TRY(add(spec(9, false, 12, C, kEpiBias, fp8 ? kOutF16E4m3 : kOutF16Chunk), oihw(pkg.first, C, 3, 1, kFirstIn, 12),
                bias(pkg.first, C), nullptr, in, &s0->t, q_of(&s0->t), sc[0], nullptr, nullptr, k_first, 0));
  }
  const ChunkedTensor* x = &s0->t;
  for (int b = 0; b < pkg.blocks; ++b) {
    const Span8Package::Block& blk = pkg.block[b];
    const bool last = b + 1 == pkg.blocks;
    const float s_in = b == 0 ? sc[0] : sc[3 * b];
    // c1: E4M3 engine -> E4M3 ReLU output (the last block's also in FP16 for conv_cat)
    const ChunkedTensor* in_x[1] = {fp8 ? q_of(x) : x};
    if (fp8) {
      if (last)
        KB2_TRY(add(spec(9, true, C, C, kEpiPrelu, kOutF16E4m3), oihw(blk.c[0], C, 3, 1, kStored, C), bias(blk.c[0], C),
                    &s_in, in_x, &r1_last->t, &r1->t, sc[1 + 3 * b], nullptr, nullptr, k_relu));
      else
        KB2_TRY(add(spec(9, true, C, C, kEpiPrelu, kOutE4m3Chunk), oihw(blk.c[0], C, 3, 1, kStored, C), bias(blk.c[0], C),
                    &s_in, in_x, nullptr, &r1->t, sc[1 + 3 * b], nullptr, nullptr, k_relu));
    } else {
      KB2_TRY(add(spec(9, false, C, C, kEpiPrelu, kOutF16Chunk), oihw(blk.c[0], C, 3, 1, kStored, C), bias(blk.c[0], C),
                  nullptr, in_x, last ? &r1_last->t : &r1->t, nullptr, 1.0f, nullptr, nullptr, k_relu, 1 + 3 * b));
    }
    // c2 reads the E4M3 ReLU output (FP16: the last block's own copy)
    const ChunkedTensor* in_1[1] = {fp8 || !last ? &r1->t : &r1_last->t};
    const float s1 = sc[1 + 3 * b], s2 = sc[2 + 3 * b];
    if (fp8)
      KB2_TRY(add(spec(9, true, C, C, kEpiPrelu, kOutE4m3Chunk), oihw(blk.c[1], C, 3, 1, kStored, C), bias(blk.c[1], C),
                  &s1, in_1, nullptr, &r2->t, s2, nullptr, nullptr, k_relu));
    else
      KB2_TRY(add(spec(9, false, C, C, kEpiPrelu, kOutF16Chunk), oihw(blk.c[1], C, 3, 1, kStored, C), bias(blk.c[1], C),
                  nullptr, in_1, &r2->t, nullptr, 1.0f, nullptr, nullptr, k_relu, 2 + 3 * b));
    const ChunkedTensor* in_2[1] = {&r2->t};
    KB2_TRY(add(spec(9, fp8, C, C, kEpiBias, kOutF16Chunk), oihw(blk.c[2], C, 3, 1, kStored, C), bias(blk.c[2], C),
                fp8 ? &s2 : nullptr, in_2, &c3->t, nullptr, 1.0f, nullptr, nullptr, k_c3));
    // the block output: block 0's is kept for conv_cat; the others alternate between two buffers
    const ChunkedTensor* xo = b == 0 ? &x1->t : (x == &xa->t ? &xb->t : &xa->t);
    const ChunkedTensor* in_3[1] = {&c3->t};
    KB2_TRY(add(spec(1, false, C, C, kEpiTanhGate, fp8 ? kOutF16E4m3 : kOutF16Chunk), oihw(blk.att, C, 1, 1, kStored, C),
                bias(blk.att, C), nullptr, in_3, xo, q_of(xo), sc[3 + 3 * b], x, &c3->t, k_gate, 3 + 3 * b));
    x = xo;
  }
  {
    ConvSpec sp = spec(1, false, C, C, kEpiBias, kOutF16Chunk);
    sp.n_sources = 4;
    const ChunkedTensor* in[4] = {&s0->t, x, &x1->t, &r1_last->t};
    KB2_TRY(add(sp, oihw(pkg.concat, C, 1, 4, kStored, C), bias(pkg.concat, C), nullptr, in, &cat->t, nullptr, 1.0f,
                nullptr, nullptr, k_cat));
  }
  {
    const ChunkedTensor* in[1] = {&cat->t};
    KB2_TRY(add(spec(9, false, C, kPixelOut, kEpiBias, kOutPixShuf4), oihw(pkg.pixel, kPixelOut, 3, 1, kStored, C),
                pkg.pixel.b, nullptr, in, nullptr, nullptr, 1.0f, nullptr, nullptr, k_pix));
  }
  for (auto* t : {&u, &s0, &xa, &xb, &x1, &r1, &r1_last, &r2, &c3, &cat, &s0q, &xaq, &xbq, &x1q})
    if (*t) tensors_.push_back(std::move(*t));
  return Status::Ok();
}

size_t Span8Net::device_bytes() const {
  size_t total = err_.bytes;
  for (const auto& t : tensors_) total += t->buf.bytes;
  for (const auto& l : layers_) total += l->wpack.bytes + l->bias.bytes + l->slope.bytes + l->scale.bytes;
  return total;
}

Status Span8Net::calibrate(cudaStream_t stream, const void* frames, int n, float* peaks_out) {
  if (fp8_) return refuse(KB2_FORMAT_UNSUPPORTED, "unshuffle SPAN: calibration runs on the FP16 engine");
  const int ns = scale_count();
  std::vector<float> best(static_cast<size_t>(ns), 0.0f);
  DeviceBuffer scratch;  // the discarded x2 frames
  KB2_TRY(scratch.alloc(static_cast<size_t>(max_batch_) * 3 * 4 * H_ * W_ * 2));
  std::vector<unsigned int> bits(static_cast<size_t>(ns));
  for (int i = 0; i < n; i += max_batch_) {
    const int batch = n - i < max_batch_ ? n - i : max_batch_;
    KB2_CUDA(cudaMemsetAsync(peaks_.ptr, 0, peaks_.bytes, stream));
    const uint8_t* src = static_cast<const uint8_t*>(frames) + static_cast<size_t>(i) * 3 * H_ * W_ * 2;
    KB2_TRY(run(stream, src, scratch.ptr, batch, peaks_.as<unsigned int>()));
    KB2_CUDA(cudaMemcpyAsync(bits.data(), peaks_.ptr, peaks_.bytes, cudaMemcpyDeviceToHost, stream));
    KB2_CUDA(cudaStreamSynchronize(stream));
    for (int k = 0; k < ns; ++k) {
      float f;
      std::memcpy(&f, &bits[static_cast<size_t>(k)], 4);
      best[static_cast<size_t>(k)] = std::fmax(best[static_cast<size_t>(k)], f);
    }
  }
  std::memcpy(peaks_out, best.data(), best.size() * sizeof(float));
  return Status::Ok();
}

Status Span8Net::run(cudaStream_t stream, const void* in, void* out, int batch, unsigned int* peaks) {
  if (batch < 1 || batch > max_batch_) return refuse(KB2_SHAPE_INVALID, "unshuffle SPAN: batch out of contract");
  {
    const int by = std::max(1, std::min(batch * h_, 65535));
    KB2_TRY(timer_.begin(stream));
    span8_unshuffle_kernel<<<dim3(static_cast<unsigned>((w_ + 127) / 128), static_cast<unsigned>(by)), 128, 0,
                             stream>>>(static_cast<const __half*>(in), unshuffled_->ptr, batch, H_, W_);
    KB2_CUDA(cudaGetLastError());
    KB2_TRY(timer_.end(k_pack_, 0.0, static_cast<double>(batch) * H_ * W_ * 6.0 + batch * h_ * w_ * 32.0, stream));
  }
  const double px = static_cast<double>(batch) * h_ * w_;
  for (const Step& s : steps_) {
    const ConvSpec& sp = s.layer->spec;
    const double flops = 2.0 * sp.taps * sp.n_sources * sp.cin * sp.n_real * px;
    // algorithmic bytes: every FP16 source pixel and residual read once, every output written once
    const double in_b = 16.0 * sp.n_sources * s.layer->args.chunks;
    const double res_b = (s.residual != nullptr ? 2.0 * ch_ : 0.0) + (s.residual2 != nullptr ? 2.0 * ch_ : 0.0);
    const double out_b = (sp.out == kOutE4m3Chunk ? 1.0 : 2.0) * sp.n_real + (s.out2 != nullptr ? sp.n_real : 0.0);
    const double bytes = (in_b + res_b + out_b) * px;
    KB2_TRY(timer_.begin(stream));
    // E4M3-only layers write their one output through `out2`'s tensor
    const ChunkedTensor* o = s.out != nullptr ? s.out : (s.out2 != nullptr && sp.out == kOutE4m3Chunk ? s.out2 : nullptr);
    void* o2 = s.out != nullptr && s.out2 != nullptr ? static_cast<void*>(s.out2->ptr) : nullptr;
    KB2_TRY(s.layer->launch(stream, batch, o != nullptr ? static_cast<void*>(o->ptr) : out,
                            s.residual != nullptr ? s.residual->ptr : nullptr, s.out_inv_scale, 1.0f, o2,
                            s.residual != nullptr ? s.residual->chunks : 0,
                            s.residual2 != nullptr ? s.residual2->ptr : nullptr));
    KB2_TRY(timer_.end(s.kind, flops, bytes, stream));
    if (peaks != nullptr && s.peak >= 0 && o != nullptr) {
      const size_t n2 = static_cast<size_t>(batch) * h_ * o->chunks * w_ * 4;  // 4 half2 per chunk
      KB2_TRY(launch_absmax(stream, o->ptr, n2, peaks + s.peak));
    }
  }
  return Status::Ok();
}

}  // namespace kb2
