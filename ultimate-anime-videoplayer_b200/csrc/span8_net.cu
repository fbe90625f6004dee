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
// ReLU is the PReLU epilogue with zero slopes. The E4M3 blocks of an FP8 package are not run: every
// package runs in FP16 (its weights are FP16 in the file; the FP8 scales are read and checked only).
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>

#include "span8_net.h"

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

Status Span8Net::make_tensor(std::unique_ptr<Tensor>& t, int chunks) {
  t = std::make_unique<Tensor>();
  t->t.batch = max_batch_;
  t->t.H = h_;
  t->t.W = w_;
  t->t.chunks = chunks;
  t->t.fp8 = false;
  KB2_TRY(t->buf.alloc(t->t.bytes()));
  KB2_CUDA(cudaMemset(t->buf.ptr, 0, t->t.bytes()));
  t->t.ptr = t->buf.as<uint8_t>();
  return Status::Ok();
}

Status Span8Net::create(const Span8Package& pkg, int max_batch, int H, int W) {
  if (H % 2 != 0 || W % 2 != 0) return refuse(KB2_SHAPE_INVALID, "unshuffle SPAN: even frame height and width");
  if (H < 4 || W < 4) return refuse(KB2_SHAPE_INVALID, "unshuffle SPAN: frame too small");
  max_batch_ = max_batch;
  H_ = H;
  W_ = W;
  h_ = H / 2;
  w_ = W / 2;
  ch_ = pkg.real;
  const int C = ch_, cc = C / 8;
  KB2_TRY(err_.alloc(sizeof(int)));
  KB2_CUDA(cudaMemset(err_.ptr, 0, sizeof(int)));
  int* err = err_.as<int>();
  k_pack_ = timer_.kind("span8.unshuffle");
  const int k_first = timer_.kind("span8.conv_1"), k_relu = timer_.kind("span8.block_relu_conv");
  const int k_c3 = timer_.kind("span8.block_c3"), k_gate = timer_.kind("span8.block_att_gate");
  const int k_cat = timer_.kind("span8.conv_cat"), k_pix = timer_.kind("span8.to_pixel");

  std::unique_ptr<Tensor> u, s0, xa, xb, x1, r1, r1_last, r2, c3, cat;
  KB2_TRY(make_tensor(u, 2));
  KB2_TRY(make_tensor(s0, cc));
  KB2_TRY(make_tensor(xa, cc));
  KB2_TRY(make_tensor(xb, cc));
  KB2_TRY(make_tensor(x1, cc));
  KB2_TRY(make_tensor(r1, cc));
  KB2_TRY(make_tensor(r1_last, cc));
  KB2_TRY(make_tensor(r2, cc));
  KB2_TRY(make_tensor(c3, cc));
  KB2_TRY(make_tensor(cat, cc));
  unshuffled_ = &u->t;

  auto add = [&](const ConvSpec& s, const std::vector<float>& w, const std::vector<float>& b,
                 const ChunkedTensor* const* inputs, const ChunkedTensor* out, const ChunkedTensor* res,
                 const ChunkedTensor* res2, int kind) -> Status {
    auto l = std::make_unique<ConvLayer>();
    KB2_TRY(l->build(s, w.data(), b.data(), nullptr, nullptr, inputs, err));
    steps_.push_back(Step{l.get(), out, res, res2, kind});
    layers_.push_back(std::move(l));
    return Status::Ok();
  };
  auto conv3 = [&](int cin, int n_pad, int epi, int out_fmt, int out_chunks) {
    ConvSpec s;
    s.taps = 9;
    s.cin = cin;
    s.n_real = n_pad;
    s.n_pad = n_pad;
    s.epi = epi;
    s.out = out_fmt;
    s.out_chunks = out_chunks;
    return s;
  };
  const std::vector<float> bias_c(pkg.first.b.begin(), pkg.first.b.begin() + C);
  {
    const ChunkedTensor* in[1] = {&u->t};
    KB2_TRY(add(conv3(12, C, kEpiBias, kOutF16Chunk, cc), oihw(pkg.first, C, 3, 1, kFirstIn, 12), bias_c, in, &s0->t,
                nullptr, nullptr, k_first));
  }
  const ChunkedTensor* x = &s0->t;
  for (int b = 0; b < pkg.blocks; ++b) {
    const Span8Package::Block& blk = pkg.block[b];
    auto bias = [&](const Span8Package::Conv& c) { return std::vector<float>(c.b.begin(), c.b.begin() + C); };
    const bool last = b + 1 == pkg.blocks;
    const ChunkedTensor* t1 = last ? &r1_last->t : &r1->t;
    const ChunkedTensor* in_x[1] = {x};
    KB2_TRY(add(conv3(C, C, kEpiPrelu, kOutF16Chunk, cc), oihw(blk.c[0], C, 3, 1, kStored, C), bias(blk.c[0]), in_x,
                t1, nullptr, nullptr, k_relu));
    const ChunkedTensor* in_1[1] = {t1};
    KB2_TRY(add(conv3(C, C, kEpiPrelu, kOutF16Chunk, cc), oihw(blk.c[1], C, 3, 1, kStored, C), bias(blk.c[1]), in_1,
                &r2->t, nullptr, nullptr, k_relu));
    const ChunkedTensor* in_2[1] = {&r2->t};
    KB2_TRY(add(conv3(C, C, kEpiBias, kOutF16Chunk, cc), oihw(blk.c[2], C, 3, 1, kStored, C), bias(blk.c[2]), in_2,
                &c3->t, nullptr, nullptr, k_c3));
    // the block output: block 0's is kept for conv_cat; the others alternate between two buffers
    const ChunkedTensor* xo = b == 0 ? &x1->t : (x == &xa->t ? &xb->t : &xa->t);
    ConvSpec g;
    g.taps = 1;
    g.cin = C;
    g.n_real = C;
    g.n_pad = C;
    g.epi = kEpiTanhGate;
    g.out = kOutF16Chunk;
    g.out_chunks = cc;
    const ChunkedTensor* in_3[1] = {&c3->t};
    KB2_TRY(add(g, oihw(blk.att, C, 1, 1, kStored, C), bias(blk.att), in_3, xo, x, &c3->t, k_gate));
    x = xo;
  }
  {
    ConvSpec s;
    s.taps = 1;
    s.n_sources = 4;
    s.cin = C;
    s.n_real = C;
    s.n_pad = C;
    s.epi = kEpiBias;
    s.out = kOutF16Chunk;
    s.out_chunks = cc;
    const ChunkedTensor* in[4] = {&s0->t, x, &x1->t, &r1_last->t};
    KB2_TRY(add(s, oihw(pkg.concat, C, 1, 4, kStored, C), std::vector<float>(pkg.concat.b.begin(), pkg.concat.b.begin() + C),
                in, &cat->t, nullptr, nullptr, k_cat));
  }
  {
    const ChunkedTensor* in[1] = {&cat->t};
    KB2_TRY(add(conv3(C, kPixelOut, kEpiBias, kOutPixShuf4, 0), oihw(pkg.pixel, kPixelOut, 3, 1, kStored, C), pkg.pixel.b,
                in, nullptr, nullptr, nullptr, k_pix));
  }
  for (auto* t : {&u, &s0, &xa, &xb, &x1, &r1, &r1_last, &r2, &c3, &cat}) tensors_.push_back(std::move(*t));
  return Status::Ok();
}

size_t Span8Net::device_bytes() const {
  size_t total = err_.bytes;
  for (const auto& t : tensors_) total += t->buf.bytes;
  for (const auto& l : layers_) total += l->wpack.bytes + l->bias.bytes + l->slope.bytes + l->scale.bytes;
  return total;
}

Status Span8Net::run(cudaStream_t stream, const void* in, void* out, int batch) {
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
    const double in_b = 2.0 * sp.n_sources * s.layer->args.chunks * 8;
    const double res_b = (s.residual != nullptr ? 2.0 * ch_ : 0.0) + (s.residual2 != nullptr ? 2.0 * ch_ : 0.0);
    const double out_b = 2.0 * sp.n_real;
    const double bytes = (in_b + res_b + out_b) * px;
    KB2_TRY(timer_.begin(stream));
    KB2_TRY(s.layer->launch(stream, batch, s.out != nullptr ? static_cast<void*>(s.out->ptr) : out,
                            s.residual != nullptr ? s.residual->ptr : nullptr, 1.0f, 1.0f, nullptr,
                            s.residual != nullptr ? s.residual->chunks : 0,
                            s.residual2 != nullptr ? s.residual2->ptr : nullptr));
    KB2_TRY(timer_.end(s.kind, flops, bytes, stream));
  }
  return Status::Ok();
}

}  // namespace kb2
