// RIFE 4.2x glue on CUDA cores, between the tensor-core convs (rife_net.cu). It replaces the
// reference's fused RIFE entry / glue / finish kernels (src/gpu/cuda/backend/rife_fused_kernels.cu:
// 70, 141, 208) and follows the graph they stand for (src/kernels/spec/rife_fused.h:1-19; its CPU
// statement src/kernels/ref/rife_fused.cpp):
//
//  * block k reads X_k at 1/d_k of the padded frame and leaves Z_k = DepthToSpace(Y_k), 13 channels
//    at 1/d_k (flow 4, mask 1, attributes 8), which the tensor-core transposed conv writes directly
//    as Z pixels of 16 FP16 (32 bytes) [n][Hp/d_k][Wp/d_k];
//  * the flow at a full-resolution pixel is the sum, in block order, of d_i x (Z_i's flow resized by
//    d_i to the pixel), half-pixel linear resize; the mask and attributes X_k reads are Z_{k-1}'s,
//    resized the same way;
//  * X_k (k >= 1), 28 channels: frames A and B warped by their flow halves (3 + 3), the encodings of
//    A and B warped the same (4 + 4), the timestep, the mask and attributes (1 + 8), the flow / d_k
//    (4); X_0, 15 channels: A, B, their encodings and the timestep, unwarped. Both are computed at
//    the full-resolution sample points of the 1/d_k resize and resized there (d_k = 1: no resize);
//  * warps are bilinear with the border clamp over the padded plane (warp_tap, glue_common.cuh);
//    the finish warps both frames by the final flow and blends with sigmoid(mask of the last block).
//
// The resize and warp arithmetic is glue_common.cuh's (resize_tap, warp_tap, lerp_rn), written with
// the _rn intrinsics in the order the network states it.
#pragma once

#include "glue_common.cuh"
#include "tc_common.cuh"

namespace kb2 {

constexpr int kRifeMaxBlocks = 5;
constexpr int kRifeZBytes = 32;  // one Z pixel: 16 FP16 channels, 13 used

// The Z outputs of the blocks so far: Z_i at 1/d_i of the padded plane.
struct RifeZ {
  const uint8_t* z[kRifeMaxBlocks];
  int h[kRifeMaxBlocks], w[kRifeMaxBlocks];
  float d[kRifeMaxBlocks];    // flow scale of block i
  float inv[kRifeMaxBlocks];  // 1 / d_i: resize position factor from the frame to Z_i
};

// Encodings of both frames of every pair, one 8-byte pixel of 4 FP16 channels each, [2 n][Hp][Wp]
// (A of pair n at image 2 n, B at 2 n + 1).
struct RifeEnc {
  const uint2* e;
  __device__ __forceinline__ const uint2* frame(int n, int f, int Hp, int Wp) const {
    return e + static_cast<size_t>(2 * n + f) * Hp * Wp;
  }
};

__device__ __forceinline__ void half4(uint2 q, float c[4]) {
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&q.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&q.y));
  c[0] = a.x;
  c[1] = a.y;
  c[2] = b.x;
  c[3] = b.y;
}

// Backward warp of the 4 channels of a padded plane of 8-byte pixels (`fr`: its first pixel) at
// (Y, X) by flow (fx, fy); the arithmetic of warp3.
__device__ __forceinline__ void warp4(const uint2* fr, int Hp, int Wp, int Y, int X, float fx, float fy, float out[4]) {
  const AxisTap tx = warp_tap(X, fx, Wp);
  const AxisTap ty = warp_tap(Y, fy, Hp);
  __half2 c01, c23;
  bilerp_h2(fr, Wp, tx, ty, c01, c23);
  const float2 a = __half22float2(c01);
  const float2 b = __half22float2(c23);
  out[0] = a.x;
  out[1] = a.y;
  out[2] = b.x;
  out[3] = b.y;
}

// Rows a glue thread walks down its column: its column's resize taps and source caches are set
// once per run; runs never cross frames.
constexpr int kRifeRunRows = 8;

// The first kCh channels of a Z pixel (4: the flow; 13: flow, mask and attributes).
template <int kCh>
__device__ __forceinline__ void load_z(const uint8_t* px, float q[kCh]) {
  if constexpr (kCh == 4) {
    half4(__ldg(reinterpret_cast<const uint2*>(px)), q);
  } else {
    const uint4 lo = __ldg(reinterpret_cast<const uint4*>(px));
    const uint4 hi = __ldg(reinterpret_cast<const uint4*>(px + 16));
    const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
    for (int j = 0; j < kCh; ++j) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j >> 1]));
      q[j] = (j & 1) ? f.y : f.x;
    }
  }
}

// Column cache of Z_i at one full-resolution column X: the x tap of its resize (fixed), the source
// row pair last loaded (lo; hi follows from it) and both rows' kCh channels interpolated in x. A
// thread walking rows down its column reloads it once per source row pair, every d_i rows; the
// value at a row is lerp(lerp(q00, q01, tx), lerp(q10, q11, tx), ty), the resize's order.
template <int kCh>
struct ZCol {
  int x0, x1, lo;
  float tx;
  float top[kCh], bot[kCh];
};

template <int kCh>
__device__ __forceinline__ void zcol_init(const RifeZ& Z, int i, int X, ZCol<kCh>& c) {
  const AxisTap t = resize_tap(X, Z.inv[i], Z.w[i]);
  c.x0 = t.lo;
  c.x1 = t.hi;
  c.tx = t.t;
  c.lo = -1;
}

template <int kCh>
__device__ __forceinline__ void zcol_at(const RifeZ& Z, int i, int n, int Y, ZCol<kCh>& c, float out[kCh]) {
  const AxisTap ty = resize_tap(Y, Z.inv[i], Z.h[i]);
  if (ty.lo != c.lo) {
    const uint8_t* base = Z.z[i] + static_cast<size_t>(n) * Z.h[i] * Z.w[i] * kRifeZBytes;
    const uint8_t* r0 = base + static_cast<size_t>(ty.lo) * Z.w[i] * kRifeZBytes;
    const uint8_t* r1 = base + static_cast<size_t>(ty.hi) * Z.w[i] * kRifeZBytes;
    float q00[kCh], q01[kCh], q10[kCh], q11[kCh];
    load_z<kCh>(r0 + c.x0 * kRifeZBytes, q00);
    load_z<kCh>(r0 + c.x1 * kRifeZBytes, q01);
    load_z<kCh>(r1 + c.x0 * kRifeZBytes, q10);
    load_z<kCh>(r1 + c.x1 * kRifeZBytes, q11);
#pragma unroll
    for (int ch = 0; ch < kCh; ++ch) {
      c.top[ch] = lerp_rn(q00[ch], q01[ch], c.tx);
      c.bot[ch] = lerp_rn(q10[ch], q11[ch], c.tx);
    }
    c.lo = ty.lo;
  }
#pragma unroll
  for (int ch = 0; ch < kCh; ++ch) out[ch] = lerp_rn(c.top[ch], c.bot[ch], ty.t);
}

// f += d_i x (Z_i's flow resized to row Y), in block order (i = 0 sets f).
template <int kCh>
__device__ __forceinline__ void add_flow(const RifeZ& Z, int i, const float (&z)[kCh], float f[4]) {
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) {
    const float s = __fmul_rn(z[ch], Z.d[i]);
    f[ch] = i == 0 ? s : __fadd_rn(f[ch], s);
  }
}

// The flow after blocks 0 .. K - 1 at row Y of the caches' column.
template <int K>
__device__ __forceinline__ void cached_flow(const RifeZ& Z, int n, int Y, ZCol<4> (&c)[K], float f[4]) {
#pragma unroll
  for (int i = 0; i < K; ++i) {
    float z[4];
    zcol_at<4>(Z, i, n, Y, c[i], z);
    add_flow<4>(Z, i, z, f);
  }
}

// The sources of block K's input at one column: Z_0 .. Z_(K-2) for the flow, Z_(K-1) for the flow,
// mask and attributes.
template <int K>
struct BlockCols {
  ZCol<4> flow[K > 1 ? K - 1 : 1];
  ZCol<13> last;
};

template <int K>
__device__ __forceinline__ void block_cols_init(const RifeZ& Z, int X, BlockCols<K>& c) {
#pragma unroll
  for (int i = 0; i + 1 < K; ++i) zcol_init<4>(Z, i, X, c.flow[i]);
  zcol_init<13>(Z, K - 1, X, c.last);
}

// Chunk q (channels 8 q .. 8 q + 7) of one X pixel into its parity-split chunk row (the layout
// conv0a's stride-2 loads read): rows of `chunks` chunks of wo pixels.
__device__ __forceinline__ void store_chunk8(uint8_t* out, int chunks, int ho, int wo, int n, int oy, int ox, int q,
                                             const float (&c)[8]) {
  uint4 o;
  o.x = pack_half2(c[0], c[1]);
  o.y = pack_half2(c[2], c[3]);
  o.z = pack_half2(c[4], c[5]);
  o.w = pack_half2(c[6], c[7]);
  const int xs = (ox & 1) * (wo >> 1) + (ox >> 1);
  *reinterpret_cast<uint4*>(out + (((static_cast<size_t>(n) * ho + oy) * chunks + q) * wo + xs) * 16) = o;
}

// The resize of a quad's four sample points (lanes 4 p + 2 sy + sx) to their output pixel, as the
// 1/d resize does it (x first, then y), by shuffles; every lane of the quad ends with the result.
__device__ __forceinline__ void quad_resize(float (&c)[8], int sx, int sy, float tx, float ty) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float p = __shfl_xor_sync(0xffffffffu, c[j], 1);
    const float h = sx ? lerp_rn(p, c[j], tx) : lerp_rn(c[j], p, tx);
    const float o = __shfl_xor_sync(0xffffffffu, h, 2);
    c[j] = sy ? lerp_rn(o, h, ty) : lerp_rn(h, o, ty);
  }
}

// Emits chunk q of an X pixel: d = 1 stores it; d >= 2 resizes it over the quad and the quad's lane
// q (sx + 2 sy) stores it. `scale`: a factor applied after the resize (the flow's 1 / d).
__device__ __forceinline__ void emit_chunk(float (&c)[8], int q, bool quad, int sx, int sy, float tx, float ty,
                                           float scale, bool live, uint8_t* out, int chunks, int ho, int wo, int n,
                                           int oy, int ox) {
  if (quad) quad_resize(c, sx, sy, tx, ty);
  if (scale != 1.0f) {
#pragma unroll
    for (int j = 0; j < 8; ++j) c[j] = __fmul_rn(c[j], scale);
  }
  if (live && (!quad || q == sx + 2 * sy)) store_chunk8(out, chunks, ho, wo, n, oy, ox, q, c);
}

// NCHW frames -> padded RGBx pixels (zeros outside the window), and the encoder's input: the same
// pixels as one chunk of 8 FP16 channels (3 used) in parity-split rows, images interleaved A, B
// per pair ([2 n][Hp][1][Wp][16 B]).
__global__ void rife_pad_frames_kernel(IfFrames F, int batch, uint8_t* __restrict__ enc_in) {
  const size_t plane = static_cast<size_t>(F.H) * F.W;
  const int X = blockIdx.x * blockDim.x + threadIdx.x;
  if (X >= F.Wp) return;
  const int xs = (X & 1) * (F.Wp >> 1) + (X >> 1);
  for (int r = blockIdx.y; r < batch * F.Hp; r += gridDim.y) {
    const int n = r / F.Hp;
    const int Y = r - n * F.Hp;
    const size_t i = static_cast<size_t>(r) * F.Wp + X;
    const int y = Y - F.top, x = X - F.left;
    uint2 p0 = make_uint2(0, 0), p1 = make_uint2(0, 0);
    if (y >= 0 && y < F.H && x >= 0 && x < F.W) {
      const size_t at = static_cast<size_t>(n) * 3 * plane + static_cast<size_t>(y) * F.W + x;
      const __half z = __float2half_rn(0.0f);
      const __half2 a01 = __halves2half2(F.img0[at], F.img0[at + plane]);
      const __half2 a2 = __halves2half2(F.img0[at + 2 * plane], z);
      const __half2 b01 = __halves2half2(F.img1[at], F.img1[at + plane]);
      const __half2 b2 = __halves2half2(F.img1[at + 2 * plane], z);
      p0 = make_uint2(*reinterpret_cast<const uint32_t*>(&a01), *reinterpret_cast<const uint32_t*>(&a2));
      p1 = make_uint2(*reinterpret_cast<const uint32_t*>(&b01), *reinterpret_cast<const uint32_t*>(&b2));
    }
    F.pad0[i] = p0;
    F.pad1[i] = p1;
    const size_t ea = (static_cast<size_t>(2 * n) * F.Hp + Y) * F.Wp + xs;
    const size_t eb = (static_cast<size_t>(2 * n + 1) * F.Hp + Y) * F.Wp + xs;
    reinterpret_cast<uint4*>(enc_in)[ea] = make_uint4(p0.x, p0.y, 0, 0);
    reinterpret_cast<uint4*>(enc_in)[eb] = make_uint4(p1.x, p1.y, 0, 0);
  }
}

// X_0 (15 channels in 2 chunks: A, B, their encodings and the timestep) at 1/d, d >= 2: four
// threads per output pixel, one per sample point of the resize (lanes 4 p + 2 sy + sx), each walking
// kRifeRunRows output rows down its sample column; the quad resizes each chunk by shuffles.
__global__ void __launch_bounds__(kGlueThreads) rife_first_input_kernel(IfFrames F, RifeEnc E, int d, int batch,
                                                                        float timestep, uint8_t* __restrict__ out) {
  const int ho = F.Hp / d, wo = F.Wp / d;
  const int runs = (ho + kRifeRunRows - 1) / kRifeRunRows;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int ox = t >> 2, sx = t & 1, sy = (t >> 1) & 1;
  const bool live = ox < wo;  // the quad agrees; the shuffles need every lane of the warp
  const AxisTap tx = resize_tap(live ? ox : wo - 1, static_cast<float>(d), F.Wp);
  const int X = sx ? tx.hi : tx.lo;
  for (int r = blockIdx.y; r < batch * runs; r += gridDim.y) {
    const int n = r / runs;
    const int oy0 = (r - n * runs) * kRifeRunRows;
    const int oy1 = min(oy0 + kRifeRunRows, ho);
    const size_t frame = static_cast<size_t>(n) * F.Hp * F.Wp;
    for (int oy = oy0; oy < oy1; ++oy) {
      const AxisTap ty = resize_tap(oy, static_cast<float>(d), F.Hp);
      const int Y = sy ? ty.hi : ty.lo;
      const size_t at = static_cast<size_t>(Y) * F.Wp + X;
      float ea[4], eb[4];
      half4(__ldg(E.frame(n, 0, F.Hp, F.Wp) + at), ea);
      half4(__ldg(E.frame(n, 1, F.Hp, F.Wp) + at), eb);
      float c[8];
      frame_rgb(F.pad0 + frame, F.Wp, Y, X, c);
      frame_rgb(F.pad1 + frame, F.Wp, Y, X, c + 3);
      c[6] = ea[0];
      c[7] = ea[1];
      emit_chunk(c, 0, true, sx, sy, tx.t, ty.t, 1.0f, live, out, 2, ho, wo, n, oy, ox);
      c[0] = ea[2];
      c[1] = ea[3];
#pragma unroll
      for (int j = 0; j < 4; ++j) c[2 + j] = eb[j];
      c[6] = timestep;
      c[7] = 0.0f;
      emit_chunk(c, 1, true, sx, sy, tx.t, ty.t, 1.0f, live, out, 2, ho, wo, n, oy, ox);
    }
  }
}

// X_K of block K >= 1 (28 channels in 4 chunks) at 1/d. d = 1: one thread per pixel column; d >= 2:
// four threads per output pixel as rife_first_input_kernel. Each thread walks kRifeRunRows output
// rows down its sample column with the column caches of Z_0 .. Z_(K-1), and emits the chunks one
// at a time: 3 (flow / d), 2 (attributes), 0 (warped A, B and encoding of A, first half), 1 (the rest
// of the encodings, the timestep and the mask).
template <int K>
__global__ void __launch_bounds__(kGlueThreads, 2)
    rife_block_input_kernel(IfFrames F, RifeEnc E, RifeZ Z, int d, int batch, float timestep,
                            uint8_t* __restrict__ out) {
  static_assert(K >= 1 && K < kRifeMaxBlocks, "block 1 .. 4");
  const int ho = F.Hp / d, wo = F.Wp / d;
  const int runs = (ho + kRifeRunRows - 1) / kRifeRunRows;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const bool quad = d >= 2;
  const int ox = quad ? t >> 2 : t;
  const int sx = quad ? (t & 1) : 0, sy = quad ? ((t >> 1) & 1) : 0;
  const bool live = ox < wo;
  if (!quad && !live) return;  // d = 1: no lane exchanges
  const AxisTap tx = quad ? resize_tap(live ? ox : wo - 1, static_cast<float>(d), F.Wp) : AxisTap{ox, ox, 0.0f};
  const int X = sx ? tx.hi : tx.lo;
  const float inv = __fdiv_rn(1.0f, static_cast<float>(d));
  BlockCols<K> cols;
  block_cols_init<K>(Z, X, cols);
  for (int r = blockIdx.y; r < batch * runs; r += gridDim.y) {
    const int n = r / runs;
    const int oy0 = (r - n * runs) * kRifeRunRows;
    const int oy1 = min(oy0 + kRifeRunRows, ho);
#pragma unroll
    for (int i = 0; i + 1 < K; ++i) cols.flow[i].lo = -1;
    cols.last.lo = -1;
    const size_t frame = static_cast<size_t>(n) * F.Hp * F.Wp;
    for (int oy = oy0; oy < oy1; ++oy) {
      const AxisTap ty = quad ? resize_tap(oy, static_cast<float>(d), F.Hp) : AxisTap{oy, oy, 0.0f};
      const int Y = sy ? ty.hi : ty.lo;
      float f[4];
#pragma unroll
      for (int i = 0; i + 1 < K; ++i) {
        float z[4];
        zcol_at<4>(Z, i, n, Y, cols.flow[i], z);
        add_flow<4>(Z, i, z, f);
      }
      float za[13];
      zcol_at<13>(Z, K - 1, n, Y, cols.last, za);
      add_flow<13>(Z, K - 1, za, f);
      float c[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        c[j] = f[j];
        c[4 + j] = 0.0f;
      }
      emit_chunk(c, 3, quad, sx, sy, tx.t, ty.t, inv, live, out, 4, ho, wo, n, oy, ox);
#pragma unroll
      for (int j = 0; j < 8; ++j) c[j] = za[5 + j];
      emit_chunk(c, 2, quad, sx, sy, tx.t, ty.t, 1.0f, live, out, 4, ho, wo, n, oy, ox);
      const float mask = za[4];
      float ea[4], eb[4];
      warp3(F.pad0 + frame, F, Y, X, f[0], f[1], c);
      warp3(F.pad1 + frame, F, Y, X, f[2], f[3], c + 3);
      warp4(E.frame(n, 0, F.Hp, F.Wp), F.Hp, F.Wp, Y, X, f[0], f[1], ea);
      warp4(E.frame(n, 1, F.Hp, F.Wp), F.Hp, F.Wp, Y, X, f[2], f[3], eb);
      c[6] = ea[0];
      c[7] = ea[1];
      emit_chunk(c, 0, quad, sx, sy, tx.t, ty.t, 1.0f, live, out, 4, ho, wo, n, oy, ox);
      c[0] = ea[2];
      c[1] = ea[3];
#pragma unroll
      for (int j = 0; j < 4; ++j) c[2 + j] = eb[j];
      c[6] = timestep;
      c[7] = mask;
      emit_chunk(c, 1, quad, sx, sy, tx.t, ty.t, 1.0f, live, out, 4, ho, wo, n, oy, ox);
    }
  }
}

// The final flow at row Y of a column: blocks 0 .. L - 1 through the column caches, then the last
// block's own (d = 1: read in place), and its mask logit.
template <int L>
__device__ __forceinline__ void final_flow(const RifeZ& Z, int n, int Y, int X, ZCol<4> (&cols)[L], float f[4],
                                           float* mask) {
  cached_flow<L>(Z, n, Y, cols, f);
  const uint8_t* px = Z.z[L] + ((static_cast<size_t>(n) * Z.h[L] + Y) * Z.w[L] + X) * kRifeZBytes;
  const uint4 q = __ldg(reinterpret_cast<const uint4*>(px));
  float a[4], b[4];
  half4(make_uint2(q.x, q.y), a);
  half4(make_uint2(q.z, q.w), b);
#pragma unroll
  for (int c = 0; c < 4; ++c) f[c] = __fadd_rn(f[c], a[c]);
  *mask = b[0];
}

// The interpolated frame in the window: out = warp(A) m + warp(B) (1 - m), m = sigmoid(mask),
// NCHW FP16 [n][3][H][W]; L = the last block's index. One thread per column walking kRifeRunRows
// rows with the column caches of Z_0 .. Z_(L-1). Four blocks an SM (64 registers, no spills): the
// gathers' latency wants the warps; at the compiler's own 128 registers the kernel ran 35 % slower.
template <int L>
__global__ void __launch_bounds__(kGlueThreads, 4) rife_finish_kernel(IfFrames F, RifeZ Z, int batch,
                                                                   __half* __restrict__ out) {
  const int x = blockIdx.x * blockDim.x + threadIdx.x;
  if (x >= F.W) return;
  const int X = x + F.left;
  ZCol<4> cols[L];
#pragma unroll
  for (int i = 0; i < L; ++i) zcol_init<4>(Z, i, X, cols[i]);
  const int runs = (F.H + kRifeRunRows - 1) / kRifeRunRows;
  for (int r = blockIdx.y; r < batch * runs; r += gridDim.y) {
    const int n = r / runs;
    const int y0 = (r - n * runs) * kRifeRunRows;
#pragma unroll
    for (int i = 0; i < L; ++i) cols[i].lo = -1;
    const size_t frame = static_cast<size_t>(n) * F.Hp * F.Wp;
    for (int y = y0; y < min(y0 + kRifeRunRows, F.H); ++y) {
      const int Y = y + F.top;
      float f[4], mask;
      final_flow<L>(Z, n, Y, X, cols, f, &mask);
      float w0[3], w1[3];
      warp3(F.pad0 + frame, F, Y, X, f[0], f[1], w0);
      warp3(F.pad1 + frame, F, Y, X, f[2], f[3], w1);
      const float m = __fdiv_rn(1.0f, __fadd_rn(1.0f, __expf(-mask)));
      const float m1 = __fsub_rn(1.0f, m);
      __half* o = out + (static_cast<size_t>(n) * 3 * F.H + y) * F.W + x;
#pragma unroll
      for (int c = 0; c < 3; ++c)
        o[static_cast<size_t>(c) * F.H * F.W] = __float2half_rn(__fadd_rn(__fmul_rn(w0[c], m), __fmul_rn(w1[c], m1)));
    }
  }
}

// The motion variant over the padded plane: the final flow [n][4][Hp][Wp] and sigmoid(mask)
// [n][1][Hp][Wp], T = float or __half; the walk of rife_finish_kernel.
template <int L, typename T>
__global__ void __launch_bounds__(kGlueThreads, 4) rife_motion_kernel(IfFrames F, RifeZ Z, int batch,
                                                                   T* __restrict__ flow, T* __restrict__ mask) {
  const int X = blockIdx.x * blockDim.x + threadIdx.x;
  if (X >= F.Wp) return;
  ZCol<4> cols[L];
#pragma unroll
  for (int i = 0; i < L; ++i) zcol_init<4>(Z, i, X, cols[i]);
  const size_t pl = static_cast<size_t>(F.Hp) * F.Wp;
  const int runs = (F.Hp + kRifeRunRows - 1) / kRifeRunRows;
  for (int r = blockIdx.y; r < batch * runs; r += gridDim.y) {
    const int n = r / runs;
    const int y0 = (r - n * runs) * kRifeRunRows;
#pragma unroll
    for (int i = 0; i < L; ++i) cols[i].lo = -1;
    for (int Y = y0; Y < min(y0 + kRifeRunRows, F.Hp); ++Y) {
      float f[4], m;
      final_flow<L>(Z, n, Y, X, cols, f, &m);
      const size_t at = static_cast<size_t>(Y) * F.Wp + X;
#pragma unroll
      for (int c = 0; c < 4; ++c) store_motion(flow + (static_cast<size_t>(n) * 4 + c) * pl + at, f[c]);
      store_motion(mask + static_cast<size_t>(n) * pl + at, __fdiv_rn(1.0f, __fadd_rn(1.0f, __expf(-m))));
    }
  }
}

}  // namespace kb2
