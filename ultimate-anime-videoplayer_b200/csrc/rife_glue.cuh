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
  const float wx1 = __fsub_rn(1.0f, tx.t), wy1 = __fsub_rn(1.0f, ty.t);
  float a[4], b[4], d[4], e[4];
  half4(__ldg(fr + (static_cast<size_t>(ty.lo) * Wp + tx.lo)), a);
  half4(__ldg(fr + (static_cast<size_t>(ty.lo) * Wp + tx.hi)), b);
  half4(__ldg(fr + (static_cast<size_t>(ty.hi) * Wp + tx.lo)), d);
  half4(__ldg(fr + (static_cast<size_t>(ty.hi) * Wp + tx.hi)), e);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float top = __fadd_rn(__fmul_rn(a[c], wx1), __fmul_rn(b[c], tx.t));
    const float bot = __fadd_rn(__fmul_rn(d[c], wx1), __fmul_rn(e[c], tx.t));
    out[c] = __fadd_rn(__fmul_rn(top, wy1), __fmul_rn(bot, ty.t));
  }
}

// The `kCh` first channels (4: the flow; 13: all) of Z_i (frame n) resized to full-resolution
// pixel (Y, X): lerp(lerp(q00, q01, tx), lerp(q10, q11, tx), ty), x first.
template <int kCh>
__device__ __forceinline__ void z_at(const RifeZ& Z, int i, int n, int Y, int X, float out[kCh]) {
  const AxisTap tx = resize_tap(X, Z.inv[i], Z.w[i]);
  const AxisTap ty = resize_tap(Y, Z.inv[i], Z.h[i]);
  const uint8_t* base = Z.z[i] + static_cast<size_t>(n) * Z.h[i] * Z.w[i] * kRifeZBytes;
  const uint8_t* px[4] = {base + (static_cast<size_t>(ty.lo) * Z.w[i] + tx.lo) * kRifeZBytes,
                          base + (static_cast<size_t>(ty.lo) * Z.w[i] + tx.hi) * kRifeZBytes,
                          base + (static_cast<size_t>(ty.hi) * Z.w[i] + tx.lo) * kRifeZBytes,
                          base + (static_cast<size_t>(ty.hi) * Z.w[i] + tx.hi) * kRifeZBytes};
  float q[4][kCh];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if constexpr (kCh == 4) {
      half4(__ldg(reinterpret_cast<const uint2*>(px[k])), q[k]);
    } else {
      const uint4 lo = __ldg(reinterpret_cast<const uint4*>(px[k]));
      const uint4 hi = __ldg(reinterpret_cast<const uint4*>(px[k] + 16));
      const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
      for (int j = 0; j < kCh; ++j) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j >> 1]));
        q[k][j] = (j & 1) ? f.y : f.x;
      }
    }
  }
#pragma unroll
  for (int c = 0; c < kCh; ++c)
    out[c] = lerp_rn(lerp_rn(q[0][c], q[1][c], tx.t), lerp_rn(q[2][c], q[3][c], tx.t), ty.t);
}

// The flow after blocks 0 .. K - 1 at full-resolution pixel (Y, X): sum of d_i x resized Z_i flow.
__device__ __forceinline__ void flow_at(const RifeZ& Z, int K, int n, int Y, int X, float f[4]) {
#pragma unroll 1
  for (int i = 0; i < K; ++i) {
    float v[4];
    z_at<4>(Z, i, n, Y, X, v);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float s = __fmul_rn(v[c], Z.d[i]);
      f[c] = i == 0 ? s : __fadd_rn(f[c], s);
    }
  }
}

// The 28 channels of X_K (K >= 1) at full-resolution pixel (Y, X), before its 1/d_K resize; the
// flow channels are not yet divided by d_K.
__device__ __forceinline__ void block_channels(const IfFrames& F, const RifeEnc& E, const RifeZ& Z, int K, int n, int Y,
                                               int X, float timestep, float v[28]) {
  float f[4];
  flow_at(Z, K, n, Y, X, f);
  const size_t frame = static_cast<size_t>(n) * F.Hp * F.Wp;
  warp3(F.pad0 + frame, F, Y, X, f[0], f[1], v);
  warp3(F.pad1 + frame, F, Y, X, f[2], f[3], v + 3);
  warp4(E.frame(n, 0, F.Hp, F.Wp), F.Hp, F.Wp, Y, X, f[0], f[1], v + 6);
  warp4(E.frame(n, 1, F.Hp, F.Wp), F.Hp, F.Wp, Y, X, f[2], f[3], v + 10);
  v[14] = timestep;
  float za[13];
  z_at<13>(Z, K - 1, n, Y, X, za);
#pragma unroll
  for (int c = 0; c < 9; ++c) v[15 + c] = za[4 + c];
#pragma unroll
  for (int c = 0; c < 4; ++c) v[24 + c] = f[c];
}

// The 15 channels of X_0 at full-resolution pixel (Y, X).
__device__ __forceinline__ void first_channels(const IfFrames& F, const RifeEnc& E, int n, int Y, int X,
                                               float timestep, float v[15]) {
  const size_t frame = static_cast<size_t>(n) * F.Hp * F.Wp;
  frame_rgb(F.pad0 + frame, F.Wp, Y, X, v);
  frame_rgb(F.pad1 + frame, F.Wp, Y, X, v + 3);
  half4(__ldg(E.frame(n, 0, F.Hp, F.Wp) + (static_cast<size_t>(Y) * F.Wp + X)), v + 6);
  half4(__ldg(E.frame(n, 1, F.Hp, F.Wp) + (static_cast<size_t>(Y) * F.Wp + X)), v + 10);
  v[14] = timestep;
}

// Chunk `q` (channels 8 q .. 8 q + 7, zeros beyond kC) of one X pixel into its parity-split chunk
// row (the layout conv0a's stride-2 loads read): rows of `chunks` chunks of wo pixels.
template <int kC>
__device__ __forceinline__ void store_x_chunk(uint8_t* out, int chunks, int ho, int wo, int n, int oy, int ox, int q,
                                              const float (&v)[kC]) {
  float c8[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) c8[j] = 0.0f;
#pragma unroll
  for (int qq = 0; qq < (kC + 7) / 8; ++qq)
    if (qq == q) {
#pragma unroll
      for (int j = 0; j < 8; ++j) c8[j] = 8 * qq + j < kC ? v[8 * qq + j] : 0.0f;
    }
  uint4 o;
  o.x = pack_half2(c8[0], c8[1]);
  o.y = pack_half2(c8[2], c8[3]);
  o.z = pack_half2(c8[4], c8[5]);
  o.w = pack_half2(c8[6], c8[7]);
  const int xs = (ox & 1) * (wo >> 1) + (ox >> 1);
  *reinterpret_cast<uint4*>(out + (((static_cast<size_t>(n) * ho + oy) * chunks + q) * wo + xs) * 16) = o;
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

// X_K of block K at 1/d (ho x wo, `chunks` chunks: 2 for X_0, 4 after) for output rows walked along
// blockIdx.y. d >= 2: four threads per output pixel, one per sample point of the resize (lanes
// 4 p + 2 sy + sx); each computes the channels at its point, the quad combines them as the resize
// does (x first, then y) by shuffles, and thread sx + 2 sy stores chunk sx + 2 sy. d = 1: one thread
// per pixel stores every chunk.
template <int kC>
__global__ void __launch_bounds__(kGlueThreads, 2)
    rife_block_input_kernel(IfFrames F, RifeEnc E, RifeZ Z, int K, int d, int batch, float timestep,
                            uint8_t* __restrict__ out) {
  static_assert(kC == 15 || kC == 28, "X_0 or X_k");
  constexpr int chunks = (kC + 7) / 8 + ((kC + 7) / 8 & 1);  // 15 -> 2, 28 -> 4
  const int ho = F.Hp / d, wo = F.Wp / d;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (d == 1) {
    const int ox = t;
    if (ox >= wo) return;
    for (int r = blockIdx.y; r < batch * ho; r += gridDim.y) {
      const int n = r / ho;
      const int oy = r - n * ho;
      float v[kC];
      if constexpr (kC == 15)
        first_channels(F, E, n, oy, ox, timestep, v);
      else
        block_channels(F, E, Z, K, n, oy, ox, timestep, v);
#pragma unroll
      for (int q = 0; q < chunks; ++q) store_x_chunk<kC>(out, chunks, ho, wo, n, oy, ox, q, v);
    }
    return;
  }
  const int ox = t >> 2;
  const int sx = t & 1, sy = (t >> 1) & 1;
  const bool live = ox < wo;  // the quad agrees; the shuffles need every lane of the warp
  const AxisTap tx = resize_tap(live ? ox : wo - 1, static_cast<float>(d), F.Wp);
  const int X = sx ? tx.hi : tx.lo;
  const float inv = __fdiv_rn(1.0f, static_cast<float>(d));
  for (int r = blockIdx.y; r < batch * ho; r += gridDim.y) {
    const int n = r / ho;
    const int oy = r - n * ho;
    const AxisTap ty = resize_tap(oy, static_cast<float>(d), F.Hp);
    const int Y = sy ? ty.hi : ty.lo;
    float v[kC];
    if constexpr (kC == 15)
      first_channels(F, E, n, Y, X, timestep, v);
    else
      block_channels(F, E, Z, K, n, Y, X, timestep, v);
#pragma unroll
    for (int c = 0; c < kC; ++c) {
      const float p = __shfl_xor_sync(0xffffffffu, v[c], 1);
      const float h = sx ? lerp_rn(p, v[c], tx.t) : lerp_rn(v[c], p, tx.t);
      const float o = __shfl_xor_sync(0xffffffffu, h, 2);
      v[c] = sy ? lerp_rn(o, h, ty.t) : lerp_rn(h, o, ty.t);
    }
    if constexpr (kC == 28) {
#pragma unroll
      for (int c = 24; c < 28; ++c) v[c] = __fmul_rn(v[c], inv);
    }
    const int q = sx + 2 * sy;
    if (live && q < chunks) store_x_chunk<kC>(out, chunks, ho, wo, n, oy, ox, q, v);
  }
}

// The final flow at (Y, X): blocks 0 .. last - 1 resized, then the last block's own (d = 1: read
// in place), and its mask logit.
__device__ __forceinline__ void final_flow(const RifeZ& Z, int last, int n, int Y, int X, float f[4], float* mask) {
  flow_at(Z, last, n, Y, X, f);
  const uint8_t* px = Z.z[last] + ((static_cast<size_t>(n) * Z.h[last] + Y) * Z.w[last] + X) * kRifeZBytes;
  const uint4 q = __ldg(reinterpret_cast<const uint4*>(px));
  float a[4], b[4];
  half4(make_uint2(q.x, q.y), a);
  half4(make_uint2(q.z, q.w), b);
#pragma unroll
  for (int c = 0; c < 4; ++c) f[c] = last == 0 ? a[c] : __fadd_rn(f[c], a[c]);
  *mask = b[0];
}

// The interpolated frame in the window: out = warp(A) m + warp(B) (1 - m), m = sigmoid(mask),
// NCHW FP16 [n][3][H][W]; one thread per column, rows along blockIdx.y.
__global__ void rife_finish_kernel(IfFrames F, RifeZ Z, int last, int batch, __half* __restrict__ out) {
  const int x = blockIdx.x * blockDim.x + threadIdx.x;
  if (x >= F.W) return;
  const int X = x + F.left;
  for (int r = blockIdx.y; r < batch * F.H; r += gridDim.y) {
    const int n = r / F.H;
    const int y = r - n * F.H;
    const int Y = y + F.top;
    float f[4], mask;
    final_flow(Z, last, n, Y, X, f, &mask);
    const size_t frame = static_cast<size_t>(n) * F.Hp * F.Wp;
    float w0[3], w1[3];
    warp3(F.pad0 + frame, F, Y, X, f[0], f[1], w0);
    warp3(F.pad1 + frame, F, Y, X, f[2], f[3], w1);
    const float m = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-mask)));
    const float m1 = __fsub_rn(1.0f, m);
    __half* o = out + (static_cast<size_t>(n) * 3 * F.H + y) * F.W + x;
#pragma unroll
    for (int c = 0; c < 3; ++c)
      o[static_cast<size_t>(c) * F.H * F.W] = __float2half_rn(__fadd_rn(__fmul_rn(w0[c], m), __fmul_rn(w1[c], m1)));
  }
}

// The motion variant over the padded plane: the final flow [n][4][Hp][Wp] and sigmoid(mask)
// [n][1][Hp][Wp], T = float or __half.
template <typename T>
__global__ void rife_motion_kernel(IfFrames F, RifeZ Z, int last, int batch, T* __restrict__ flow,
                                   T* __restrict__ mask) {
  const int X = blockIdx.x * blockDim.x + threadIdx.x;
  if (X >= F.Wp) return;
  const size_t pl = static_cast<size_t>(F.Hp) * F.Wp;
  for (int r = blockIdx.y; r < batch * F.Hp; r += gridDim.y) {
    const int n = r / F.Hp;
    const int Y = r - n * F.Hp;
    float f[4], m;
    final_flow(Z, last, n, Y, X, f, &m);
    const size_t at = static_cast<size_t>(Y) * F.Wp + X;
#pragma unroll
    for (int c = 0; c < 4; ++c) store_motion(flow + (static_cast<size_t>(n) * 4 + c) * pl + at, f[c]);
    store_motion(mask + static_cast<size_t>(n) * pl + at, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-m))));
  }
}

}  // namespace kb2
