// Device helpers of the interpolators' glue kernels (ifnet_glue.cuh for classic IFNet, rife_glue.cuh
// for RIFE 4.2x): the padded frames, the half-pixel resize and bilinear warp taps, the 3-channel warp
// and the motion-plane stores. The arithmetic follows the reference's warp library and the IR's
// Resize, as ifnet_glue.cuh states.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace kb2 {

// Input frames: caller's NCHW FP16 [n][3][H][W], placed at (top, left) in a zero padded Hp x Wp
// plane. `pad0` / `pad1`: the same frames padded, one 8-byte RGBx FP16 pixel each
// ([n][Hp][Wp] uint2, filled by ifnet_pad_frames_kernel), so that a warp tap is one load.
struct IfFrames {
  const __half* img0;
  const __half* img1;
  int H, W, Hp, Wp, top, left;
  uint2* pad0;
  uint2* pad1;
};

// The glue kernels run on a grid of rows: blockIdx.x * blockDim.x + threadIdx.x is the column and
// blockIdx.y walks the rows (frame-major) in steps of gridDim.y, so no thread divides a 64-bit
// pixel index.
constexpr int kGlueThreads = 256;
constexpr int kGlueMaxRowBlocks = 65535;

__device__ __forceinline__ float lerp_rn(float a, float b, float t) {
  // (1 - t) * a + t * b
  return __fadd_rn(__fmul_rn(__fsub_rn(1.0f, t), a), __fmul_rn(t, b));
}

struct AxisTap {
  int lo, hi;
  float t;
};

// Half-pixel resize tap of output index o along an axis of n_in -> n_out samples, inv = n_in / n_out
// a power of two (so that the division by the scale n_out / n_in is this exact product).
__device__ __forceinline__ AxisTap resize_tap(int o, float inv, int n_in) {
  float pos = __fsub_rn(__fmul_rn(__fadd_rn(static_cast<float>(o), 0.5f), inv), 0.5f);
  pos = fminf(fmaxf(pos, 0.0f), static_cast<float>(n_in - 1));
  AxisTap r;
  r.lo = static_cast<int>(pos);
  r.hi = min(r.lo + 1, n_in - 1);
  r.t = __fsub_rn(pos, static_cast<float>(r.lo));
  return r;
}

// Bilinear tap of the warp at integer position p displaced by f, over [0, n).
__device__ __forceinline__ AxisTap warp_tap(int p, float f, int n) {
  float i = __fadd_rn(static_cast<float>(p), f);
  i = fminf(fmaxf(i, 0.0f), static_cast<float>(n - 1));  // fmaxf(NaN, 0) = 0: NaN goes to the low bound
  AxisTap r;
  r.lo = static_cast<int>(i);
  r.hi = min(r.lo + 1, n - 1);
  r.t = __fsub_rn(i, static_cast<float>(r.lo));
  return r;
}

// The three channels of pixel (Y, X) of one padded frame (`fr`: the frame's first pixel).
__device__ __forceinline__ void frame_rgb(const uint2* fr, int Wp, int Y, int X, float c[3]) {
  const uint2 q = __ldg(fr + (Y * Wp + X));
  const float2 rg = __half22float2(*reinterpret_cast<const __half2*>(&q.x));
  c[0] = rg.x;
  c[1] = rg.y;
  c[2] = __low2float(*reinterpret_cast<const __half2*>(&q.y));
}

// The bilinear mix of the four 8-byte FP16 pixels (4 channels) around a warp position, in packed
// FP16 pairs: lerp(lerp(a, b, wx), lerp(d, e, wx), wy), each lerp as p + w (q - p). The positions
// (tap indices and weights, warp_tap) are computed in FP32 as the reference states them; only the
// mixing of the pixel values, which are FP16 like the results' consumers, runs on pairs.
__device__ __forceinline__ void bilerp_h2(const uint2* fr, int Wp, const AxisTap& tx, const AxisTap& ty, __half2& c01,
                                          __half2& c23) {
  const __half2 wx = __float2half2_rn(tx.t), wy = __float2half2_rn(ty.t);
  const uint2 qa = __ldg(fr + (ty.lo * Wp + tx.lo));
  const uint2 qb = __ldg(fr + (ty.lo * Wp + tx.hi));
  const uint2 qd = __ldg(fr + (ty.hi * Wp + tx.lo));
  const uint2 qe = __ldg(fr + (ty.hi * Wp + tx.hi));
  auto h = [](uint32_t u) { return *reinterpret_cast<const __half2*>(&u); };
  const __half2 t0 = __hfma2(wx, __hsub2(h(qb.x), h(qa.x)), h(qa.x));
  const __half2 t1 = __hfma2(wx, __hsub2(h(qb.y), h(qa.y)), h(qa.y));
  const __half2 b0 = __hfma2(wx, __hsub2(h(qe.x), h(qd.x)), h(qd.x));
  const __half2 b1 = __hfma2(wx, __hsub2(h(qe.y), h(qd.y)), h(qd.y));
  c01 = __hfma2(wy, __hsub2(b0, t0), t0);
  c23 = __hfma2(wy, __hsub2(b1, t1), t1);
}

// Backward warp of the 3 channels of a padded frame (`fr`: its first pixel) at pixel (Y, X) by
// flow (fx, fy).
__device__ __forceinline__ void warp3(const uint2* fr, const IfFrames& F, int Y, int X, float fx, float fy,
                                      float out[3]) {
  const AxisTap tx = warp_tap(X, fx, F.Wp);
  const AxisTap ty = warp_tap(Y, fy, F.Hp);
  __half2 c01, c23;
  bilerp_h2(fr, F.Wp, tx, ty, c01, c23);
  const float2 rg = __half22float2(c01);
  out[0] = rg.x;
  out[1] = rg.y;
  out[2] = __low2float(c23);
}

__device__ __forceinline__ void store_motion(float* p, float v) { *p = v; }
__device__ __forceinline__ void store_motion(__half* p, float v) { *p = __float2half_rn(v); }

}  // namespace kb2
