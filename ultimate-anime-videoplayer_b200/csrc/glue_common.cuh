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

// Backward warp of the 3 channels of a padded frame (`fr`: its first pixel) at pixel (Y, X) by
// flow (fx, fy).
__device__ __forceinline__ void warp3(const uint2* fr, const IfFrames& F, int Y, int X, float fx, float fy,
                                      float out[3]) {
  const AxisTap tx = warp_tap(X, fx, F.Wp);
  const AxisTap ty = warp_tap(Y, fy, F.Hp);
  const float wx1 = __fsub_rn(1.0f, tx.t), wy1 = __fsub_rn(1.0f, ty.t);
  float a[3], b[3], d[3], e[3];
  frame_rgb(fr, F.Wp, ty.lo, tx.lo, a);
  frame_rgb(fr, F.Wp, ty.lo, tx.hi, b);
  frame_rgb(fr, F.Wp, ty.hi, tx.lo, d);
  frame_rgb(fr, F.Wp, ty.hi, tx.hi, e);
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    // (a (1 - wx) + b wx) (1 - wy) + (d (1 - wx) + e wx) wy
    const float top = __fadd_rn(__fmul_rn(a[c], wx1), __fmul_rn(b[c], tx.t));
    const float bot = __fadd_rn(__fmul_rn(d[c], wx1), __fmul_rn(e[c], tx.t));
    out[c] = __fadd_rn(__fmul_rn(top, wy1), __fmul_rn(bot, ty.t));
  }
}

__device__ __forceinline__ void store_motion(float* p, float v) { *p = v; }
__device__ __forceinline__ void store_motion(__half* p, float v) { *p = __float2half_rn(v); }

}  // namespace kb2
