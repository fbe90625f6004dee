// Frames at any instant from one mid-pair motion, and the motion's size: the reference's
// warp_blend_at and flow_max (src/kernels/ref/warp.cpp:261, :290; the law and its constants in
// src/kernels/spec/warp.h:50-110), which let the player run RIFE once per calm pair and synthesise
// the other instants from that one motion.
//
// warp_blend_at, per output pixel (x, y) of frame n (H x W), with the motion's window ww x wh:
//   sx = W / ww, u = (x + 0.5) / sx - 0.5 (the same in y): the pixel's point in the motion grid;
//   t = 1/2: f = flow(u, v), m = mask(u, v);
//   other t: (u2, v2) = (u, v) - ((1 - t) f0 + t f1)(u, v); d = f1(u2, v2) - f0(u2, v2);
//            to a -t d, to b (1 - t) d; mm = clamp(mask(u2, v2), 1e-4, 1 - 1e-4);
//            m = 1 / (1 + exp(-(A ln(mm / (1 - mm)) + B ln((1 - t) / t) + C)));
//   out = a(x + sx dax, y + sy day) m + b(x + sx dbx, y + sy dby) (1 - m), bilinear reads clamped to
//   the window (motion) or the frame (images). FP32 arithmetic in the reference's order with the
//   _rn intrinsics (no contraction); ln and exp are CUDA's logf / expf.
// warp_blend_poses (keep the poses, spec/poses.h): per pixel, two iterations of: the point seen at the
// pixel at instant tp, its displacement D now and D' in the previous pair (q = pa - f1'(q), two steps;
// D' = 0 for a held pair), r = (|D'| + e) / (|D'| + |D| + 2e), tp = pose_time(t, r) clamped; then the
// straight-line blend at tp. |.| is CUDA's hypotf.
// The pan lock (spec/warp_pan.h, ref/warp_pan.cpp): per pair, a Lucas-Kanade translation of the luma
// on a 32 x 32 grid (3 iterations); where it is sure, RIFE's flow is replaced by it where small and
// close; and the blend weight fades to the linear blend under half a pixel of motion
// (logit m = w law + (1 - w) ln((1 - t) / t), w = smoothstep(0.5, 2, |d|)).
// flow_max: per pair, a 256-bin histogram of max |flow component| over the window (bins of 0.25 px,
// the last taking the rest), then the 99.9th percentile's bin edge.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <vector>

#include "engine.h"

namespace kb2 {

namespace {

constexpr float kLawA = 1.0f, kLawB = 2.591f, kLawC = 0.0f, kMaskEps = 1e-4f;
// keep the poses (spec/poses.h): iterations, distance epsilon (grid pixels), instant limit
constexpr int kPoseIterations = 2;
constexpr float kPoseEps = 0.01f, kPoseTimeLimit = 1e-3f;
// the pair's global translation (spec/warp_pan.h): grid, iterations, luma, limits, slow fade
constexpr int kPanGrid = 32, kPanIterations = 3;
constexpr float kPanLumaR = 0.2126f, kPanLumaG = 0.7152f, kPanLumaB = 0.0722f;
constexpr float kPanDetRatio = 1e-6f, kPanMaxShift = 8.0f, kPanFlowLimit = 2.0f, kPanAgreement = 1.0f;
constexpr float kSlowFadeLo = 0.5f, kSlowFadeHi = 2.0f;

// A pair's pan: the flow g that replaces RIFE's where it is small and close to it (on), and the
// slow fade towards the linear blend (always, with the pan lock).
struct Pan {
  float g[4];
  int on;
};

// The pairs' pans of a pan-locked call, estimated and read on the call's stream (pan-locked calls
// that overlap on the GPU race on them).
constexpr int kMaxPanPairs = 64;
__device__ Pan g_pan_slots[kMaxPanPairs];
constexpr int kFlowBins = 256;
constexpr float kFlowBinStep = 0.25f;
constexpr double kFlowPercentile = 0.999;

struct MotionView {
  const float* flow;  // [n][4][ph][pw]
  const float* mask;  // [n][ph][pw]
  int ph, pw, wx, wy, ww, wh;
};

// Bilinear read of plane p (row pitch pw) relative to the corner (wx, wy) of a ww x wh window:
// clamp (NaN to 0, as fmaxf), truncate, right / bottom neighbour clamped.
template <class T>
__device__ __forceinline__ float load_f(const T* p, size_t i);
template <>
__device__ __forceinline__ float load_f<float>(const float* p, size_t i) {
  return __ldg(p + i);
}
template <>
__device__ __forceinline__ float load_f<__half>(const __half* p, size_t i) {
  return __half2float(p[i]);
}

template <class T>
__device__ __forceinline__ float bilinear(const T* p, int pw, int wx, int wy, int ww, int wh, float x, float y) {
  x = fminf(fmaxf(x, 0.0f), static_cast<float>(ww - 1));
  y = fminf(fmaxf(y, 0.0f), static_cast<float>(wh - 1));
  const int x0 = static_cast<int>(x), y0 = static_cast<int>(y);
  const int x1 = min(x0 + 1, ww - 1), y1 = min(y0 + 1, wh - 1);
  const float fx = __fsub_rn(x, static_cast<float>(x0));
  const float fy = __fsub_rn(y, static_cast<float>(y0));
  const size_t r0 = static_cast<size_t>(wy + y0) * pw + wx, r1 = static_cast<size_t>(wy + y1) * pw + wx;
  const float gx = __fsub_rn(1.0f, fx), gy = __fsub_rn(1.0f, fy);
  const float top = __fadd_rn(__fmul_rn(load_f(p, r0 + x0), gx), __fmul_rn(load_f(p, r0 + x1), fx));
  const float bot = __fadd_rn(__fmul_rn(load_f(p, r1 + x0), gx), __fmul_rn(load_f(p, r1 + x1), fx));
  return __fadd_rn(__fmul_rn(top, gy), __fmul_rn(bot, fy));
}

__device__ __forceinline__ float luma_at(const __half* a, size_t plane, int w, int x, int y) {
  const size_t i = static_cast<size_t>(y) * w + x;
  return __fadd_rn(__fadd_rn(__fmul_rn(kPanLumaR, __half2float(a[i])), __fmul_rn(kPanLumaG, __half2float(a[plane + i]))),
                   __fmul_rn(kPanLumaB, __half2float(a[2 * plane + i])));
}

__device__ __forceinline__ float luma_bilinear(const __half* a, size_t plane, int w, int h, float x, float y) {
  x = fminf(fmaxf(x, 0.0f), static_cast<float>(w - 1));
  y = fminf(fmaxf(y, 0.0f), static_cast<float>(h - 1));
  const int x0 = static_cast<int>(x), y0 = static_cast<int>(y);
  const int x1 = min(x0 + 1, w - 1), y1 = min(y0 + 1, h - 1);
  const float fx = __fsub_rn(x, static_cast<float>(x0)), fy = __fsub_rn(y, static_cast<float>(y0));
  const float gx = __fsub_rn(1.0f, fx), gy = __fsub_rn(1.0f, fy);
  const float top = __fadd_rn(__fmul_rn(luma_at(a, plane, w, x0, y0), gx), __fmul_rn(luma_at(a, plane, w, x1, y0), fx));
  const float bot = __fadd_rn(__fmul_rn(luma_at(a, plane, w, x0, y1), gx), __fmul_rn(luma_at(a, plane, w, x1, y1), fx));
  return __fadd_rn(__fmul_rn(top, gy), __fmul_rn(bot, fy));
}

__device__ __forceinline__ int pan_point(int i, int n) {
  const int m = n / 12 > 4 ? n / 12 : 4;
  return m + (i * (n - 2 * m)) / kPanGrid;
}

// smoothstep(0.5, 2, d): the weight of the fitted blend law against the linear fade
__device__ __forceinline__ float slow_fade_weight(float d) {
  float s = __fdiv_rn(__fsub_rn(d, kSlowFadeLo), kSlowFadeHi - kSlowFadeLo);
  s = s < 0.0f ? 0.0f : (s > 1.0f ? 1.0f : s);
  return __fmul_rn(__fmul_rn(s, s), __fsub_rn(3.0f, __fmul_rn(2.0f, s)));
}

// One block of kPanGrid^2 threads per pair: Lucas-Kanade on the luma of a and b at a 32 x 32 grid
// (ref/warp_pan.cpp pan_estimate), sums in double (the reference's are sequential, these a tree:
// a last-bit difference at most), then the pair's g for the flow read at the middle (s = 1/2).
__global__ void __launch_bounds__(kPanGrid * kPanGrid) pan_estimate_kernel(const __half* __restrict__ a,
                                                                           const __half* __restrict__ b, int H, int W,
                                                                           float sx, float sy, float sm,
                                                                           Pan* __restrict__ pans) {
  const int n = blockIdx.x;
  const int q = threadIdx.x;
  __shared__ double red[5][kPanGrid * kPanGrid / 32];
  __shared__ float s_dx, s_dy;
  __shared__ int s_valid;
  if (W < 16 || H < 16) {
    if (q == 0) pans[n] = Pan{{0.0f, 0.0f, 0.0f, 0.0f}, 0};
    return;
  }
  const size_t plane = static_cast<size_t>(H) * W;
  const __half* fa = a + static_cast<size_t>(n) * 3 * plane;
  const __half* fb = b + static_cast<size_t>(n) * 3 * plane;
  const int px = pan_point(q % kPanGrid, W), py = pan_point(q / kPanGrid, H);
  const float la = luma_at(fa, plane, W, px, py);
  const float gx = __fmul_rn(0.5f, __fsub_rn(luma_at(fa, plane, W, px + 1, py), luma_at(fa, plane, W, px - 1, py)));
  const float gy = __fmul_rn(0.5f, __fsub_rn(luma_at(fa, plane, W, px, py + 1), luma_at(fa, plane, W, px, py - 1)));
  if (q == 0) {
    s_dx = 0.0f;
    s_dy = 0.0f;
    s_valid = 0;
  }
  __syncthreads();
  for (int it = 0; it < kPanIterations; ++it) {
    const float r = __fsub_rn(luma_bilinear(fb, plane, W, H, __fadd_rn(static_cast<float>(px), s_dx),
                                            __fadd_rn(static_cast<float>(py), s_dy)),
                              la);
    double v[5] = {__fmul_rn(gx, gx), __fmul_rn(gx, gy), __fmul_rn(gy, gy), __fmul_rn(gx, r), __fmul_rn(gy, r)};
#pragma unroll
    for (int k = 0; k < 5; ++k)
      for (int o = 16; o > 0; o >>= 1) v[k] += __shfl_xor_sync(0xffffffffu, v[k], o);
    if ((q & 31) == 0)
#pragma unroll
      for (int k = 0; k < 5; ++k) red[k][q >> 5] = v[k];
    __syncthreads();
    if (q == 0) {
      double sm[5] = {0, 0, 0, 0, 0};
      for (int w = 0; w < kPanGrid * kPanGrid / 32; ++w)
#pragma unroll
        for (int k = 0; k < 5; ++k) sm[k] += red[k][w];
      const double sxx = sm[0], sxy = sm[1], syy = sm[2], sxr = sm[3], syr = sm[4];
      const double det = sxx * syy - sxy * sxy;
      const bool valid = det > static_cast<double>(kPanDetRatio) * (sxx + syy) * (sxx + syy) && det > 0.0;
      s_valid = valid ? 1 : 0;
      if (valid) {
        s_dx = __fsub_rn(s_dx, static_cast<float>((syy * sxr - sxy * syr) / det));
        s_dy = __fsub_rn(s_dy, static_cast<float>((sxx * syr - sxy * sxr) / det));
      }
    }
    __syncthreads();
    if (!s_valid) break;
  }
  if (q == 0) {
    const float dx = s_dx, dy = s_dy;
    const bool sure = s_valid != 0 && hypotf(dx, dy) < kPanMaxShift;
    pans[n] = Pan{{__fdiv_rn(__fmul_rn(-sm, dx), sx), __fdiv_rn(__fmul_rn(-sm, dy), sy),
                   __fdiv_rn(__fmul_rn(__fsub_rn(1.0f, sm), dx), sx), __fdiv_rn(__fmul_rn(__fsub_rn(1.0f, sm), dy), sy)},
                  sure ? 1 : 0};
  }
}

// The flow read f replaced by the pan's g where it is small (max |f| < 2) and close (max |f - g| < 1).
__device__ __forceinline__ void pan_substitute(float (&f)[4], const Pan& p) {
  if (!p.on) return;
  float m = 0.0f, e = 0.0f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    m = fmaxf(m, fabsf(f[c]));
    e = fmaxf(e, fabsf(__fsub_rn(f[c], p.g[c])));
  }
  if (m < kPanFlowLimit && e < kPanAgreement)
#pragma unroll
    for (int c = 0; c < 4; ++c) f[c] = p.g[c];
}

// Catmull-Rom read of plane p (w x h, row pitch w) at (x, y) (spec/warp.h RifeWarp::CatmullRom): the
// position clamped to the plane, points -1 .. 2 around the truncation with clamped indices, weights
// (-0.5 t3 + t2 - 0.5 t, 1.5 t3 - 2.5 t2 + 1, -1.5 t3 + 2 t2 + 0.5 t, 0.5 t3 - 0.5 t2), rows then
// columns, the result clamped to the four central samples' range (ref/warp.cpp catmull_rom_at).
__device__ __forceinline__ void cr_weights(float t, float (&w)[4]) {
  const float t2 = __fmul_rn(t, t), t3 = __fmul_rn(t2, t);
  w[0] = __fsub_rn(__fadd_rn(__fmul_rn(-0.5f, t3), t2), __fmul_rn(0.5f, t));
  w[1] = __fadd_rn(__fsub_rn(__fmul_rn(1.5f, t3), __fmul_rn(2.5f, t2)), 1.0f);
  w[2] = __fadd_rn(__fadd_rn(__fmul_rn(-1.5f, t3), __fmul_rn(2.0f, t2)), __fmul_rn(0.5f, t));
  w[3] = __fsub_rn(__fmul_rn(0.5f, t3), __fmul_rn(0.5f, t2));
}

__device__ __forceinline__ float catmull_rom(const __half* p, int w, int h, float x, float y) {
  x = fminf(fmaxf(x, 0.0f), static_cast<float>(w - 1));
  y = fminf(fmaxf(y, 0.0f), static_cast<float>(h - 1));
  const int x0 = static_cast<int>(x), y0 = static_cast<int>(y);
  float wx[4], wy[4];
  cr_weights(__fsub_rn(x, static_cast<float>(x0)), wx);
  cr_weights(__fsub_rn(y, static_cast<float>(y0)), wy);
  float sum = 0.0f, lo = __int_as_float(0x7f800000), hi = -__int_as_float(0x7f800000);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int yy = min(max(y0 - 1 + j, 0), h - 1);
    float row = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float v = __half2float(__ldg(p + static_cast<size_t>(yy) * w + min(max(x0 - 1 + i, 0), w - 1)));
      row = __fadd_rn(row, __fmul_rn(v, wx[i]));
      if ((i == 1 || i == 2) && (j == 1 || j == 2)) {
        lo = fminf(lo, v);
        hi = fmaxf(hi, v);
      }
    }
    sum = __fadd_rn(sum, __fmul_rn(row, wy[j]));
  }
  return fminf(fmaxf(sum, lo), hi);
}

// kMode 0: t = 1/2, flow and mask as they are; 1: straight-line motion from the middle at t; 2: keep the
// poses: each pixel's instant adjusted by the distance ratio to the previous pair's motion `pm`
// (pm.flow null: a held previous pair), then mode 1 at that instant.
// kCatmull: frames a and b read by Catmull-Rom instead of bilinearly (the motion stays bilinear).
// pans: the pairs' pans with the pan lock (modes 0 and 1), else null.
template <int kMode, bool kCatmull>
__global__ void warp_blend_at_kernel(const __half* __restrict__ a, const __half* __restrict__ b, MotionView m,
                                     MotionView pm, int batch, int H, int W, float t, const Pan* __restrict__ pans,
                                     __half* __restrict__ out) {
  constexpr bool kMiddle = kMode == 0;
  const int x = blockIdx.x * blockDim.x + threadIdx.x;
  if (x >= W) return;
  const float sx = __fdiv_rn(static_cast<float>(W), static_cast<float>(m.ww));
  const float sy = __fdiv_rn(static_cast<float>(H), static_cast<float>(m.wh));
  const float fx = static_cast<float>(x);
  const float u = __fsub_rn(__fdiv_rn(__fadd_rn(fx, 0.5f), sx), 0.5f);
  const size_t plane = static_cast<size_t>(m.ph) * m.pw;
  const size_t frame = static_cast<size_t>(H) * W;
  for (int r = blockIdx.y; r < batch * H; r += gridDim.y) {
    const int n = r / H;
    const int y = r - n * H;
    const float fy = static_cast<float>(y);
    const float v = __fsub_rn(__fdiv_rn(__fadd_rn(fy, 0.5f), sy), 0.5f);
    const float* fl = m.flow + static_cast<size_t>(n) * 4 * plane;
    const float* mk = m.mask + static_cast<size_t>(n) * plane;
    float f[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) f[c] = bilinear(fl + c * plane, m.pw, m.wx, m.wy, m.ww, m.wh, u, v);
    Pan pan{};
    const bool fade = kMode != 2 && pans != nullptr;
    if (fade) {
      pan = pans[n];
      pan_substitute(f, pan);
    }
    float tq = t;  // the pixel's instant
    if constexpr (kMode == 2) {
      const float* pf = pm.flow != nullptr ? pm.flow + static_cast<size_t>(n) * 4 * plane : nullptr;
      for (int k = 0; k < kPoseIterations; ++k) {
        const float s = __fsub_rn(1.0f, tq);
        const float u2 = __fsub_rn(u, __fadd_rn(__fmul_rn(s, f[0]), __fmul_rn(tq, f[2])));
        const float v2 = __fsub_rn(v, __fadd_rn(__fmul_rn(s, f[1]), __fmul_rn(tq, f[3])));
        const float dx = __fsub_rn(bilinear(fl + 2 * plane, m.pw, m.wx, m.wy, m.ww, m.wh, u2, v2),
                                   bilinear(fl, m.pw, m.wx, m.wy, m.ww, m.wh, u2, v2));
        const float dy = __fsub_rn(bilinear(fl + 3 * plane, m.pw, m.wx, m.wy, m.ww, m.wh, u2, v2),
                                   bilinear(fl + plane, m.pw, m.wx, m.wy, m.ww, m.wh, u2, v2));
        float before = 0.0f;
        if (pf != nullptr) {
          // where the point was in the previous pair: q = pa - f1'(q), two steps from pa
          const float ax = __fsub_rn(u, __fmul_rn(tq, dx)), ay = __fsub_rn(v, __fmul_rn(tq, dy));
          float qx = ax, qy = ay;
          for (int step = 0; step < 2; ++step) {
            const float nx = __fsub_rn(ax, bilinear(pf + 2 * plane, pm.pw, pm.wx, pm.wy, pm.ww, pm.wh, qx, qy));
            const float ny = __fsub_rn(ay, bilinear(pf + 3 * plane, pm.pw, pm.wx, pm.wy, pm.ww, pm.wh, qx, qy));
            qx = nx;
            qy = ny;
          }
          before = hypotf(__fsub_rn(bilinear(pf + 2 * plane, pm.pw, pm.wx, pm.wy, pm.ww, pm.wh, qx, qy),
                                    bilinear(pf, pm.pw, pm.wx, pm.wy, pm.ww, pm.wh, qx, qy)),
                          __fsub_rn(bilinear(pf + 3 * plane, pm.pw, pm.wx, pm.wy, pm.ww, pm.wh, qx, qy),
                                    bilinear(pf + plane, pm.pw, pm.wx, pm.wy, pm.ww, pm.wh, qx, qy)));
        }
        const float now = hypotf(dx, dy);
        const float r = __fdiv_rn(__fadd_rn(before, kPoseEps), __fadd_rn(__fadd_rn(before, now), 2.0f * kPoseEps));
        const float pt = t < 0.5f ? __fmul_rn(__fmul_rn(2.0f, t), r)
                                  : __fsub_rn(1.0f, __fmul_rn(__fmul_rn(2.0f, __fsub_rn(1.0f, t)), r));
        tq = fminf(fmaxf(pt, kPoseTimeLimit), 1.0f - kPoseTimeLimit);
      }
    }
    float dax, day, dbx, dby, wgt;
    if constexpr (kMiddle) {
      dax = f[0];
      day = f[1];
      dbx = f[2];
      dby = f[3];
      wgt = bilinear(mk, m.pw, m.wx, m.wy, m.ww, m.wh, u, v);
      if (fade) {  // under half a pixel of motion the blend slides to the linear fade
        const float mm = fminf(fmaxf(wgt, kMaskEps), __fsub_rn(1.0f, kMaskEps));
        const float w = slow_fade_weight(hypotf(__fsub_rn(f[2], f[0]), __fsub_rn(f[3], f[1])));
        const float z = __fadd_rn(__fmul_rn(w, logf(__fdiv_rn(mm, __fsub_rn(1.0f, mm)))),
                                  __fmul_rn(__fsub_rn(1.0f, w), logf(__fdiv_rn(__fsub_rn(1.0f, t), t))));
        wgt = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-z)));
      }
    } else {
      const float s = __fsub_rn(1.0f, tq);
      const float u2 = __fsub_rn(u, __fadd_rn(__fmul_rn(s, f[0]), __fmul_rn(tq, f[2])));
      const float v2 = __fsub_rn(v, __fadd_rn(__fmul_rn(s, f[1]), __fmul_rn(tq, f[3])));
      float g[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) g[c] = bilinear(fl + c * plane, m.pw, m.wx, m.wy, m.ww, m.wh, u2, v2);
      if (fade) pan_substitute(g, pan);
      const float tx = __fsub_rn(g[2], g[0]);
      const float ty = __fsub_rn(g[3], g[1]);
      const float mm =
          fminf(fmaxf(bilinear(mk, m.pw, m.wx, m.wy, m.ww, m.wh, u2, v2), kMaskEps), __fsub_rn(1.0f, kMaskEps));
      float z = __fadd_rn(__fadd_rn(__fmul_rn(kLawA, logf(__fdiv_rn(mm, __fsub_rn(1.0f, mm)))),
                                    __fmul_rn(kLawB, logf(__fdiv_rn(s, tq)))),
                          kLawC);
      if (fade) {
        const float w = slow_fade_weight(hypotf(tx, ty));
        z = __fadd_rn(__fmul_rn(w, z), __fmul_rn(__fsub_rn(1.0f, w), logf(__fdiv_rn(s, tq))));
      }
      wgt = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-z)));
      dax = __fmul_rn(-tq, tx);
      day = __fmul_rn(-tq, ty);
      dbx = __fmul_rn(s, tx);
      dby = __fmul_rn(s, ty);
    }
    const float xa = __fadd_rn(fx, __fmul_rn(sx, dax)), ya = __fadd_rn(fy, __fmul_rn(sy, day));
    const float xb = __fadd_rn(fx, __fmul_rn(sx, dbx)), yb = __fadd_rn(fy, __fmul_rn(sy, dby));
    const float w1 = __fsub_rn(1.0f, wgt);
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const size_t pc = (static_cast<size_t>(n) * 3 + c) * frame;
      const float va = kCatmull ? catmull_rom(a + pc, W, H, xa, ya) : bilinear(a + pc, W, 0, 0, W, H, xa, ya);
      const float vb = kCatmull ? catmull_rom(b + pc, W, H, xb, yb) : bilinear(b + pc, W, 0, 0, W, H, xb, yb);
      out[pc + static_cast<size_t>(y) * W + x] = __float2half_rn(__fadd_rn(__fmul_rn(va, wgt), __fmul_rn(vb, w1)));
    }
  }
}

// Histogram of max |flow component| over each pair's window (block histogram in shared memory).
__global__ void flow_hist_kernel(MotionView m, int batch, unsigned int* __restrict__ bins) {
  __shared__ unsigned int h[kFlowBins];
  for (int i = threadIdx.x; i < kFlowBins; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const size_t plane = static_cast<size_t>(m.ph) * m.pw;
  const int x = blockIdx.x * blockDim.x + threadIdx.x;
  // every block keeps to one pair: blockIdx.z
  const int n = blockIdx.z;
  if (x < m.ww) {
    const float* fl = m.flow + static_cast<size_t>(n) * 4 * plane;
    for (int y = blockIdx.y; y < m.wh; y += gridDim.y) {
      const size_t at = static_cast<size_t>(m.wy + y) * m.pw + m.wx + x;
      float mx = 0.0f;
#pragma unroll
      for (int c = 0; c < 4; ++c) mx = fmaxf(mx, fabsf(__ldg(fl + c * plane + at)));
      int bin = 0;
      if (mx > 0.0f) {
        const float scaled = __fdiv_rn(mx, kFlowBinStep);
        bin = scaled >= static_cast<float>(kFlowBins - 1) ? kFlowBins - 1 : static_cast<int>(scaled);
      }
      atomicAdd(&h[bin], 1u);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kFlowBins; i += blockDim.x)
    if (h[i] != 0) atomicAdd(&bins[static_cast<size_t>(n) * kFlowBins + i], h[i]);
}

Status motion_view(const kb2_motion* motion, MotionView& m) {
  if (motion == nullptr || motion->flow == nullptr || motion->mask == nullptr)
    return refuse(KB2_INVALID_ARGUMENT, "motion: null pointer");
  const kb2_motion& q = *motion;
  if (q.warp != 0 && q.warp != 1) return refuse(KB2_INVALID_ARGUMENT, "motion: warp filter 0 or 1");
  if (q.pan_lock != 0 && q.pan_lock != 1) return refuse(KB2_INVALID_ARGUMENT, "motion: pan_lock 0 or 1");
  if (q.at_instant != 0 && q.at_instant != 1) return refuse(KB2_INVALID_ARGUMENT, "motion: at_instant 0 or 1");
  if (q.plane_h < 1 || q.plane_w < 1 || q.plane_h > 16384 || q.plane_w > 16384)
    return refuse(KB2_SHAPE_INVALID, "motion: plane size out of range");
  // written without x + width, which could overflow
  if (q.x < 0 || q.y < 0 || q.width < 1 || q.height < 1 || q.width > q.plane_w - q.x || q.height > q.plane_h - q.y)
    return refuse(KB2_SHAPE_INVALID, "motion: window outside the planes");
  m = MotionView{q.flow, q.mask, q.plane_h, q.plane_w, q.x, q.y, q.width, q.height};
  return Status::Ok();
}

dim3 rows_grid(int width, int rows) {
  const int bx = (width + 127) / 128;
  const int by = std::max(1, std::min({rows, 65535, (16 * 148 + bx - 1) / bx}));
  return dim3(static_cast<unsigned>(bx), static_cast<unsigned>(by));
}

}  // namespace

Status warp_blend_at(cudaStream_t stream, const kb2_tensor* a, const kb2_tensor* b, const kb2_motion* motion, float t,
                     const kb2_tensor* out, bool keep_poses, const kb2_motion* previous) {
  if (a == nullptr || b == nullptr || out == nullptr) return refuse(KB2_INVALID_ARGUMENT, "null tensor");
  if (!(t > 0.0f && t < 1.0f)) return refuse(KB2_INVALID_ARGUMENT, "warp_blend_at: t outside (0, 1)");
  MotionView m{};
  KB2_TRY(motion_view(motion, m));
  for (const kb2_tensor* x : {a, b, out}) {
    if (x->type != KB2_F16 || x->dims[1] != 3) return refuse(KB2_INPUT_MISMATCH, "warp_blend_at: F16 [n,3,H,W]");
    if (x->dims[0] != a->dims[0] || x->dims[2] != a->dims[2] || x->dims[3] != a->dims[3])
      return refuse(KB2_INPUT_MISMATCH, "warp_blend_at: frames of different shapes");
    if (x->handle + x->offset == 0 || ((x->handle + x->offset) & 1u) != 0)
      return refuse(KB2_INPUT_MISMATCH, "warp_blend_at: null or misaligned frame");
  }
  const long long n = a->dims[0], H = a->dims[2], W = a->dims[3];
  if (n < 1 || H < 1 || W < 1 || H > 16384 || W > 16384 || n * H > (1LL << 30))
    return refuse(KB2_SHAPE_INVALID, "warp_blend_at: frame size out of range");
  const auto* pa = reinterpret_cast<const __half*>(a->handle + a->offset);
  const auto* pb = reinterpret_cast<const __half*>(b->handle + b->offset);
  auto* po = reinterpret_cast<__half*>(out->handle + out->offset);
  MotionView pm{};
  if (keep_poses && previous != nullptr) {
    KB2_TRY(motion_view(previous, pm));
    if (pm.ph != m.ph || pm.pw != m.pw || pm.wx != m.wx || pm.wy != m.wy || pm.ww != m.ww || pm.wh != m.wh)
      return refuse(KB2_INPUT_MISMATCH, "warp_blend_poses: the two pairs' motions differ in size or window");
  }
  const dim3 g = rows_grid(static_cast<int>(W), static_cast<int>(n * H));
  const int nn = static_cast<int>(n), hh = static_cast<int>(H), w = static_cast<int>(W);
  // a motion estimated at the output instant is read as it is at any t (ref/warp.cpp:265)
  const int mode = keep_poses ? 2 : (t == 0.5f || motion->at_instant != 0 ? 0 : 1);
  // the pan lock (not with keep-the-poses): one estimate per pair into the library's pan slots
  const Pan* pans = nullptr;
  if (motion->pan_lock != 0 && !keep_poses) {
    if (n > kMaxPanPairs) return refuse(KB2_SHAPE_INVALID, "warp_blend_at: pan lock on more than 64 pairs");
    Pan* slots = nullptr;
    KB2_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&slots), g_pan_slots));
    const float sx = static_cast<float>(W) / static_cast<float>(m.ww), sy = static_cast<float>(H) / static_cast<float>(m.wh);
    // the instant of the flow read: RIFE's middle, or t for a motion estimated at the output instant
    const float s_read = motion->at_instant != 0 ? t : 0.5f;
    pan_estimate_kernel<<<nn, kPanGrid * kPanGrid, 0, stream>>>(pa, pb, hh, w, sx, sy, s_read, slots);
    KB2_CUDA(cudaGetLastError());
    pans = slots;
  }
  if (motion->warp == 1) {
    if (mode == 2) warp_blend_at_kernel<2, true><<<g, 128, 0, stream>>>(pa, pb, m, pm, nn, hh, w, t, pans, po);
    else if (mode == 0) warp_blend_at_kernel<0, true><<<g, 128, 0, stream>>>(pa, pb, m, pm, nn, hh, w, t, pans, po);
    else warp_blend_at_kernel<1, true><<<g, 128, 0, stream>>>(pa, pb, m, pm, nn, hh, w, t, pans, po);
  } else {
    if (mode == 2) warp_blend_at_kernel<2, false><<<g, 128, 0, stream>>>(pa, pb, m, pm, nn, hh, w, t, pans, po);
    else if (mode == 0) warp_blend_at_kernel<0, false><<<g, 128, 0, stream>>>(pa, pb, m, pm, nn, hh, w, t, pans, po);
    else warp_blend_at_kernel<1, false><<<g, 128, 0, stream>>>(pa, pb, m, pm, nn, hh, w, t, pans, po);
  }
  return cuda_status(cudaGetLastError(), "warp_blend_at launch");
}

Status flow_max(cudaStream_t stream, const kb2_motion* motion, int n, unsigned int* bins, float* out) {
  if (bins == nullptr || out == nullptr) return refuse(KB2_INVALID_ARGUMENT, "flow_max: null pointer");
  if (n < 1 || n > 65535) return refuse(KB2_SHAPE_INVALID, "flow_max: pair count out of range");
  MotionView m{};
  KB2_TRY(motion_view(motion, m));
  KB2_CUDA(cudaMemsetAsync(bins, 0, static_cast<size_t>(n) * kFlowBins * sizeof(unsigned int), stream));
  dim3 g = rows_grid(m.ww, m.wh);
  g.y = std::max(1u, std::min(g.y, 64u));
  g.z = static_cast<unsigned>(n);
  flow_hist_kernel<<<g, 128, 0, stream>>>(m, n, bins);
  KB2_CUDA(cudaGetLastError());
  std::vector<unsigned int> h(static_cast<size_t>(n) * kFlowBins);
  KB2_CUDA(cudaMemcpyAsync(h.data(), bins, h.size() * sizeof(unsigned int), cudaMemcpyDeviceToHost, stream));
  KB2_CUDA(cudaStreamSynchronize(stream));
  const unsigned long long points = static_cast<unsigned long long>(m.ww) * static_cast<unsigned long long>(m.wh);
  for (int i = 0; i < n; ++i) {
    // the bin of the percentile's rank (spec/warp.h flow_percentile): rank = ceil(points * 0.999), >= 1
    auto rank = static_cast<unsigned long long>(static_cast<double>(points) * kFlowPercentile);
    if (static_cast<double>(rank) < static_cast<double>(points) * kFlowPercentile) ++rank;
    if (rank == 0) rank = 1;
    unsigned long long seen = 0;
    float v = static_cast<float>(kFlowBins - 1) * kFlowBinStep;
    for (int k = 0; k < kFlowBins; ++k) {
      seen += h[static_cast<size_t>(i) * kFlowBins + k];
      if (seen >= rank) {
        v = static_cast<float>(k) * kFlowBinStep;
        break;
      }
    }
    out[i] = v;
  }
  return Status::Ok();
}

}  // namespace kb2
