// IFNet glue on CUDA cores, between the tensor-core convs: the input of each IFNet block and the
// final blend. They replace the reference's fused entry / glue / finish kernels
// (src/gpu/cuda/backend/rife_fused_kernels.cu:70,141,208), whose arithmetic is kept:
//
//  * bilinear warp with the reference's tap rule (tap_at, src/gpu/cuda/backend/warp_lib.cuh:45-58;
//    kernels/spec/warp.h:44-49): ix = x + fx in FP32 round-to-nearest, clamped to [0, W - 1],
//    x0 = trunc(ix), x1 = min(x0 + 1, W - 1), weight ix - x0, the same along y. The clamp window is
//    the whole padded plane, as the reference IR's GridSample (border, align_corners = 0);
//  * half-pixel linear resize (src/gpu/ir/op_sample.cpp:88-170): position (o + 0.5) / scale - 0.5
//    in FP32 with scale = n_out / n_in, clamped to [0, n_in - 1], truncated;
//  * the transposed conv of block j leaves a small FP32 tensor (5 planes at 1/(2 s_j) of the
//    frame). After each block, one pass adds it, resized to full resolution and scaled by 2 s_j,
//    to the full-resolution FP32 flow / mask planes: the network's sequential
//    `flow = flow + resize(...)`, in the same order.
//
// Every product and sum is written with the _rn intrinsics, in the order the network states it,
// so that no multiply-add contraction changes a warp position.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace kb2 {

constexpr int kIfBlocks = 4;
// Scale of block k: the block works on the frame at 1/8, 1/4, 1/2, 1/1.
__host__ __device__ constexpr int if_scale(int k) { return 8 >> k; }

// The outputs of the transposed convs so far, FP32 planes [n][5][h][w] at 1/(2 s) of the padded frame.
struct IfFlowLevels {
  const float* t[kIfBlocks];
  int h[kIfBlocks], w[kIfBlocks];
  float mul[kIfBlocks];  // 2 s: flow scale of block j
};

// Input frames: caller's NCHW FP16 [n][3][H][W], placed at (top, left) in a zero padded
// Hp x Wp plane.
struct IfFrames {
  const __half* img0;
  const __half* img1;
  int H, W, Hp, Wp, top, left;
};

__device__ __forceinline__ float lerp_rn(float a, float b, float t) {
  // (1 - t) * a + t * b
  return __fadd_rn(__fmul_rn(__fsub_rn(1.0f, t), a), __fmul_rn(t, b));
}

struct AxisTap {
  int lo, hi;
  float t;
};

// Half-pixel resize tap of output index o along an axis of n_in -> n_out samples.
__device__ __forceinline__ AxisTap resize_tap(int o, int n_in, int n_out) {
  const float scale = __fdiv_rn(static_cast<float>(n_out), static_cast<float>(n_in));
  float pos = __fsub_rn(__fdiv_rn(__fadd_rn(static_cast<float>(o), 0.5f), scale), 0.5f);
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

// Adds block j's contribution at padded pixel (Y, X) of frame n to the flow (4) and mask; block 0
// sets them.
__device__ __forceinline__ void flow_step(const IfFlowLevels& L, int j, int n, int Y, int X, int Hp, int Wp,
                                          float f[4], float* mask) {
  const AxisTap ty = resize_tap(Y, L.h[j], Hp);
  const AxisTap tx = resize_tap(X, L.w[j], Wp);
  const size_t plane = static_cast<size_t>(L.h[j]) * L.w[j];
  const float* base = L.t[j] + static_cast<size_t>(n) * 5 * plane;
  float v[5];
#pragma unroll
  for (int c = 0; c < 5; ++c) {
    const float* p = base + c * plane;
    const float a = __ldg(p + static_cast<size_t>(ty.lo) * L.w[j] + tx.lo);
    const float b = __ldg(p + static_cast<size_t>(ty.lo) * L.w[j] + tx.hi);
    const float d = __ldg(p + static_cast<size_t>(ty.hi) * L.w[j] + tx.lo);
    const float e = __ldg(p + static_cast<size_t>(ty.hi) * L.w[j] + tx.hi);
    v[c] = lerp_rn(lerp_rn(a, b, tx.t), lerp_rn(d, e, tx.t), ty.t);
  }
  if (j == 0) {
#pragma unroll
    for (int c = 0; c < 4; ++c) f[c] = __fmul_rn(v[c], L.mul[j]);
    *mask = v[4];
  } else {
#pragma unroll
    for (int c = 0; c < 4; ++c) f[c] = __fadd_rn(f[c], __fmul_rn(v[c], L.mul[j]));
    *mask = __fadd_rn(*mask, v[4]);
  }
}

// Full-resolution flow (planes 0-3) and mask (plane 4) after the blocks so far: FP32 [n][5][Hp][Wp].
struct IfFlowField {
  float* f;
  int Hp, Wp;
  __device__ __forceinline__ size_t at(int n, int c, int Y, int X) const {
    return ((static_cast<size_t>(n) * 5 + c) * Hp + Y) * Wp + X;
  }
};

// flow / mask += block k's transposed-conv output resized to full resolution (flow x 2 s); block 0
// sets them.
__global__ void ifnet_flow_update_kernel(IfFlowLevels L, int k, int batch, IfFlowField F) {
  const long long total = static_cast<long long>(batch) * F.Hp * F.Wp;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int X = static_cast<int>(i % F.Wp);
    const int Y = static_cast<int>((i / F.Wp) % F.Hp);
    const int n = static_cast<int>(i / (static_cast<long long>(F.Wp) * F.Hp));
    float f[4], mask;
    if (k > 0) {
#pragma unroll
      for (int c = 0; c < 4; ++c) f[c] = F.f[F.at(n, c, Y, X)];
      mask = F.f[F.at(n, 4, Y, X)];
    }
    flow_step(L, k, n, Y, X, F.Hp, F.Wp, f, &mask);
#pragma unroll
    for (int c = 0; c < 4; ++c) F.f[F.at(n, c, Y, X)] = f[c];
    F.f[F.at(n, 4, Y, X)] = mask;
  }
}

// Frame pixel (Y, X) of the zero padded plane, channel c.
__device__ __forceinline__ float frame_px(const __half* img, const IfFrames& F, int n, int c, int Y, int X) {
  const int y = Y - F.top, x = X - F.left;
  if (y < 0 || y >= F.H || x < 0 || x >= F.W) return 0.0f;
  return __half2float(img[((static_cast<size_t>(n) * 3 + c) * F.H + y) * F.W + x]);
}

// Backward warp of the 3 channels of `img` at padded pixel (Y, X) by flow (fx, fy).
__device__ __forceinline__ void warp3(const __half* img, const IfFrames& F, int n, int Y, int X, float fx, float fy,
                                      float out[3]) {
  const AxisTap tx = warp_tap(X, fx, F.Wp);
  const AxisTap ty = warp_tap(Y, fy, F.Hp);
  const float wx1 = __fsub_rn(1.0f, tx.t), wy1 = __fsub_rn(1.0f, ty.t);
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    const float a = frame_px(img, F, n, c, ty.lo, tx.lo);
    const float b = frame_px(img, F, n, c, ty.lo, tx.hi);
    const float d = frame_px(img, F, n, c, ty.hi, tx.lo);
    const float e = frame_px(img, F, n, c, ty.hi, tx.hi);
    // (a (1 - wx) + b wx) (1 - wy) + (d (1 - wx) + e wx) wy
    const float top = __fadd_rn(__fmul_rn(a, wx1), __fmul_rn(b, tx.t));
    const float bot = __fadd_rn(__fmul_rn(d, wx1), __fmul_rn(e, tx.t));
    out[c] = __fadd_rn(__fmul_rn(top, wy1), __fmul_rn(bot, ty.t));
  }
}

// The 12 input planes of block k >= 1 at padded full-resolution pixel (Y, X): warped frames (6),
// timestep, mask, flow (4, not yet divided by the block scale).
__device__ __forceinline__ void block_planes(const IfFrames& F, const IfFlowField& FF, int n, int Y, int X,
                                             float timestep, float v[12]) {
  float f[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) f[c] = __ldg(FF.f + FF.at(n, c, Y, X));
  const float mask = __ldg(FF.f + FF.at(n, 4, Y, X));
  warp3(F.img0, F, n, Y, X, f[0], f[1], v);
  warp3(F.img1, F, n, Y, X, f[2], f[3], v + 3);
  v[6] = timestep;
  v[7] = mask;
#pragma unroll
  for (int c = 0; c < 4; ++c) v[8 + c] = f[c];
}

// Input of block k as row-chunked FP16 [n][Hp/s][2][Wp/s][8 halves] (16 channels, 12 or 7 used):
// the block's planes resized to 1/s (not for s = 1), the flow planes then divided by s.
__global__ void ifnet_block_input_kernel(IfFrames F, IfFlowField FF, int k, int batch, float timestep,
                                         uint8_t* __restrict__ out) {
  const int s = if_scale(k);
  const int ho = F.Hp / s, wo = F.Wp / s;
  const long long total = static_cast<long long>(batch) * ho * wo;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int ox = static_cast<int>(i % wo);
    const int oy = static_cast<int>((i / wo) % ho);
    const int n = static_cast<int>(i / (static_cast<long long>(wo) * ho));
    float v[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) v[c] = 0.0f;
    const int nc = k == 0 ? 7 : 12;
    if (s == 1) {
      block_planes(F, FF, n, oy, ox, timestep, v);
    } else {
      const AxisTap ty = resize_tap(oy, F.Hp, ho);
      const AxisTap tx = resize_tap(ox, F.Wp, wo);
      float q[4][12];
      const int ys[2] = {ty.lo, ty.hi}, xs[2] = {tx.lo, tx.hi};
#pragma unroll
      for (int yy = 0; yy < 2; ++yy)
#pragma unroll
        for (int xx = 0; xx < 2; ++xx) {
          float* p = q[yy * 2 + xx];
          if (k == 0) {
            for (int c = 0; c < 3; ++c) {
              p[c] = frame_px(F.img0, F, n, c, ys[yy], xs[xx]);
              p[3 + c] = frame_px(F.img1, F, n, c, ys[yy], xs[xx]);
            }
            p[6] = timestep;
          } else {
            block_planes(F, FF, n, ys[yy], xs[xx], timestep, p);
          }
        }
      for (int c = 0; c < nc; ++c)
        v[c] = lerp_rn(lerp_rn(q[0][c], q[1][c], tx.t), lerp_rn(q[2][c], q[3][c], tx.t), ty.t);
    }
    if (k > 0) {
      const float inv = __fdiv_rn(1.0f, static_cast<float>(s));
#pragma unroll
      for (int c = 8; c < 12; ++c) v[c] = __fmul_rn(v[c], inv);
    }
    uint8_t* row = out + (static_cast<size_t>(n) * ho + oy) * 2 * wo * 16;
#pragma unroll
    for (int ch = 0; ch < 2; ++ch) {
      uint4 o;
      __half2 h0 = __floats2half2_rn(v[8 * ch + 0], v[8 * ch + 1]);
      __half2 h1 = __floats2half2_rn(v[8 * ch + 2], v[8 * ch + 3]);
      __half2 h2 = __floats2half2_rn(v[8 * ch + 4], v[8 * ch + 5]);
      __half2 h3 = __floats2half2_rn(v[8 * ch + 6], v[8 * ch + 7]);
      o.x = *reinterpret_cast<uint32_t*>(&h0);
      o.y = *reinterpret_cast<uint32_t*>(&h1);
      o.z = *reinterpret_cast<uint32_t*>(&h2);
      o.w = *reinterpret_cast<uint32_t*>(&h3);
      *reinterpret_cast<uint4*>(row + (static_cast<size_t>(ch) * wo + ox) * 16) = o;
    }
  }
}

// The interpolated frame: warp both frames by the final flow, blend with sigmoid(mask), crop the
// window: out = w0 * m + w1 * (1 - m), NCHW FP16 [n][3][H][W].
__global__ void ifnet_blend_kernel(IfFrames F, IfFlowField FF, int batch, __half* __restrict__ out) {
  const long long total = static_cast<long long>(batch) * F.H * F.W;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int x = static_cast<int>(i % F.W);
    const int y = static_cast<int>((i / F.W) % F.H);
    const int n = static_cast<int>(i / (static_cast<long long>(F.W) * F.H));
    const int Y = y + F.top, X = x + F.left;
    float f[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) f[c] = __ldg(FF.f + FF.at(n, c, Y, X));
    const float mask = __ldg(FF.f + FF.at(n, 4, Y, X));
    float w0[3], w1[3];
    warp3(F.img0, F, n, Y, X, f[0], f[1], w0);
    warp3(F.img1, F, n, Y, X, f[2], f[3], w1);
    const float m = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-mask)));
    const float m1 = __fsub_rn(1.0f, m);
#pragma unroll
    for (int c = 0; c < 3; ++c)
      out[((static_cast<size_t>(n) * 3 + c) * F.H + y) * F.W + x] =
          __float2half_rn(__fadd_rn(__fmul_rn(w0[c], m), __fmul_rn(w1[c], m1)));
  }
}

// Warp taps of a flow field [n][2][h][w] (FP32): x0, x1, y0, y1 as int32 planes [n][4][h][w] and
// the weights wx, wy as FP32 planes [n][2][h][w] (kb2_warp_taps).
__global__ void warp_taps_kernel(const float* __restrict__ flow, int batch, int h, int w, int32_t* __restrict__ taps,
                                 float* __restrict__ weights) {
  const long long plane = static_cast<long long>(h) * w;
  const long long total = batch * plane;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int x = static_cast<int>(i % w);
    const int y = static_cast<int>((i / w) % h);
    const long long n = i / plane;
    const long long p = i % plane;
    const AxisTap tx = warp_tap(x, flow[(n * 2 + 0) * plane + p], w);
    const AxisTap ty = warp_tap(y, flow[(n * 2 + 1) * plane + p], h);
    taps[(n * 4 + 0) * plane + p] = tx.lo;
    taps[(n * 4 + 1) * plane + p] = tx.hi;
    taps[(n * 4 + 2) * plane + p] = ty.lo;
    taps[(n * 4 + 3) * plane + p] = ty.hi;
    weights[(n * 2 + 0) * plane + p] = tx.t;
    weights[(n * 2 + 1) * plane + p] = ty.t;
  }
}

}  // namespace kb2
