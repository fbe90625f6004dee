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
//    frame). The flow at a pixel is the sum, in block order, of those tensors resized to the pixel
//    and scaled by 2 s_j: the network's sequential `flow = flow + resize(...)`. Blocks 1 and 2 need
//    it only at their resize sample points and compute it there; block 3 computes it at every pixel
//    and leaves it in FP32 planes, to which the blend adds block 3's own part;
//  * every resize of this network has a power-of-two scale (the padded frame is a multiple of 32),
//    so the position (o + 0.5) / scale is computed as (o + 0.5) * (1 / scale): exact, the same value.
//
// Every product and sum is written with the _rn intrinsics, in the order the network states it,
// so that no multiply-add contraction changes a warp position.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "glue_common.cuh"

namespace kb2 {

constexpr int kIfBlocks = 4;
// Scale of block k: the block works on the frame at 1/8, 1/4, 1/2, 1/1.
__host__ __device__ constexpr int if_scale(int k) { return 8 >> k; }

// The outputs of the transposed convs so far, FP32 [n][h][w][8] (5 used) at 1/(2 s) of the padded frame.
struct IfFlowLevels {
  const float* t[kIfBlocks];
  int h[kIfBlocks], w[kIfBlocks];
  float mul[kIfBlocks];  // 2 s: flow scale of block j
  float inv[kIfBlocks];  // 1 / (2 s): resize position factor from the frame to block j's tensor
};


// NCHW frames -> padded RGBx pixels (zeros outside the window).
__global__ void ifnet_pad_frames_kernel(IfFrames F, int batch) {
  const size_t plane = static_cast<size_t>(F.H) * F.W;
  const int X = blockIdx.x * blockDim.x + threadIdx.x;
  if (X >= F.Wp) return;
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
  }
}

// The video-stream form of the padding: pair n is frames n and n + 1 of one buffer (img1 = img0 one
// frame on), so each of the `frames` = batch + 1 frames is padded once, into consecutive planes of
// pad0, and pad1 = pad0 one plane on. Same pixels as ifnet_pad_frames_kernel, half the traffic.
__global__ void ifnet_pad_stream_kernel(IfFrames F, int frames) {
  const size_t plane = static_cast<size_t>(F.H) * F.W;
  const int X = blockIdx.x * blockDim.x + threadIdx.x;
  if (X >= F.Wp) return;
  for (int r = blockIdx.y; r < frames * F.Hp; r += gridDim.y) {
    const int n = r / F.Hp;
    const int Y = r - n * F.Hp;
    const int y = Y - F.top, x = X - F.left;
    uint2 p = make_uint2(0, 0);
    if (y >= 0 && y < F.H && x >= 0 && x < F.W) {
      const size_t at = static_cast<size_t>(n) * 3 * plane + static_cast<size_t>(y) * F.W + x;
      const __half2 c01 = __halves2half2(F.img0[at], F.img0[at + plane]);
      const __half2 c2 = __halves2half2(F.img0[at + 2 * plane], __float2half_rn(0.0f));
      p = make_uint2(*reinterpret_cast<const uint32_t*>(&c01), *reinterpret_cast<const uint32_t*>(&c2));
    }
    F.pad0[static_cast<size_t>(r) * F.Wp + X] = p;
  }
}

// The x half of block j's flow resize at one full-resolution column, cached along a column: the
// column's x tap (fixed), and for the source row pair last used (lo, hi) both rows' 5 channels
// interpolated in x. Output rows that resample the same source rows (2, 4 or 8 in a row at
// scales 2, 4 and 8 of the flow tensor) then only interpolate in y. The arithmetic is that of the
// resize, x first: lerp(lerp(q00, q01, tx), lerp(q10, q11, tx), ty).
struct LevelCol {
  AxisTap tx;
  int lo, hi;
  float top[5], bot[5];
};

__device__ __forceinline__ void level_col_init(const IfFlowLevels& L, int j, int X, LevelCol& c) {
  c.tx = resize_tap(X, L.inv[j], L.w[j]);
  c.lo = -1;
  c.hi = -1;
}

// Adds block j's contribution at padded row Y of column c (frame n) to the flow (4) and mask;
// block 0 sets them. The threads of a warp share Y, so the refill branch is uniform.
__device__ __forceinline__ void flow_step_col(const IfFlowLevels& L, int j, int n, int Y, LevelCol& c, float f[4],
                                              float* mask) {
  const AxisTap ty = resize_tap(Y, L.inv[j], L.h[j]);
  if (ty.lo != c.lo || ty.hi != c.hi) {
    const float* base = L.t[j] + static_cast<size_t>(n) * L.h[j] * L.w[j] * 8;
    const float* ra = base + static_cast<size_t>(ty.lo) * L.w[j] * 8;
    const float* rb = base + static_cast<size_t>(ty.hi) * L.w[j] * 8;
    const float* px[4] = {ra + c.tx.lo * 8, ra + c.tx.hi * 8, rb + c.tx.lo * 8, rb + c.tx.hi * 8};
    float q[4][5];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4 u = __ldg(reinterpret_cast<const float4*>(px[k]));
      q[k][0] = u.x;
      q[k][1] = u.y;
      q[k][2] = u.z;
      q[k][3] = u.w;
      q[k][4] = __ldg(px[k] + 4);
    }
#pragma unroll
    for (int ch = 0; ch < 5; ++ch) {
      c.top[ch] = lerp_rn(q[0][ch], q[1][ch], c.tx.t);
      c.bot[ch] = lerp_rn(q[2][ch], q[3][ch], c.tx.t);
    }
    c.lo = ty.lo;
    c.hi = ty.hi;
  }
  float v[5];
#pragma unroll
  for (int ch = 0; ch < 5; ++ch) v[ch] = lerp_rn(c.top[ch], c.bot[ch], ty.t);
  if (j == 0) {
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) f[ch] = __fmul_rn(v[ch], L.mul[j]);
    *mask = v[4];
  } else {
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) f[ch] = __fadd_rn(f[ch], __fmul_rn(v[ch], L.mul[j]));
    *mask = __fadd_rn(*mask, v[4]);
  }
}

// Full-resolution flow (planes 0-3) and mask (plane 4) after blocks 0-2: FP32 [n][5][Hp][Wp],
// written by block 3's input kernel, read by the blend.
struct IfFlowField {
  float* f;
  int Hp, Wp;
  __device__ __forceinline__ float* pixel(int n, int Y, int X) const {
    return f + static_cast<size_t>(n) * 5 * Hp * Wp + static_cast<size_t>(Y) * Wp + X;
  }
  __device__ __forceinline__ size_t plane() const { return static_cast<size_t>(Hp) * Wp; }
};


// The 12 input planes of block K >= 1 at padded full-resolution pixel (Y, X) of frame n: warped
// frames (6), timestep, mask, flow (4, not yet divided by the block scale), the flow from the
// column caches of blocks 0 .. K - 1. Block 3 also stores the flow.
template <int K>
__device__ __forceinline__ void block_planes(const IfFrames& F, const IfFlowLevels& L, const IfFlowField& FF, int n,
                                             int Y, int X, LevelCol (&cols)[K], float timestep, float v[12]) {
  float f[4], mask;
#pragma unroll
  for (int j = 0; j < K; ++j) flow_step_col(L, j, n, Y, cols[j], f, &mask);
  if constexpr (K == kIfBlocks - 1) {
    float* p = FF.pixel(n, Y, X);
    const size_t pl = FF.plane();
#pragma unroll
    for (int c = 0; c < 4; ++c) p[c * pl] = f[c];
    p[4 * pl] = mask;
  }
  const size_t frame = static_cast<size_t>(n) * F.Hp * F.Wp;
  warp3(F.pad0 + frame, F, Y, X, f[0], f[1], v);
  warp3(F.pad1 + frame, F, Y, X, f[2], f[3], v + 3);
  v[6] = timestep;
  v[7] = mask;
#pragma unroll
  for (int c = 0; c < 4; ++c) v[8 + c] = f[c];
}

// Output rows per thread in the glue kernels: a thread walks a run of rows down one column (runs
// never cross frames), so the flow caches are refilled once per source row pair.
constexpr int kGlueRunRows = 8;

// Block K's input row run: rows per run at the block's scale (8 full-resolution rows).
template <int K>
constexpr int glue_run() {
  return kGlueRunRows / if_scale(K) > 0 ? kGlueRunRows / if_scale(K) : 1;
}

// Stores the 16 planes of one output pixel as two FP16 chunks. Each chunk row is parity-split,
// the even pixels then the odd ones (wo even), which is the layout conv0a's stride-2 loads read.
__device__ __forceinline__ void store_chunks(uint8_t* row, int wo, int ox, const float v[16]) {
  const int xs = (ox & 1) * (wo >> 1) + (ox >> 1);
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
    *reinterpret_cast<uint4*>(row + (static_cast<size_t>(ch) * wo + xs) * 16) = o;
  }
}

// store_chunks of 16 planes already paired as FP16.
__device__ __forceinline__ void store_chunks_h2(uint8_t* row, int wo, int ox, const __half2 v[8]) {
  const int xs = (ox & 1) * (wo >> 1) + (ox >> 1);
  const uint32_t* u = reinterpret_cast<const uint32_t*>(v);
#pragma unroll
  for (int ch = 0; ch < 2; ++ch)
    *reinterpret_cast<uint4*>(row + (static_cast<size_t>(ch) * wo + xs) * 16) =
        make_uint4(u[4 * ch], u[4 * ch + 1], u[4 * ch + 2], u[4 * ch + 3]);
}

// Input of block K as row-chunked FP16 [n][Hp/s][2][Wp/s][8 halves] (16 channels, 12 or 7 used;
// each chunk row parity-split):
// the block's planes resized to 1/s (not for s = 1), the flow planes then divided by s. One
// instantiation per block, so that every plane array stays in registers; 64 registers a thread
// (4 blocks of 256 per SM: measured 19-27 % faster than 80-88 registers at 2-3 blocks, no spills).
//  * s = 1: one thread per column, walking glue_run<K>() rows;
//  * s > 1: two threads per output column, one per resize sample column (lo, hi); each computes
//    the planes at its column for both sample rows, and the pair exchanges them by a shuffle so
//    that both hold lerp(q(x lo), q(x hi), tx) for each row; the even thread stores.
template <int K>
__global__ void __launch_bounds__(kGlueThreads, 4)
    ifnet_block_input_kernel(IfFrames F, IfFlowLevels L, IfFlowField FF, int batch, float timestep,
                             uint8_t* __restrict__ out) {
  constexpr int s = if_scale(K);
  constexpr int R = glue_run<K>();
  constexpr int nc = K == 0 ? 7 : 12;
  const int ho = F.Hp / s, wo = F.Wp / s;
  const int runs = (ho + R - 1) / R;
  if constexpr (s == 1) {
    const int X = blockIdx.x * blockDim.x + threadIdx.x;
    if (X >= wo) return;
    LevelCol cols[K];
#pragma unroll
    for (int j = 0; j < K; ++j) level_col_init(L, j, X, cols[j]);
    for (int r = blockIdx.y; r < batch * runs; r += gridDim.y) {
      const int n = r / runs;
      const int y0 = (r - n * runs) * R;
#pragma unroll
      for (int j = 0; j < K; ++j) cols[j].lo = -1;
      for (int y = y0; y < y0 + R && y < ho; ++y) {
        float v[16];
#pragma unroll
        for (int c = 12; c < 16; ++c) v[c] = 0.0f;
        block_planes<K>(F, L, FF, n, y, X, cols, timestep, v);
        // the flow planes divided by s = 1: unchanged
        store_chunks(out + (static_cast<size_t>(n) * ho + y) * 2 * wo * 16, wo, X, v);
      }
    }
  } else {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    const int ox = t >> 1;
    const int side = t & 1;
    const bool live = ox < wo;  // both threads of a pair agree; the shuffles need every lane
    const AxisTap tx = resize_tap(live ? ox : wo - 1, static_cast<float>(s), F.Wp);
    const int X = side ? tx.hi : tx.lo;
    LevelCol cols[K > 0 ? K : 1];
#pragma unroll
    for (int j = 0; j < K; ++j) level_col_init(L, j, X, cols[j]);
    const float inv = __fdiv_rn(1.0f, static_cast<float>(s));
    for (int r = blockIdx.y; r < batch * runs; r += gridDim.y) {
      const int n = r / runs;
      const int y0 = (r - n * runs) * R;
#pragma unroll
      for (int j = 0; j < K; ++j) cols[j].lo = -1;
      for (int oy = y0; oy < y0 + R && oy < ho; ++oy) {
        const AxisTap ty = resize_tap(oy, static_cast<float>(s), F.Hp);
        // the planes' resize (x by the pair's shuffle, then y) as packed FP16 pairs: the block
        // input is stored in FP16, and no tap position depends on it
        constexpr int np = (nc + 1) / 2;
        const __half2 wx = __float2half2_rn(tx.t), wy = __float2half2_rn(ty.t);
        __half2 h[2][np];
#pragma unroll
        for (int yy = 0; yy < 2; ++yy) {
          const int Y = yy ? ty.hi : ty.lo;
          float q[12];
          if constexpr (K == 0) {
            const size_t frame = static_cast<size_t>(n) * F.Hp * F.Wp;
            frame_rgb(F.pad0 + frame, F.Wp, Y, X, q);
            frame_rgb(F.pad1 + frame, F.Wp, Y, X, q + 3);
            q[6] = timestep;
            q[7] = 0.0f;
          } else {
            block_planes<K>(F, L, FF, n, Y, X, cols, timestep, q);
          }
#pragma unroll
          for (int i = 0; i < np; ++i) {
            const __half2 mine = __floats2half2_rn(q[2 * i], q[2 * i + 1]);
            const uint32_t mu = *reinterpret_cast<const uint32_t*>(&mine);
            const uint32_t pu = __shfl_xor_sync(0xffffffffu, mu, 1);
            const __half2 other = *reinterpret_cast<const __half2*>(&pu);
            const __half2 lo = side ? other : mine, hi = side ? mine : other;
            h[yy][i] = __hfma2(wx, __hsub2(hi, lo), lo);
          }
        }
        __half2 v2[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          v2[i] = i < np ? __hfma2(wy, __hsub2(h[1][i], h[0][i]), h[0][i]) : __floats2half2_rn(0.0f, 0.0f);
        if constexpr (K > 0) {  // the flow planes 8-11 divided by s (a power of two: exact)
          const __half2 inv2 = __float2half2_rn(inv);
          v2[4] = __hmul2(v2[4], inv2);
          v2[5] = __hmul2(v2[5], inv2);
        }
        if (live && side == 0) store_chunks_h2(out + (static_cast<size_t>(n) * ho + oy) * 2 * wo * 16, wo, ox, v2);
      }
    }
  }
}

// The interpolated frame: warp both frames by the final flow, blend with sigmoid(mask) (as
// 1 / (1 + __expf(-mask)), the reference's fused finish, rife_finish.cuh:46), crop the
// window: out = w0 * m + w1 * (1 - m), NCHW FP16 [n][3][H][W]. One thread per column walking
// kGlueRunRows rows, with block 3's flow resize cached along the column.
__global__ void ifnet_blend_kernel(IfFrames F, IfFlowLevels L, IfFlowField FF, int batch, __half* __restrict__ out) {
  const int x = blockIdx.x * blockDim.x + threadIdx.x;
  if (x >= F.W) return;
  const int X = x + F.left;
  LevelCol col;
  level_col_init(L, kIfBlocks - 1, X, col);
  const int runs = (F.H + kGlueRunRows - 1) / kGlueRunRows;
  const size_t pl = FF.plane();
  for (int r = blockIdx.y; r < batch * runs; r += gridDim.y) {
    const int n = r / runs;
    const int y0 = (r - n * runs) * kGlueRunRows;
    col.lo = -1;
    const size_t frame = static_cast<size_t>(n) * F.Hp * F.Wp;
    for (int y = y0; y < y0 + kGlueRunRows && y < F.H; ++y) {
      const int Y = y + F.top;
      const float* p = FF.pixel(n, Y, X);
      float f[4], mask;
#pragma unroll
      for (int c = 0; c < 4; ++c) f[c] = __ldg(p + c * pl);
      mask = __ldg(p + 4 * pl);
      flow_step_col(L, kIfBlocks - 1, n, Y, col, f, &mask);
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

// The motion variant's outputs in place of the blend (the reference's motion finish,
// src/gpu/cuda/backend/rife_finish.cuh:40-55, called from fused_finish, rife_fused_kernels.cu:208):
// over the whole padded plane, the final flow (FP32 planes of blocks 0-2 plus block 3's part, in
// the network's order) into flow [n][4][Hp][Wp] and sigmoid(mask), the weight of frame A, into
// mask [n][1][Hp][Wp]; T = float, or __half as the reference's engine writes them. One thread per
// column walking kGlueRunRows rows, with block 3's flow resize cached along the column; each plane
// row is one coalesced run of stores.

template <typename T>
__global__ void ifnet_motion_kernel(IfFrames F, IfFlowLevels L, IfFlowField FF, int batch, T* __restrict__ flow,
                                    T* __restrict__ mask) {
  const int X = blockIdx.x * blockDim.x + threadIdx.x;
  if (X >= F.Wp) return;
  LevelCol col;
  level_col_init(L, kIfBlocks - 1, X, col);
  const int runs = (F.Hp + kGlueRunRows - 1) / kGlueRunRows;
  const size_t pl = FF.plane();
  for (int r = blockIdx.y; r < batch * runs; r += gridDim.y) {
    const int n = r / runs;
    const int y0 = (r - n * runs) * kGlueRunRows;
    col.lo = -1;
    for (int Y = y0; Y < y0 + kGlueRunRows && Y < F.Hp; ++Y) {
      const float* p = FF.pixel(n, Y, X);
      float f[4], m;
#pragma unroll
      for (int c = 0; c < 4; ++c) f[c] = __ldg(p + c * pl);
      m = __ldg(p + 4 * pl);
      flow_step_col(L, kIfBlocks - 1, n, Y, col, f, &m);
      const size_t at = static_cast<size_t>(Y) * F.Wp + X;
#pragma unroll
      for (int c = 0; c < 4; ++c) store_motion(flow + (static_cast<size_t>(n) * 4 + c) * pl + at, f[c]);
      store_motion(mask + static_cast<size_t>(n) * pl + at, __fdiv_rn(1.0f, __fadd_rn(1.0f, __expf(-m))));
    }
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
