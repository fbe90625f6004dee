// Display-ring pixel codes (the reference's ring store contract, src/kernels/spec/ring_pack.h and
// color.h unorm16), shared by the packing pass (display_pack.cu) and the SPAN upsampler's display
// epilogue (conv_tc.cuh, kOutPixShuf2Display):
//   RGBA16 UNORM: unorm16(v) = trunc(clamp(v, 0, 1) * 65535 + 0.5) per channel (NaN -> 0), alpha 65535;
//   RGB10A2 UNORM: r | g << 10 | b << 20 | 3 << 30 with unorm10(v) = trunc(clamp(v, 0, 1) * 1023 + 0.5);
//   RGB10A2 dithered: clamp(v, 0, 1) * 1023 + 0.5 + n, n the pixel's fixed TPDF noise in (-1, 1) (the
//   sum of two uniforms of an integer hash of (x, y), minus 1), brought into [0, 1023] and truncated.
// Products and sums are written with the _rn intrinsics: the contract's roundings, no contraction.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "kirari_b200.h"

namespace kb2 {

__device__ __forceinline__ float clamp_unit(float v) { return v != v ? 0.0f : fminf(fmaxf(v, 0.0f), 1.0f); }

__device__ __forceinline__ uint16_t unorm16(float v) {
  return static_cast<uint16_t>(__fadd_rn(__fmul_rn(clamp_unit(v), 65535.0f), 0.5f));
}
__device__ __forceinline__ uint32_t unorm10(float v) {
  return static_cast<uint32_t>(__fadd_rn(__fmul_rn(clamp_unit(v), 1023.0f), 0.5f));
}
// the pixel hash (a PCG step) and its uniform in [0, 1) (spec/ring_pack.h)
__device__ __forceinline__ uint32_t ring_hash(uint32_t x, uint32_t y, uint32_t salt) {
  uint32_t v = x * 0x9E3779B1u ^ y * 0x85EBCA77u ^ salt * 0xC2B2AE3Du;
  v = v * 747796405u + 2891336453u;
  v = ((v >> ((v >> 28u) + 4u)) ^ v) * 277803737u;
  return (v >> 22u) ^ v;
}
__device__ __forceinline__ float ring_uniform(uint32_t x, uint32_t y, uint32_t salt) {
  return __fmul_rn(static_cast<float>(ring_hash(x, y, salt) >> 8u), 1.0f / 16777216.0f);
}
__device__ __forceinline__ uint32_t unorm10_dithered(float v, float noise) {
  const float biased = __fadd_rn(__fadd_rn(__fmul_rn(clamp_unit(v), 1023.0f), 0.5f), noise);
  if (!(biased > 0.0f)) return 0u;
  return biased >= 1023.0f ? 1023u : static_cast<uint32_t>(biased);
}

// One RGB10A2 word of pixel (x, y) of a frame, plain or dithered.
__device__ __forceinline__ uint32_t rgb10a2(float r, float g, float b, bool dither, uint32_t x, uint32_t y) {
  uint32_t pr, pg, pb;
  if (!dither) {
    pr = unorm10(r);
    pg = unorm10(g);
    pb = unorm10(b);
  } else {
    const float noise = __fadd_rn(__fadd_rn(ring_uniform(x, y, 5u), ring_uniform(x, y, 6u)), -1.0f);
    pr = unorm10_dithered(r, noise);
    pg = unorm10_dithered(g, noise);
    pb = unorm10_dithered(b, noise);
  }
  return pr | pg << 10 | pb << 20 | 3u << 30;
}

// One RGBA16 pixel as two words (r | g << 16, b | alpha << 16).
__device__ __forceinline__ uint2 rgba16(float r, float g, float b) {
  return make_uint2(static_cast<uint32_t>(unorm16(r)) | static_cast<uint32_t>(unorm16(g)) << 16,
                    static_cast<uint32_t>(unorm16(b)) | 0xFFFF0000u);
}

}  // namespace kb2
