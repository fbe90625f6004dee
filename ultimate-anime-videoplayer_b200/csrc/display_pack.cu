// Display-ring pixels from the engines' FP16 frames: the reference's ring store (pixel_kernels.cuh
// store_ring; its contract src/kernels/spec/ring_pack.h and color.h unorm16), as a pass over NCHW
// frames into a pitched buffer of packed pixels:
//   RGBA16 UNORM: unorm16(v) = trunc(clamp(v, 0, 1) * 65535 + 0.5) per channel (NaN -> 0), alpha 65535;
//   RGB10A2 UNORM: r | g << 10 | b << 20 | 3 << 30 with unorm10(v) = trunc(clamp(v, 0, 1) * 1023 + 0.5);
//   RGB10A2 dithered: clamp(v, 0, 1) * 1023 + 0.5 + n, n the pixel's fixed TPDF noise in (-1, 1) (the
//   sum of two uniforms of an integer hash of (x, y), minus 1), brought into [0, 1023] and truncated.
// Products and sums are written with the _rn intrinsics: the contract's roundings, no contraction.
#include <cuda_fp16.h>

#include <algorithm>

#include "engine.h"

namespace kb2 {

namespace {

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

template <int kFormat>
__global__ void display_pack_kernel(const __half* __restrict__ in, int batch, int H, int W, uint8_t* __restrict__ out,
                                    long long pitch) {
  const int x = blockIdx.x * blockDim.x + threadIdx.x;
  if (x >= W) return;
  const size_t plane = static_cast<size_t>(H) * W;
  for (int r = blockIdx.y; r < batch * H; r += gridDim.y) {
    const int n = r / H;
    const int y = r - n * H;
    const __half* p = in + static_cast<size_t>(n) * 3 * plane + static_cast<size_t>(y) * W + x;
    const float cr = __half2float(p[0]), cg = __half2float(p[plane]), cb = __half2float(p[2 * plane]);
    uint8_t* row = out + static_cast<size_t>(r) * static_cast<size_t>(pitch);
    if constexpr (kFormat == KB2_DISPLAY_RGBA16) {
      const uint32_t lo = static_cast<uint32_t>(unorm16(cr)) | static_cast<uint32_t>(unorm16(cg)) << 16;
      const uint32_t hi = static_cast<uint32_t>(unorm16(cb)) | 0xFFFF0000u;
      reinterpret_cast<uint2*>(row)[x] = make_uint2(lo, hi);
    } else {
      uint32_t pr, pg, pb;
      if constexpr (kFormat == KB2_DISPLAY_RGB10A2) {
        pr = unorm10(cr);
        pg = unorm10(cg);
        pb = unorm10(cb);
      } else {
        const uint32_t ux = static_cast<uint32_t>(x), uy = static_cast<uint32_t>(y);
        const float noise = __fadd_rn(__fadd_rn(ring_uniform(ux, uy, 5u), ring_uniform(ux, uy, 6u)), -1.0f);
        pr = unorm10_dithered(cr, noise);
        pg = unorm10_dithered(cg, noise);
        pb = unorm10_dithered(cb, noise);
      }
      reinterpret_cast<uint32_t*>(row)[x] = pr | pg << 10 | pb << 20 | 3u << 30;
    }
  }
}

}  // namespace

Status pack_display(cudaStream_t stream, const kb2_tensor* frames, int format, void* out, long long pitch) {
  if (frames == nullptr || out == nullptr) return refuse(KB2_INVALID_ARGUMENT, "pack_display: null pointer");
  if (format != KB2_DISPLAY_RGBA16 && format != KB2_DISPLAY_RGB10A2 && format != KB2_DISPLAY_RGB10A2_DITHER)
    return refuse(KB2_FORMAT_UNSUPPORTED, "pack_display: unknown display format");
  if (frames->type != KB2_F16 || frames->dims[1] != 3) return refuse(KB2_INPUT_MISMATCH, "pack_display: F16 [n,3,H,W]");
  const long long n = frames->dims[0], H = frames->dims[2], W = frames->dims[3];
  if (n < 1 || H < 1 || W < 1 || H > 16384 || W > 16384 || n * H > (1LL << 30))
    return refuse(KB2_SHAPE_INVALID, "pack_display: frame size out of range");
  const long long px_bytes = format == KB2_DISPLAY_RGBA16 ? 8 : 4;
  if (pitch < W * px_bytes || pitch % px_bytes != 0 || (reinterpret_cast<uintptr_t>(out) % px_bytes) != 0)
    return refuse(KB2_INPUT_MISMATCH, "pack_display: pitch below a row or misaligned output");
  const uint64_t addr = frames->handle + frames->offset;
  if (addr == 0 || (addr & 1u) != 0) return refuse(KB2_INPUT_MISMATCH, "pack_display: null or misaligned frames");
  const auto* in = reinterpret_cast<const __half*>(addr);
  auto* o = static_cast<uint8_t*>(out);
  const int bx = static_cast<int>((W + 127) / 128);
  const dim3 g(static_cast<unsigned>(bx),
               static_cast<unsigned>(std::max(1LL, std::min({n * H, 65535LL, (16LL * 148 + bx - 1) / bx}))));
  const int nn = static_cast<int>(n), hh = static_cast<int>(H), ww = static_cast<int>(W);
  if (format == KB2_DISPLAY_RGBA16)
    display_pack_kernel<KB2_DISPLAY_RGBA16><<<g, 128, 0, stream>>>(in, nn, hh, ww, o, pitch);
  else if (format == KB2_DISPLAY_RGB10A2)
    display_pack_kernel<KB2_DISPLAY_RGB10A2><<<g, 128, 0, stream>>>(in, nn, hh, ww, o, pitch);
  else
    display_pack_kernel<KB2_DISPLAY_RGB10A2_DITHER><<<g, 128, 0, stream>>>(in, nn, hh, ww, o, pitch);
  return cuda_status(cudaGetLastError(), "pack_display launch");
}

}  // namespace kb2
