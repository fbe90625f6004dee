// Display-ring pixels from the engines' FP16 frames: the reference's ring store (pixel_kernels.cuh
// store_ring; its contract src/kernels/spec/ring_pack.h and color.h unorm16, display_pixel.cuh), as a
// pass over NCHW frames into a pitched buffer of packed pixels.
#include <cuda_fp16.h>

#include <algorithm>

#include "display_pixel.cuh"
#include "engine.h"

namespace kb2 {

namespace {

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
      reinterpret_cast<uint2*>(row)[x] = rgba16(cr, cg, cb);
    } else {
      reinterpret_cast<uint32_t*>(row)[x] = rgb10a2(cr, cg, cb, kFormat == KB2_DISPLAY_RGB10A2_DITHER,
                                                    static_cast<uint32_t>(x), static_cast<uint32_t>(y));
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
