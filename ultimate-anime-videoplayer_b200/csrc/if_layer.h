// One tensor-core convolution of the interpolators (classic IFNet and RIFE 4.2x): packed weights,
// constants, tensor map and launch shape of ifconv_kernel (ifnet_conv.cuh), or of the paired
// stacked kernel (conv3p.cuh) for 64-channel residual convs. Built once per engine for a fixed
// input geometry (if_layer.cu).
#pragma once

#include <vector>

#include "conv_layer.h"
#include "ifnet_conv.cuh"

namespace kb2 {

struct IfKernel;  // one ifconv_kernel instantiation (if_layer.cu)

struct IfLayer {
  IfConvArgs args{};
  IfMaps maps{};
  const IfKernel* k = nullptr;
  DeviceBuffer wpack, bias, slope;
  size_t smem = 0;
  int per_sm = 1;
  int kind = 0;                           // layer timer kind
  double flops_px = 0.0, bytes_px = 0.0;  // algorithmic work per output pixel of the conv grid
  // 64-channel residual convs run on the paired stacked kernel (conv3p.cuh) instead: one M = 256
  // MMA for two SMs, the three kernel rows stacked in N = 192
  ConvLayer pair;
  bool paired = false;
  uint8_t* pair_out = nullptr;
  const uint8_t* pair_res = nullptr;
  int pair_res_chunks = 0;

  // The residual conv (PReLU(conv(x) + bias + x), C -> C, stride 1) of `c` = 64 channels on the
  // pair kernel: w OIHW [c][c][3][3]; the tensors are [n][h][c / 8][w][8] FP16.
  Status build_paired(int c, const float* w, const float* b, const float* prelu, uint8_t* in, int batch, int h,
                      int wd, uint8_t* out, int* err);

  // A 3x3 conv (pad 1) of `stride` over the row-chunked FP16 input `in` ([batch][h_in][in_chunks]
  // [w_in][16 B], parity-split rows when stride is 2) into N = n_pad columns with epilogue `epi`.
  // w: dense weights [n_pad][cin][3][3] (columns beyond cout zero); b, prelu: n_pad values (prelu
  // may be null). `out` / `out_chunks` / `out_f32` as IfConvArgs states for the epilogue. g: input
  // chunks per K group (0: the largest even divisor of in_chunks up to 8); a g above in_chunks
  // reads the missing chunks as zeros (the tensor map's out-of-bounds fill).
  Status build(int n_pad, int stride, int epi, const std::vector<float>& w, int cout, int cin, const float* b,
               const float* prelu, uint8_t* in, int batch, int h_in, int w_in, int in_chunks, int h_out, int w_out,
               uint8_t* out, int out_chunks, float* out_f32, int* err, int g = 0);

  Status launch(cudaStream_t stream, int batch);
};

// Dense [n][cin][3][3] weights of a 4x4 stride-2 (pad 1) transposed conv as a 3x3 conv whose N
// columns are its four output phases: output (2y + py, 2x + px) takes input row y + dy - 1 with
// kernel row kmap[py][dy] (py = 0: dy 0 -> 3, dy 1 -> 1; py = 1: dy 1 -> 2, dy 2 -> 0), the same
// along x. `column(n, &phase, &co)` names the phase (0..3 = 2 py + px) and the transposed conv's
// output channel of column n (co < 0: a zero column). wt: ONNX ConvTranspose [cin][cout][4][4].
template <class Column>
std::vector<float> convt_phase_weights(const float* wt, int cin, int cout, int n_pad, Column column) {
  static constexpr int kmap[2][3] = {{3, 1, -1}, {-1, 2, 0}};
  std::vector<float> w(static_cast<size_t>(n_pad) * cin * 9, 0.0f);
  for (int n = 0; n < n_pad; ++n) {
    int ph = 0, co = -1;
    column(n, &ph, &co);
    if (co < 0) continue;
    for (int ci = 0; ci < cin; ++ci)
      for (int dy = 0; dy < 3; ++dy)
        for (int dx = 0; dx < 3; ++dx) {
          const int ky = kmap[ph >> 1][dy], kx = kmap[ph & 1][dx];
          if (ky < 0 || kx < 0) continue;
          w[((static_cast<size_t>(n) * cin + ci) * 3 + dy) * 3 + dx] =
              wt[((static_cast<size_t>(ci) * cout + co) * 4 + ky) * 4 + kx];
        }
  }
  return w;
}

// Dense weights of an OIHW 3x3 conv [cout][cin][3][3], padded to n_pad columns and scaled per
// output channel by `scale` (null: 1).
std::vector<float> dense_conv_weights(const float* w, int cout, int cin, int n_pad, const float* scale = nullptr);

}  // namespace kb2
