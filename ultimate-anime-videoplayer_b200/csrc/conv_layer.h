// One tensor-core convolution layer: K-step table, packed weights, tensor maps and the launch of
// conv_tc_kernel (conv_tc.cuh) for a fixed input geometry.
#pragma once

#include <vector>

#include "conv_tc.cuh"
#include "host_util.h"

namespace kb2 {

struct ConvSpec {
  int taps = 9;           // 9: 3x3 pad 1; 1: 1x1
  bool fp8 = false;       // E4M3 operands (else FP16)
  int n_sources = 1;      // 1, or 4: the concat-free 1x1 (conv_cat), or kEpiColsBias (conv_cat + upsampler)
  int cin = 48;           // real input channels per source
  int n_real = 48;        // real output channels
  int n_pad = 48;         // N of the MMA (multiple of 16, <= 64)
  int epi = kEpiBias;
  int out = kOutF16Chunk;
  int out_chunks = 6;     // chunks per output pixel (chunked outputs)
  int out2_chunks = 3;    // kOutF16E4m3: chunks of the E4M3 copy
};

struct ConvLayer {
  ConvSpec spec;
  ConvArgs args{};
  ConvMaps maps{};
  DeviceBuffer wpack, bias, scale, slope;
  size_t smem = 0;
  int grid = 0;
  int kind = 0;  // kernel family: 0 conv_tc.cuh, 2 conv3p.cuh (paired stacked 3x3)

  // W: [n_real][n_sources * cin][k][k] (OIHW), b: [n_real]. act_scales: per-source E4M3 scale of
  // the input tensors (FP8 only; folded into the per-output-channel weight scales).
  Status build(const ConvSpec& s, const float* W, const float* b, const float* prelu_slope,
               const float* act_scales, const ChunkedTensor* const* inputs, int* err_word);
  // kEpiColsBias: the bias term of each tap, [9][n_real] (tap ky * 3 + kx), dropped where that tap
  // falls outside the image (ConvArgs::tap_bias)
  void set_tap_bias(const float* tb);
  // residual / out: device pointers for this launch (residual may be null); residual2: the second
  // addend of kEpiTanhGate.
  // display: kOutPixShuf2Display's row pitch and kb2_display_format.
  Status launch(cudaStream_t stream, int batch, void* out, const void* residual, float out_inv_scale,
                float res_scale, void* out2 = nullptr, int res_chunks = 0, const void* residual2 = nullptr,
                long long out_pitch = 0, int display_format = 0) const;
};

int num_sms();

}  // namespace kb2
