// One E4M3 SPAN block (three 3x3 convolutions and the gate) as a single fused kernel launch.
#pragma once

#include "conv_layer.h"
#include "spab8.cuh"

namespace kb2 {

struct SpabLayer {
  SpabArgs args{};
  size_t smem = 0;

  // c1..c3: the block's built E4M3 layers (their weights, scales and K steps are used as they are);
  // x_in: the block input (E4M3, 3 chunks). inv1 / inv2: 1 / E4M3 scale of the two activations,
  // inv3: of the block output (unused for the last block, which writes FP16), res_scale: scale of
  // the block input.
  Status build(const ConvLayer& c1, const ConvLayer& c2, const ConvLayer& c3, const ChunkedTensor& x_in, float inv1,
               float inv2, float inv3, float res_scale, bool last, int* err);
  // out: block output; t1_f16: the last block's FP16 copy of its first activation (else null).
  Status launch(cudaStream_t stream, int batch, void* out, void* t1_f16) const;

 private:
  bool last_ = false;
  CUtensorMap map_{};
};

}  // namespace kb2
