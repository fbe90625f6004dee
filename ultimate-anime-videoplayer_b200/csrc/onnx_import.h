// RIFE 4.2x weights read from ONNX (onnx_import.cu): the pieces of a split RIFE model (the encoder
// and one piece per block) as the reference's native RIFE path reads them (src/prepare/rife_native.h
// rife_native_layers), written out as the weight blob v1 of KB2_MODEL_RIFE_FUSED.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "host_util.h"

namespace kb2 {

// One layer of a piece, in the blob's layouts: Conv 3x3 (pad 1, stride 1 or 2) OIHW
// [cout][cin][3][3]; ConvTranspose 4x4 (stride 2, pad 1) [cin][cout][4][4].
struct OnnxLayer {
  bool transposed = false;
  int cin = 0, cout = 0, stride = 1;
  std::vector<float> w, b;
  std::vector<float> slope;  // negative slope per output channel; empty: no activation
  std::vector<float> scale;  // residual act(scale (conv + b) + x); empty: no residual
};

// The layer chain of one ONNX piece (a ModelProto's bytes): from its single input to its single
// output, Conv (+ LeakyRelu / PRelu / Relu, + Mul by a per-channel constant and Add of the conv's
// input), ending with a ConvTranspose; Cast and Identity pass through. Refuses anything else.
Status onnx_piece_layers(const uint8_t* model, size_t bytes, std::vector<OnnxLayer>& layers);

// The blob of KB2_MODEL_RIFE_FUSED from the encoder piece and `blocks` block pieces, with the
// plan's input reductions `reduce` (the block widths come from the weights).
Status rife_blob_from_onnx(const uint8_t* const* pieces, const uint64_t* sizes, int blocks, const int32_t* reduce,
                           std::vector<uint8_t>& blob);

}  // namespace kb2
