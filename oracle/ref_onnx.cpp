// TEST INFRASTRUCTURE ONLY: a C entry point over the reference's own reader of RIFE ONNX pieces
// (Ta2b/Ultimate-Anime-VideoPlayer src/prepare/rife_native.cpp rife_native_layers, over its ONNX
// reader src/gpu/ir/onnx_reader.cpp / onnx_tensor.cpp / protobuf.cpp, compiled in place by
// oracle/Makefile). The tests compare the library's kb2_rife_blob_from_onnx against it piece by
// piece. Nothing in the product path links or loads it.
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <span>
#include <string>

#include "prepare/rife_native.h"

namespace {

void set_error(char* err, int cap, const std::string& what) {
  if (err == nullptr || cap <= 0) return;
  const size_t n = std::min(static_cast<size_t>(cap - 1), what.size());
  std::memcpy(err, what.data(), n);
  err[n] = '\0';
}

}  // namespace

extern "C" {

// The layers of one piece. meta receives 9 int32 per layer (transposed, cin, cout, kernel, stride,
// then the float counts of weights, bias, slope and scale); vals receives each layer's weights in
// the reference's [cout][kernel^2][cin] order, then bias, slope and scale. Returns the layer count,
// -1 when the reference refuses the piece (err holds its refusal detail), -2 when a buffer is short.
int kref_rife_native_layers(const void* bytes, uint64_t size, int32_t* meta, int max_layers, float* vals,
                            uint64_t max_vals, char* err, int err_cap) {
  const auto piece = std::span<const std::byte>(static_cast<const std::byte*>(bytes), static_cast<size_t>(size));
  auto layers = kirari::prepare::rife_native_layers(piece);
  if (!layers) {
    set_error(err, err_cap, layers.error().detail);
    return -1;
  }
  if (static_cast<int>(layers->size()) > max_layers) return -2;
  uint64_t used = 0;
  int i = 0;
  for (const auto& l : *layers) {
    int32_t* m = meta + 9 * i++;
    m[0] = l.transposed ? 1 : 0;
    m[1] = l.cin;
    m[2] = l.cout;
    m[3] = l.kernel;
    m[4] = l.stride;
    m[5] = static_cast<int32_t>(l.weights.size());
    m[6] = static_cast<int32_t>(l.bias.size());
    m[7] = static_cast<int32_t>(l.slope.size());
    m[8] = static_cast<int32_t>(l.scale.size());
    for (const auto* v : {&l.weights, &l.bias, &l.slope, &l.scale}) {
      if (used + v->size() > max_vals) return -2;
      std::memcpy(vals + used, v->data(), v->size() * sizeof(float));
      used += v->size();
    }
  }
  return static_cast<int>(layers->size());
}

}  // extern "C"
