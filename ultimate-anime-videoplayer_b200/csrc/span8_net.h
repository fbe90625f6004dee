// The AnimeJaNai "unshuffle" SPAN (b5f48, b8f64 and the like) read from a .span8 package, on the
// tensor-core conv layers (see span8_net.cu).
#pragma once

#include <memory>
#include <string>
#include <vector>

#include "conv_layer.h"
#include "layer_timer.h"

namespace kb2 {

// The package, as read by parse_span8: FP16 weights widened to float, in the package's order
// ([out][ky][kx][in] over the stored channels), and the f32 biases.
struct Span8Package {
  struct Conv {
    std::vector<float> w, b;
  };
  struct Block {
    Conv c[3], att;
  };
  int version = 0, blocks = 0, real = 0;
  uint32_t flags = 0;
  std::vector<float> scales;
  Conv first, concat, pixel;
  std::vector<Block> block;
};

// Reads and checks a .span8 package (the reference's span_fp8::parse, src/gpu/span_fp8/package.cpp:143):
// magic, version 1 or 2, 2..8 blocks (8 in version 1) stored in 64 channels with 48 or 64 real,
// known flags, payload size, CRC-32, finite weights and biases, positive scales, nothing left over.
// Refusals: KB2_WEIGHTS_INVALID where the reference says FileUnreadable (size, truncation, CRC),
// KB2_FORMAT_UNSUPPORTED where it says FormatUnsupported (magic, version, flags, shape, contents).
Status parse_span8(const void* bytes, uint64_t n, Span8Package& out);

class Span8Net {
 public:
  // fp8: the blocks' 3x3 convs in E4M3 with the package's activation scales (an FP8 package);
  // otherwise every layer in FP16.
  Status create(const Span8Package& pkg, bool fp8, int max_batch, int H, int W);
  // in: NCHW F16 [batch][3][H][W]; out: NCHW F16 [batch][3][2H][2W] (device pointers).
  // peaks: raise the package's 1 + 3 * blocks activation peaks there (FP16 engine only).
  Status run(cudaStream_t stream, const void* in, void* out, int batch, unsigned int* peaks = nullptr);
  // The FP16 engine over n frames: max |v| of each tensor the package scales (package.h:15-17:
  // [0] conv_1's output, per block b [1 + 3b] and [2 + 3b] its two ReLU outputs, [3 + 3b] its output),
  // the peaks the reference's span_fp8::derive collects (derive.h:42-46). Synchronous on `stream`.
  Status calibrate(cudaStream_t stream, const void* frames, int n, float* peaks_out);
  int scale_count() const { return 1 + 3 * blocks_; }
  size_t device_bytes() const;
  int* err_word() const { return err_.as<int>(); }
  int height() const { return H_; }
  int width() const { return W_; }
  int max_batch() const { return max_batch_; }
  int launches_per_run() const { return 1 + static_cast<int>(steps_.size()); }
  LayerTimer& timer() { return timer_; }

 private:
  struct Tensor {
    ChunkedTensor t;
    DeviceBuffer buf;
  };
  struct Step {
    ConvLayer* layer;
    const ChunkedTensor* out;  // null: the caller's output frame
    const ChunkedTensor* out2;  // E4M3 copy (dual-output layers), or null
    float out_inv_scale;        // 1 / scale of the E4M3 output
    const ChunkedTensor* residual;
    const ChunkedTensor* residual2;
    int kind;
    int peak;  // index of `out` among the package's scaled tensors, -1 none
  };
  Status make_tensor(std::unique_ptr<Tensor>& t, int chunks, bool fp8 = false);

  int max_batch_ = 0, H_ = 0, W_ = 0, h_ = 0, w_ = 0, ch_ = 0;
  bool fp8_ = false;
  int blocks_ = 0;
  DeviceBuffer err_, peaks_;
  std::vector<std::unique_ptr<Tensor>> tensors_;
  std::vector<std::unique_ptr<ConvLayer>> layers_;
  std::vector<Step> steps_;
  const ChunkedTensor* unshuffled_ = nullptr;
  LayerTimer timer_;
  int k_pack_ = 0;
};

}  // namespace kb2
