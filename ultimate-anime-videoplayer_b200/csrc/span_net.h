// Canonical SPAN x2 network on the tensor-core conv layers (see span_net.cu).
#pragma once

#include <memory>
#include <string>
#include <vector>

#include "conv_layer.h"

namespace kb2 {

constexpr size_t kSpanParams = KB2_SPAN_X2_PARAMS;  // the blob order of include/kirari_b200.h
constexpr int kSpanScales = 19;         // 1 + 3 * 6 E4M3 activation scales
constexpr int kSpanBlocks = 6;

// max |v| over n_half2 FP16 pairs raised into *dst (atomicMax on the float bits; *dst starts at 0).
Status launch_absmax(cudaStream_t stream, const void* f16, size_t n_half2, unsigned int* dst);

class SpanNet {
 public:
  // shared_err: another network's device error word to report into (null: its own).
  Status create(const std::vector<float>& params, int precision, int max_batch, int H, int W,
                const float* act_scales, int n_scales, int* shared_err = nullptr);
  // in: NCHW F16 [batch][3][H][W]; out: NCHW F16 [batch][3][2H][2W] (device pointers).
  // peaks_dst: where capture_peaks collects the 19 peak words (null: the engine's own words).
  Status run(cudaStream_t stream, const void* in, void* out, int batch, bool capture_peaks = false,
             unsigned int* peaks_dst = nullptr);
  Status calibrate(cudaStream_t stream, const void* frames, int n, float* peaks_out);
  // 0: run() writes NCHW F16 frames; a kb2_display_format: packed display pixels from the
  // upsampler's epilogue, rows of 2W pixels (display_bytes() each) at out + row * 2W * bytes.
  Status set_output_format(int format);
  int output_format() const { return out_format_; }
  int display_bytes() const { return out_format_ == KB2_DISPLAY_RGBA16 ? 8 : 4; }
  // calibrate() with the caller's device scratch in place of its per-call allocation: the peak
  // words at the start of `scratch`, the discarded x2 frames after them (kb2_span_calibrate_static).
  Status calibrate_in(cudaStream_t stream, const void* frames, int n, float* peaks_out, uint8_t* scratch,
                      size_t scratch_bytes);
  size_t device_bytes() const;
  int* err_word() const { return err_ptr_; }
  int height() const { return H_; }
  int width() const { return W_; }
  int max_batch() const { return max_batch_; }
  bool fp8() const { return fp8_; }
  // Kernel launches per run(): the frame repack + one per conv layer.
  int launches_per_run() const { return 1 + static_cast<int>(steps_.size()); }
  // Block b runs in E4M3 (FP8 engine: every block but the first).
  bool block_fp8(int b) const { return fp8_ && b >= 1; }

  // Per-layer-kind device timing (kb2_set_profiling / kb2_read_profile).
  struct Profile {
    std::string name;
    uint64_t launches = 0;
    double ms = 0.0, flops = 0.0, bytes = 0.0;
  };
  void set_profiling(bool on) { profiling_ = on; }
  Status read_profile(std::vector<Profile>& out);

 private:
  struct Tensor {
    ChunkedTensor t;
    DeviceBuffer buf;
  };
  // One launch of the network: layer, destination(s), residual, scales, calibration tap.
  struct Step {
    ConvLayer* layer;
    const ChunkedTensor* out;   // null: the caller's output frame
    const ChunkedTensor* out2;  // E4M3 copy (dual-output layers)
    const ChunkedTensor* residual;
    float out_inv_scale, res_scale;
    int peak;  // calibration index of `out`, -1 none
    int kind;  // profile record
    double flops_px, bytes_px;  // algorithmic work per output pixel
  };
  int kind_index(const char* name);
  Status timed(int kind, double flops, double bytes, cudaStream_t stream, bool begin);
  Status make_tensor(std::unique_ptr<Tensor>& t, int chunks, bool fp8);

  bool fp8_ = false;
  int max_batch_ = 0, H_ = 0, W_ = 0;
  std::vector<float> scales_;
  DeviceBuffer err_, peaks_;
  int* err_ptr_ = nullptr;
  std::vector<std::unique_ptr<Tensor>> tensors_;
  std::vector<std::unique_ptr<ConvLayer>> layers_;
  std::vector<Step> steps_;
  const ChunkedTensor* img_ = nullptr;
  ConvLayer* up_display_ = nullptr;  // the upsampler with the display epilogue (same weights)
  int k_display_ = 0;
  int out_format_ = 0;
  bool profiling_ = false;
  std::vector<Profile> kinds_;
  struct Pending {
    int kind;
    cudaEvent_t start, stop;
    double flops, bytes;
  };
  std::vector<Pending> pending_;
  std::vector<cudaEvent_t> event_pool_;
  cudaEvent_t open_start_ = nullptr;

 public:
  ~SpanNet();
};

}  // namespace kb2
