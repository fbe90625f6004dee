// RIFE 4.2x (4.25, 4.26, 4.25 lite, 4.22 lite) on the tensor-core interpolator convs and the RIFE
// glue kernels (rife_net.cu): the reference's fused RIFE (RifeFusedEngine, src/gpu/cuda/backend/
// rife_fused_engine.h:41; its plan src/kernels/spec/rife_fused.h:7-19) with its native block
// kernels (--rife-native, src/prepare/rife_native.h) in place of the TensorRT engines.
#pragma once

#include <memory>
#include <vector>

#include "layer_timer.h"

namespace kb2 {

struct IfLayer;

// The plan: blocks (2..5), the input reduction d_k of each block (powers of two, the first >= 2,
// the last 1) and its width C_k (32, 64, 96, 128 or 192).
struct RifePlan {
  int blocks = 0;
  int reduce[5] = {};
  int channels[5] = {};
};

// Parameters after the 12 plan floats, for a plan (include/kirari_b200.h, KB2_MODEL_RIFE_FUSED).
size_t rife_param_count(const RifePlan& plan);
// Reads and checks the plan floats of a parameter array.
Status rife_read_plan(const std::vector<float>& params, RifePlan& plan);

class RifeNet {
 public:
  RifeNet();
  ~RifeNet();
  Status create(const std::vector<float>& params, int max_batch, int H, int W);
  // img0 / img1: NCHW F16 [batch][3][H][W]; out: NCHW F16 [batch][3][H][W] (device pointers).
  Status run(cudaStream_t stream, const void* img0, const void* img1, void* out, int batch);
  // The motion variant: flow [batch][4][Hp][Wp] and sigmoid(mask) [batch][1][Hp][Wp] over the
  // padded plane (FP32, or FP16 when `f16`) in place of the frame.
  Status run_motion(cudaStream_t stream, const void* img0, const void* img1, void* flow, void* mask, bool f16,
                    int batch);
  int plane_height() const { return Hp_; }
  int plane_width() const { return Wp_; }
  int window_x() const { return left_; }
  int window_y() const { return top_; }
  Status set_timestep(float t);
  size_t device_bytes() const;
  int* err_word() const { return err_.as<int>(); }
  int height() const { return H_; }
  int width() const { return W_; }
  int max_batch() const { return max_batch_; }
  int launches_per_run() const;
  LayerTimer& timer() { return timer_; }

 private:
  struct Finish {
    void* image;
    void* flow;
    void* mask;
    bool f16;
  };
  Status run_impl(cudaStream_t stream, const void* img0, const void* img1, const Finish& finish, int batch);
  Status buffer(DeviceBuffer& b, size_t bytes);

  RifePlan plan_;
  int max_batch_ = 0, H_ = 0, W_ = 0, Hp_ = 0, Wp_ = 0, top_ = 0, left_ = 0;
  float timestep_ = 0.5f;
  DeviceBuffer err_;
  std::vector<std::unique_ptr<DeviceBuffer>> buffers_;
  std::vector<std::unique_ptr<IfLayer>> enc_layers_;       // cnn0 .. cnn3 over 2 x batch images
  std::vector<std::unique_ptr<IfLayer>> layers_[5];        // per block: conv0a, conv0b, 8 ResConv, convT
  uint8_t* x_[5] = {};                                     // block inputs X_k
  uint8_t* z_[5] = {};                                     // block outputs Z_k
  uint8_t* enc_in_ = nullptr;                              // encoder input, [2 n][Hp][1][Wp][16 B]
  uint8_t* enc_ = nullptr;                                 // encodings, [2 n][Hp][Wp] 4 x FP16
  DeviceBuffer pad_;                                       // both frames, padded RGBx [2][n][Hp][Wp]
  LayerTimer timer_;
  int k_pad_ = 0, k_glue_[5] = {}, k_c0a_ = 0, k_c0b_ = 0, k_res_ = 0, k_ct_ = 0, k_finish_ = 0, k_motion_ = 0;
};

}  // namespace kb2
