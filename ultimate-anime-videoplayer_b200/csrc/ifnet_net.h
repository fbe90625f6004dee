// Classic IFNet (RIFE 4.x, four blocks at 1/8 .. 1/1) on the tensor-core IFNet convs and the glue
// kernels (see ifnet_net.cu).
#pragma once

#include <memory>
#include <vector>

#include "layer_timer.h"

namespace kb2 {

constexpr size_t kIfnetParams = KB2_IFNET_PARAMS;  // the blob order of include/kirari_b200.h
// Padded frame: multiples of 32, what the network needs (its coarsest level is 1/32 of the frame).
// The reference pads to 64 for its RIFE 4.x models (src/kernels/spec/rife.h:33); for 1920x1080 both
// give 1920x1088.
constexpr int kIfnetAlign = 32;

struct IfLayer;

class IfnetNet {
 public:
  IfnetNet();
  ~IfnetNet();
  Status create(const std::vector<float>& params, int max_batch, int H, int W);
  // img0 / img1: NCHW F16 [batch][3][H][W]; out: NCHW F16 [batch][3][H][W] (device pointers).
  Status run(cudaStream_t stream, const void* img0, const void* img1, void* out, int batch);
  // The motion variant: the same network with the final flow [batch][4][Hp][Wp] and sigmoid(mask)
  // [batch][1][Hp][Wp] over the padded plane (FP32, or FP16 when `f16`) in place of the frame.
  Status run_motion(cudaStream_t stream, const void* img0, const void* img1, void* flow, void* mask, bool f16,
                    int batch);
  // The padded plane and the frame's window in it (the reference's rife_geometry).
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
  struct Tensor {
    uint8_t* ptr = nullptr;
    int H = 0, W = 0, chunks = 0;
    DeviceBuffer buf;
  };
  Status tensor(std::unique_ptr<Tensor>& t, int H, int W, int chunks);
  // What the last kernel writes: the blended frame (image), or the motion (flow and mask).
  struct Finish {
    void* image;
    void* flow;
    void* mask;
    bool f16;
  };
  Status run_impl(cudaStream_t stream, const void* img0, const void* img1, const Finish& finish, int batch);

  int max_batch_ = 0, H_ = 0, W_ = 0, Hp_ = 0, Wp_ = 0, top_ = 0, left_ = 0;
  float timestep_ = 0.5f;
  DeviceBuffer err_;
  std::vector<std::unique_ptr<Tensor>> tensors_;
  std::vector<std::unique_ptr<IfLayer>> layers_;  // per block: conv0a, conv0b, 8 residual, convT
  const Tensor* x_[4] = {};                       // block inputs
  DeviceBuffer flows_[4];                         // transposed-conv outputs, FP32 [n][Hp/2s][Wp/2s][8]
  DeviceBuffer flow_full_;                        // flow / mask after blocks 0-2, FP32 [n][5][Hp][Wp]
  DeviceBuffer pad_;                              // both frames, padded RGBx FP16 pixels [2][n][Hp][Wp]
  LayerTimer timer_;
  int k_glue_[4] = {}, k_blend_ = 0, k_pad_ = 0, k_motion_ = 0;
};

// Bilinear backward-warp taps of a flow field [n][2][h][w] (FP32, device): x0, x1, y0, y1 as int32
// planes [n][4][h][w] and wx, wy as FP32 planes [n][2][h][w] (kb2_warp_taps).
Status warp_taps(cudaStream_t stream, const float* flow, int n, int h, int w, int32_t* taps, float* weights);

}  // namespace kb2
