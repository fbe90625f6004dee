// C++ engines behind the C ABI: the shape of the reference's gpu::Engine (src/gpu/backend.h:381-413)
// with the per-model enqueue of TensorRtBackend (tensorrt_backend.cpp:527-548) folded in.
#pragma once

#include <memory>
#include <string>
#include <vector>

#include "host_util.h"

namespace kb2 {

class Engine {
 public:
  virtual ~Engine() = default;
  virtual std::vector<std::string> input_names() const = 0;   // Engine::input_names (backend.h:385)
  virtual std::vector<std::string> output_names() const = 0;  // Engine::output_names (backend.h:386)
  virtual int max_batch() const = 0;
  virtual int height() const = 0;
  virtual int width() const = 0;
  virtual size_t device_bytes() const = 0;
  virtual Status enqueue(cudaStream_t stream, const kb2_tensor* inputs, int n_inputs, const kb2_tensor* outputs,
                         int n_outputs) = 0;
  virtual Status set_timestep(float) { return refuse(KB2_FORMAT_UNSUPPORTED, "this engine has no timestep"); }
  virtual Status calibrate(cudaStream_t, const kb2_tensor&, float*, int) {
    return refuse(KB2_FORMAT_UNSUPPORTED, "this engine does not calibrate");
  }
  // calibrate() with its scratch in the library's static device array (kb2_span_calibrate_static)
  virtual Status calibrate_static(cudaStream_t, const kb2_tensor&, float*, int) {
    return refuse(KB2_FORMAT_UNSUPPORTED, "this engine does not calibrate");
  }
  Status check_device(cudaStream_t stream, int32_t* code);
  // kb2_span_tile_grid / kb2_next_span_tiles: moving tiles (SPAN x2 only)
  virtual Status tile_grid(kb2_tile_grid*) const {
    return refuse(KB2_FORMAT_UNSUPPORTED, "this engine computes whole frames only");
  }
  virtual Status next_tiles(const uint8_t*, int, int, int, const kb2_tensor*) {
    return refuse(KB2_FORMAT_UNSUPPORTED, "this engine computes whole frames only");
  }
  // kb2_set_row_tiles (SPAN x2 only)
  virtual Status set_row_tiles(int, int) { return refuse(KB2_FORMAT_UNSUPPORTED, "this engine runs whole frames"); }
  // kb2_set_output_format: 0 = F16 frames, else a kb2_display_format (SPAN x2 only)
  virtual Status set_output_format(int) { return refuse(KB2_FORMAT_UNSUPPORTED, "this engine writes F16 frames only"); }
  virtual Status set_profiling(bool) { return refuse(KB2_FORMAT_UNSUPPORTED, "no profiling"); }
  virtual Status read_profile(kb2_layer_profile*, int, int* count) {
    *count = 0;
    return refuse(KB2_FORMAT_UNSUPPORTED, "no profiling");
  }
  virtual int launches_per_enqueue() const = 0;
  // IFNet: the padded plane of the motion outputs and the frame's window in it (kb2_rife_geometry)
  virtual Status geometry(int32_t*, int32_t*, int32_t*, int32_t*) const {
    return refuse(KB2_FORMAT_UNSUPPORTED, "this engine has no motion plane");
  }

 protected:
  // Validates the frame tensors of an enqueue: n_frames_in inputs F16 [n,3,H,W], one output
  // F16 [n,3,H*out_scale,W*out_scale] (display_bytes > 0: display pixels, U8
  // [n,display_bytes,H*out_scale,W*out_scale]), n <= max_batch, 16-byte aligned.
  Status frame_io(const kb2_tensor* inputs, int n_in, const kb2_tensor* outputs, int n_out, int n_frames_in,
                  int out_scale, void** in_ptrs, void** out_ptr, int* batch, int display_bytes = 0) const;
  // Validates the IFNet motion variant's tensors: two F16 frames [n,3,H,W] in; out flow [n,4,ph,pw]
  // and mask [n,1,ph,pw], both F32 or both F16 (*f16).
  Status motion_io(const kb2_tensor* inputs, int n_in, const kb2_tensor* outputs, int n_out, int ph, int pw,
                   void** in_ptrs, void** flow, void** mask, bool* f16, int* batch) const;
  virtual int* err_word() const = 0;
};

Status make_engine(const kb2_engine_desc& desc, std::unique_ptr<Engine>& out);

// kb2_selftest_bounded_wait (selftest.cu): KB2_KERNEL_TIMEOUT with the wait's error code and the time
// the device waited, when the bounded wait gave up as designed.
Status selftest_bounded_wait(int device, int32_t* code, double* waited_s);

// kb2_warp_blend_at / kb2_flow_max (warp_blend.cu).
Status warp_blend_at(cudaStream_t stream, const kb2_tensor* a, const kb2_tensor* b, const kb2_motion* motion, float t,
                     const kb2_tensor* out, bool keep_poses = false, const kb2_motion* previous = nullptr);
Status flow_max(cudaStream_t stream, const kb2_motion* motion, int n, unsigned int* bins, float* out);

// kb2_pack_display (display_pack.cu).
Status pack_display(cudaStream_t stream, const kb2_tensor* frames, int format, void* out, long long pitch);

}  // namespace kb2
