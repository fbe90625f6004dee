// The C ABI of include/kirari_b200.h over the C++ engines. Every entry point catches everything:
// nothing throws across the boundary (the reference's rule for its module entry points,
// src/gpu/backend.h:575-587).
#include <cstring>
#include <memory>
#include <new>
#include <string>
#include <vector>

#include "kirari_b200.h"
#include "engine.h"
#include "ifnet_net.h"
#include "onnx_import.h"

namespace {
thread_local std::string g_create_error;

int set_error(kb2_engine* e, const kb2::Status& s);
}  // namespace

struct kb2_engine {
  std::unique_ptr<kb2::Engine> impl;
  std::string error;
};

namespace {
int set_error(kb2_engine* e, const kb2::Status& s) {
  if (e != nullptr) e->error = s.ok() ? std::string() : s.detail;
  return s.code;
}

kb2::Status tensor_ptr(const kb2_tensor& t, int type, const int64_t (&dims)[4], void** out) {
  if (t.type != type) return kb2::refuse(KB2_INPUT_MISMATCH, "tensor type mismatch");
  for (int i = 0; i < 4; ++i)
    if (t.dims[i] != dims[i]) return kb2::refuse(KB2_INPUT_MISMATCH, "tensor shape mismatch");
  const uint64_t addr = t.handle + t.offset;
  if (addr == 0 || (addr & 15u) != 0) return kb2::refuse(KB2_INPUT_MISMATCH, "tensor address null or not 16-byte aligned");
  *out = reinterpret_cast<void*>(addr);
  return kb2::Status::Ok();
}
}  // namespace

namespace kb2 {
Status Engine::frame_io(const kb2_tensor* inputs, int n_in, const kb2_tensor* outputs, int n_out, int n_frames_in,
                        int out_scale, void** in_ptrs, void** out_ptr, int* batch, int display_bytes) const {
  if (inputs == nullptr || outputs == nullptr || n_in != n_frames_in || n_out != 1)
    return refuse(KB2_INPUT_MISMATCH, "wrong number of input / output tensors");
  const int64_t n = inputs[0].dims[0];
  if (n < 1 || n > max_batch()) return refuse(KB2_SHAPE_INVALID, "batch out of contract");
  const int64_t din[4] = {n, 3, height(), width()};
  for (int i = 0; i < n_in; ++i) KB2_TRY(tensor_ptr(inputs[i], KB2_F16, din, &in_ptrs[i]));
  if (display_bytes > 0) {
    const int64_t dpix[4] = {n, display_bytes, height() * out_scale, width() * out_scale};
    KB2_TRY(tensor_ptr(outputs[0], KB2_U8, dpix, out_ptr));
  } else {
    const int64_t dout[4] = {n, 3, height() * out_scale, width() * out_scale};
    KB2_TRY(tensor_ptr(outputs[0], KB2_F16, dout, out_ptr));
  }
  *batch = static_cast<int>(n);
  return Status::Ok();
}

Status Engine::motion_io(const kb2_tensor* inputs, int n_in, const kb2_tensor* outputs, int n_out, int ph, int pw,
                         void** in_ptrs, void** flow, void** mask, bool* f16, int* batch) const {
  if (inputs == nullptr || outputs == nullptr || n_in != 2 || n_out != 2)
    return refuse(KB2_INPUT_MISMATCH, "motion: two frames in, flow and mask out");
  const int64_t n = inputs[0].dims[0];
  if (n < 1 || n > max_batch()) return refuse(KB2_SHAPE_INVALID, "batch out of contract");
  const int64_t din[4] = {n, 3, height(), width()};
  for (int i = 0; i < n_in; ++i) KB2_TRY(tensor_ptr(inputs[i], KB2_F16, din, &in_ptrs[i]));
  const int type = outputs[0].type;
  if (type != KB2_F32 && type != KB2_F16) return refuse(KB2_INPUT_MISMATCH, "motion outputs: F32 or F16");
  const int64_t dflow[4] = {n, 4, ph, pw};
  const int64_t dmask[4] = {n, 1, ph, pw};
  KB2_TRY(tensor_ptr(outputs[0], type, dflow, flow));
  KB2_TRY(tensor_ptr(outputs[1], type, dmask, mask));
  *f16 = type == KB2_F16;
  *batch = static_cast<int>(n);
  return Status::Ok();
}
}  // namespace kb2

extern "C" {

int kb2_abi_version(void) { return KB2_ABI_VERSION; }

const char* kb2_create_error(void) { return g_create_error.c_str(); }

int kb2_rife_blob_from_onnx(const void* const* pieces, const uint64_t* piece_bytes, int32_t blocks,
                            const int32_t* reduce, void* blob, uint64_t* blob_bytes) {
  try {
    g_create_error.clear();
    if (pieces == nullptr || piece_bytes == nullptr || reduce == nullptr || blob_bytes == nullptr || blocks < 0 ||
        blocks > 5) {
      g_create_error = "null or out-of-range argument";
      return KB2_INVALID_ARGUMENT;
    }
    std::vector<const uint8_t*> p(static_cast<size_t>(blocks) + 1);
    for (size_t i = 0; i < p.size(); ++i) p[i] = static_cast<const uint8_t*>(pieces[i]);
    std::vector<uint8_t> out;
    const kb2::Status st = kb2::rife_blob_from_onnx(p.data(), piece_bytes, blocks, reduce, out);
    if (!st.ok()) {
      g_create_error = st.detail;
      return st.code;
    }
    const uint64_t capacity = *blob_bytes;
    *blob_bytes = out.size();
    if (blob == nullptr) return KB2_OK;
    if (capacity < out.size()) {
      g_create_error = "blob buffer too small";
      return KB2_INVALID_ARGUMENT;
    }
    std::memcpy(blob, out.data(), out.size());
    return KB2_OK;
  } catch (const std::exception& ex) {
    g_create_error = ex.what();
    return KB2_VENDOR_CALL_FAILED;
  } catch (...) {
    g_create_error = "unknown failure";
    return KB2_VENDOR_CALL_FAILED;
  }
}

int kb2_create(const kb2_engine_desc* desc, kb2_engine** out) {
  try {
    g_create_error.clear();
    if (out == nullptr || desc == nullptr) {
      g_create_error = "null argument";
      return KB2_INVALID_ARGUMENT;
    }
    *out = nullptr;
    std::unique_ptr<kb2::Engine> impl;
    const kb2::Status st = kb2::make_engine(*desc, impl);
    if (!st.ok()) {
      g_create_error = st.detail;
      return st.code;
    }
    auto* e = new (std::nothrow) kb2_engine;
    if (e == nullptr) {
      g_create_error = "host allocation failed";
      return KB2_GPU_MEMORY_EXHAUSTED;
    }
    e->impl = std::move(impl);
    *out = e;
    return KB2_OK;
  } catch (const std::exception& ex) {
    g_create_error = ex.what();
    return KB2_VENDOR_CALL_FAILED;
  } catch (...) {
    g_create_error = "unknown failure";
    return KB2_VENDOR_CALL_FAILED;
  }
}

int kb2_destroy(kb2_engine* engine) {
  if (engine == nullptr) return KB2_INVALID_ARGUMENT;
  try {
    cudaDeviceSynchronize();
    delete engine;
    return KB2_OK;
  } catch (...) {
    return KB2_VENDOR_CALL_FAILED;
  }
}

const char* kb2_last_error(const kb2_engine* engine) { return engine == nullptr ? "" : engine->error.c_str(); }

int kb2_workspace_bytes(const kb2_engine* engine, uint64_t* bytes) {
  if (engine == nullptr || bytes == nullptr) return KB2_INVALID_ARGUMENT;
  *bytes = engine->impl->device_bytes();
  return KB2_OK;
}

int kb2_enqueue(kb2_engine* engine, void* stream, const kb2_tensor* inputs, int32_t n_inputs,
                const kb2_tensor* outputs, int32_t n_outputs) {
  if (engine == nullptr) return KB2_INVALID_ARGUMENT;
  try {
    return set_error(engine, engine->impl->enqueue(static_cast<cudaStream_t>(stream), inputs, n_inputs, outputs,
                                                   n_outputs));
  } catch (const std::exception& ex) {
    return set_error(engine, kb2::refuse(KB2_VENDOR_CALL_FAILED, ex.what()));
  }
}

int kb2_set_output_format(kb2_engine* engine, int32_t format) {
  if (engine == nullptr) return KB2_INVALID_ARGUMENT;
  try {
    return set_error(engine, engine->impl->set_output_format(format));
  } catch (const std::exception& ex) {
    return set_error(engine, kb2::refuse(KB2_VENDOR_CALL_FAILED, ex.what()));
  }
}

int kb2_span_tile_grid(const kb2_engine* engine, kb2_tile_grid* grid) {
  if (engine == nullptr || grid == nullptr) return KB2_INVALID_ARGUMENT;
  try {
    *grid = kb2_tile_grid{};
    return engine->impl->tile_grid(grid).code;
  } catch (...) {
    return KB2_VENDOR_CALL_FAILED;
  }
}

int kb2_next_span_tiles(kb2_engine* engine, const uint8_t* core, int32_t count, int32_t shift_x, int32_t shift_y,
                        const kb2_tensor* previous) {
  if (engine == nullptr) return KB2_INVALID_ARGUMENT;
  try {
    return set_error(engine, engine->impl->next_tiles(core, count, shift_x, shift_y, previous));
  } catch (const std::exception& ex) {
    return set_error(engine, kb2::refuse(KB2_VENDOR_CALL_FAILED, ex.what()));
  }
}

int kb2_set_row_tiles(kb2_engine* engine, int32_t tiles, int32_t halo) {
  if (engine == nullptr) return KB2_INVALID_ARGUMENT;
  try {
    return set_error(engine, engine->impl->set_row_tiles(tiles, halo));
  } catch (const std::exception& ex) {
    return set_error(engine, kb2::refuse(KB2_VENDOR_CALL_FAILED, ex.what()));
  }
}

int kb2_set_timestep(kb2_engine* engine, float timestep) {
  if (engine == nullptr) return KB2_INVALID_ARGUMENT;
  return set_error(engine, engine->impl->set_timestep(timestep));
}

int kb2_check_device(kb2_engine* engine, void* stream, int32_t* code) {
  if (engine == nullptr) return KB2_INVALID_ARGUMENT;
  try {
    return set_error(engine, engine->impl->check_device(static_cast<cudaStream_t>(stream), code));
  } catch (const std::exception& ex) {
    return set_error(engine, kb2::refuse(KB2_VENDOR_CALL_FAILED, ex.what()));
  }
}

int kb2_span_calibrate(kb2_engine* engine, void* stream, const kb2_tensor* frames, float* peaks, int32_t n_peaks) {
  if (engine == nullptr || frames == nullptr || peaks == nullptr) return KB2_INVALID_ARGUMENT;
  try {
    return set_error(engine, engine->impl->calibrate(static_cast<cudaStream_t>(stream), *frames, peaks, n_peaks));
  } catch (const std::exception& ex) {
    return set_error(engine, kb2::refuse(KB2_VENDOR_CALL_FAILED, ex.what()));
  }
}

int kb2_span_calibrate_static(kb2_engine* engine, void* stream, const kb2_tensor* frames, float* peaks,
                              int32_t n_peaks) {
  if (engine == nullptr || frames == nullptr || peaks == nullptr) return KB2_INVALID_ARGUMENT;
  try {
    return set_error(engine,
                     engine->impl->calibrate_static(static_cast<cudaStream_t>(stream), *frames, peaks, n_peaks));
  } catch (const std::exception& ex) {
    return set_error(engine, kb2::refuse(KB2_VENDOR_CALL_FAILED, ex.what()));
  }
}

int kb2_warp_taps(void* stream, const float* flow, int32_t n, int32_t h, int32_t w, int32_t* taps, float* weights) {
  try {
    return kb2::warp_taps(static_cast<cudaStream_t>(stream), flow, n, h, w, taps, weights).code;
  } catch (...) {
    return KB2_VENDOR_CALL_FAILED;
  }
}

int kb2_warp_blend_at(void* stream, const kb2_tensor* a, const kb2_tensor* b, const kb2_motion* motion, float t,
                      const kb2_tensor* out) {
  try {
    return kb2::warp_blend_at(static_cast<cudaStream_t>(stream), a, b, motion, t, out).code;
  } catch (...) {
    return KB2_VENDOR_CALL_FAILED;
  }
}

int kb2_warp_blend_poses(void* stream, const kb2_tensor* a, const kb2_tensor* b, const kb2_motion* motion,
                         const kb2_motion* previous, float t, const kb2_tensor* out) {
  try {
    return kb2::warp_blend_at(static_cast<cudaStream_t>(stream), a, b, motion, t, out, true, previous).code;
  } catch (...) {
    return KB2_VENDOR_CALL_FAILED;
  }
}

int kb2_pack_display(void* stream, const kb2_tensor* frames, int32_t format, void* out, int64_t pitch) {
  try {
    return kb2::pack_display(static_cast<cudaStream_t>(stream), frames, format, out, pitch).code;
  } catch (...) {
    return KB2_VENDOR_CALL_FAILED;
  }
}

int kb2_flow_max(void* stream, const kb2_motion* motion, int32_t n, uint32_t* bins, float* out) {
  try {
    return kb2::flow_max(static_cast<cudaStream_t>(stream), motion, n, bins, out).code;
  } catch (...) {
    return KB2_VENDOR_CALL_FAILED;
  }
}

int kb2_selftest_bounded_wait(int32_t device, int32_t* code, double* waited_seconds) {
  try {
    return kb2::selftest_bounded_wait(device, code, waited_seconds).code;
  } catch (...) {
    return KB2_VENDOR_CALL_FAILED;
  }
}

int kb2_set_profiling(kb2_engine* engine, int32_t enable) {
  if (engine == nullptr) return KB2_INVALID_ARGUMENT;
  return set_error(engine, engine->impl->set_profiling(enable != 0));
}

int kb2_read_profile(kb2_engine* engine, kb2_layer_profile* records, int32_t capacity, int32_t* count) {
  if (engine == nullptr || count == nullptr || (records == nullptr && capacity > 0) || capacity < 0)
    return KB2_INVALID_ARGUMENT;
  try {
    int n = 0;
    const int rc = set_error(engine, engine->impl->read_profile(records, capacity, &n));
    *count = n;
    return rc;
  } catch (const std::exception& ex) {
    return set_error(engine, kb2::refuse(KB2_VENDOR_CALL_FAILED, ex.what()));
  }
}

int kb2_rife_geometry(const kb2_engine* engine, int32_t* plane_h, int32_t* plane_w, int32_t* window_x,
                      int32_t* window_y) {
  if (engine == nullptr || plane_h == nullptr || plane_w == nullptr || window_x == nullptr || window_y == nullptr)
    return KB2_INVALID_ARGUMENT;
  try {
    return engine->impl->geometry(plane_h, plane_w, window_x, window_y).code;
  } catch (...) {
    return KB2_VENDOR_CALL_FAILED;
  }
}

int kb2_launches_per_enqueue(const kb2_engine* engine, int32_t* launches) {
  if (engine == nullptr || launches == nullptr) return KB2_INVALID_ARGUMENT;
  *launches = engine->impl->launches_per_enqueue();
  return KB2_OK;
}

}  // extern "C"
