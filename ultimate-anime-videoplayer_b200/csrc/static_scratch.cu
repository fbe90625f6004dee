// Fixed device scratch for callers that must not allocate (kb2_span_calibrate_static).
//
// kb2_span_calibrate needs device scratch for two things on every call: the 19 peak words that
// the peak reduction raises with atomicMax, and the x2 output frames of the calibration passes,
// which nobody reads. It allocates that scratch on every call and frees it on return. A caller
// that sizes its device memory once, up front, cannot allow that: a player that has handed the
// rest of the GPU to its decoder and frame ring, or a process running under a hard memory cap.
// For such callers this file provides one scratch array compiled into the library, so that the
// calibration itself allocates nothing.
//
// The array is kStaticScratchBytes (64 MiB) of __device__ memory. The driver reserves it on a
// device when it loads this file's module there. That happens on the first static_scratch() call
// made with that device current: cudaGetSymbolAddress loads the module. The memory stays reserved
// until the context ends. Nothing else in the library touches this module, so engines that never
// use the static path never pay for the array.
//
// One array per device, shared by every engine on it: overlapping calls on the same device race
// on it.
#include <mutex>

#include "static_scratch.h"

namespace kb2 {

namespace {
__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {};  // g_static_scratch's address on each device, once looked up
}  // namespace

Status static_scratch(void** ptr) {
  int dev = -1;
  KB2_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return refuse(KB2_FORMAT_UNSUPPORTED, "static scratch: device ordinal >= 64");
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_addr[dev] == nullptr) {
    void* p = nullptr;
    KB2_CUDA(cudaGetSymbolAddress(&p, g_static_scratch));  // with `dev` current: loads the module there
    if (p == nullptr) return refuse(KB2_VENDOR_CALL_FAILED, "static scratch: null symbol address");
    g_addr[dev] = p;
  }
  *ptr = g_addr[dev];
  return Status::Ok();
}

}  // namespace kb2
