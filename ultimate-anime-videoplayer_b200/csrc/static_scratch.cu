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
// device when it loads this file's module there. With lazy module loading (CUDA's default,
// CUDA_MODULE_LOADING=LAZY) that happens on the first static_scratch() call made with that device
// current, so engines that never use the static path never pay for the array. With
// CUDA_MODULE_LOADING=EAGER every context that loads the library reserves the 64 MiB on each device
// it uses, whether or not the static path ever runs. The memory stays reserved until the context
// ends.
//
// One array per device, shared by every engine on it: overlapping calls on the same device race
// on it.
#include "static_scratch.h"

namespace kb2 {

namespace {
__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];
}  // namespace

Status static_scratch(void** ptr) {
  // Looked up on every call, not cached: the address belongs to the module as loaded in the
  // current context, and a context that is destroyed and made again (cudaDeviceReset, or another
  // driver-API context made current) may load the module at another address. Once the module is
  // loaded the lookup is cheap.
  void* p = nullptr;
  KB2_CUDA(cudaGetSymbolAddress(&p, g_static_scratch));
  if (p == nullptr) return refuse(KB2_VENDOR_CALL_FAILED, "static scratch: null symbol address");
  *ptr = p;
  return Status::Ok();
}

}  // namespace kb2
