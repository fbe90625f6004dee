// Fixed device scratch for the no-allocation entry point (static_scratch.cu).
#pragma once

#include "host_util.h"

namespace kb2 {

constexpr size_t kStaticScratchBytes = static_cast<size_t>(64) << 20;  // 64 MiB per device

// Device address of the static scratch in the current device's current context, looked up with
// cudaGetSymbolAddress on every call. The first call in a context loads the array's module there
// (the one-time setup, under lazy module loading); later calls are a cheap lookup.
Status static_scratch(void** ptr);

}  // namespace kb2
