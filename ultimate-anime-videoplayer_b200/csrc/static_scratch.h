// Fixed device scratch for the no-allocation entry point (static_scratch.cu).
#pragma once

#include "host_util.h"

namespace kb2 {

constexpr size_t kStaticScratchBytes = static_cast<size_t>(64) << 20;  // 64 MiB per device

// Device address of the static scratch on the current device. The first call on a device looks it
// up with cudaGetSymbolAddress, which loads the array's module on that device (the one-time setup);
// later calls only read a cached address.
Status static_scratch(void** ptr);

}  // namespace kb2
