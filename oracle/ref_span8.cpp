// TEST INFRASTRUCTURE ONLY (oracle): a C entry point over the reference's own .span8 reader and FP32
// CPU forward of the AnimeJaNai "unshuffle" SPAN (Ta2b/Ultimate-Anime-VideoPlayer
// src/gpu/span_fp8/package.cpp:143 parse, src/gpu/span_fp8/forward.cpp:144 forward), compiled in
// place by oracle/Makefile. The tests use it to pin the numpy restatement (oracle/nets.py
// span8_forward) and the library's own package reader; nothing in the product path loads it.
#include <cstddef>
#include <cstring>
#include <span>
#include <string>
#include <vector>

#include "gpu/span_fp8/forward.h"
#include "gpu/span_fp8/package.h"

namespace {
std::string g_error;
}

extern "C" {

const char* kref_span8_last_error() { return g_error.c_str(); }

// Parses a package; returns 0 and the block count / real channels / flags, or the reference's
// refusal code + 1 (its message in kref_span8_last_error).
int kref_span8_parse(const unsigned char* bytes, long n, int* blocks, int* real_channels, int* fp16) {
  namespace s8 = kirari::gpu::span_fp8;
  auto pkg = s8::parse(std::span<const std::byte>(reinterpret_cast<const std::byte*>(bytes), static_cast<size_t>(n)));
  if (!pkg) {
    g_error = pkg.error().detail;
    return static_cast<int>(pkg.error().code) + 1;
  }
  *blocks = static_cast<int>(pkg->blocks.size());
  *real_channels = pkg->real_channels;
  *fp16 = pkg->fp16 ? 1 : 0;
  return 0;
}

// The reference's FP32 forward of one frame: rgb 3 planes of h x w, out 3 planes of 2h x 2w.
int kref_span8_forward(const unsigned char* bytes, long n, const float* rgb, int h, int w, float* out) {
  namespace s8 = kirari::gpu::span_fp8;
  auto pkg = s8::parse(std::span<const std::byte>(reinterpret_cast<const std::byte*>(bytes), static_cast<size_t>(n)));
  if (!pkg) {
    g_error = pkg.error().detail;
    return static_cast<int>(pkg.error().code) + 1;
  }
  const std::vector<float> y = s8::forward(*pkg, std::span<const float>(rgb, static_cast<size_t>(3) * h * w), h, w);
  if (y.size() != static_cast<size_t>(12) * h * w) {
    g_error = "forward refused the frame size";
    return -1;
  }
  std::memcpy(out, y.data(), y.size() * sizeof(float));
  return 0;
}

}  // extern "C"
