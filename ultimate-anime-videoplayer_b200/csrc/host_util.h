// Host-side helpers: status/refusal plumbing, TMA tensor-map encoding, E4M3 rounding, CRC-32 and
// the weight blob.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "kirari_b200.h"

namespace kb2 {

// A refusal: status code + message, the C restatement of the reference's Refusal
// (src/core/types.h:102-116).
struct Status {
  int code = KB2_OK;
  std::string detail;
  bool ok() const { return code == KB2_OK; }
  static Status Ok() { return {}; }
};

inline Status refuse(int code, std::string detail) { return Status{code, std::move(detail)}; }

inline Status cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return Status::Ok();
  const int code = e == cudaErrorMemoryAllocation ? KB2_GPU_MEMORY_EXHAUSTED : KB2_VENDOR_CALL_FAILED;
  return refuse(code, std::string(what) + ": " + cudaGetErrorString(e));
}

#define KB2_TRY(expr)                  \
  do {                                 \
    ::kb2::Status st_ = (expr);        \
    if (!st_.ok()) return st_;         \
  } while (0)
#define KB2_CUDA(call) KB2_TRY(::kb2::cuda_status((call), #call))

// ---------------------------------------------------------------- TMA tensor maps
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// Row-chunked activation tensor [batch][H][chunks][W][16 bytes].
struct ChunkedTensor {
  uint8_t* ptr = nullptr;
  int batch = 0, H = 0, W = 0, chunks = 0;
  bool fp8 = false;
  size_t bytes() const { return static_cast<size_t>(batch) * H * chunks * W * 16; }
};

// One row of one image: kRowBoxPx consecutive pixels x all channel chunks, as ONE TMA box. The
// tensor is viewed as 64-bit words ([n][y][chunk][2 * x]) so that 128 pixels (2 KB per chunk) fit
// the 256-element box limit; the box lands in shared memory as [chunk][128 px][16 B], the row slot
// layout of the conv kernels. One request per row matters: issuing a TMA instruction costs the
// producer ~170 cycles, so many small boxes per row starve the MMAs. Tile mode copies bytes, so the
// word type does not change the FP16 / E4M3 payload.
constexpr int kRowBoxPx = 128;

inline Status encode_row_map(CUtensorMap* map, const ChunkedTensor& t) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr) return refuse(KB2_VENDOR_CALL_FAILED, "cuTensorMapEncodeTiled unavailable");
  if (t.chunks < 1 || t.chunks > 256) return refuse(KB2_FORMAT_UNSUPPORTED, "row box: 1..256 chunks");
  const cuuint64_t row = static_cast<cuuint64_t>(t.W) * 16;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(t.W) * 2, static_cast<cuuint64_t>(t.chunks),
                              static_cast<cuuint64_t>(t.H), static_cast<cuuint64_t>(t.batch)};
  const cuuint64_t strides[3] = {row, row * static_cast<cuuint64_t>(t.chunks),
                                 row * static_cast<cuuint64_t>(t.chunks) * static_cast<cuuint64_t>(t.H)};
  const cuuint32_t box[4] = {static_cast<cuuint32_t>(kRowBoxPx) * 2, static_cast<cuuint32_t>(t.chunks), 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 4, t.ptr, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return refuse(KB2_VENDOR_CALL_FAILED, "cuTensorMapEncodeTiled failed: " + std::to_string(r));
  return Status::Ok();
}

// ---------------------------------------------------------------- E4M3 (host)
// Round to the nearest E4M3 value, ties to the even code, saturating to +-448 (the rounding of
// span_fp8::e4m3_round, src/gpu/span_fp8/quantize.h:14-18). Built from the format: 1 sign bit,
// 4 exponent bits (bias 7), 3 mantissa bits, no infinities, code 0x7F = NaN.
inline float e4m3_decode(uint8_t code) {
  const int e = (code >> 3) & 0xF;
  const int m = code & 7;
  const float mag = e == 0 ? std::ldexp(static_cast<float>(m) / 8.0f, -6)
                           : std::ldexp(1.0f + static_cast<float>(m) / 8.0f, e - 7);
  return (code & 0x80) ? -mag : mag;
}

inline uint8_t e4m3_encode(float x) {
  if (std::isnan(x)) return 0x7F;
  const uint8_t sign = std::signbit(x) ? 0x80 : 0x00;
  float a = std::fabs(x);
  if (a >= 448.0f) return sign | 0x7E;
  // positive codes 0..0x7E are increasing in value: binary search the neighbours
  int lo = 0, hi = 0x7E;
  while (hi - lo > 1) {
    const int mid = (lo + hi) / 2;
    if (e4m3_decode(static_cast<uint8_t>(mid)) <= a) lo = mid; else hi = mid;
  }
  const float vlo = e4m3_decode(static_cast<uint8_t>(lo));
  const float vhi = e4m3_decode(static_cast<uint8_t>(hi));
  int pick;
  if (a - vlo < vhi - a) pick = lo;
  else if (a - vlo > vhi - a) pick = hi;
  else pick = (lo % 2 == 0) ? lo : hi;
  if (a < vlo) pick = lo;
  return sign | static_cast<uint8_t>(pick);
}

inline float e4m3_round(float x) { return e4m3_decode(e4m3_encode(x)); }

// ---------------------------------------------------------------- CRC-32 (IEEE 802.3, reflected)
inline uint32_t crc32(const uint8_t* data, size_t n) {
  static uint32_t table[256];
  static bool init = false;
  if (!init) {
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int k = 0; k < 8; ++k) c = (c & 1u) ? 0xEDB88320u ^ (c >> 1) : c >> 1;
      table[i] = c;
    }
    init = true;
  }
  uint32_t c = 0xFFFFFFFFu;
  for (size_t i = 0; i < n; ++i) c = table[(c ^ data[i]) & 0xFFu] ^ (c >> 8);
  return c ^ 0xFFFFFFFFu;
}

// ---------------------------------------------------------------- weight blob v1
// 32-byte little-endian header: "KB2WGT01", u32 version (1), u32 model (kb2_model), u64 float count,
// u32 CRC-32 of the payload, u32 reserved (0); then `count` float32 parameters in the model's order.
constexpr uint32_t kBlobVersion = 1;
constexpr size_t kBlobHeader = 32;

inline Status parse_blob(const void* blob, uint64_t bytes, int model, std::vector<float>& out) {
  if (blob == nullptr || bytes < kBlobHeader) return refuse(KB2_WEIGHTS_INVALID, "weight blob missing or short");
  const uint8_t* p = static_cast<const uint8_t*>(blob);
  if (std::memcmp(p, "KB2WGT01", 8) != 0) return refuse(KB2_WEIGHTS_INVALID, "weight blob: bad magic");
  uint32_t version, blob_model, crc, reserved;
  uint64_t count;
  std::memcpy(&version, p + 8, 4);
  std::memcpy(&blob_model, p + 12, 4);
  std::memcpy(&count, p + 16, 8);
  std::memcpy(&crc, p + 24, 4);
  std::memcpy(&reserved, p + 28, 4);
  if (version != kBlobVersion) return refuse(KB2_WEIGHTS_INVALID, "weight blob: unknown version");
  if (static_cast<int>(blob_model) != model) return refuse(KB2_WEIGHTS_INVALID, "weight blob: other model");
  if (reserved != 0) return refuse(KB2_WEIGHTS_INVALID, "weight blob: reserved field set");
  if (count > (bytes - kBlobHeader) / 4 || kBlobHeader + count * 4 != bytes)
    return refuse(KB2_WEIGHTS_INVALID, "weight blob: payload size mismatch");
  if (crc32(p + kBlobHeader, count * 4) != crc) return refuse(KB2_WEIGHTS_INVALID, "weight blob: CRC mismatch");
  out.resize(count);
  std::memcpy(out.data(), p + kBlobHeader, count * 4);
  for (float v : out)
    if (!std::isfinite(v)) return refuse(KB2_WEIGHTS_INVALID, "weight blob: non-finite parameter");
  return Status::Ok();
}

// Device buffer owned by an engine.
struct DeviceBuffer {
  void* ptr = nullptr;
  size_t bytes = 0;
  DeviceBuffer() = default;
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  ~DeviceBuffer() {
    if (ptr != nullptr) cudaFree(ptr);
  }
  Status alloc(size_t n) {
    bytes = n;
    return cuda_status(cudaMalloc(&ptr, n == 0 ? 16 : n), "cudaMalloc");
  }
  template <class T>
  T* as() const { return static_cast<T*>(ptr); }
};

}  // namespace kb2
