// Implicit-GEMM convolution on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces the reference's mma.sync conv family (src/gpu/cuda/backend/span_native_conv.cuh:99
// `conv_kernel`, its kPlain / kGate / kPixel / Sources=4 modes) and the FP8 CUTLASS Sm89 blocks
// (span_fp8_kernels.cuh:304-330) with one B200-native kernel:
//
//  * Activations live in HBM as row-chunked NHWC: [n][y][chunk][x][16 bytes], a chunk being 8 FP16
//    or 16 E4M3 channels. TMA brings one input row of one source into a shared-memory slot as
//    [chunk][pixel][16 B] (1 KB boxes of 64 pixels): pixels sit at a 16-byte pitch, the row pitch of
//    the UMMA no-swizzle K-major core matrix, so the A operand of tap (dy, dx) is the row of dy
//    shifted by dx pixels -- a descriptor start-address offset, no im2col. Zero padding comes from
//    the TMA out-of-bounds fill.
//  * M = 128 output pixels of one row, N = output channels (16..64), K = taps x channels in steps
//    of 32 bytes (two 16-byte halves, LBO apart). A host-built K-step table says which input row and
//    which A tile each instruction uses; the packed weights (B, resident in shared memory) follow it.
//  * A operand from TMEM (3x3 layers). With N = 48 an MMA whose A (128 x 32 B) is read from shared
//    memory is bound by the 128 B/clk shared-memory read, not by the tensor pipe (measured on B200:
//    ~44 clk per M128 N48 K16 instruction instead of 24). So each input row is copied once into
//    TMEM (tcgen05.cp) as the few distinct (dx, channel-pair) tiles the K steps use, into a ring of
//    four row regions, and the three output rows that need that input row read it from TMEM; the
//    shared-memory slot is released as soon as the copy is done. 1x1 layers (no reuse across rows)
//    read A from shared memory.
//  * Warp roles: warp 0 = TMA producer, warp 1 = TMEM owner + single-thread MMA / copy issuer,
//    warps 2.. = epilogue, 4 per 16 accumulator columns. An epilogue warp reads the 32 TMEM lanes
//    of its quadrant (warp id mod 4) and 16 columns, and applies the fused epilogue (bias, SiLU,
//    SPAN gate, PReLU, pixel shuffle, E4M3 requantisation). The accumulator is double-buffered so
//    the epilogue of row y overlaps the MMAs of row y+1.
//  * Persistent CTAs walk work items (image, band of rows, 128-pixel strip).
#pragma once

#include "display_pixel.cuh"
#include "tc_common.cuh"

namespace kb2 {

constexpr int kMaxKSteps = 40;
constexpr int kMaxTiles = 16;
constexpr int kTileM = 128;
constexpr int kMaxN = 64;
constexpr uint32_t kTmemRegions = 4;       // TMEM ring of input rows (A operand)
constexpr uint32_t kTmemRegionBase = 128;  // columns [0, 128) hold the two accumulators

template <int kN>
struct ConvShape {
  static constexpr int epi_warps = 4 * (kN / 16);
  static constexpr int threads = 64 + 32 * epi_warps;
  static constexpr uint32_t col_stride = kN <= 32 ? 32 : 64;  // accumulator buffer stride
};

enum Epi : int {
  kEpiBias = 0,      // acc*scale + bias
  kEpiSilu = 1,      // SiLU(acc*scale + bias)
  kEpiSpanAttn = 2,  // (v + x) * (sigmoid(v) - 0.5), x = the block input (residual tensor)
  kEpiPrelu = 3,     // PReLU(v)
  kEpiResPrelu = 4,  // PReLU(v + residual)
  kEpiTanhGate = 5,  // (residual + residual2) * tanh(v): the unshuffle SPAN's block end (x + c3) * tanh(att)
  // 3x3 conv with its kernel columns in N (pair kernel only, conv3p.cuh): accumulator column
  // 16 kx + c of MMA row m holds kernel column kx of output channel c applied at slot pixel m; the
  // epilogue sums D[m - 1][c] + D[m][16 + c] + D[m + 1][32 + c] across neighbouring lanes, then adds
  // the bias and the border terms of ConvArgs::tap_bias
  kEpiColsBias = 6,
};

enum OutFmt : int {
  kOutF16Chunk = 0,   // [n][y][C/8][x][8] half
  kOutE4m3Chunk = 1,  // [n][y][C/16][x][16] e4m3, value * out_inv_scale
  kOutPixShuf2 = 2,   // NCHW half [n][3][2H][2W], DepthToSpace(2, CRD) of 12 channels
  kOutF16E4m3 = 3,    // both: half chunks to `out`, E4M3 chunks (value * out_inv_scale) to `out2`
  kOutPixShuf4 = 4,   // NCHW half [n][3][4H][4W], DepthToSpace(4, CRD) of 48 channels
  // DepthToSpace(2, CRD) of 12 channels as display pixels (display_pixel.cuh, format a.display_format),
  // rows of 2W pixels at a.out + (n * 2H + row) * a.out_pitch: each value rounded to FP16 first, so the
  // pixels are those the packing pass makes of the FP16 frame
  kOutPixShuf2Display = 5,
};

struct KStep {
  uint32_t a_off;  // byte offset of the first K half inside the input row slot
  uint32_t lbo;    // byte distance to the second K half
  int32_t row;     // input row of the window (0 .. in_rows-1)
  int32_t tile;    // TMEM tile of this (a_off, lbo) pair within a row region (TMEM-A mode)
};

struct ConvArgs {
  int batch, H, W;  // output rows / columns (input has the same size: stride 1)
  int strips, bands, band_rows, items;
  int pairs;  // paired stacked kernel (conv3p.cuh): strip pairs per row band
  int strip_w;  // output pixels per strip (128 minus the pixels the shifted A tiles read past the slot)
  int n_sources, chunks, px, halo, in_rows, row_off;
  uint32_t src_bytes, slot_bytes, ring, w_smem;
  int n_ksteps;
  KStep ks[kMaxKSteps];
  int tmem_a;                    // 1: A from TMEM (3x3 layers)
  int n_tiles;                   // distinct A tiles per input row (TMEM-A mode)
  uint32_t tile_off[kMaxTiles];  // slot byte offset of tile t
  uint32_t tile_lbo[kMaxTiles];  // its K-half distance
  uint32_t idesc;
  uint32_t idesc_n[3];  // stacked 3x3 kernel: instruction descriptors for 1, 2, 3 row blocks
  int acc_slots;        // stacked 3x3 kernel: TMEM ring of output-row accumulators
  const uint8_t* wpack;  // n_ksteps * 2 * N * 16 bytes
  uint32_t wbytes;
  const float* bias;        // N entries (zero padded)
  const float* chan_scale;  // N entries or null
  const float* slope;       // N entries (PReLU) or null
  // The epilogue's per-channel bias and scale (1 where the layer has none), in the parameter space:
  // every warp reads the same values, which the constant cache serves without the shared-memory
  // pipe the MMAs' operands use. SiLU and gate layers hold them halved (epi_halved).
  float cbias[kMaxN];
  float cscale[kMaxN];
  // kEpiColsBias: the part of cbias that tap (ky, kx) = (t / 3, t % 3) contributes, per output
  // channel. cbias holds the interior sum; an output pixel whose tap falls outside the image
  // subtracts that tap's term (the layer this conv replaces zero-pads its input, bias included).
  float tap_bias[9][16];
  float out_inv_scale;      // E4M3 output: 1 / scale
  float res_scale;          // E4M3 residual dequantisation scale
  const uint8_t* residual;  // same pixels and channels as the output, chunked
  const uint8_t* residual2;  // kEpiTanhGate: the second addend (FP16 chunks like `residual`)
  int res_fp8;              // residual chunk format: 0 = f16, 1 = e4m3
  int res_chunks;           // chunks per residual pixel
  uint8_t* out;
  int out_chunks;  // chunks per output pixel (chunked formats)
  uint8_t* out2;   // kOutF16E4m3: the E4M3 copy
  int out2_chunks;
  long long out_pitch;  // kOutPixShuf2Display: bytes per output row
  int display_format;   // kOutPixShuf2Display: kb2_display_format
  int* err;
};

// Tensor maps of the sources (one 128-pixel row box each, host_util.h encode_row_map).
struct ConvMaps {
  CUtensorMap m[4];
};

// Shared-memory bytes besides the weights and the ring: alignment slack, barriers, K-step and tile
// tables, per-channel constants, TMEM address.
constexpr uint32_t kConvSmemExtra = 1024 + 64 * 8 + (kMaxKSteps + 1) * 8 + kMaxTiles * 8 + 3 * kMaxN * 4 + 64;

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t{1023});
}

// Epilogue of kCols accumulator columns [col0, col0 + kCols) of one pixel, in groups of 8 columns.
// Per-channel constants are read at kc0 + j; the output channel of column j is col0 + j (col0
// defaults to kc0; a caller holding its constants in a register array passes kc0 = 0).
// The residual words of kCols channels [col0, col0 + kCols) of one pixel (same pixel and channels as
// the output, in the block input's format): 4 words per 8 channels for FP16, 2 for E4M3. Loaded
// ahead of the accumulator wait by the paired kernel, so the load latency hides behind the wait.
// kResFp8: the residual is E4M3 (the E4M3 layers' block inputs), else FP16.
template <int kCols, bool kResFp8>
__device__ __forceinline__ void load_residual_words(const ConvArgs& a, int n, int y, int x, int col0,
                                                    uint32_t (&w)[kCols / 2]) {
  const size_t pix_row = static_cast<size_t>(n) * a.H + y;
  if (kCols % 16 == 0 && kResFp8 && (col0 & 15) == 0) {
    // whole 16-channel E4M3 chunks: one 16-byte load each (groups 2 g2 and 2 g2 + 1)
#pragma unroll
    for (int g2 = 0; g2 < kCols / 16; ++g2) {
      const uint4 q = __ldg(reinterpret_cast<const uint4*>(
          a.residual + ((pix_row * a.res_chunks + (col0 + 16 * g2) / 16) * a.W + x) * 16));
      w[8 * g2] = q.x;
      w[8 * g2 + 1] = q.y;
      w[8 * g2 + 4] = q.z;
      w[8 * g2 + 5] = q.w;
    }
    return;
  }
#pragma unroll
  for (int g = 0; g < kCols / 8; ++g) {
    const int c = col0 + 8 * g;
    if (kResFp8) {
      const uint2 q = __ldg(reinterpret_cast<const uint2*>(
          a.residual + ((pix_row * a.res_chunks + c / 16) * a.W + x) * 16 + (c % 16)));
      w[4 * g] = q.x;
      w[4 * g + 1] = q.y;
    } else {
      const uint4 q =
          __ldg(reinterpret_cast<const uint4*>(a.residual + ((pix_row * a.res_chunks + c / 8) * a.W + x) * 16));
      w[4 * g] = q.x;
      w[4 * g + 1] = q.y;
      w[4 * g + 2] = q.z;
      w[4 * g + 3] = q.w;
    }
  }
}

// SiLU and the SPAN gate work on h = v / 2, the argument of their tanh: the host stores those
// layers' bias and channel scale halved (exact, ConvArgs::cbias / cscale), so the constant step
// yields h, and
//   SiLU(v) = v sigmoid(v) = h tanh(h) + h,
//   (v + x)(sigmoid(v) - 1/2) = (h + x / 2) tanh(h),
// two multiplies fewer per value than from v.
template <int kEpi>
__host__ __device__ constexpr bool epi_halved() { return kEpi == kEpiSilu || kEpi == kEpiSpanAttn; }

// How the per-channel constants are applied: kConstsAny, v * scale + bias from both arrays;
// kConstsBias, the bias array alone with the layer's constant scale (1, or 1/2 for the halved
// epilogues): FP16 layers, whose scale array holds only that constant.
enum ConstsMode : int { kConstsAny = 0, kConstsBias = 1 };

template <int kEpi, int kOut, int kCols, int kConsts = kConstsAny>
__device__ __forceinline__ void epilogue_cols(const ConvArgs& a, const float* bias, const float* scale,
                                              const float* s_slope, float* v, int kc0, int n, int y, int x,
                                              int col0_override = -1, const uint32_t* res_pre = nullptr) {
  const int col0 = col0_override >= 0 ? col0_override : kc0;
  const size_t pix_row = static_cast<size_t>(n) * a.H + y;
  if constexpr (kConsts == kConstsAny) {
#pragma unroll
    for (int j = 0; j < kCols; ++j) v[j] = fmaf(v[j], scale[kc0 + j], bias[kc0 + j]);
  } else {
    constexpr float kScale = epi_halved<kEpi>() ? 0.5f : 1.0f;
#pragma unroll
    for (int j = 0; j < kCols; ++j) v[j] = fmaf(v[j], kScale, bias[kc0 + j]);
  }
  // PReLU slopes of this pixel's channels, read from shared memory where they are used (held in
  // registers for the whole residual loop they made the 64-channel residual conv spill)
  auto slope_at = [&](int j) -> float { return s_slope[kc0 + j]; };
  if constexpr (kEpi == kEpiSilu) {
#pragma unroll
    for (int j = 0; j < kCols; ++j) v[j] = fmaf(v[j], tanh_approx(v[j]), v[j]);  // v holds h = v / 2
  } else if constexpr (kEpi == kEpiPrelu) {
#pragma unroll
    for (int j = 0; j < kCols; ++j) v[j] = v[j] >= 0.0f ? v[j] : v[j] * slope_at(j);
  } else if constexpr (kEpi == kEpiSpanAttn || kEpi == kEpiResPrelu) {
    // residual: same pixel and channels, in the block input's format
    // r holds the residual's stored values (E4M3 codes decoded, or FP16); its factor in the sum:
    // the dequantisation scale (E4M3), halved for the gate, which adds x / 2 to h
    const float rc = (a.res_fp8 ? a.res_scale : 1.0f) * (kEpi == kEpiSpanAttn ? 0.5f : 1.0f);
#pragma unroll
    for (int g = 0; g < kCols / 8; ++g) {
      const int c = col0 + 8 * g;
      float r[8];
      if (a.res_fp8) {
        const uint2 q = res_pre != nullptr ? make_uint2(res_pre[4 * g], res_pre[4 * g + 1])
                                           : __ldg(reinterpret_cast<const uint2*>(
                                                 a.residual + ((pix_row * a.res_chunks + c / 16) * a.W + x) * 16 +
                                                 (c % 16)));
        const uint32_t w2[2] = {q.x, q.y};
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const float2 lo = unpack_e4m3x2(static_cast<uint16_t>(w2[k] & 0xFFFFu));
          const float2 hi = unpack_e4m3x2(static_cast<uint16_t>(w2[k] >> 16));
          r[4 * k + 0] = lo.x;
          r[4 * k + 1] = lo.y;
          r[4 * k + 2] = hi.x;
          r[4 * k + 3] = hi.y;
        }
      } else {
        const uint4 q = res_pre != nullptr
                            ? make_uint4(res_pre[4 * g], res_pre[4 * g + 1], res_pre[4 * g + 2], res_pre[4 * g + 3])
                            : __ldg(reinterpret_cast<const uint4*>(
                                  a.residual + ((pix_row * a.res_chunks + c / 8) * a.W + x) * 16));
        const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = unpack_half2(w4[k]);
          r[2 * k] = f.x;
          r[2 * k + 1] = f.y;
        }
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float& t = v[8 * g + k];
        if constexpr (kEpi == kEpiSpanAttn) {
          t = fmaf(rc, r[k], t) * tanh_approx(t);  // t holds h = v / 2
        } else {
          const float u = fmaf(rc, r[k], t);
          t = u >= 0.0f ? u : u * slope_at(8 * g + k);
        }
      }
    }
  }

  if constexpr (kEpi == kEpiTanhGate) {
    // (x + c3) * tanh(att): both addends FP16 chunks of the same pixel and channels
#pragma unroll
    for (int g = 0; g < kCols / 8; ++g) {
      const size_t at = ((pix_row * a.res_chunks + (col0 + 8 * g) / 8) * a.W + x) * 16;
      const uint4 qa = __ldg(reinterpret_cast<const uint4*>(a.residual + at));
      const uint4 qb = __ldg(reinterpret_cast<const uint4*>(a.residual2 + at));
      const uint32_t wa[4] = {qa.x, qa.y, qa.z, qa.w};
      const uint32_t wb[4] = {qb.x, qb.y, qb.z, qb.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 fa = unpack_half2(wa[k]);
        const float2 fb = unpack_half2(wb[k]);
        v[8 * g + 2 * k] = (fa.x + fb.x) * tanh_approx(v[8 * g + 2 * k]);
        v[8 * g + 2 * k + 1] = (fa.y + fb.y) * tanh_approx(v[8 * g + 2 * k + 1]);
      }
    }
  }

  if constexpr (kOut == kOutF16Chunk || kOut == kOutF16E4m3) {
#pragma unroll
    for (int g = 0; g < kCols / 8; ++g) {
      const float* f = v + 8 * g;
      uint4 q;
      q.x = pack_half2(f[0], f[1]);
      q.y = pack_half2(f[2], f[3]);
      q.z = pack_half2(f[4], f[5]);
      q.w = pack_half2(f[6], f[7]);
      *reinterpret_cast<uint4*>(a.out + ((pix_row * a.out_chunks + (col0 + 8 * g) / 8) * a.W + x) * 16) = q;
    }
  }
  if constexpr (kOut == kOutE4m3Chunk || kOut == kOutF16E4m3) {
    uint8_t* dst = kOut == kOutE4m3Chunk ? a.out : a.out2;
    const int dst_chunks = kOut == kOutE4m3Chunk ? a.out_chunks : a.out2_chunks;
    const float is = a.out_inv_scale;
    auto e4m3x8 = [&](const float* f) {
      uint2 q;
      q.x = static_cast<uint32_t>(pack_e4m3x2(f[0] * is, f[1] * is)) |
            (static_cast<uint32_t>(pack_e4m3x2(f[2] * is, f[3] * is)) << 16);
      q.y = static_cast<uint32_t>(pack_e4m3x2(f[4] * is, f[5] * is)) |
            (static_cast<uint32_t>(pack_e4m3x2(f[6] * is, f[7] * is)) << 16);
      return q;
    };
    if (kCols % 16 == 0 && (col0 & 15) == 0) {
      // whole 16-channel chunks: one 16-byte store each
#pragma unroll
      for (int g = 0; g < kCols / 16; ++g) {
        const uint2 lo = e4m3x8(v + 16 * g), hi = e4m3x8(v + 16 * g + 8);
        *reinterpret_cast<uint4*>(dst + ((pix_row * dst_chunks + (col0 + 16 * g) / 16) * a.W + x) * 16) =
            make_uint4(lo.x, lo.y, hi.x, hi.y);
      }
    } else {
#pragma unroll
      for (int g = 0; g < kCols / 8; ++g) {
        const int c = col0 + 8 * g;
        *reinterpret_cast<uint2*>(dst + ((pix_row * dst_chunks + c / 16) * a.W + x) * 16 + (c % 16)) = e4m3x8(v + 8 * g);
      }
    }
  }
  if constexpr (kOut == kOutPixShuf4) {
    // channel 16p + 4i + j -> pixel (4y + i, 4x + j) of plane p: four adjacent halves per (p, i)
    const size_t W4 = static_cast<size_t>(a.W) * 4;
    const size_t H4 = static_cast<size_t>(a.H) * 4;
#pragma unroll
    for (int q = 0; q < kCols / 4; ++q) {
      const int c = col0 + 4 * q;
      const int plane = c / 16, i = (c % 16) / 4;
      if (plane < 3) {
        const size_t at = ((static_cast<size_t>(n) * 3 + plane) * H4 + 4 * static_cast<size_t>(y) + i) * W4 + 4 * x;
        *reinterpret_cast<uint2*>(a.out + at * 2) =
            make_uint2(pack_half2(v[4 * q], v[4 * q + 1]), pack_half2(v[4 * q + 2], v[4 * q + 3]));
      }
    }
  }
  if constexpr (kOut == kOutPixShuf2Display) {
    // channel 4p + 2i + j -> display pixel (2y + i, 2x + j), p = r, g, b: the thread holds all 12
    // channels of its input pixel (col0 = 0), so each output row gets its two pixels in one store
    static_assert(kCols >= 12, "the display epilogue needs the pixel's 12 channels");
    const int fmt = a.display_format;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint32_t oy = 2u * static_cast<uint32_t>(y) + static_cast<uint32_t>(i);
      uint8_t* row = a.out + (static_cast<size_t>(n) * 2 * a.H + oy) * static_cast<size_t>(a.out_pitch);
      float c[2][3];
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int p = 0; p < 3; ++p) c[j][p] = __half2float(__float2half_rn(v[4 * p + 2 * i + j]));
      const uint32_t ox = 2u * static_cast<uint32_t>(x);
      if (fmt == KB2_DISPLAY_RGBA16) {
        const uint2 p0 = rgba16(c[0][0], c[0][1], c[0][2]);
        const uint2 p1 = rgba16(c[1][0], c[1][1], c[1][2]);
        *reinterpret_cast<uint4*>(row + static_cast<size_t>(ox) * 8) = make_uint4(p0.x, p0.y, p1.x, p1.y);
      } else {
        const bool dither = fmt == KB2_DISPLAY_RGB10A2_DITHER;
        *reinterpret_cast<uint2*>(row + static_cast<size_t>(ox) * 4) =
            make_uint2(rgb10a2(c[0][0], c[0][1], c[0][2], dither, ox, oy),
                       rgb10a2(c[1][0], c[1][1], c[1][2], dither, ox + 1u, oy));
      }
    }
  }
  if constexpr (kOut == kOutPixShuf2) {
    // channel 4p + 2i + j -> pixel (2y + i, 2x + j) of plane p (p < 3)
    const size_t W2 = static_cast<size_t>(a.W) * 2;
    const size_t H2 = static_cast<size_t>(a.H) * 2;
#pragma unroll
    for (int q = 0; q < kCols / 4; ++q) {
      const int plane = (col0 + 4 * q) / 4;
      if (plane < 3) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const size_t at =
              ((static_cast<size_t>(n) * 3 + plane) * H2 + 2 * static_cast<size_t>(y) + i) * W2 + 2 * x;
          *reinterpret_cast<uint32_t*>(a.out + at * 2) = pack_half2(v[4 * q + 2 * i], v[4 * q + 2 * i + 1]);
        }
      }
    }
  }
}

template <bool kFp8, int kN, int kEpi, int kOut>
__global__ void __launch_bounds__(ConvShape<kN>::threads, 1)
    conv_tc_kernel(const __grid_constant__ ConvMaps maps, const __grid_constant__ ConvArgs a) {
  static_assert(kN % 16 == 0 && kN >= 16 && kN <= kMaxN, "N must be 16..64 in steps of 16");
  constexpr int kEpiWarps = ConvShape<kN>::epi_warps;
  constexpr uint32_t kColStride = ConvShape<kN>::col_stride;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sw = smem;
  uint8_t* ring = smem + a.w_smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + a.ring * a.slot_bytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + a.ring;
  uint64_t* acc_full = bars + 2 * a.ring;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* wbar = acc_empty + 2;
  uint64_t* drain = wbar + 1;
  // per K step: (a_off >> 4) | (lbo >> 4) << 16 | row << 56 | tile << 58 (bits 56-63 are not part
  // of the descriptor fields the delta is added to, and are masked off before use)
  uint64_t* s_kstep = bars + 64;
  uint64_t* s_tile = s_kstep + kMaxKSteps + 1;  // per A tile: (off >> 4) | (lbo >> 4) << 16
  // PReLU slopes (bias and scale are read from the parameter space, ConvArgs::cbias / cscale)
  float* s_slope = reinterpret_cast<float*>(s_tile + kMaxTiles) + 2 * kMaxN;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(s_slope + kMaxN);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t tmem_cols = a.tmem_a ? 512u : 2u * kColStride;

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < a.ring; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&acc_full[0], 1);
    mbar_init(&acc_full[1], 1);
    mbar_init(&acc_empty[0], kEpiWarps);
    mbar_init(&acc_empty[1], kEpiWarps);
    mbar_init(wbar, 1);
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  for (int j = threadIdx.x; j < kMaxN; j += blockDim.x) {
    s_slope[j] = (a.slope != nullptr && j < kN) ? a.slope[j] : 0.0f;
  }
  for (int j = threadIdx.x; j <= kMaxKSteps; j += blockDim.x) {
    uint64_t e = 0;
    if (j < a.n_ksteps) {
      const KStep& s = a.ks[j];
      e = static_cast<uint64_t>(s.a_off >> 4) | (static_cast<uint64_t>(s.lbo >> 4) << 16) |
          (static_cast<uint64_t>(s.row & 3) << 56) | (static_cast<uint64_t>(s.tile & 15) << 58);
    }
    s_kstep[j] = e;
  }
  for (int t = threadIdx.x; t < kMaxTiles; t += blockDim.x)
    s_tile[t] = t < a.n_tiles
                    ? (static_cast<uint64_t>(a.tile_off[t] >> 4) | (static_cast<uint64_t>(a.tile_lbo[t] >> 4) << 16))
                    : 0;
  if (warp == 0 && lane < a.n_sources) prefetch_tmap(&maps.m[lane]);
  if (warp == 1) {
    tmem_alloc(tmem_holder, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ producer
      bool ok = true;
      mbar_arrive_expect_tx(wbar, a.wbytes);
      for (uint32_t off = 0; off < a.wbytes; off += 32768u) {
        const uint32_t len = a.wbytes - off < 32768u ? a.wbytes - off : 32768u;
        bulk_load(sw + off, a.wpack + off, len, wbar);
      }
      uint32_t cnt = 0;
      for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x) {
        const int strip = item % a.strips;
        const int t = item / a.strips;
        const int band = t % a.bands;
        const int n = t / a.bands;
        const int y0 = band * a.band_rows;
        const int y1 = min(a.H, y0 + a.band_rows);
        const int x0 = strip * a.strip_w;
        const int r_end = (y1 - 1) + a.row_off + a.in_rows;
        for (int r = y0 + a.row_off; r < r_end; ++r, ++cnt) {
          const uint32_t slot = cnt % a.ring;
          const uint32_t use = cnt / a.ring;
          if (!wait_bar(&empty[slot], (use & 1u) ^ 1u, a.err, kErrWaitProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[slot], a.slot_bytes);
          uint8_t* dst = ring + slot * a.slot_bytes;
          // one box per source: 128 pixels from x0 - halo (a 16-byte-aligned word coordinate,
          // negative at the left edge: zero fill), all chunks
          for (int s = 0; s < a.n_sources; ++s)
            tma_load_4d(dst + s * a.src_bytes, &maps.m[s], &full[slot], (x0 - a.halo) * 2, 0, r, n);
        }
      }
      // every copy issued has landed before the block may exit
      for (uint32_t k = cnt > a.ring ? cnt - a.ring : 0; k < cnt; ++k)
        wait_bar(&full[k % a.ring], (k / a.ring) & 1u, a.err, kErrWaitDrain);
      wait_bar(wbar, 0, a.err, kErrWaitDrain);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA / copy issuer
      bool ok = wait_bar(wbar, 0, a.err, kErrWaitMma);
      const uint32_t ring_base = smem_u32(ring);
      // descriptor template: SBO = 128 B (8 rows x 16 B), version 1, no swizzle; the start address
      // and LBO fields are added per K step (the fields cannot carry into each other)
      const uint64_t desc_hi = make_sdesc(0, 0, 128);
      const uint64_t b_desc0 = make_sdesc(smem_u32(sw), kN * 16, 128);
      constexpr uint64_t kBStep16 = (2u * kN * 16u) >> 4;
      const int n_ksteps = a.n_ksteps;
      const int n_tiles = a.n_tiles;
      const uint32_t region_cols = static_cast<uint32_t>(n_tiles) * 8u;
      const uint32_t tmem_a_base = tmem_base + kTmemRegionBase;
      uint32_t in_cnt = 0;
      uint32_t acc_cnt = 0;
      for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x) {
        const int t = item / a.strips;
        const int band = t % a.bands;
        const int y0 = band * a.band_rows;
        const int y1 = min(a.H, y0 + a.band_rows);
        const uint32_t base = in_cnt;
        uint32_t ready = 0;  // rows of this item available (loaded, and copied to TMEM in TMEM-A mode)
        for (int y = y0; y < y1; ++y) {
          const uint32_t rel = static_cast<uint32_t>(y - y0);
          // Wait for the accumulator first: its release by the epilogue also proves that the MMAs
          // of two rows ago are complete, so the TMEM region the copies below overwrite (the input
          // row four rows back, last read by those MMAs) is no longer in use.
          const uint32_t buf = acc_cnt & 1u;
          const uint32_t use = acc_cnt >> 1;
          if (!wait_bar(&acc_empty[buf], (use & 1u) ^ 1u, a.err, kErrWaitMma)) {
            ok = false;
            break;
          }
          for (; ready < rel + static_cast<uint32_t>(a.in_rows); ++ready) {
            const uint32_t k = base + ready;
            const uint32_t slot = k % a.ring;
            if (!wait_bar(&full[slot], (k / a.ring) & 1u, a.err, kErrWaitMma)) {
              ok = false;
              break;
            }
            if (a.tmem_a) {
              tc_fence_after();
              const uint64_t row_desc = desc_hi | static_cast<uint64_t>((ring_base + slot * a.slot_bytes) >> 4);
              const uint32_t dst = tmem_a_base + (k % kTmemRegions) * region_cols;
              for (int tt = 0; tt < n_tiles; ++tt) tmem_cp_128x256b(dst + 8u * tt, row_desc + s_tile[tt]);
              mma_commit(&empty[slot]);  // the slot is free once copied
            }
          }
          if (!ok) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + buf * kColStride;
          uint64_t bdesc = b_desc0;
          uint64_t e = s_kstep[0];
          if (a.tmem_a) {
            const uint32_t r0 = tmem_a_base + ((base + rel) % kTmemRegions) * region_cols;
            const uint32_t r1 = tmem_a_base + ((base + rel + 1) % kTmemRegions) * region_cols;
            const uint32_t r2 = tmem_a_base + ((base + rel + 2) % kTmemRegions) * region_cols;
            for (int j = 0; j < n_ksteps; ++j) {
              const uint64_t next = s_kstep[j + 1];  // prefetched (the table is padded by one entry)
              const uint32_t row = static_cast<uint32_t>(e >> 56) & 3u;
              const uint32_t tile = static_cast<uint32_t>(e >> 58) & 15u;
              const uint32_t a_tmem = (row == 0 ? r0 : (row == 1 ? r1 : r2)) + 8u * tile;
              mma_ts<kFp8>(d_tmem, a_tmem, bdesc, a.idesc, j > 0 ? 1u : 0u);
              bdesc += kBStep16;
              e = next;
            }
          } else {
            auto row_desc = [&](uint32_t r) {
              const uint32_t slot = (base + rel + r) % a.ring;
              return desc_hi | static_cast<uint64_t>((ring_base + slot * a.slot_bytes) >> 4);
            };
            const uint64_t d0 = row_desc(0), d1 = row_desc(1), d2 = row_desc(2);
            for (int j = 0; j < n_ksteps; ++j) {
              const uint64_t next = s_kstep[j + 1];
              const uint32_t row = static_cast<uint32_t>(e >> 56) & 3u;
              const uint64_t adesc = (row == 0 ? d0 : (row == 1 ? d1 : d2)) + (e & 0x3FFF3FFFull);
              mma_ss<kFp8>(d_tmem, adesc, bdesc, a.idesc, j > 0 ? 1u : 0u);
              bdesc += kBStep16;
              e = next;
            }
          }
          mma_commit(&acc_full[buf]);
          if (!a.tmem_a) mma_commit(&empty[(base + rel) % a.ring]);  // the oldest row of this window is done
          ++acc_cnt;
        }
        if (!ok) break;
        const uint32_t rows_out = static_cast<uint32_t>(y1 - y0);
        const uint32_t total = rows_out - 1 + static_cast<uint32_t>(a.in_rows);
        if (!a.tmem_a)
          for (uint32_t r = rows_out; r < total; ++r) mma_commit(&empty[(base + r) % a.ring]);
        in_cnt = base + total;
      }
      mma_commit(drain);
      wait_bar(drain, 0, a.err, kErrWaitDrain);
    }
    __syncwarp();
  } else {
    // -------------------------------------------------------------------- epilogue
    const int quad = warp & 3;
    const int col0 = ((warp - 2) >> 2) * 16;
    uint32_t acc_cnt = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x) {
      const int strip = item % a.strips;
      const int t = item / a.strips;
      const int band = t % a.bands;
      const int n = t / a.bands;
      const int y0 = band * a.band_rows;
      const int y1 = min(a.H, y0 + a.band_rows);
      const int m = quad * 32 + lane;
      const int x = strip * a.strip_w + m;
      const bool store = m < a.strip_w && x < a.W;
      for (int y = y0; y < y1; ++y) {
        const uint32_t buf = acc_cnt & 1u;
        const uint32_t use = acc_cnt >> 1;
        const bool got = wait_bar(&acc_full[buf], use & 1u, a.err, kErrWaitEpilogue);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float v[16];
        tmem_ld16(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + buf * kColStride + static_cast<uint32_t>(col0),
                  v);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
        if (store) epilogue_cols<kEpi, kOut, 16>(a, a.cbias, a.cscale, s_slope, v, col0, n, y, x);
        ++acc_cnt;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

}  // namespace kb2
