// Implicit-GEMM convolution on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces the reference's mma.sync conv family (src/gpu/cuda/backend/span_native_conv.cuh:99
// `conv_kernel`, its kPlain / kGate / kPixel / Sources=4 modes) and the FP8 CUTLASS Sm89 blocks
// (span_fp8_kernels.cuh:304-330) with one B200-native kernel:
//
//  * Activations live in HBM as row-chunked NHWC: [n][y][chunk][x][16 bytes], a chunk being 8 FP16
//    or 16 E4M3 channels. One TMA box brings one input row of one source into shared memory as
//    [chunk][pixel][16 B]: pixels sit at a 16-byte pitch, which is exactly the row pitch of the UMMA
//    no-swizzle K-major core matrix, so the A operand of tap (dy, dx) is the row slot of dy shifted
//    by dx pixels -- a descriptor start-address offset, no im2col copy. Zero padding comes from the
//    TMA out-of-bounds fill.
//  * M = 128 output pixels of one row, N = output channels (<= 64 here), K = taps x channels in
//    steps of 32 bytes (two 16-byte halves, LBO apart). A host-built K-step table says, per
//    instruction, which input row slot, byte offset and LBO the A operand uses; the packed weights
//    (B, resident in shared memory) follow the same table.
//  * Warp roles: warp 0 = TMA producer, warp 1 = TMEM owner + single-thread MMA issuer, warps 2-5 =
//    epilogue (TMEM -> registers -> fused bias / SiLU / SPAN attention / PReLU / pixel shuffle /
//    E4M3 requantisation -> global). The accumulator is double-buffered in TMEM so the epilogue of
//    row y overlaps the MMAs of row y+1; input rows stream through a ring of slots, each output row
//    loading one new input row.
//  * Persistent CTAs walk work items (image, band of rows, 128-pixel strip).
#pragma once

#include "tc_common.cuh"

namespace kb2 {

constexpr int kMaxKSteps = 40;
constexpr int kTileM = 128;

enum Epi : int {
  kEpiBias = 0,      // acc*scale + bias
  kEpiSilu = 1,      // SiLU(acc*scale + bias)
  kEpiSpanAttn = 2,  // (v + x) * (sigmoid(v) - 0.5), x = the block input (residual tensor)
  kEpiPrelu = 3,     // PReLU(v)
  kEpiResPrelu = 4,  // PReLU(v + residual)
};

enum OutFmt : int {
  kOutF16Chunk = 0,   // [n][y][C/8][x][8] half
  kOutE4m3Chunk = 1,  // [n][y][C/16][x][16] e4m3, value * out_inv_scale
  kOutPixShuf2 = 2,   // NCHW half [n][n_real/4][2H][2W], DepthToSpace(2, CRD)
  kOutF16E4m3 = 3,    // both: half chunks to `out`, E4M3 chunks (value * out_inv_scale) to `out2`
};

struct KStep {
  uint32_t a_off;  // byte offset of the first K half inside the input row slot
  uint32_t lbo;    // byte distance to the second K half
  int32_t row;     // input row of the window (0 .. in_rows-1)
  int32_t pad_;
};

struct ConvArgs {
  int batch, H, W;        // output rows / columns (input has the same size: stride 1)
  int strips, bands, band_rows, items;
  int n_sources, chunks, px, halo, in_rows, row_off;
  uint32_t src_bytes, slot_bytes, ring, w_smem;
  int n_ksteps;
  KStep ks[kMaxKSteps];
  uint32_t idesc;
  const uint8_t* wpack;  // n_ksteps * 2 * N * 16 bytes
  uint32_t wbytes;
  const float* bias;        // N entries (zero padded)
  const float* chan_scale;  // N entries or null
  const float* slope;       // N entries (PReLU) or null
  float out_inv_scale;      // E4M3 output: 1 / scale
  float res_scale;          // E4M3 residual dequantisation scale
  const uint8_t* residual;  // same geometry as the output, chunked
  int res_fp8;              // residual chunk format: 0 = f16, 1 = e4m3
  uint8_t* out;
  int out_chunks;  // chunks per output pixel (chunked formats)
  uint8_t* out2;   // kOutF16E4m3: the E4M3 copy
  int out2_chunks;
  int* err;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t{1023});
}

template <int kN>
struct TmemCols {
  static constexpr uint32_t stride = kN <= 32 ? 32 : (kN <= 64 ? 64 : (kN <= 128 ? 128 : 256));
  static constexpr uint32_t total = 2 * stride;
};

template <int kEpi, int kOut, int kN>
__device__ __forceinline__ void epilogue_store(const ConvArgs& a, float* v, int n, int y, int x) {
  // scale, bias, activation
#pragma unroll
  for (int j = 0; j < kN; ++j) {
    float s = a.chan_scale != nullptr ? __ldg(a.chan_scale + j) : 1.0f;
    v[j] = fmaf(v[j], s, __ldg(a.bias + j));
  }
  const size_t pix_row = static_cast<size_t>(n) * a.H + y;
  if constexpr (kEpi == kEpiSilu) {
#pragma unroll
    for (int j = 0; j < kN; ++j) v[j] = v[j] * sigmoidf_fast(v[j]);
  } else if constexpr (kEpi == kEpiPrelu) {
#pragma unroll
    for (int j = 0; j < kN; ++j) v[j] = v[j] >= 0.0f ? v[j] : v[j] * __ldg(a.slope + j);
  } else if constexpr (kEpi == kEpiSpanAttn || kEpi == kEpiResPrelu) {
    float r[kN];
    if (a.res_fp8) {
#pragma unroll
      for (int c = 0; c < kN / 16; ++c) {
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(
            a.residual + ((pix_row * (kN / 16) + c) * a.W + x) * 16));
        const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 lo = unpack_e4m3x2(static_cast<uint16_t>(w4[k] & 0xFFFFu));
          const float2 hi = unpack_e4m3x2(static_cast<uint16_t>(w4[k] >> 16));
          r[c * 16 + 4 * k + 0] = lo.x * a.res_scale;
          r[c * 16 + 4 * k + 1] = lo.y * a.res_scale;
          r[c * 16 + 4 * k + 2] = hi.x * a.res_scale;
          r[c * 16 + 4 * k + 3] = hi.y * a.res_scale;
        }
      }
    } else {
#pragma unroll
      for (int c = 0; c < kN / 8; ++c) {
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(
            a.residual + ((pix_row * (kN / 8) + c) * a.W + x) * 16));
        const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = unpack_half2(w4[k]);
          r[c * 8 + 2 * k] = f.x;
          r[c * 8 + 2 * k + 1] = f.y;
        }
      }
    }
    if constexpr (kEpi == kEpiSpanAttn) {
#pragma unroll
      for (int j = 0; j < kN; ++j) v[j] = (v[j] + r[j]) * (sigmoidf_fast(v[j]) - 0.5f);
    } else {
#pragma unroll
      for (int j = 0; j < kN; ++j) {
        const float t = v[j] + r[j];
        v[j] = t >= 0.0f ? t : t * __ldg(a.slope + j);
      }
    }
  }

  if constexpr (kOut == kOutF16Chunk || kOut == kOutF16E4m3) {
#pragma unroll
    for (int c = 0; c < kN / 8; ++c) {
      uint4 q;
      q.x = pack_half2(v[c * 8 + 0], v[c * 8 + 1]);
      q.y = pack_half2(v[c * 8 + 2], v[c * 8 + 3]);
      q.z = pack_half2(v[c * 8 + 4], v[c * 8 + 5]);
      q.w = pack_half2(v[c * 8 + 6], v[c * 8 + 7]);
      *reinterpret_cast<uint4*>(a.out + ((pix_row * a.out_chunks + c) * a.W + x) * 16) = q;
    }
  }
  if constexpr (kOut == kOutE4m3Chunk || kOut == kOutF16E4m3) {
    uint8_t* dst = kOut == kOutE4m3Chunk ? a.out : a.out2;
    const int dst_chunks = kOut == kOutE4m3Chunk ? a.out_chunks : a.out2_chunks;
    const float is = a.out_inv_scale;
#pragma unroll
    for (int c = 0; c < kN / 16; ++c) {
      uint32_t w4[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float* f = v + c * 16 + 4 * k;
        w4[k] = static_cast<uint32_t>(pack_e4m3x2(f[0] * is, f[1] * is)) |
                (static_cast<uint32_t>(pack_e4m3x2(f[2] * is, f[3] * is)) << 16);
      }
      *reinterpret_cast<uint4*>(dst + ((pix_row * dst_chunks + c) * a.W + x) * 16) =
          make_uint4(w4[0], w4[1], w4[2], w4[3]);
    }
  }
  if constexpr (kOut == kOutPixShuf2) {  // channel 4c + 2i + j -> pixel (2y + i, 2x + j) of plane c
    const int planes = kN / 4 < 3 ? kN / 4 : 3;
    const size_t W2 = static_cast<size_t>(a.W) * 2;
    const size_t H2 = static_cast<size_t>(a.H) * 2;
#pragma unroll
    for (int c = 0; c < planes; ++c) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const size_t at = ((static_cast<size_t>(n) * 3 + c) * H2 + 2 * static_cast<size_t>(y) + i) * W2 + 2 * x;
        *reinterpret_cast<uint32_t*>(a.out + at * 2) = pack_half2(v[4 * c + 2 * i], v[4 * c + 2 * i + 1]);
      }
    }
  }
}

template <bool kFp8, int kN, int kEpi, int kOut>
__global__ void __launch_bounds__(192, 2)
    conv_tc_kernel(const __grid_constant__ CUtensorMap map0, const __grid_constant__ CUtensorMap map1,
                   const __grid_constant__ CUtensorMap map2, const __grid_constant__ CUtensorMap map3,
                   const __grid_constant__ ConvArgs a) {
  static_assert(kN % 16 == 0 && kN >= 16 && kN <= 64, "N must be 16..64 in steps of 16");
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
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr uint32_t kColStride = TmemCols<kN>::stride;
  constexpr uint32_t kTmemCols = TmemCols<kN>::total;

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < a.ring; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&acc_full[0], 1);
    mbar_init(&acc_full[1], 1);
    mbar_init(&acc_empty[0], 4);
    mbar_init(&acc_empty[1], 4);
    mbar_init(wbar, 1);
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&map0);
    if (a.n_sources > 1) {
      prefetch_tmap(&map1);
      prefetch_tmap(&map2);
      prefetch_tmap(&map3);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemCols);
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
        const int x0 = strip * kTileM;
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
          tma_load_5d(dst, &map0, &full[slot], 0, x0 - a.halo, 0, r, n);
          if (a.n_sources > 1) {
            tma_load_5d(dst + a.src_bytes, &map1, &full[slot], 0, x0 - a.halo, 0, r, n);
            tma_load_5d(dst + 2 * a.src_bytes, &map2, &full[slot], 0, x0 - a.halo, 0, r, n);
            tma_load_5d(dst + 3 * a.src_bytes, &map3, &full[slot], 0, x0 - a.halo, 0, r, n);
          }
        }
      }
      // every copy issued has landed before the block may exit
      for (uint32_t k = cnt > a.ring ? cnt - a.ring : 0; k < cnt; ++k)
        wait_bar(&full[k % a.ring], (k / a.ring) & 1u, a.err, kErrWaitDrain);
      wait_bar(wbar, 0, a.err, kErrWaitDrain);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA issuer
      bool ok = wait_bar(wbar, 0, a.err, kErrWaitMma);
      const uint32_t ring_base = smem_u32(ring);
      const uint32_t w_base = smem_u32(sw);
      constexpr uint32_t kBStep = 2u * kN * 16u;
      uint32_t in_cnt = 0;
      uint32_t acc_cnt = 0;
      for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x) {
        const int t = item / a.strips;
        const int band = t % a.bands;
        const int y0 = band * a.band_rows;
        const int y1 = min(a.H, y0 + a.band_rows);
        const uint32_t base = in_cnt;
        uint32_t waited = 0;
        for (int y = y0; y < y1; ++y) {
          const uint32_t rel = static_cast<uint32_t>(y - y0);
          for (; waited < rel + static_cast<uint32_t>(a.in_rows); ++waited) {
            const uint32_t k = base + waited;
            if (!wait_bar(&full[k % a.ring], (k / a.ring) & 1u, a.err, kErrWaitMma)) {
              ok = false;
              break;
            }
          }
          if (!ok) break;
          const uint32_t buf = acc_cnt & 1u;
          const uint32_t use = acc_cnt >> 1;
          if (!wait_bar(&acc_empty[buf], (use & 1u) ^ 1u, a.err, kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + buf * kColStride;
          for (int j = 0; j < a.n_ksteps; ++j) {
            const KStep& s = a.ks[j];
            const uint32_t slot = (base + rel + static_cast<uint32_t>(s.row)) % a.ring;
            const uint32_t a_addr = ring_base + slot * a.slot_bytes + s.a_off;
            const uint64_t adesc = make_sdesc(a_addr, s.lbo, 128);
            const uint64_t bdesc = make_sdesc(w_base + static_cast<uint32_t>(j) * kBStep, kN * 16, 128);
            mma_ss<kFp8>(d_tmem, adesc, bdesc, a.idesc, j > 0 ? 1u : 0u);
          }
          mma_commit(&acc_full[buf]);
          mma_commit(&empty[(base + rel) % a.ring]);  // the oldest row of this window is done
          ++acc_cnt;
        }
        if (!ok) break;
        const uint32_t rows_out = static_cast<uint32_t>(y1 - y0);
        const uint32_t total = rows_out - 1 + static_cast<uint32_t>(a.in_rows);
        for (uint32_t r = rows_out; r < total; ++r) mma_commit(&empty[(base + r) % a.ring]);
        in_cnt = base + total;
      }
      mma_commit(drain);
      wait_bar(drain, 0, a.err, kErrWaitDrain);
    }
    __syncwarp();
  } else {
    // -------------------------------------------------------------------- epilogue (warps 2..5)
    const int quad = warp & 3;
    uint32_t acc_cnt = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x) {
      const int strip = item % a.strips;
      const int t = item / a.strips;
      const int band = t % a.bands;
      const int n = t / a.bands;
      const int y0 = band * a.band_rows;
      const int y1 = min(a.H, y0 + a.band_rows);
      const int x = strip * kTileM + quad * 32 + lane;
      for (int y = y0; y < y1; ++y) {
        const uint32_t buf = acc_cnt & 1u;
        const uint32_t use = acc_cnt >> 1;
        const bool got = wait_bar(&acc_full[buf], use & 1u, a.err, kErrWaitEpilogue);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float v[kN];
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + buf * kColStride;
#pragma unroll
        for (int c = 0; c < kN; c += 16) tmem_ld16(taddr + c, v + c);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
        if (x < a.W) epilogue_store<kEpi, kOut, kN>(a, v, n, y, x);
        ++acc_cnt;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace kb2
