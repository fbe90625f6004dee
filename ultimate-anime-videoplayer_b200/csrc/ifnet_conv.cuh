// IFNet convolutions on sm_100a tensor cores: one streaming implicit-GEMM kernel for every conv of
// the classic IFNet block: the two stride-2 entry convs, the residual convs and the 4x4 stride-2
// transposed conv. It replaces the reference's native RIFE conv kinds (3x3 s2 conv0, ResConv with
// the residual and PReLU at the store, 4x4 s2 deconv as four phases; src/gpu/cuda/backend/
// rife_native_plan.h:20-29, rife_native_kernels.cuh:35-55).
//
//  * Activations are row-chunked NHWC FP16, [n][y][chunk][x][16 B] (8 channels per chunk), as in
//    the SPAN kernels. A work item is one output row strip of 126 pixels. M = 128 pixels, N = the
//    output channels (32..192, one MMA), K = 3 x 3 taps x input channels.
//  * The K loop runs over (kernel row dy, group of g input chunks). Each step stages, through one
//    ring slot, the input row's g chunks for 128 pixels (TMA) and the matching weights for the
//    three dx taps (bulk copy). Weights are read from L2 for every item: the wide layers (N = 192,
//    K = 1728) do not fit in shared memory next to the input rows.
//  * The three dx taps are shifts of the staged row: a descriptor start-address offset of 16 B per
//    pixel. Stride 2 stages the row as two boxes, even and odd pixels (a 5-D tensor-map view that
//    splits x into pixel pairs), so that every tap again reads 128 consecutive 16-byte rows. Rows
//    above or below the image contribute nothing: their K steps are skipped by both the producer
//    and the MMA issuer. Zero padding at the left and right comes from the TMA out-of-bounds fill.
//  * Warp 0: producer. Warp 1: TMEM owner + MMA issuer. Warps 2..9: epilogue, two per TMEM lane
//    quadrant, each half of the columns. The accumulator is double-buffered in TMEM. Fused
//    epilogues: bias + PReLU; bias + residual + PReLU; transposed-conv phases scattered as FP32
//    pixels of 8 floats (+ bias; 5 used); for RIFE 4.2x, the encoder's transposed conv as FP16
//    pixels of 4 channels, and the blocks' transposed conv with the DepthToSpace(2) after it folded
//    into the store (Z pixels of 16 FP16 channels, 13 used).
#pragma once

#include "tc_common.cuh"

namespace kb2 {

enum IfEpi : int {
  kIfPrelu = 0,     // PReLU(acc + bias)
  kIfResPrelu = 1,  // PReLU(acc + bias + residual), residual = the conv input (same shape)
  kIfConvT = 2,     // 4 phases x 8 columns (5 used): out[co][2y+py][2x+px] = acc + bias, FP32 planes
  // RIFE 4.2x encoder cnn3: 4 phases x 8 columns (4 used): acc + bias as one 8-byte FP16 pixel of 4
  // channels at (2y + py, 2x + px) of an image [n][2 h_out][2 w_out] (`out`)
  kIfConvTEnc = 3,
  // RIFE 4.2x block transposed conv to Y (52 channels) and DepthToSpace(2, CRD) to Z (13 channels):
  // column n = 64 phase + 16 (2 qy + qx) + c holds Y channel 4 c + 2 qy + qx of ConvT output phase
  // (py, px) = (phase / 2, phase % 2), i.e. Z channel c of Z pixel (4y + 2py + qy, 4x + 2px + qx);
  // acc + bias stored as Z pixels of 16 FP16 (32 bytes, c < 13 used) [n][4 h_out][4 w_out] (`out`)
  kIfConvTZ = 4,
};

constexpr int kIfEpiWarps = 8;
constexpr int kIfThreads = 64 + 32 * kIfEpiWarps;
constexpr int kIfMaxStages = 4;
constexpr int kIfStrip = 126;  // output pixels per item: the shifted A tiles stay in a 128-pixel box
constexpr int kIfMaxN = 256;
constexpr uint32_t kIfChunkBytes = 128 * 16;  // one chunk of a 128-pixel box

struct IfConvArgs {
  int batch, h_in, w_in, h_out, w_out;
  int g;         // input chunks per K group (even, <= 8)
  int n_groups;  // input chunks / g
  int strips, items;
  uint32_t a_bytes;      // A bytes per ring slot: g chunks x 2 KB (x 2 boxes at stride 2)
  uint32_t b_bytes;      // weight bytes per K group: 3 dx x g/2 K steps x 2 halves x N x 16 B
  uint32_t stage_bytes;  // a_bytes + b_bytes, rounded up to 1 KB
  uint32_t stages;
  const uint8_t* wpack;  // [3 dy][n_groups][b_bytes]
  const float* bias;     // N (zero padded)
  const float* slope;    // N (PReLU)
  const uint8_t* residual;  // kIfResPrelu: chunked FP16 like out
  uint8_t* out;             // chunked FP16 [n][h_out][out_chunks][w_out][16 B]
  int out_chunks;
  int out_split;            // 1: each chunk row stored parity-split, even pixels then odd (the
                            // layout a stride-2 conv reads); w_out even
  float* out_f32;  // kIfConvT: FP32 [n][2 h_out][2 w_out][8] (5 used: flow x0 y0 x1 y1, mask)
                   // (kIfConvTEnc / kIfConvTZ store through `out`, their layouts above)
  int* err;
};

struct IfMaps {
  CUtensorMap a;  // stride 1: 3-D {2 W u64, chunks, batch*H}; stride 2 (parity-split rows): 4-D
                  // {W u64, 2 parities, chunks, batch*H}
};

// Dynamic shared memory of a launch besides its ring: alignment slack, barriers, the TMEM holder,
// bias and slopes of N columns (at least 192 columns' room, the budget of the classic layers).
__host__ __device__ constexpr uint32_t if_smem_extra(int n) {
  return 1024 + 16 * 8 + 16 + 2 * static_cast<uint32_t>(n > 192 ? n : 192) * 4;
}

template <int kN>
struct IfShape {
  static_assert(kN % 16 == 0 && kN >= 16 && kN <= kIfMaxN, "N");
  static constexpr uint32_t tmem_cols = 2 * kN <= 64 ? 64 : (2 * kN <= 128 ? 128 : (2 * kN <= 256 ? 256 : 512));
  static constexpr int groups_per_warp = kN / 16;  // 8-column groups per epilogue warp (half of N)
};

// Accumulating MMAs kFrom .. kCount - 1 of a stage's descriptor lists, from one or two asm blocks
// (at most 9 MMAs per block).
template <int kFrom, int kCount>
__device__ __forceinline__ void if_issue(uint32_t d, const uint64_t (&ad)[12], const uint64_t (&bd)[12], uint32_t idesc) {
  constexpr int n = kCount - kFrom;
  constexpr int n1 = n < 9 ? n : 9;
  uint64_t a1[9], b1[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) {
    a1[i] = i < n1 ? ad[kFrom + i] : 0;
    b1[i] = i < n1 ? bd[kFrom + i] : 0;
  }
  mma_ss_block<false, n1>(d, a1, b1, idesc);
  if constexpr (n > 9) {
    uint64_t a2[9], b2[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) {
      a2[i] = i < n - 9 ? ad[kFrom + 9 + i] : 0;
      b2[i] = i < n - 9 ? bd[kFrom + 9 + i] : 0;
    }
    mma_ss_block<false, (n > 9 ? n - 9 : 1)>(d, a2, b2, idesc);
  }
}

// kG: input chunks per K group (2, 4, 6 or 8), so that a stage's 3 x kG / 2 MMAs are known at
// compile time and issue from asm blocks with nothing in between (an instruction between two MMAs
// costs the single issuing thread ~60 cycles).
template <int kN, int kStride, int kEpi, int kG>
__global__ void __launch_bounds__(kIfThreads, 1)
    ifconv_kernel(const __grid_constant__ IfMaps maps, const __grid_constant__ IfConvArgs a) {
  static_assert(kG == 2 || kG == 4 || kG == 6 || kG == 8, "group of 2..8 chunks");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t{1023});
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + a.stages * a.stage_bytes);
  uint64_t* empty = full + kIfMaxStages;
  uint64_t* acc_full = empty + kIfMaxStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  float* s_bias = reinterpret_cast<float*>(tmem_holder + 4);
  float* s_slope = s_bias + kN;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&acc_full[0], 1);
    mbar_init(&acc_full[1], 1);
    mbar_init(&acc_empty[0], kIfEpiWarps);
    mbar_init(&acc_empty[1], kIfEpiWarps);
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  for (int j = threadIdx.x; j < kN; j += blockDim.x) {
    s_bias[j] = a.bias[j];
    s_slope[j] = a.slope != nullptr ? a.slope[j] : 0.0f;
  }
  if (warp == 0 && lane == 0) prefetch_tmap(&maps.a);
  if (warp == 1) {
    tmem_alloc(tmem_holder, IfShape<kN>::tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ producer
      RingPos st{0, 0};
      uint32_t issued = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x) {
        const int strip = item % a.strips;
        const int t = item / a.strips;
        const int oy = t % a.h_out;
        const int n = t / a.h_out;
        const int p0 = strip * kIfStrip - 1;  // first pixel (stride 1) / pixel pair (stride 2) of the box
        for (int dy = 0; dy < 3 && ok; ++dy) {
          const int iy = oy * kStride + dy - 1;
          if (iy < 0 || iy >= a.h_in) continue;
          const int row = n * a.h_in + iy;
          for (int grp = 0; grp < a.n_groups; ++grp) {
            if (!wait_bar(&empty[st.idx], st.phase ^ 1u, a.err, kErrWaitProducer)) {
              ok = false;
              break;
            }
            uint64_t* bar = &full[st.idx];
            uint8_t* dst = ring + st.idx * a.stage_bytes;
            mbar_arrive_expect_tx(bar, a.a_bytes + a.b_bytes);
            if constexpr (kStride == 1) {
              tma_load_3d(dst, &maps.a, bar, p0 * 2, grp * a.g, row);
            } else {
              tma_load_4d(dst, &maps.a, bar, p0 * 2, 0, grp * a.g, row);  // even pixels
              tma_load_4d(dst + a.g * kIfChunkBytes, &maps.a, bar, p0 * 2, 1, grp * a.g, row);  // odd pixels
            }
            const uint8_t* src = a.wpack + static_cast<size_t>(dy * a.n_groups + grp) * a.b_bytes;
            for (uint32_t off = 0; off < a.b_bytes; off += 32768u) {
              const uint32_t len = a.b_bytes - off < 32768u ? a.b_bytes - off : 32768u;
              bulk_load(dst + a.a_bytes + off, src + off, len, bar);
            }
            st.advance(a.stages);
            ++issued;
          }
        }
      }
      // every copy issued has landed before the block may exit
      RingPos d = st;
      const uint32_t pending = issued < a.stages ? issued : a.stages;
      for (uint32_t k = 0; k < pending; ++k) {
        d.retreat(a.stages);
        wait_bar(&full[d.idx], d.phase, a.err, kErrWaitDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = make_idesc(128, kN);
      constexpr uint32_t kStep = 2u * kN * 16u;  // B bytes per K step
      RingPos st{0, 0}, acc{0, 0};
      bool ok = true;
      constexpr int kHs = kG / 2;     // K steps per tap (chunk pairs)
      constexpr int kNm = 3 * kHs;    // MMAs per stage
      for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x) {
        const int t = item / a.strips;
        const int oy = t % a.h_out;
        if (!wait_bar(&acc_empty[acc.idx], acc.phase ^ 1u, a.err, kErrWaitMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc.idx * kN;
        bool first = true;
        for (int dy = 0; dy < 3 && ok; ++dy) {
          const int iy = oy * kStride + dy - 1;
          if (iy < 0 || iy >= a.h_in) continue;
          for (int grp = 0; grp < a.n_groups; ++grp) {
            if (!wait_bar(&full[st.idx], st.phase, a.err, kErrWaitMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(ring + st.idx * a.stage_bytes);
            const uint32_t b_base = a_base + a.a_bytes;
            uint64_t ad[12], bd[12];
#pragma unroll
            for (int dx = 0; dx < 3; ++dx) {
              // tap dx: which staged box and how many pixels into it
              uint32_t tile;
              if constexpr (kStride == 1) {
                tile = a_base + static_cast<uint32_t>(dx) * 16u;
              } else {
                const uint32_t odd = a_base + static_cast<uint32_t>(kG) * kIfChunkBytes;
                tile = dx == 0 ? odd : (dx == 1 ? a_base + 16u : odd + 16u);
              }
#pragma unroll
              for (int j = 0; j < kHs; ++j) {
                ad[dx * kHs + j] = make_sdesc(tile + static_cast<uint32_t>(2 * j) * kIfChunkBytes, kIfChunkBytes, 128);
                bd[dx * kHs + j] = make_sdesc(b_base + static_cast<uint32_t>(dx * kHs + j) * kStep, kN * 16u, 128);
              }
            }
#pragma unroll
            for (int i = kNm; i < 12; ++i) ad[i] = bd[i] = 0;
            if (first) {  // the item's first MMA overwrites the accumulator, the rest accumulate
              mma_ss<false>(d_tmem, ad[0], bd[0], idesc, 0u);
              if_issue<1, kNm>(d_tmem, ad, bd, idesc);
              first = false;
            } else {
              if_issue<0, kNm>(d_tmem, ad, bd, idesc);
            }
            mma_commit(&empty[st.idx]);
            st.advance(a.stages);
          }
        }
        if (!ok) break;
        mma_commit(&acc_full[acc.idx]);
        acc.advance(2);
      }
      mma_commit(drain);
      wait_bar(drain, 0, a.err, kErrWaitDrain);
    }
    __syncwarp();
  } else {
    // -------------------------------------------------------------------- epilogue
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    RingPos acc{0, 0};
    for (int item = blockIdx.x; item < a.items; item += gridDim.x) {
      const int strip = item % a.strips;
      const int t = item / a.strips;
      const int oy = t % a.h_out;
      const int n = t / a.h_out;
      const bool got = wait_bar(&acc_full[acc.idx], acc.phase, a.err, kErrWaitEpilogue);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const int m = quad * 32 + lane;
      const int x = strip * kIfStrip + m;
      const bool store = m < kIfStrip && x < a.w_out;
      const int xs = a.out_split ? (x & 1) * (a.w_out >> 1) + (x >> 1) : x;  // stored column
#pragma unroll 1
      for (int q = 0; q < IfShape<kN>::groups_per_warp; ++q) {
        const int cg = half * IfShape<kN>::groups_per_warp + q;  // 8-column group = output chunk
        float v[8];
        __syncwarp();  // tcgen05.ld is warp-collective: every lane arrives here together
        tmem_ld8(tmem_base + lane_addr + acc.idx * kN + static_cast<uint32_t>(cg * 8), v);
        tmem_ld_wait();
        if (!store) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] += s_bias[cg * 8 + j];
        if constexpr (kEpi == kIfConvT) {
          const int py = cg >> 1, px = cg & 1;
          float* dst = a.out_f32 + ((static_cast<size_t>(n) * (2 * a.h_out) + 2 * oy + py) * (2 * a.w_out) + (2 * x + px)) * 8;
          *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
          *reinterpret_cast<float4*>(dst + 4) = make_float4(v[4], 0.0f, 0.0f, 0.0f);
        } else if constexpr (kEpi == kIfConvTEnc) {
          const int py = cg >> 1, px = cg & 1;
          const size_t pix = (static_cast<size_t>(n) * (2 * a.h_out) + 2 * oy + py) * (2 * a.w_out) + (2 * x + px);
          *reinterpret_cast<uint2*>(a.out + pix * 8) = make_uint2(pack_half2(v[0], v[1]), pack_half2(v[2], v[3]));
        } else if constexpr (kEpi == kIfConvTZ) {
          const int phase = cg >> 3, par = (cg >> 1) & 3, part = cg & 1;
          const int zy = 4 * oy + 2 * (phase >> 1) + (par >> 1);
          const int zx = 4 * x + 2 * (phase & 1) + (par & 1);
          const size_t pix = (static_cast<size_t>(n) * (4 * a.h_out) + zy) * (4 * a.w_out) + zx;
          uint4 o;
          o.x = pack_half2(v[0], v[1]);
          o.y = pack_half2(v[2], v[3]);
          o.z = pack_half2(v[4], v[5]);
          o.w = pack_half2(v[6], v[7]);
          *reinterpret_cast<uint4*>(a.out + pix * 32 + part * 16) = o;
        } else {
          const size_t pix = ((static_cast<size_t>(n) * a.h_out + oy) * a.out_chunks + cg) * a.w_out + xs;
          if constexpr (kEpi == kIfResPrelu) {
            const uint4 r = __ldg(reinterpret_cast<const uint4*>(a.residual + pix * 16));
            const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f = unpack_half2(rw[j]);
              v[2 * j] += f.x;
              v[2 * j + 1] += f.y;
            }
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] = v[j] >= 0.0f ? v[j] : v[j] * s_slope[cg * 8 + j];
          uint4 o;
          o.x = pack_half2(v[0], v[1]);
          o.y = pack_half2(v[2], v[3]);
          o.z = pack_half2(v[4], v[5]);
          o.w = pack_half2(v[6], v[7]);
          *reinterpret_cast<uint4*>(a.out + pix * 16) = o;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc.idx]);
      acc.advance(2);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, IfShape<kN>::tmem_cols);
  }
}

}  // namespace kb2
