// Host side of the tensor-core convolution: the K-step table (which input row, pixel shift and
// channel chunk each 32-byte K step of an MMA reads), the matching weight packing (FP16, or E4M3 with
// per-output-channel scales as span_fp8::channel_scales, src/gpu/span_fp8/quantize.h:1-5), the TMA
// tensor maps and the persistent launch.
#include <algorithm>
#include <array>
#include <cstdio>

#include "conv3p.cuh"
#include "conv_layer.h"

namespace kb2 {

namespace {

struct Half {
  int src, dy, dx, chunk;
  bool zero;  // pads the instruction: weights are zero, the data read is in bounds and finite
};

std::vector<std::array<Half, 2>> make_ksteps(const ConvSpec& s, int chunks) {
  std::vector<std::array<Half, 2>> steps;
  if (s.epi == kEpiColsBias) {
    // kernel columns in N: every step reads the slot unshifted (dx = -1: slot pixel m for MMA row m)
    for (int src = 0; src < s.n_sources; ++src)
      for (int c = 0; c + 1 < chunks; c += 2) steps.push_back({Half{src, 0, -1, c, false}, Half{src, 0, -1, c + 1, false}});
    return steps;
  }
  if (s.taps == 1) {
    std::vector<Half> seq;
    for (int src = 0; src < s.n_sources; ++src)
      for (int c = 0; c < chunks; ++c) seq.push_back({src, 0, 0, c, false});
    if (seq.size() % 2 != 0) {
      const Half last = seq.back();
      seq.push_back({last.src, 0, 1, last.chunk, true});
    }
    for (size_t i = 0; i < seq.size(); i += 2) steps.push_back({seq[i], seq[i + 1]});
    return steps;
  }
  for (int dy = -1; dy <= 1; ++dy) {
    for (int dx = -1; dx <= 1; ++dx)
      for (int c = 0; c + 1 < chunks; c += 2) steps.push_back({Half{0, dy, dx, c, false}, Half{0, dy, dx, c + 1, false}});
    if (chunks % 2 != 0) {
      const int cl = chunks - 1;
      // the odd chunk of horizontally adjacent taps: one pixel (16 bytes) apart in the slot
      steps.push_back({Half{0, dy, -1, cl, false}, Half{0, dy, 0, cl, false}});
      steps.push_back({Half{0, dy, 1, cl, false}, Half{0, dy, 2, cl, true}});
    }
  }
  return steps;
}

using LaunchFn = void (*)(dim3, size_t, cudaStream_t, const ConvMaps&, const ConvArgs&);

template <bool F8, int N, int E, int O>
void launch_impl(dim3 grid, size_t smem, cudaStream_t s, const ConvMaps& m, const ConvArgs& a) {
  conv_tc_kernel<F8, N, E, O><<<grid, ConvShape<N>::threads, smem, s>>>(m, a);
}
template <bool F8, int N, int E, int O>
void launch_paired(dim3 grid, size_t smem, cudaStream_t s, const ConvMaps& m, const ConvArgs& a) {
  conv3p_kernel<F8, N, E, O><<<grid, PairShape<N, E, F8>::threads, smem, s>>>(m, a);  // clusters of 2 (__cluster_dims__)
}

constexpr int kKindGeneric = 0, kKindPaired = 2;

struct KernelEntry {
  int kind;  // kKindGeneric: conv_tc.cuh; kKindPaired: conv3p.cuh
  bool fp8;
  int n, epi, out;
  LaunchFn launch;
  const void* fn;
  int threads;
};

#define KB2_KERNEL(F8, N, E, O)                                                                          \
  KernelEntry {                                                                                          \
    kKindGeneric, F8, N, E, O, &launch_impl<F8, N, E, O>,                                                \
        reinterpret_cast<const void*>(&conv_tc_kernel<F8, N, E, O>), ConvShape<N>::threads               \
  }
#define KB2_PAIRED(F8, N, E, O)                                                                          \
  KernelEntry {                                                                                          \
    kKindPaired, F8, N, E, O, &launch_paired<F8, N, E, O>,                                               \
        reinterpret_cast<const void*>(&conv3p_kernel<F8, N, E, O>), PairShape<N, E, F8>::threads             \
  }

// The instantiations the engines use: 3x3 layers on the pair kernel, the 1x1 convs (conv_cat, the
// unshuffle SPAN's attention) on the generic one.
const KernelEntry kKernels[] = {
    KB2_KERNEL(false, 48, kEpiBias, kOutF16Chunk),
    KB2_PAIRED(false, 48, kEpiBias, kOutF16Chunk),
    KB2_PAIRED(false, 48, kEpiSilu, kOutF16Chunk),
    KB2_PAIRED(false, 48, kEpiSpanAttn, kOutF16Chunk),
    // SPAN's conv_cat folded into its upsampler: one 3x3 conv over the four sources, kernel columns in N
    KB2_PAIRED(false, 48, kEpiColsBias, kOutPixShuf2),
    KB2_PAIRED(false, 48, kEpiColsBias, kOutPixShuf2Display),
    KB2_PAIRED(false, 48, kEpiSpanAttn, kOutF16E4m3),
    KB2_PAIRED(true, 48, kEpiSilu, kOutE4m3Chunk),
    KB2_PAIRED(true, 48, kEpiSilu, kOutF16E4m3),
    KB2_PAIRED(true, 48, kEpiSpanAttn, kOutE4m3Chunk),
    KB2_PAIRED(true, 48, kEpiSpanAttn, kOutF16Chunk),
    // the IFNet residual convs of 64 channels (ifnet_net.cu): pair kernel only
    KB2_PAIRED(false, 64, kEpiResPrelu, kOutF16Chunk),
    // the unshuffle SPAN (span8_net.cu): ReLU convs (PReLU, slope 0), c3 and conv_1 at 64
    // channels, to_pixel with DepthToSpace(4), the 1x1 attention with its tanh gate, conv_cat at 64
    KB2_PAIRED(false, 48, kEpiPrelu, kOutF16Chunk),
    KB2_PAIRED(false, 64, kEpiPrelu, kOutF16Chunk),
    KB2_PAIRED(false, 64, kEpiBias, kOutF16Chunk),
    KB2_PAIRED(false, 48, kEpiBias, kOutPixShuf4),
    KB2_KERNEL(false, 48, kEpiTanhGate, kOutF16Chunk),
    KB2_KERNEL(false, 64, kEpiTanhGate, kOutF16Chunk),
    KB2_KERNEL(false, 64, kEpiBias, kOutF16Chunk),
    // its E4M3 blocks: ReLU convs to E4M3 (the last block's first one to FP16 as well, a conv_cat
    // source), c3 to FP16, the gate and conv_1 writing FP16 and E4M3 copies of the block input
    KB2_PAIRED(true, 48, kEpiPrelu, kOutE4m3Chunk),
    KB2_PAIRED(true, 48, kEpiPrelu, kOutF16E4m3),
    KB2_PAIRED(true, 48, kEpiBias, kOutF16Chunk),
    KB2_PAIRED(true, 64, kEpiPrelu, kOutE4m3Chunk),
    KB2_PAIRED(true, 64, kEpiPrelu, kOutF16E4m3),
    KB2_PAIRED(true, 64, kEpiBias, kOutF16Chunk),
    KB2_PAIRED(false, 48, kEpiBias, kOutF16E4m3),
    KB2_PAIRED(false, 64, kEpiBias, kOutF16E4m3),
    KB2_KERNEL(false, 48, kEpiTanhGate, kOutF16E4m3),
    KB2_KERNEL(false, 64, kEpiTanhGate, kOutF16E4m3),
};

bool wants_stacked(const ConvSpec& s) {
  if (s.epi == kEpiColsBias) return s.taps == 9 && s.n_sources == 4 && s.n_pad == 48 && !s.fp8;
  return s.taps == 9 && s.n_sources == 1 && (s.n_pad == 48 || s.n_pad == 16 || s.n_pad == 64);
}

// K steps per input row the pair kernel runs (conv3p.cuh): 64 output channels 12 or 3 in FP16, 6 in
// E4M3 (64 inputs); 48 channels 2, 3, 5, 9, or 12 in FP16 (64 FP16 inputs); 16 channels 2, 3, 5 or 9
bool pair_admits(const ConvSpec& s, int nk) {
  if (s.n_pad == 64) return s.fp8 ? nk == 6 : (nk == 12 || nk == 3);
  if (nk == 12) return !s.fp8 && s.n_pad == 48;
  return nk == 2 || nk == 3 || nk == 5 || nk == 9;
}

const KernelEntry* find_kernel(const ConvSpec& s, int kind) {
  for (const KernelEntry& k : kKernels)
    if (k.kind == kind && k.fp8 == s.fp8 && k.n == s.n_pad && k.epi == s.epi && k.out == s.out) return &k;
  return nullptr;
}

uint32_t tmem_cols(int n) {
  const uint32_t stride = n <= 32 ? 32 : (n <= 64 ? 64 : (n <= 128 ? 128 : 256));
  return 2 * stride;
}

uint16_t f32_to_f16_bits(float f) {
  const __half h = __float2half_rn(f);
  return *reinterpret_cast<const uint16_t*>(&h);
}

}  // namespace

int num_sms() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

Status ConvLayer::build(const ConvSpec& s, const float* W, const float* b, const float* prelu_slope,
                        const float* act_scales, const ChunkedTensor* const* inputs, int* err_word) {
  spec = s;
  // 3x3 layers run stacked on the pair kernel (conv3p.cuh), the rest on the generic one
  const bool stacked = wants_stacked(s);
  kind = stacked ? kKindPaired : kKindGeneric;
  const KernelEntry* k = find_kernel(s, kind);
  if (k == nullptr) return refuse(KB2_FORMAT_UNSUPPORTED, "no tensor-core kernel for this layer shape");
  const ChunkedTensor& in0 = *inputs[0];
  for (int i = 0; i < s.n_sources; ++i) {
    const ChunkedTensor& t = *inputs[i];
    if (t.fp8 != s.fp8 || t.chunks != in0.chunks || t.H != in0.H || t.W != in0.W || t.batch != in0.batch)
      return refuse(KB2_INPUT_MISMATCH, "conv sources of different geometry");
  }
  const int chunks = in0.chunks;
  const int epc = s.fp8 ? 16 : 8;
  const int halo = s.taps == 9 ? 1 : 0;
  if (chunks * epc < s.cin) return refuse(KB2_INPUT_MISMATCH, "input tensor narrower than the conv");

  auto steps = make_ksteps(s, chunks);
  if (stacked) {
    // one input row per instruction group: the dy = 0 steps (every dy uses the same pixel shifts
    // and channel pairs); the three kernel rows go into N instead
    std::vector<std::array<Half, 2>> row_steps;
    for (const auto& st : steps)
      if (st[0].dy == 0) row_steps.push_back(st);
    steps = row_steps;
    // the pair kernel (one MMA for two SMs) runs rows of the K-step counts it admits
    if (!pair_admits(s, static_cast<int>(steps.size())))
      return refuse(KB2_FORMAT_UNSUPPORTED, "no tensor-core kernel for this row shape");
  }
  const bool paired = kind == kKindPaired;
  if (static_cast<int>(steps.size()) > kMaxKSteps) return refuse(KB2_FORMAT_UNSUPPORTED, "too many K steps");
  // the row slot is one 128-pixel TMA box starting at x0 - halo; an A tile shifted by dx reads slot
  // pixels m + halo + dx (+1 for the second half of a zero-partnered step) for MMA row m, so the
  // strip keeps only the rows whose reads stay inside the box
  int reach = 0;  // furthest slot pixel an A half reads for MMA row 0
  for (const auto& st : steps)
    for (const Half& h : st) reach = std::max(reach, h.dx + halo);
  const int px = kRowBoxPx;
  // kernel columns in N: MMA row m is slot pixel m, and output m - 1 needs rows m - 1 .. m + 1
  const bool cols = s.epi == kEpiColsBias;
  if (cols && (s.n_real > 16 || s.cin % 16 != 0 || chunks * epc != s.cin))
    return refuse(KB2_FORMAT_UNSUPPORTED, "columns in N: up to 16 outputs from whole 16-channel input pairs");
  const int strip_w = cols ? px - 2 : px - reach;
  if (strip_w < 64) return refuse(KB2_FORMAT_UNSUPPORTED, "row slot too narrow for the taps");
  const uint32_t src_bytes = static_cast<uint32_t>(chunks) * px * 16;
  const uint32_t slot_bytes = src_bytes * static_cast<uint32_t>(s.n_sources);

  ConvArgs& a = args;
  a = ConvArgs{};
  a.batch = in0.batch;
  a.H = in0.H;
  a.W = in0.W;
  a.strip_w = strip_w;
  a.strips = (in0.W + strip_w - 1) / strip_w;
  a.n_sources = s.n_sources;
  a.chunks = chunks;
  a.px = px;
  a.halo = halo;
  a.in_rows = s.taps == 9 ? 3 : 1;
  a.row_off = s.taps == 9 ? -1 : 0;
  a.src_bytes = src_bytes;
  a.slot_bytes = slot_bytes;
  a.ring = 0;  // sized below from the shared memory left for two blocks per SM
  a.n_ksteps = static_cast<int>(steps.size());
  for (size_t j = 0; j < steps.size(); ++j) {
    auto addr = [&](const Half& h) {
      return static_cast<int64_t>(h.src) * src_bytes + static_cast<int64_t>(h.chunk) * px * 16 +
             static_cast<int64_t>(h.dx + halo) * 16;
    };
    const int64_t a0 = addr(steps[j][0]);
    const int64_t a1 = addr(steps[j][1]);
    if (steps[j][0].dy != steps[j][1].dy || a1 <= a0 || (a1 - a0) % 16 != 0 || (a1 - a0) >= (1 << 18))
      return refuse(KB2_FORMAT_UNSUPPORTED, "K step halves not expressible as one descriptor");
    a.ks[j].a_off = static_cast<uint32_t>(a0);
    a.ks[j].lbo = static_cast<uint32_t>(a1 - a0);
    a.ks[j].row = s.taps == 9 ? steps[j][0].dy + 1 : 0;
    // the distinct (offset, LBO) pairs of a row are the A tiles copied to TMEM once per input row
    int tile = -1;
    for (int t = 0; t < a.n_tiles; ++t)
      if (a.tile_off[t] == a.ks[j].a_off && a.tile_lbo[t] == a.ks[j].lbo) tile = t;
    if (tile < 0 && a.n_tiles < kMaxTiles) {
      tile = a.n_tiles++;
      a.tile_off[tile] = a.ks[j].a_off;
      a.tile_lbo[tile] = a.ks[j].lbo;
    }
    a.ks[j].tile = tile < 0 ? 0 : tile;
  }
  // A from TMEM for 3x3 layers (rows reused by three output rows) when the tiles of four input
  // rows fit beside the accumulators in the 512 TMEM columns
  a.tmem_a = (s.taps == 9 && a.n_tiles <= kMaxTiles &&
              kTmemRegionBase + kTmemRegions * 8u * static_cast<uint32_t>(a.n_tiles) <= 512u)
                 ? 1
                 : 0;
  a.idesc = make_idesc(kTileM, s.n_pad);
  if (stacked) {
    a.tmem_a = 0;
    a.n_tiles = 0;
    for (int i = 0; i < 3; ++i) a.idesc_n[i] = make_idesc(kTileM, (i + 1) * s.n_pad);
    a.acc_slots = static_cast<int>(kStackSlots);
    if (static_cast<int>(steps.size()) > kPairMaxK)
      return refuse(KB2_FORMAT_UNSUPPORTED, "stacked: too many K steps per row");
  }
  const int n_rows_b = stacked ? 3 * s.n_pad : s.n_pad;  // rows of B per K step

  // ---- weights
  const int kk = s.taps == 9 ? 3 : 1;
  const int cin_total = s.n_sources * s.cin;
  auto w_at = [&](int co, int ci_total, int ky, int kx) {
    return W[((static_cast<size_t>(co) * cin_total + ci_total) * kk + ky) * kk + kx];
  };
  std::vector<float> wscale(static_cast<size_t>(s.n_pad), 1.0f);
  auto src_scale = [&](int src) { return act_scales != nullptr ? act_scales[src] : 1.0f; };
  if (s.fp8) {
    for (int co = 0; co < s.n_real; ++co) {
      float mx = 0.0f;
      for (int src = 0; src < s.n_sources; ++src)
        for (int ci = 0; ci < s.cin; ++ci)
          for (int ky = 0; ky < kk; ++ky)
            for (int kx = 0; kx < kk; ++kx)
              mx = std::fmax(mx, std::fabs(w_at(co, src * s.cin + ci, ky, kx) * src_scale(src)));
      wscale[co] = mx > 0.0f ? mx / 448.0f : 1.0f;
    }
  }
  // B of K step j: [half][row][16 bytes]; stacked layers have 3 row blocks, block b holding the
  // kernel row ky = 2 - b (dy = +1, 0, -1) so that its results land on output rows o = t - 2 + b
  const size_t step_bytes = 2u * static_cast<size_t>(n_rows_b) * 16u;
  std::vector<uint8_t> packed(steps.size() * step_bytes, 0);
  for (size_t j = 0; j < steps.size(); ++j) {
    for (int h = 0; h < 2; ++h) {
      const Half& hf = steps[j][h];
      for (int row = 0; row < n_rows_b; ++row) {
        const int blk = row / s.n_pad;
        // with the kernel columns in N, row 16 kx + c of a kernel-row block is column kx, channel c
        const int col_kx = cols ? (row % s.n_pad) / 16 : 0;
        const int co = cols ? row % 16 : row % s.n_pad;
        if (co >= s.n_real) continue;
        for (int e = 0; e < epc; ++e) {
          const int ci = hf.chunk * epc + e;
          float v = 0.0f;
          if (!hf.zero && ci < s.cin) {
            const int ky = stacked ? 2 - blk : (s.taps == 9 ? hf.dy + 1 : 0);
            const int kx = cols ? col_kx : (s.taps == 9 ? hf.dx + 1 : 0);
            v = w_at(co, hf.src * s.cin + ci, ky, kx);
          }
          // paired kernel: block r of the pair holds B rows [r N/2, (r + 1) N/2) of every step
          const int half_rows = n_rows_b / 2;
          uint8_t* dst = paired ? packed.data() + static_cast<size_t>(row / half_rows) * (packed.size() / 2) +
                                      j * (step_bytes / 2) + static_cast<size_t>(h) * half_rows * 16 +
                                      static_cast<size_t>(row % half_rows) * 16
                                : packed.data() + j * step_bytes + static_cast<size_t>(h) * n_rows_b * 16 +
                                      static_cast<size_t>(row) * 16;
          if (s.fp8) {
            dst[e] = e4m3_encode(v * src_scale(hf.src) / wscale[co]);
          } else {
            const uint16_t bits = f32_to_f16_bits(v);
            std::memcpy(dst + 2 * e, &bits, 2);
          }
        }
      }
    }
  }
  KB2_TRY(wpack.alloc(packed.size()));
  KB2_CUDA(cudaMemcpy(wpack.ptr, packed.data(), packed.size(), cudaMemcpyHostToDevice));
  std::vector<float> bias_h(static_cast<size_t>(s.n_pad), 0.0f), slope_h(static_cast<size_t>(s.n_pad), 0.0f);
  for (int co = 0; co < s.n_real; ++co) {
    bias_h[co] = b != nullptr ? b[co] : 0.0f;
    slope_h[co] = prelu_slope != nullptr ? prelu_slope[co] : 0.0f;
  }
  KB2_TRY(bias.alloc(bias_h.size() * 4));
  KB2_CUDA(cudaMemcpy(bias.ptr, bias_h.data(), bias_h.size() * 4, cudaMemcpyHostToDevice));
  KB2_TRY(slope.alloc(slope_h.size() * 4));
  KB2_CUDA(cudaMemcpy(slope.ptr, slope_h.data(), slope_h.size() * 4, cudaMemcpyHostToDevice));
  if (s.fp8) {
    KB2_TRY(scale.alloc(wscale.size() * 4));
    KB2_CUDA(cudaMemcpy(scale.ptr, wscale.data(), wscale.size() * 4, cudaMemcpyHostToDevice));
  }
  a.wpack = wpack.as<uint8_t>();
  a.wbytes = static_cast<uint32_t>(packed.size());
  a.w_smem = ((paired ? a.wbytes / 2u : a.wbytes) + 1023u) / 1024u * 1024u;
  a.bias = bias.as<float>();
  a.slope = slope.as<float>();
  a.chan_scale = s.fp8 ? scale.as<float>() : nullptr;
  {
    // SiLU and gate layers hold their constants halved (exact): their epilogue works on v / 2
    const float half = (s.epi == kEpiSilu || s.epi == kEpiSpanAttn) ? 0.5f : 1.0f;
    for (int co = 0; co < kMaxN; ++co) {
      a.cbias[co] = co < s.n_pad ? half * bias_h[co] : 0.0f;
      a.cscale[co] = half * ((s.fp8 && co < static_cast<int>(wscale.size())) ? wscale[co] : 1.0f);
    }
  }
  a.out_chunks = s.out_chunks;
  a.out2_chunks = s.out2_chunks;
  a.err = err_word;

  // ---- tensor maps (single-source layers repeat map 0)
  for (int i = 0; i < 4; ++i) KB2_TRY(encode_row_map(&maps.m[i], *inputs[i < s.n_sources ? i : 0]));

  // ---- launch shape
  // ring: as many row slots as fit beside the weights with two blocks per SM (at least the window
  // plus one row of prefetch, at most 12)
  // TMEM-A layers own all 512 TMEM columns: one block per SM, and a ring as deep as shared memory
  // allows (slots are released as soon as copied, so the producer runs that many rows ahead);
  // stacked layers run kStackBlocksPerSm blocks per SM, each with its share of TMEM
  const bool one_per_sm = a.tmem_a != 0 || (stacked && kStackBlocksPerSm == 1);
  {
    const size_t fixed = a.w_smem + (stacked ? kStackSmemExtra : kConvSmemExtra);
    const int min_ring = a.in_rows + 1;
    auto fit = [&](size_t per_block) {
      return per_block > fixed ? static_cast<int>((per_block - fixed) / slot_bytes) : 0;
    };
    int ring = one_per_sm ? fit(200u * 1024u) : fit((228u * 1024u) / 2 - 2048u);
    if (!one_per_sm && !stacked && ring < min_ring + 2) ring = fit(227u * 1024u);  // wide slots: one block per SM
    ring = std::min(ring, 12);
    // the pair issuer's ring is fixed by its 12-row periods (checked against shared memory below)
    if (paired) ring = static_cast<int>(cols ? kColsRing : steps.size() == 12 ? pair_ring<12>() : pair_ring<9>());
    a.ring = static_cast<uint32_t>(std::max(ring, min_ring));
  }
  smem = a.w_smem + static_cast<size_t>(a.ring) * slot_bytes + (stacked ? kStackSmemExtra : kConvSmemExtra) +
         (cols ? kStackXchgBytes : 0u);
  // a block that allocates all 512 TMEM columns asks for more than half the SM's shared memory, so
  // two of them are never co-resident (the second would only wait in tcgen05.alloc)
  if (one_per_sm) smem = std::max<size_t>(smem, 120u * 1024u);
  int dev = 0;
  KB2_CUDA(cudaGetDevice(&dev));
  int optin = 0;
  KB2_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  if (smem > static_cast<size_t>(optin)) return refuse(KB2_FORMAT_UNSUPPORTED, "layer needs too much shared memory");
  KB2_CUDA(cudaFuncSetAttribute(k->fn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin));
  KB2_CUDA(cudaFuncSetAttribute(k->fn, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
  int per_sm = 0;
  KB2_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k->fn, k->threads, smem));
  if (per_sm < 1) return refuse(KB2_FORMAT_UNSUPPORTED, "layer does not fit on an SM");
  // resident blocks per SM: shared memory (228 KB per SM, 1 KB reserved per block) and TMEM
  // (512 columns; a TMEM-A block takes them all) permitting
  const int smem_fit = static_cast<int>((228u * 1024u) / (smem + 1024u));
  const int tmem_fit = a.tmem_a ? 1 : (stacked ? kStackBlocksPerSm : static_cast<int>(512u / tmem_cols(s.n_pad)));
  per_sm = std::min({per_sm, smem_fit, tmem_fit});
  if (per_sm < 1) per_sm = 1;
  int slots = num_sms() * per_sm;
  a.pairs = (a.strips + 1) / 2;
  if (paired) {
    // resident pairs: clusters need both SMs of a pair free, so ask the runtime instead of
    // halving the SM count
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(2 * (num_sms() / 2)));
    cfg.blockDim = dim3(static_cast<unsigned>(k->threads));
    cfg.dynamicSmemBytes = smem;
    int clusters = 0;
    KB2_CUDA(cudaOccupancyMaxActiveClusters(&clusters, k->fn, &cfg));
    if (clusters < 1) return refuse(KB2_FORMAT_UNSUPPORTED, "paired layer: no cluster of two fits");
    slots = clusters;
  }
  const int units = paired ? a.pairs : a.strips;  // work units across a row band
  // bands: about 16 work items per resident block (pair), 4..64 rows each (8.. for the stacked
  // kernels, whose two halo rows per band are extra MMA work)
  const long long rows_total = static_cast<long long>(a.batch) * a.H * units;
  int band = static_cast<int>(rows_total / (16LL * slots));
  const int band_min = stacked ? 8 : 4;
  band = band < band_min ? band_min : (band > 64 ? 64 : band);
  // 1x1 layers (no halo rows, so short bands cost nothing): bands of 8 rows keep the blocks that
  // run at once on neighbouring rows of the same frames (conv_cat 2 % faster on 8 x 1080p)
  if (!stacked && a.in_rows == 1) band = std::min(band, 8);
  a.band_rows = band;
  a.bands = (a.H + band - 1) / band;
  a.items = a.batch * a.bands * units;
  grid = a.items < slots ? a.items : slots;
  if (paired) grid = 2 * slots;  // two blocks per cluster; the launch trims it to the rows
  return Status::Ok();
}

void ConvLayer::set_tap_bias(const float* tb) {
  for (int t = 0; t < 9; ++t)
    for (int c = 0; c < 16; ++c) args.tap_bias[t][c] = c < spec.n_real ? tb[t * spec.n_real + c] : 0.0f;
}

Status ConvLayer::launch(cudaStream_t stream, int batch, void* out, const void* residual, float out_inv_scale,
                         float res_scale, void* out2, int res_chunks, const void* residual2, long long out_pitch,
                         int display_format) const {
  const KernelEntry* k = find_kernel(spec, kind);
  if (k == nullptr) return refuse(KB2_FORMAT_UNSUPPORTED, "no kernel");
  const bool paired = kind == kKindPaired;
  ConvArgs a = args;
  a.batch = batch;
  a.items = batch * a.bands * (paired ? a.pairs : a.strips);
  a.out = static_cast<uint8_t*>(out);
  a.out2 = static_cast<uint8_t*>(out2);
  a.residual = static_cast<const uint8_t*>(residual);
  a.residual2 = static_cast<const uint8_t*>(residual2);
  a.res_fp8 = spec.fp8 ? 1 : 0;
  a.res_chunks = res_chunks;
  a.out_inv_scale = out_inv_scale;
  a.res_scale = res_scale;
  a.out_pitch = out_pitch;
  a.display_format = display_format;
  int g = a.items < grid ? a.items : grid;
  if (paired) {
    // pair kernel: contiguous row ranges, one per cluster (conv3p.cuh PairSpan)
    const long long rows = static_cast<long long>(batch) * a.pairs * a.H;
    const long long clusters = grid / 2;
    g = 2 * static_cast<int>(rows < clusters ? rows : clusters);
  }
  k->launch(dim3(static_cast<unsigned>(g)), smem, stream, maps, a);
  return cuda_status(cudaGetLastError(), "conv_tc_kernel launch");
}

}  // namespace kb2
