// One tensor-core conv of the interpolators (if_layer.h): the ifconv_kernel instantiations every
// layer shape of classic IFNet and RIFE 4.2x needs, the weight packing, the tensor map of the input
// rows and the launch shape.
#include <algorithm>
#include <cstring>

#include "if_layer.h"

namespace kb2 {

using IfLaunchFn = void (*)(dim3, size_t, cudaStream_t, const IfMaps&, const IfConvArgs&);

struct IfKernel {
  int n, stride, epi, g;
  IfLaunchFn launch;
  const void* fn;
};

namespace {

template <int N, int S, int E, int G>
void if_launch(dim3 grid, size_t smem, cudaStream_t s, const IfMaps& m, const IfConvArgs& a) {
  ifconv_kernel<N, S, E, G><<<grid, kIfThreads, smem, s>>>(m, a);
}

#define KB2_IFK(N, S, E, G) \
  IfKernel { N, S, E, G, &if_launch<N, S, E, G>, reinterpret_cast<const void*>(&ifconv_kernel<N, S, E, G>) }

// every conv shape of the interpolators: (N, stride, epilogue, input chunks per K group)
const IfKernel kIfKernels[] = {
    // classic IFNet conv0a: 12 (7) channels -> C/2, stride 2; RIFE 4.2x block 0 (15 channels)
    KB2_IFK(96, 2, kIfPrelu, 2), KB2_IFK(64, 2, kIfPrelu, 2), KB2_IFK(48, 2, kIfPrelu, 2), KB2_IFK(32, 2, kIfPrelu, 2),
    KB2_IFK(16, 2, kIfPrelu, 2),
    // RIFE 4.2x conv0a of blocks 1.. (28 channels in 4 chunks)
    KB2_IFK(96, 2, kIfPrelu, 4), KB2_IFK(64, 2, kIfPrelu, 4), KB2_IFK(48, 2, kIfPrelu, 4), KB2_IFK(32, 2, kIfPrelu, 4),
    KB2_IFK(16, 2, kIfPrelu, 4),
    // conv0b: C/2 -> C, stride 2
    KB2_IFK(192, 2, kIfPrelu, 6), KB2_IFK(128, 2, kIfPrelu, 8), KB2_IFK(96, 2, kIfPrelu, 6),
    KB2_IFK(64, 2, kIfPrelu, 4), KB2_IFK(32, 2, kIfPrelu, 2),
    // residual convs: C -> C (64 channels: the pair kernel)
    KB2_IFK(192, 1, kIfResPrelu, 8), KB2_IFK(128, 1, kIfResPrelu, 8), KB2_IFK(96, 1, kIfResPrelu, 6),
    KB2_IFK(64, 1, kIfResPrelu, 8), KB2_IFK(32, 1, kIfResPrelu, 4),
    // classic transposed conv: C -> 4 phases x 8
    KB2_IFK(32, 1, kIfConvT, 8), KB2_IFK(32, 1, kIfConvT, 6),
    // RIFE 4.2x transposed conv: C -> 4 phases x 4 DepthToSpace parities x 16 (13 used)
    KB2_IFK(256, 1, kIfConvTZ, 4),
    // RIFE 4.2x encoder: cnn0 (3 -> 16, stride 2), cnn1 / cnn2 (16 -> 16), cnn3 (16 -> 4 phases x 8)
    KB2_IFK(16, 1, kIfPrelu, 2), KB2_IFK(32, 1, kIfConvTEnc, 2),
};

const IfKernel* find_if_kernel(int n, int stride, int epi, int g) {
  for (const IfKernel& k : kIfKernels)
    if (k.n == n && k.stride == stride && k.epi == epi && k.g == g) return &k;
  return nullptr;
}

uint16_t f16_bits(float f) {
  const __half h = __float2half_rn(f);
  uint16_t b;
  std::memcpy(&b, &h, 2);
  return b;
}

// Largest even divisor of `chunks` that is at most 8: the chunks staged per K group.
int group_chunks(int chunks) {
  for (int g = 8; g >= 2; g -= 2)
    if (chunks % g == 0) return g;
  return 0;
}

}  // namespace

Status IfLayer::build_paired(int c, const float* w, const float* b, const float* prelu, uint8_t* in, int batch,
                             int h, int wd, uint8_t* out, int* err) {
  ConvSpec s;
  s.taps = 9;
  s.fp8 = false;
  s.n_sources = 1;
  s.cin = c;
  s.n_real = c;
  s.n_pad = c;
  s.epi = kEpiResPrelu;
  s.out = kOutF16Chunk;
  s.out_chunks = c / 8;
  ChunkedTensor t;
  t.ptr = in;
  t.batch = batch;
  t.H = h;
  t.W = wd;
  t.chunks = c / 8;
  t.fp8 = false;
  const ChunkedTensor* inputs[1] = {&t};
  KB2_TRY(pair.build(s, w, b, prelu, nullptr, inputs, err));
  if (pair.kind != 2) return refuse(KB2_FORMAT_UNSUPPORTED, "IFNet: residual conv did not map to the pair kernel");
  paired = true;
  pair_out = out;
  pair_res = in;
  pair_res_chunks = c / 8;
  args.h_out = h;
  args.w_out = wd;
  flops_px = 2.0 * 9.0 * c * c;
  bytes_px = 3.0 * (c / 8) * 16.0;  // input, residual and output: one FP16 pixel each
  return Status::Ok();
}

Status IfLayer::build(int n_pad, int stride, int epi, const std::vector<float>& w, int cout, int cin, const float* b,
                      const float* prelu, uint8_t* in, int batch, int h_in, int w_in, int in_chunks, int h_out,
                      int w_out, uint8_t* out, int out_chunks, float* out_f32, int* err, int g) {
  if (g == 0) g = group_chunks(in_chunks);
  if (g == 0 || (in_chunks > g && in_chunks % g != 0) || in_chunks * 8 < cin ||
      w.size() != static_cast<size_t>(n_pad) * cin * 9)
    return refuse(KB2_FORMAT_UNSUPPORTED, "IFNet: input channel layout");
  k = find_if_kernel(n_pad, stride, epi, g);
  if (k == nullptr) return refuse(KB2_FORMAT_UNSUPPORTED, "IFNet: no conv kernel for this layer shape");
  IfConvArgs& a = args;
  a.h_in = h_in;
  a.w_in = w_in;
  a.h_out = h_out;
  a.w_out = w_out;
  a.g = g;
  a.n_groups = (in_chunks + g - 1) / g;
  a.strips = (w_out + kIfStrip - 1) / kIfStrip;
  a.a_bytes = static_cast<uint32_t>(g) * kIfChunkBytes * (stride == 2 ? 2u : 1u);
  a.b_bytes = static_cast<uint32_t>(3 * g * n_pad * 16);
  a.stage_bytes = (a.a_bytes + a.b_bytes + 1023u) & ~1023u;
  a.out = out;
  a.out_chunks = out_chunks;
  a.out_split = 0;
  a.out_f32 = out_f32;
  a.residual = epi == kIfResPrelu ? in : nullptr;
  if (epi == kIfConvTZ && (n_pad != 256 || out == nullptr)) return refuse(KB2_FORMAT_UNSUPPORTED, "IFNet: Z layout");
  if (epi == kIfConvTEnc && (n_pad != 32 || out == nullptr)) return refuse(KB2_FORMAT_UNSUPPORTED, "IFNet: encoding layout");
  a.err = err;

  // weights: [dy][group][dx][K step j][half][n][8 channels], FP16
  const size_t wbytes = static_cast<size_t>(3) * a.n_groups * a.b_bytes;
  std::vector<uint16_t> pack(wbytes / 2, 0);
  for (int dy = 0; dy < 3; ++dy)
    for (int grp = 0; grp < a.n_groups; ++grp)
      for (int dx = 0; dx < 3; ++dx)
        for (int j = 0; j < g / 2; ++j)
          for (int h = 0; h < 2; ++h)
            for (int n = 0; n < cout; ++n)
              for (int e = 0; e < 8; ++e) {
                const int ci = (grp * g + 2 * j + h) * 8 + e;
                if (ci >= cin) continue;
                const size_t off = (static_cast<size_t>(dy * a.n_groups + grp) * a.b_bytes +
                                    static_cast<size_t>((dx * (g / 2) + j) * 2 + h) * n_pad * 16 + n * 16 + e * 2) /
                                   2;
                pack[off] = f16_bits(w[((static_cast<size_t>(n) * cin + ci) * 3 + dy) * 3 + dx]);
              }
  KB2_TRY(wpack.alloc(wbytes));
  KB2_CUDA(cudaMemcpy(wpack.ptr, pack.data(), wbytes, cudaMemcpyHostToDevice));
  std::vector<float> bv(n_pad, 0.0f), sv(n_pad, 0.0f);
  for (int n = 0; n < n_pad; ++n) {
    bv[n] = b[n];
    sv[n] = prelu != nullptr ? prelu[n] : 0.0f;
  }
  KB2_TRY(bias.alloc(n_pad * sizeof(float)));
  KB2_TRY(slope.alloc(n_pad * sizeof(float)));
  KB2_CUDA(cudaMemcpy(bias.ptr, bv.data(), n_pad * sizeof(float), cudaMemcpyHostToDevice));
  KB2_CUDA(cudaMemcpy(slope.ptr, sv.data(), n_pad * sizeof(float), cudaMemcpyHostToDevice));
  a.wpack = wpack.as<uint8_t>();
  a.bias = bias.as<float>();
  a.slope = slope.as<float>();

  // tensor map of the input rows (UINT64 words: tile mode copies bytes)
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr) return refuse(KB2_VENDOR_CALL_FAILED, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t row = static_cast<cuuint64_t>(w_in) * 16;
  const cuuint64_t rows = static_cast<cuuint64_t>(batch) * h_in;
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r;
  if (stride == 1) {
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(w_in) * 2, static_cast<cuuint64_t>(in_chunks), rows};
    const cuuint64_t strides[2] = {row, row * in_chunks};
    const cuuint32_t box[3] = {256, static_cast<cuuint32_t>(g), 1};
    r = fn(&maps.a, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, in, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    // parity-split rows: a chunk row is its W/2 even pixels then its W/2 odd pixels, so each
    // parity box is one contiguous 2 KB run per chunk
    if (w_in % 2 != 0) return refuse(KB2_FORMAT_UNSUPPORTED, "IFNet: stride-2 input of odd width");
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(w_in), 2, static_cast<cuuint64_t>(in_chunks), rows};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(w_in / 2) * 16, row, row * in_chunks};
    const cuuint32_t box[4] = {256, 1, static_cast<cuuint32_t>(g), 1};
    r = fn(&maps.a, CU_TENSOR_MAP_DATA_TYPE_UINT64, 4, in, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS)
    return refuse(KB2_VENDOR_CALL_FAILED, "IFNet: cuTensorMapEncodeTiled failed: " + std::to_string(r));

  // launch shape: as many ring slots as fit (2..4), blocks per SM by shared memory and TMEM.
  // Where TMEM holds two blocks' accumulators and two ring slots fit in half the SM's shared
  // memory, the ring is cut to that half so two blocks share the SM: one block's epilogue then
  // overlaps the other's MMAs (measured faster on the 96- and 128-channel 1080p layers).
  int dev = 0, optin = 0;
  KB2_CUDA(cudaGetDevice(&dev));
  KB2_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  const uint32_t extra = if_smem_extra(n_pad);
  const size_t budget = static_cast<size_t>(optin) - extra;
  a.stages = static_cast<uint32_t>(std::min<size_t>(kIfMaxStages, budget / a.stage_bytes));
  if (a.stages < 2) return refuse(KB2_FORMAT_UNSUPPORTED, "IFNet: layer stage does not fit in shared memory");
  const uint32_t tmem_cols = 2 * n_pad <= 64 ? 64 : (2 * n_pad <= 128 ? 128 : (2 * n_pad <= 256 ? 256 : 512));
  {
    const size_t half = (228u * 1024u) / 2 - 1024u - extra;
    const uint32_t st2 = static_cast<uint32_t>(std::min<size_t>(kIfMaxStages, half / a.stage_bytes));
    if (512u / tmem_cols >= 2 && st2 >= 2) a.stages = std::min(a.stages, st2);
  }
  smem = static_cast<size_t>(a.stages) * a.stage_bytes + extra;
  KB2_CUDA(cudaFuncSetAttribute(k->fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  const int smem_fit = static_cast<int>((228u * 1024u) / (smem + 1024u));
  per_sm = std::max(1, std::min(smem_fit, static_cast<int>(512u / tmem_cols)));
  // algorithmic work per output pixel of this conv grid (the transposed conv: 16 taps x 5 outputs
  // per input pixel, whatever the phase layout)
  // algorithmic work per output pixel of this conv grid; the transposed convs: 16 taps x their
  // outputs per input pixel (5 classic, 52 RIFE 4.2x, 4 for the encoder), whatever the phase layout
  const double t_out = epi == kIfConvT ? 5.0 : epi == kIfConvTZ ? 52.0 : 4.0;
  const bool convt = epi == kIfConvT || epi == kIfConvTZ || epi == kIfConvTEnc;
  flops_px = convt ? 2.0 * 16.0 * cin * t_out : 2.0 * 9.0 * cin * cout;
  const double out_px = epi == kIfConvT ? 4.0 * 32.0 : epi == kIfConvTZ ? 16.0 * 32.0 : epi == kIfConvTEnc ? 4.0 * 8.0
                                                                                                       : out_chunks * 16.0;
  bytes_px = out_px + (epi == kIfResPrelu ? out_chunks * 16.0 : 0.0) +
             in_chunks * 16.0 * stride * stride;
  return Status::Ok();
}

Status IfLayer::launch(cudaStream_t stream, int batch) {
  if (paired) return pair.launch(stream, batch, pair_out, pair_res, 1.0f, 1.0f, nullptr, pair_res_chunks);
  IfConvArgs a = args;
  a.batch = batch;
  a.items = batch * a.h_out * a.strips;
  const int grid = std::min(a.items, num_sms() * per_sm);
  k->launch(dim3(grid), smem, stream, maps, a);
  return cuda_status(cudaGetLastError(), "IFNet conv launch");
}

std::vector<float> dense_conv_weights(const float* w, int cout, int cin, int n_pad, const float* scale) {
  std::vector<float> d(static_cast<size_t>(n_pad) * cin * 9, 0.0f);
  for (int n = 0; n < cout; ++n) {
    const float s = scale != nullptr ? scale[n] : 1.0f;
    for (size_t i = 0; i < static_cast<size_t>(cin) * 9; ++i)
      d[static_cast<size_t>(n) * cin * 9 + i] = w[static_cast<size_t>(n) * cin * 9 + i] * s;
  }
  return d;
}

}  // namespace kb2
