// Host side of the fused E4M3 SPAN block (spab8.cuh): built from the block's three E4M3 stacked
// conv layers, whose packed weights, scales and K-step table it reuses as they are.
#include <algorithm>

#include "spab8.cuh"
#include "spab_layer.h"

namespace kb2 {

namespace {
template <bool kLast>
void spab_launch(dim3 grid, size_t smem, cudaStream_t s, const CUtensorMap& m, const SpabArgs& a) {
  spab8_kernel<kLast><<<grid, kSpabThreads, smem, s>>>(m, a);
}
}  // namespace

Status SpabLayer::build(const ConvLayer& c1, const ConvLayer& c2, const ConvLayer& c3, const ChunkedTensor& x_in,
                        float inv1, float inv2, float inv3, float res_scale, bool last, int* err) {
  const ConvLayer* cs[3] = {&c1, &c2, &c3};
  for (const ConvLayer* c : cs) {
    if (!c->spec.fp8 || c->spec.taps != 9 || c->spec.n_pad != 48 || c->spec.n_sources != 1)
      return refuse(KB2_FORMAT_UNSUPPORTED, "fused SPAB: E4M3 3x3 48-channel layers only");
    if (c->kind != 1)  // the fused kernel reads the single-SM stacked packing of B
      return refuse(KB2_FORMAT_UNSUPPORTED, "fused SPAB: layers packed for the pair kernel");
    if (c->args.n_ksteps != c1.args.n_ksteps || c->args.wbytes != c1.args.wbytes)
      return refuse(KB2_FORMAT_UNSUPPORTED, "fused SPAB: layers of different shapes");
    for (int j = 0; j < c1.args.n_ksteps; ++j)
      if (c->args.ks[j].a_off != c1.args.ks[j].a_off || c->args.ks[j].lbo != c1.args.ks[j].lbo)
        return refuse(KB2_FORMAT_UNSUPPORTED, "fused SPAB: layers with different K steps");
  }
  if (c1.args.n_ksteps > kRowMaxK) return refuse(KB2_FORMAT_UNSUPPORTED, "fused SPAB: too many K steps");
  if (x_in.chunks != 3 || !x_in.fp8) return refuse(KB2_FORMAT_UNSUPPORTED, "fused SPAB: E4M3 48-channel input");
  last_ = last;
  SpabArgs& a = args;
  a = SpabArgs{};
  a.batch = x_in.batch;
  a.H = x_in.H;
  a.W = x_in.W;
  a.strips = (x_in.W + kSpabStrip - 1) / kSpabStrip;
  a.n_k = c1.args.n_ksteps;
  for (int j = 0; j < a.n_k; ++j)
    a.ks[j] = static_cast<uint64_t>(c1.args.ks[j].a_off >> 4) | (static_cast<uint64_t>(c1.args.ks[j].lbo >> 4) << 16);
  for (int i = 0; i < 3; ++i) a.idesc_n[i] = c1.args.idesc_n[i];
  for (int i = 0; i < 3; ++i) {
    a.wpack[i] = cs[i]->wpack.as<uint8_t>();
    a.bias[i] = cs[i]->bias.as<float>();
    a.scale[i] = cs[i]->scale.as<float>();
    if (a.scale[i] == nullptr) return refuse(KB2_FORMAT_UNSUPPORTED, "fused SPAB: missing channel scales");
  }
  a.wbytes = c1.args.wbytes;
  a.wstride = (a.wbytes + 1023u) & ~1023u;
  a.inv1 = inv1;
  a.inv2 = inv2;
  a.inv3 = inv3;
  a.res_scale = res_scale;
  a.x_in = x_in.ptr;
  a.err = err;
  map_ = c1.maps.m[0];  // the block input, one 128-pixel row box of all 3 chunks

  smem = 3 * static_cast<size_t>(a.wstride) + (kSpabInRing + 2 * kSpabTRing) * kSpabRowBytes + kSpabSmemExtra;
  int dev = 0, optin = 0;
  KB2_CUDA(cudaGetDevice(&dev));
  KB2_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  if (smem > static_cast<size_t>(optin)) return refuse(KB2_FORMAT_UNSUPPORTED, "fused SPAB: shared memory");
  const void* fn = last ? reinterpret_cast<const void*>(&spab8_kernel<true>)
                        : reinterpret_cast<const void*>(&spab8_kernel<false>);
  KB2_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  // bands: about 6 work items per SM, as tall as possible (each band re-reads 6 halo rows and
  // drains the three-conv pipeline once)
  const long long rows_total = static_cast<long long>(a.batch) * a.H * a.strips;
  int band = static_cast<int>(rows_total / (6LL * num_sms()));
  band = std::max(16, std::min(band, a.H));
  a.band_rows = band;
  a.bands = (a.H + band - 1) / band;
  a.items = a.batch * a.bands * a.strips;
  return Status::Ok();
}

Status SpabLayer::launch(cudaStream_t stream, int batch, void* out, void* t1_f16) const {
  SpabArgs a = args;
  a.batch = batch;
  a.items = batch * a.bands * a.strips;
  a.out = static_cast<uint8_t*>(out);
  a.t1_f16 = static_cast<uint8_t*>(t1_f16);
  if (last_ && t1_f16 == nullptr) return refuse(KB2_INVALID_ARGUMENT, "fused SPAB: last block needs the T1 copy");
  const int grid = std::min(a.items, num_sms());
  if (last_) spab_launch<true>(dim3(grid), smem, stream, map_, a);
  else spab_launch<false>(dim3(grid), smem, stream, map_, a);
  return cuda_status(cudaGetLastError(), "spab8_kernel launch");
}

}  // namespace kb2
