// TEST INFRASTRUCTURE ONLY (oracle): the reference's display-ring pixel packing
// (Ta2b/Ultimate-Anime-VideoPlayer src/kernels/spec/ring_pack.h, color.h unorm16), evaluated on the
// CPU over a frame, compiled in place by oracle/Makefile with -ffp-contract=off (the reference
// compiles its kernels and tests that way). Used to make golden vectors; nothing in the product
// path loads it.
#include <cstdint>
#include <cstring>

#include "kernels/spec/ring_pack.h"

extern "C" {

// rgb: 3 FP32 planes of h x w. format 1: RGBA16 (4 x u16 a pixel, alpha 65535); 2: RGB10A2 (u32);
// 3: RGB10A2 with the TPDF dither of pixel (x, y). out: h x w pixels, rows packed.
int kref_pack_display(const float* rgb, int h, int w, int format, void* out) {
  namespace k = kirari::kernels;
  const size_t plane = static_cast<size_t>(h) * w;
  for (int y = 0; y < h; ++y)
    for (int x = 0; x < w; ++x) {
      const size_t i = static_cast<size_t>(y) * w + x;
      const float r = rgb[i], g = rgb[plane + i], b = rgb[2 * plane + i];
      if (format == 1) {
        const uint16_t p[4] = {k::unorm16(r), k::unorm16(g), k::unorm16(b), 65535};
        std::memcpy(static_cast<uint8_t*>(out) + i * 8, p, 8);
      } else if (format == 2 || format == 3) {
        uint32_t pr, pg, pb;
        if (format == 2) {
          pr = k::unorm10(r);
          pg = k::unorm10(g);
          pb = k::unorm10(b);
        } else {
          const float noise = k::ring_tpdf(static_cast<uint32_t>(x), static_cast<uint32_t>(y));
          pr = k::unorm10_dithered(r, noise);
          pg = k::unorm10_dithered(g, noise);
          pb = k::unorm10_dithered(b, noise);
        }
        const uint32_t p = k::pack_rgb10a2(pr, pg, pb);
        std::memcpy(static_cast<uint8_t*>(out) + i * 4, &p, 4);
      } else {
        return 1;
      }
    }
  return 0;
}

}  // extern "C"
