// TEST INFRASTRUCTURE ONLY (oracle): C entry points over the reference's own CPU warp_blend_at and
// flow_max (Ta2b/Ultimate-Anime-VideoPlayer src/kernels/ref/warp.cpp:261, :290), compiled in place by
// oracle/Makefile. The tests use them to make golden vectors and to pin oracle/nets.py's
// restatement; nothing in the product path loads them.
#include <cstring>
#include <string>

#include "kernels/ref/warp.h"

namespace {
std::string g_error;

kirari::kernels::ref::Motion motion_of(const float* flow, const float* mask, int ph, int pw, int wx, int wy, int ww,
                                        int wh, int filter = 0, int pan_lock = 0, int at_instant = 0) {
  kirari::kernels::ref::Motion m;
  for (int c = 0; c < 4; ++c) {
    m.flow[c] = kirari::kernels::PlaneF(pw, ph);
    std::memcpy(m.flow[c].data.data(), flow + static_cast<size_t>(c) * ph * pw, sizeof(float) * ph * pw);
  }
  m.mask = kirari::kernels::PlaneF(pw, ph);
  std::memcpy(m.mask.data.data(), mask, sizeof(float) * ph * pw);
  m.area = kirari::kernels::Window{.x = wx, .y = wy, .width = ww, .height = wh};
  m.warp = filter == 1 ? kirari::kernels::RifeWarp::CatmullRom : kirari::kernels::RifeWarp::Bilinear;
  m.pan_lock = pan_lock != 0;
  m.at_instant = at_instant != 0;
  return m;
}
}  // namespace

extern "C" {

const char* kref_warp_last_error() { return g_error.c_str(); }

// a, b, out: 3 FP32 planes of h x w; flow: 4 planes and mask: 1 plane of ph x pw; window (wx, wy,
// ww, wh) of the frame in the planes.
int kref_warp_blend_at(const float* a, const float* b, int h, int w, const float* flow, const float* mask, int ph,
                       int pw, int wx, int wy, int ww, int wh, float t, int filter, int pan_lock, int at_instant,
                       float* out) {
  using kirari::kernels::RgbImage;
  RgbImage ia(w, h), ib(w, h);
  for (int c = 0; c < 3; ++c) {
    std::memcpy(ia.planes[c].data.data(), a + static_cast<size_t>(c) * h * w, sizeof(float) * h * w);
    std::memcpy(ib.planes[c].data.data(), b + static_cast<size_t>(c) * h * w, sizeof(float) * h * w);
  }
  auto r = kirari::kernels::ref::warp_blend_at(
      ia, ib, motion_of(flow, mask, ph, pw, wx, wy, ww, wh, filter, pan_lock, at_instant), t);
  if (!r) {
    g_error = r.error().detail;
    return 1;
  }
  for (int c = 0; c < 3; ++c)
    std::memcpy(out + static_cast<size_t>(c) * h * w, r->planes[c].data.data(), sizeof(float) * h * w);
  return 0;
}

// warp_blend_poses (warp.cpp:270): prev_flow / prev_mask the previous pair's motion (same planes and
// window), or null for a held previous pair.
int kref_warp_blend_poses(const float* a, const float* b, int h, int w, const float* flow, const float* mask,
                          const float* prev_flow, const float* prev_mask, int ph, int pw, int wx, int wy, int ww,
                          int wh, float t, int filter, float* out) {
  using kirari::kernels::RgbImage;
  RgbImage ia(w, h), ib(w, h);
  for (int c = 0; c < 3; ++c) {
    std::memcpy(ia.planes[c].data.data(), a + static_cast<size_t>(c) * h * w, sizeof(float) * h * w);
    std::memcpy(ib.planes[c].data.data(), b + static_cast<size_t>(c) * h * w, sizeof(float) * h * w);
  }
  const auto m = motion_of(flow, mask, ph, pw, wx, wy, ww, wh, filter);
  kirari::kernels::ref::Motion prev;
  const bool has_prev = prev_flow != nullptr && prev_mask != nullptr;
  if (has_prev) prev = motion_of(prev_flow, prev_mask, ph, pw, wx, wy, ww, wh);
  auto r = kirari::kernels::ref::warp_blend_poses(ia, ib, m, has_prev ? &prev : nullptr, t);
  if (!r) {
    g_error = r.error().detail;
    return 1;
  }
  for (int c = 0; c < 3; ++c)
    std::memcpy(out + static_cast<size_t>(c) * h * w, r->planes[c].data.data(), sizeof(float) * h * w);
  return 0;
}

// The reference's pan estimate of two frames (warp_pan.cpp): dx, dy, sure.
int kref_pan_estimate(const float* a, const float* b, int h, int w, float* out3) {
  using kirari::kernels::RgbImage;
  RgbImage ia(w, h), ib(w, h);
  for (int c = 0; c < 3; ++c) {
    std::memcpy(ia.planes[c].data.data(), a + static_cast<size_t>(c) * h * w, sizeof(float) * h * w);
    std::memcpy(ib.planes[c].data.data(), b + static_cast<size_t>(c) * h * w, sizeof(float) * h * w);
  }
  const auto e = kirari::kernels::ref::pan_estimate(ia, ib);
  out3[0] = e.dx;
  out3[1] = e.dy;
  out3[2] = e.sure ? 1.0f : 0.0f;
  return 0;
}

int kref_flow_max(const float* flow, const float* mask, int ph, int pw, int wx, int wy, int ww, int wh, float* out) {
  auto r = kirari::kernels::ref::flow_max(motion_of(flow, mask, ph, pw, wx, wy, ww, wh));
  if (!r) {
    g_error = r.error().detail;
    return 1;
  }
  *out = *r;
  return 0;
}

}  // extern "C"
