// Engine implementations: SPAN x2 (FP16 / FP8), IFNet, the unshuffle SPAN of a .span8 package, and
// the factory.
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "engine.h"
#include "ifnet_net.h"
#include "rife_net.h"
#include "span8_net.h"
#include "span_net.h"
#include "span_tiles.h"
#include "static_scratch.h"

namespace kb2 {

Status Engine::check_device(cudaStream_t stream, int32_t* code) {
  KB2_CUDA(cudaStreamSynchronize(stream));
  int word = 0;
  KB2_CUDA(cudaMemcpy(&word, err_word(), sizeof(int), cudaMemcpyDeviceToHost));
  if (code != nullptr) *code = word;
  if (word != 0) {
    KB2_CUDA(cudaMemset(err_word(), 0, sizeof(int)));
    return refuse(KB2_KERNEL_TIMEOUT, "a device-side wait gave up (code " + std::to_string(word) + ")");
  }
  return Status::Ok();
}

namespace {

class SpanEngine final : public Engine {
 public:
  Status init(const kb2_engine_desc& d, const std::vector<float>& params) {
    params_ = params;
    precision_ = d.precision;
    if (d.act_scales != nullptr && d.act_scale_count > 0)
      scales_.assign(d.act_scales, d.act_scales + d.act_scale_count);
    return net_.create(params, d.precision, d.max_batch, d.height, d.width, d.act_scales, d.act_scale_count);
  }
  // kb2_set_row_tiles: every frame of the following enqueues runs as `tiles` row tiles, each read
  // with `halo` rows of context above and below (fewer at the frame's top and bottom, where the
  // window stays inside the frame), on a second network of the tile's height; the tiles' core rows
  // are stitched into the output. tiles = 1 (or 0): whole frames.
  Status set_row_tiles(int tiles, int halo) override {
    const int H = net_.height();
    if (tiles < 0 || halo < 0 || halo > 64 || tiles > H / 2)
      return refuse(KB2_SHAPE_INVALID, "row tiles: 1 <= tiles <= H / 2 and 0 <= halo <= 64");
    tile_net_.reset();
    tile_in_.reset();
    tiles_ = tiles <= 1 ? 0 : tiles;
    halo_ = halo;
    if (tiles_ == 0) return Status::Ok();
    core_ = (H + tiles_ - 1) / tiles_;
    tile_h_ = std::min(H, core_ + 2 * halo_);
    auto net = std::make_unique<SpanNet>();
    KB2_TRY(net->create(params_, precision_, net_.max_batch() * tiles_, tile_h_, net_.width(),
                        scales_.empty() ? nullptr : scales_.data(), static_cast<int>(scales_.size()),
                        net_.err_word()));
    KB2_TRY(net->set_output_format(net_.output_format()));
    net->set_profiling(profiling_);
    auto in = std::make_unique<DeviceBuffer>();
    KB2_TRY(in->alloc(static_cast<size_t>(net_.max_batch()) * tiles_ * 3 * tile_h_ * net_.width() * 2));
    tile_out_bytes_ = static_cast<size_t>(net_.max_batch()) * tiles_ * 4 * tile_h_ * net_.width() * 8;
    auto out = std::make_unique<DeviceBuffer>();
    KB2_TRY(out->alloc(tile_out_bytes_));  // room for F16 frames (6 B / px) or RGBA16 pixels (8 B / px)
    tile_net_ = std::move(net);
    tile_in_ = std::move(in);
    tile_out_ = std::move(out);
    return Status::Ok();
  }
  std::vector<std::string> input_names() const override { return {"input"}; }
  std::vector<std::string> output_names() const override { return {"output"}; }
  int max_batch() const override { return net_.max_batch(); }
  int height() const override { return net_.height(); }
  int width() const override { return net_.width(); }
  size_t device_bytes() const override { return net_.device_bytes(); }
  Status enqueue(cudaStream_t stream, const kb2_tensor* inputs, int n_inputs, const kb2_tensor* outputs,
                 int n_outputs) override {
    void* in = nullptr;
    void* out = nullptr;
    int batch = 0;
    KB2_TRY(frame_io(inputs, n_inputs, outputs, n_outputs, 1, 2, &in, &out, &batch,
                     net_.output_format() != 0 ? net_.display_bytes() : 0));
    if (moving_.has) {  // one enqueue only, as the reference's next_span_tiles
      MovingJob job = std::move(moving_);
      moving_ = MovingJob{};
      if (tiles_ == 0) return run_moving(stream, in, out, batch, outputs[0], job);
    }
    if (tiles_ > 0) return run_tiled(stream, in, out, batch);
    return net_.run(stream, in, out, batch);
  }
  Status tile_grid(kb2_tile_grid* g) const override {
    g->tile_w = kMoveTile;
    g->tile_h = kMoveTile;
    g->cols = (net_.width() + kMoveTile - 1) / kMoveTile;
    g->rows = (net_.height() + kMoveTile - 1) / kMoveTile;
    g->reach_cols = (kSpanReach + kMoveTile - 1) / kMoveTile;
    g->reach_rows = g->reach_cols;
    g->shift_step = 1;
    g->scale = 2;
    return Status::Ok();
  }
  // kb2_next_span_tiles: the next enqueue computes only what the core tiles need, and writes only them
  // (after copying `previous`, moved by (sx, sy) input pixels, into its output).
  Status next_tiles(const uint8_t* core, int count, int sx, int sy, const kb2_tensor* previous) override {
    moving_ = MovingJob{};
    kb2_tile_grid g{};
    KB2_TRY(tile_grid(&g));
    if (core == nullptr || count != g.cols * g.rows)
      return refuse(KB2_INPUT_MISMATCH, "moving tiles: core must hold cols x rows bytes");
    if (tiles_ != 0) return refuse(KB2_FORMAT_UNSUPPORTED, "moving tiles: not with row tiles");
    if ((sx != 0 || sy != 0) && previous == nullptr)
      return refuse(KB2_FORMAT_UNSUPPORTED, "moving tiles: a shift needs the previous output");
    if (std::abs(sx) >= net_.width() || std::abs(sy) >= net_.height())
      return refuse(KB2_SHAPE_INVALID, "moving tiles: shift beyond the frame");
    bool any = false;
    for (int i = 0; i < count; ++i) any = any || core[i] != 0;
    if (!any) return refuse(KB2_FORMAT_UNSUPPORTED, "moving tiles: empty core (the request is cancelled)");
    KB2_TRY(ensure_moving());
    moving_.core.assign(core, core + count);
    moving_.sx = sx;
    moving_.sy = sy;
    moving_.has_prev = previous != nullptr;
    if (previous != nullptr) moving_.prev = *previous;
    moving_.has = true;
    return Status::Ok();
  }
  Status set_output_format(int format) override {
    KB2_TRY(net_.set_output_format(format));
    if (tile_net_ != nullptr) KB2_TRY(tile_net_->set_output_format(format));
    return Status::Ok();
  }
  Status calibrate(cudaStream_t stream, const kb2_tensor& frames, float* peaks, int n_peaks) override {
    if (n_peaks != kSpanScales) return refuse(KB2_INPUT_MISMATCH, "SPAN calibration returns 19 peaks");
    if (frames.type != KB2_F16 || frames.dims[1] != 3 || frames.dims[2] != height() || frames.dims[3] != width() ||
        frames.dims[0] < 1)
      return refuse(KB2_INPUT_MISMATCH, "calibration frames: F16 [n,3,H,W] expected");
    const uint64_t addr = frames.handle + frames.offset;
    if (addr == 0 || (addr & 15u) != 0) return refuse(KB2_INPUT_MISMATCH, "calibration frames misaligned");
    return net_.calibrate(stream, reinterpret_cast<const void*>(addr), static_cast<int>(frames.dims[0]), peaks);
  }
  Status calibrate_static(cudaStream_t stream, const kb2_tensor& frames, float* peaks, int n_peaks) override {
    if (n_peaks != kSpanScales) return refuse(KB2_INPUT_MISMATCH, "SPAN calibration returns 19 peaks");
    if (frames.type != KB2_F16 || frames.dims[1] != 3 || frames.dims[2] != height() || frames.dims[3] != width() ||
        frames.dims[0] < 1)
      return refuse(KB2_INPUT_MISMATCH, "calibration frames: F16 [n,3,H,W] expected");
    const uint64_t addr = frames.handle + frames.offset;
    if (addr == 0 || (addr & 15u) != 0) return refuse(KB2_INPUT_MISMATCH, "calibration frames misaligned");
    // the scratch must be looked up on the engine's device, so that device has to be the current one
    cudaPointerAttributes attr{};
    KB2_CUDA(cudaPointerGetAttributes(&attr, err_word()));
    int cur = -1;
    KB2_CUDA(cudaGetDevice(&cur));
    if (cur != attr.device)
      return refuse(KB2_INPUT_MISMATCH, "static calibration: make the engine's device the current device");
    void* scratch = nullptr;
    KB2_TRY(static_scratch(&scratch));
    return net_.calibrate_in(stream, reinterpret_cast<const void*>(addr), static_cast<int>(frames.dims[0]), peaks,
                             static_cast<uint8_t*>(scratch), kStaticScratchBytes);
  }
  Status set_profiling(bool on) override {
    profiling_ = on;
    net_.set_profiling(on);
    if (tile_net_ != nullptr) tile_net_->set_profiling(on);
    return Status::Ok();
  }
  Status read_profile(kb2_layer_profile* records, int capacity, int* count) override {
    std::vector<SpanNet::Profile> kinds;
    KB2_TRY((tile_net_ != nullptr ? *tile_net_ : net_).read_profile(kinds));
    *count = static_cast<int>(kinds.size());
    for (int i = 0; i < *count && i < capacity; ++i) {
      kb2_layer_profile& r = records[i];
      std::memset(&r, 0, sizeof(r));
      std::strncpy(r.name, kinds[i].name.c_str(), sizeof(r.name) - 1);
      r.launches = kinds[i].launches;
      r.total_ms = kinds[i].ms;
      r.flops = kinds[i].flops;
      r.bytes = kinds[i].bytes;
    }
    return Status::Ok();
  }
  int launches_per_enqueue() const override {
    return tile_net_ != nullptr ? tile_net_->launches_per_run() : net_.launches_per_run();
  }

 protected:
  int* err_word() const override { return net_.err_word(); }  // the tile network reports into it too

 private:
  // Tile t of a frame: core rows [t * core, min(H, (t + 1) * core)), read from the window of tile_h
  // rows starting at core start - halo, moved inside the frame at its top and bottom.
  int tile_window(int t) const { return std::clamp(t * core_ - halo_, 0, net_.height() - tile_h_); }

  Status run_tiled(cudaStream_t stream, const void* in, void* out, int batch) {
    const int H = net_.height(), W = net_.width();
    const size_t plane = static_cast<size_t>(H) * W * 2;          // one input channel, bytes
    const size_t tile_plane = static_cast<size_t>(tile_h_) * W * 2;
    // cut: frame f, tile t -> tile frame f * tiles + t (3 channels of tile_h contiguous rows each)
    for (int f = 0; f < batch; ++f)
      for (int t = 0; t < tiles_; ++t) {
        const uint8_t* src = static_cast<const uint8_t*>(in) + f * 3 * plane + static_cast<size_t>(tile_window(t)) * W * 2;
        uint8_t* dst = tile_in_->as<uint8_t>() + (static_cast<size_t>(f) * tiles_ + t) * 3 * tile_plane;
        KB2_CUDA(cudaMemcpy2DAsync(dst, tile_plane, src, plane, tile_plane, 3, cudaMemcpyDeviceToDevice, stream));
      }
    KB2_TRY(tile_net_->run(stream, tile_in_->ptr, tile_out_->ptr, batch * tiles_));
    // stitch the core rows: F16 frames plane by plane, display pixels row by row
    const bool display = net_.output_format() != 0;
    const size_t row_bytes = display ? static_cast<size_t>(2 * W) * net_.display_bytes() : static_cast<size_t>(2 * W) * 2;
    const int planes = display ? 1 : 3;
    const size_t out_plane = row_bytes * 2 * H, tile_out_plane = row_bytes * 2 * tile_h_;
    for (int f = 0; f < batch; ++f)
      for (int t = 0; t < tiles_; ++t) {
        const int c0 = t * core_, c1 = std::min(H, c0 + core_);
        if (c1 <= c0) continue;
        const int ys = tile_window(t);
        const uint8_t* src = tile_out_->as<uint8_t>() + (static_cast<size_t>(f) * tiles_ + t) * planes * tile_out_plane +
                             static_cast<size_t>(2 * (c0 - ys)) * row_bytes;
        uint8_t* dst = static_cast<uint8_t*>(out) + static_cast<size_t>(f) * planes * out_plane +
                       static_cast<size_t>(2 * c0) * row_bytes;
        KB2_CUDA(cudaMemcpy2DAsync(dst, out_plane, src, tile_out_plane, static_cast<size_t>(2 * (c1 - c0)) * row_bytes,
                                   planes, cudaMemcpyDeviceToDevice, stream));
      }
    return Status::Ok();
  }

  // ---- moving tiles
  static constexpr int kMoveTile = 64;  // tile side, input pixels
  static constexpr int kSpanReach = 20;  // receptive radius of the network, input pixels
  struct MovingJob {
    bool has = false, has_prev = false;
    std::vector<uint8_t> core;
    int sx = 0, sy = 0;
    kb2_tensor prev{};
  };
  int move_rows() const { return std::min(net_.height(), kMoveTile + 2 * kSpanReach); }  // a window's rows
  int move_windows() const { return net_.max_batch() * std::max(1, (net_.height() - 1) / move_rows()); }

  // The window network, its buffers and the tile list's staging, made once (at the first request).
  Status ensure_moving() {
    if (win_net_ != nullptr) return Status::Ok();
    const int H = net_.height(), W = net_.width(), hw = move_rows();
    auto net = std::make_unique<SpanNet>();
    KB2_TRY(net->create(params_, precision_, move_windows(), hw, W, scales_.empty() ? nullptr : scales_.data(),
                        static_cast<int>(scales_.size()), net_.err_word()));
    auto win_in = std::make_unique<DeviceBuffer>();
    KB2_TRY(win_in->alloc(static_cast<size_t>(move_windows()) * 3 * hw * W * 2));
    auto win_out = std::make_unique<DeviceBuffer>();  // F16 frames (24 B / input px) or RGBA16 (32)
    KB2_TRY(win_out->alloc(static_cast<size_t>(move_windows()) * 32 * hw * W));
    auto full_out = std::make_unique<DeviceBuffer>();
    KB2_TRY(full_out->alloc(static_cast<size_t>(net_.max_batch()) * 32 * H * W));
    const int cols = (W + kMoveTile - 1) / kMoveTile, rows = (H + kMoveTile - 1) / kMoveTile;
    const size_t list = static_cast<size_t>(net_.max_batch()) * cols * rows;
    auto tiles = std::make_unique<DeviceBuffer>();
    KB2_TRY(tiles->alloc(list * sizeof(TileCopy)));
    TileCopy* host = nullptr;
    KB2_CUDA(cudaMallocHost(reinterpret_cast<void**>(&host), list * sizeof(TileCopy)));
    cudaEvent_t ev = nullptr;
    if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
      cudaFreeHost(host);
      return refuse(KB2_VENDOR_CALL_FAILED, "moving tiles: cudaEventCreate");
    }
    win_net_ = std::move(net);
    win_in_ = std::move(win_in);
    win_out_ = std::move(win_out);
    full_out_ = std::move(full_out);
    tile_list_ = std::move(tiles);
    tile_host_ = host;
    tile_sent_ = ev;
    return Status::Ok();
  }

  Status run_moving(cudaStream_t stream, const void* in, void* out, int batch, const kb2_tensor& out_t,
                    const MovingJob& job) {
    const int H = net_.height(), W = net_.width(), hw = move_rows();
    const bool display = net_.output_format() != 0;
    const int planes = display ? 1 : 3, pxb = display ? net_.display_bytes() : 2;
    const size_t row_bytes = static_cast<size_t>(2 * W) * pxb;
    const size_t frame_bytes = row_bytes * 2 * H * planes;
    KB2_TRY(win_net_->set_output_format(net_.output_format()));
    // the previous output into this one, moved by the pan
    if (job.has_prev) {
      const kb2_tensor& p = job.prev;
      for (int i = 0; i < 4; ++i)
        if (p.dims[i] != out_t.dims[i] || p.type != out_t.type)
          return refuse(KB2_INPUT_MISMATCH, "moving tiles: previous output of another shape");
      const void* prev = reinterpret_cast<const void*>(p.handle + p.offset);
      if (prev == out && (job.sx != 0 || job.sy != 0)) return net_.run(stream, in, out, batch);  // no shift in place
      if (prev != out) {
        if (job.sx == 0 && job.sy == 0)
          KB2_CUDA(cudaMemcpyAsync(out, prev, frame_bytes * batch, cudaMemcpyDeviceToDevice, stream));
        else
          KB2_TRY(shift_frames(stream, prev, out, batch, planes, 2 * H, static_cast<int>(row_bytes), pxb, 2 * job.sx,
                               2 * job.sy));
      }
    }
    const int cols = (W + kMoveTile - 1) / kMoveTile, rows = (H + kMoveTile - 1) / kMoveTile;
    std::vector<int> dirty;
    for (int r = 0; r < rows; ++r) {
      bool d = false;
      for (int c = 0; c < cols; ++c) d = d || job.core[static_cast<size_t>(r) * cols + c] != 0;
      if (d) dirty.push_back(r);
    }
    const int nd = static_cast<int>(dirty.size());
    // windows of the dirty tile rows, or the whole frames when that costs less
    const bool whole = static_cast<long long>(nd) * hw >= H || nd * batch > move_windows();
    const void* win = nullptr;
    int win_rows = 0;
    std::vector<int> ys(static_cast<size_t>(nd));
    if (whole) {
      KB2_TRY(net_.run(stream, in, full_out_->ptr, batch));
      win = full_out_->ptr;
      win_rows = 2 * H;
    } else {
      const size_t plane = static_cast<size_t>(H) * W * 2, wplane = static_cast<size_t>(hw) * W * 2;
      for (int k = 0; k < nd; ++k) ys[k] = std::clamp(dirty[k] * kMoveTile - kSpanReach, 0, H - hw);
      for (int f = 0; f < batch; ++f)
        for (int k = 0; k < nd; ++k) {
          const uint8_t* src = static_cast<const uint8_t*>(in) + f * 3 * plane + static_cast<size_t>(ys[k]) * W * 2;
          uint8_t* dst = win_in_->as<uint8_t>() + (static_cast<size_t>(f) * nd + k) * 3 * wplane;
          KB2_CUDA(cudaMemcpy2DAsync(dst, wplane, src, plane, wplane, 3, cudaMemcpyDeviceToDevice, stream));
        }
      KB2_TRY(win_net_->run(stream, win_in_->ptr, win_out_->ptr, batch * nd));
      win = win_out_->ptr;
      win_rows = 2 * hw;
    }
    // the core tiles, from their windows into the output
    KB2_CUDA(cudaEventSynchronize(tile_sent_));  // the staging's previous list has been copied
    const int unit = display ? 1 : 2;               // output pixels a unit of the copy's columns
    int n = 0;
    for (int f = 0; f < batch; ++f)
      for (int k = 0; k < nd; ++k) {
        const int r = dirty[k];
        const int y0 = r * kMoveTile, y1 = std::min(H, y0 + kMoveTile);
        for (int c = 0; c < cols; ++c) {
          if (job.core[static_cast<size_t>(r) * cols + c] == 0) continue;
          const int x0 = c * kMoveTile, x1 = std::min(W, x0 + kMoveTile);
          TileCopy& t = tile_host_[n++];
          t.frame = f;
          t.window = whole ? f : f * nd + k;
          t.out_y = 2 * y0;
          t.win_y = whole ? 2 * y0 : 2 * (y0 - ys[k]);
          t.x = 2 * x0 / unit;
          t.cols = 2 * (x1 - x0) / unit;
          t.rows = 2 * (y1 - y0);
        }
      }
    KB2_CUDA(cudaMemcpyAsync(tile_list_->ptr, tile_host_, n * sizeof(TileCopy), cudaMemcpyHostToDevice, stream));
    KB2_CUDA(cudaEventRecord(tile_sent_, stream));
    return copy_tiles(stream, tile_list_->as<TileCopy>(), n, planes, win, out, static_cast<int>(row_bytes), 2 * H,
                      win_rows, pxb);
  }

  MovingJob moving_;
  std::unique_ptr<SpanNet> win_net_;
  std::unique_ptr<DeviceBuffer> win_in_, win_out_, full_out_, tile_list_;
  TileCopy* tile_host_ = nullptr;
  cudaEvent_t tile_sent_ = nullptr;

 public:
  ~SpanEngine() override {
    if (tile_sent_ != nullptr) cudaEventDestroy(tile_sent_);
    if (tile_host_ != nullptr) cudaFreeHost(tile_host_);
  }

 private:
  SpanNet net_;
  std::vector<float> params_, scales_;
  int precision_ = KB2_PREC_FP16;
  bool profiling_ = false;
  int tiles_ = 0, halo_ = 0, core_ = 0, tile_h_ = 0;
  size_t tile_out_bytes_ = 0;
  std::unique_ptr<SpanNet> tile_net_;
  std::unique_ptr<DeviceBuffer> tile_in_, tile_out_;
};

// The interpolators: classic IFNet (IfnetNet) and RIFE 4.2x (RifeNet), the same enqueue contract.
template <class Net>
class InterpEngine final : public Engine {
 public:
  Status init(const kb2_engine_desc& d, const std::vector<float>& params) {
    if (d.precision != KB2_PREC_FP16) return refuse(KB2_FORMAT_UNSUPPORTED, "the interpolators run in FP16 only");
    return net_.create(params, d.max_batch, d.height, d.width);
  }
  std::vector<std::string> input_names() const override { return {"img0", "img1"}; }
  std::vector<std::string> output_names() const override { return {"output"}; }  // motion: {"flow", "mask"}
  int max_batch() const override { return net_.max_batch(); }
  int height() const override { return net_.height(); }
  int width() const override { return net_.width(); }
  size_t device_bytes() const override { return net_.device_bytes(); }
  Status enqueue(cudaStream_t stream, const kb2_tensor* inputs, int n_inputs, const kb2_tensor* outputs,
                 int n_outputs) override {
    void* in[2] = {nullptr, nullptr};
    int batch = 0;
    if (n_outputs == 2) {  // the motion variant: flow and mask (upscale_motion.cpp:71-84)
      void *flow = nullptr, *mask = nullptr;
      bool f16 = false;
      KB2_TRY(motion_io(inputs, n_inputs, outputs, n_outputs, net_.plane_height(), net_.plane_width(), in, &flow,
                        &mask, &f16, &batch));
      if (inputs[1].dims[0] != inputs[0].dims[0]) return refuse(KB2_INPUT_MISMATCH, "IFNet: frame counts differ");
      return net_.run_motion(stream, in[0], in[1], flow, mask, f16, batch);
    }
    void* out = nullptr;
    KB2_TRY(frame_io(inputs, n_inputs, outputs, n_outputs, 2, 1, in, &out, &batch));
    if (inputs[1].dims[0] != inputs[0].dims[0]) return refuse(KB2_INPUT_MISMATCH, "IFNet: frame counts differ");
    return net_.run(stream, in[0], in[1], out, batch);
  }
  Status geometry(int32_t* ph, int32_t* pw, int32_t* x, int32_t* y) const override {
    *ph = net_.plane_height();
    *pw = net_.plane_width();
    *x = net_.window_x();
    *y = net_.window_y();
    return Status::Ok();
  }
  Status set_timestep(float t) override { return net_.set_timestep(t); }
  Status set_profiling(bool on) override {
    net_.timer().enable(on);
    return Status::Ok();
  }
  Status read_profile(kb2_layer_profile* records, int capacity, int* count) override {
    std::vector<LayerTimer::Record> kinds;
    KB2_TRY(net_.timer().read(kinds));
    *count = static_cast<int>(kinds.size());
    for (int i = 0; i < *count && i < capacity; ++i) {
      kb2_layer_profile& r = records[i];
      std::memset(&r, 0, sizeof(r));
      std::strncpy(r.name, kinds[i].name.c_str(), sizeof(r.name) - 1);
      r.launches = kinds[i].launches;
      r.total_ms = kinds[i].ms;
      r.flops = kinds[i].flops;
      r.bytes = kinds[i].bytes;
    }
    return Status::Ok();
  }
  int launches_per_enqueue() const override { return net_.launches_per_run(); }

 protected:
  int* err_word() const override { return net_.err_word(); }

 private:
  Net net_;
};

// The unshuffle SPAN of a .span8 package (KB2_MODEL_SPAN_UNSHUFFLE): FP16, or E4M3 blocks for an FP8
// package.
class Span8Engine final : public Engine {
 public:
  Status init(const kb2_engine_desc& d, const Span8Package& pkg) {
    const bool fp8 = d.precision == KB2_PREC_FP8_E4M3;
    if (!fp8 && d.precision != KB2_PREC_FP16) return refuse(KB2_FORMAT_UNSUPPORTED, "unknown precision");
    // an FP16-native package carries unit scales that mean nothing for E4M3 (package.h:61-66)
    if (fp8 && (pkg.flags & 2u) != 0u)
      return refuse(KB2_FORMAT_UNSUPPORTED, "unshuffle SPAN: an FP16 package has no E4M3 activation scales");
    return net_.create(pkg, fp8, d.max_batch, d.height, d.width);
  }
  std::vector<std::string> input_names() const override { return {"input"}; }
  std::vector<std::string> output_names() const override { return {"output"}; }
  int max_batch() const override { return net_.max_batch(); }
  int height() const override { return net_.height(); }
  int width() const override { return net_.width(); }
  size_t device_bytes() const override { return net_.device_bytes(); }
  Status enqueue(cudaStream_t stream, const kb2_tensor* inputs, int n_inputs, const kb2_tensor* outputs,
                 int n_outputs) override {
    void* in = nullptr;
    void* out = nullptr;
    int batch = 0;
    KB2_TRY(frame_io(inputs, n_inputs, outputs, n_outputs, 1, 2, &in, &out, &batch));
    return net_.run(stream, in, out, batch);
  }
  Status calibrate(cudaStream_t stream, const kb2_tensor& frames, float* peaks, int n_peaks) override {
    if (n_peaks != net_.scale_count())
      return refuse(KB2_INPUT_MISMATCH, "unshuffle SPAN calibration returns 1 + 3 * blocks peaks");
    if (frames.type != KB2_F16 || frames.dims[1] != 3 || frames.dims[2] != height() || frames.dims[3] != width() ||
        frames.dims[0] < 1)
      return refuse(KB2_INPUT_MISMATCH, "calibration frames: F16 [n,3,H,W] expected");
    const uint64_t addr = frames.handle + frames.offset;
    if (addr == 0 || (addr & 15u) != 0) return refuse(KB2_INPUT_MISMATCH, "calibration frames misaligned");
    return net_.calibrate(stream, reinterpret_cast<const void*>(addr), static_cast<int>(frames.dims[0]), peaks);
  }
  Status set_profiling(bool on) override {
    net_.timer().enable(on);
    return Status::Ok();
  }
  Status read_profile(kb2_layer_profile* records, int capacity, int* count) override {
    std::vector<LayerTimer::Record> kinds;
    KB2_TRY(net_.timer().read(kinds));
    *count = static_cast<int>(kinds.size());
    for (int i = 0; i < *count && i < capacity; ++i) {
      kb2_layer_profile& r = records[i];
      std::memset(&r, 0, sizeof(r));
      std::strncpy(r.name, kinds[i].name.c_str(), sizeof(r.name) - 1);
      r.launches = kinds[i].launches;
      r.total_ms = kinds[i].ms;
      r.flops = kinds[i].flops;
      r.bytes = kinds[i].bytes;
    }
    return Status::Ok();
  }
  int launches_per_enqueue() const override { return net_.launches_per_run(); }

 protected:
  int* err_word() const override { return net_.err_word(); }

 private:
  Span8Net net_;
};

}  // namespace

Status make_engine(const kb2_engine_desc& d, std::unique_ptr<Engine>& out) {
  // Everything that needs no device is checked first: the blob and the shapes.
  if (d.model != KB2_MODEL_SPAN_X2 && d.model != KB2_MODEL_IFNET && d.model != KB2_MODEL_SPAN_UNSHUFFLE &&
      d.model != KB2_MODEL_RIFE_FUSED)
    return refuse(KB2_FORMAT_UNSUPPORTED, "unknown model");
  std::vector<float> params;
  Span8Package pkg;
  if (d.model == KB2_MODEL_SPAN_UNSHUFFLE)
    KB2_TRY(parse_span8(d.weights, d.weights_bytes, pkg));
  else
    KB2_TRY(parse_blob(d.weights, d.weights_bytes, d.model, params));
  if (d.model == KB2_MODEL_RIFE_FUSED) {
    RifePlan plan;
    KB2_TRY(rife_read_plan(params, plan));
  }
  if (d.max_batch < 1 || d.height < 1 || d.width < 1 || d.height > 8192 || d.width > 8192)
    return refuse(KB2_SHAPE_INVALID, "frame size or batch out of contract");
  int count = 0;
  KB2_CUDA(cudaGetDeviceCount(&count));
  if (d.device < 0 || d.device >= count) return refuse(KB2_INPUT_MISMATCH, "no such CUDA device");
  KB2_CUDA(cudaSetDevice(d.device));
  int major = 0, minor = 0;
  KB2_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d.device));
  KB2_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, d.device));
  if (major != 10 || minor != 0)
    return refuse(KB2_FORMAT_UNSUPPORTED, "this library runs on sm_100 (B200) only");
  if (d.model == KB2_MODEL_SPAN_X2) {
    auto e = std::make_unique<SpanEngine>();
    KB2_TRY(e->init(d, params));
    out = std::move(e);
    return Status::Ok();
  }
  if (d.model == KB2_MODEL_SPAN_UNSHUFFLE) {
    auto e = std::make_unique<Span8Engine>();
    KB2_TRY(e->init(d, pkg));
    out = std::move(e);
    return Status::Ok();
  }
  if (d.model == KB2_MODEL_IFNET) {
    auto e = std::make_unique<InterpEngine<IfnetNet>>();
    KB2_TRY(e->init(d, params));
    out = std::move(e);
    return Status::Ok();
  }
  if (d.model == KB2_MODEL_RIFE_FUSED) {
    auto e = std::make_unique<InterpEngine<RifeNet>>();
    KB2_TRY(e->init(d, params));
    out = std::move(e);
    return Status::Ok();
  }
  return refuse(KB2_FORMAT_UNSUPPORTED, "unknown model");
}

}  // namespace kb2
