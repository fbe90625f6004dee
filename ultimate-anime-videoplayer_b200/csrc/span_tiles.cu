// Moving tiles of SPAN x2 (the reference's contract src/kernels/spec/span_tiles.h; its engine side
// src/gpu/cuda/backend/span_fp8_tiles.cpp): the two copies around the recomputation of the changed
// tiles. Both move 4-byte words of the output's layout, which is either F16 NCHW frames (3 planes of
// halves) or display pixels (one plane of 4- or 8-byte pixels); rows are 2W pixels, so every tile
// row is a whole number of words.
#include <cuda_runtime.h>

#include <algorithm>

#include "span_tiles.h"

namespace kb2 {

namespace {

// out = prev moved by (sx, sy) output pixels: out[y][x] = prev[y - sy][x - sx] wherever that source
// is inside the frame; pixels whose source is outside are left as they are (their tiles are core).
// A grid of rows; x over 4-byte words of a row.
__global__ void shift_frames_kernel(const uint32_t* __restrict__ prev, uint32_t* __restrict__ out, int planes,
                                    int rows, int words, int px_words, int sx, int sy, int n_rows_total) {
  const int w = blockIdx.x * blockDim.x + threadIdx.x;
  if (w >= words) return;
  const int x = w / px_words;  // output pixel of this word
  const int sxw = w - sx * px_words;
  if (x - sx < 0 || x - sx >= words / px_words) return;
  for (int r = blockIdx.y; r < n_rows_total; r += gridDim.y) {
    const int y = r % rows;
    const int ys = y - sy;
    if (ys < 0 || ys >= rows) continue;
    const size_t plane_row = static_cast<size_t>(r - y);  // first row of this plane
    out[static_cast<size_t>(r) * words + w] = prev[(plane_row + ys) * words + sxw];
  }
  (void)planes;
}

// One block per (listed tile, plane): copies the tile's rows from its window's output to the frame.
__global__ void copy_tiles_kernel(const TileCopy* __restrict__ tiles, int planes, const uint32_t* __restrict__ win,
                                  uint32_t* __restrict__ out, int words, int out_rows, int win_rows, int px_words) {
  const TileCopy t = tiles[blockIdx.x];
  const int p = blockIdx.y;
  const int row_words = t.cols * px_words;
  const size_t out_plane = (static_cast<size_t>(t.frame) * planes + p) * out_rows;
  const size_t win_plane = (static_cast<size_t>(t.window) * planes + p) * win_rows;
  for (int i = threadIdx.x; i < t.rows * row_words; i += blockDim.x) {
    const int r = i / row_words, c = i - r * row_words;
    out[(out_plane + t.out_y + r) * words + t.x * px_words + c] = win[(win_plane + t.win_y + r) * words + t.x * px_words + c];
  }
}

}  // namespace

Status shift_frames(cudaStream_t stream, const void* prev, void* out, int frames, int planes, int rows, int row_bytes,
                    int px_bytes, int sx, int sy) {
  if (row_bytes % 4 != 0 || px_bytes % 2 != 0) return refuse(KB2_FORMAT_UNSUPPORTED, "shift: rows of whole words");
  const int words = row_bytes / 4;
  // 2-byte pixels (F16 planes) move by pairs: the shift is a whole number of words when sx is even
  int px_words = px_bytes / 4;
  int sxs = sx;
  if (px_bytes == 2) {
    if (sx % 2 != 0) return refuse(KB2_FORMAT_UNSUPPORTED, "shift: F16 rows move by even pixels");
    px_words = 1;
    sxs = sx / 2;
  }
  const int total = frames * planes * rows;
  const dim3 g(static_cast<unsigned>((words + 255) / 256), static_cast<unsigned>(std::min(total, 65535)));
  shift_frames_kernel<<<g, 256, 0, stream>>>(static_cast<const uint32_t*>(prev), static_cast<uint32_t*>(out), planes,
                                             rows, words, px_words, sxs, sy, total);
  return cuda_status(cudaGetLastError(), "shift_frames launch");
}

Status copy_tiles(cudaStream_t stream, const TileCopy* tiles, int n_tiles, int planes, const void* win, void* out,
                  int row_bytes, int out_rows, int win_rows, int px_bytes) {
  if (n_tiles <= 0) return Status::Ok();
  if (row_bytes % 4 != 0) return refuse(KB2_FORMAT_UNSUPPORTED, "copy_tiles: rows of whole words");
  // tile columns are counted in pixels for 4- and 8-byte pixels, in pixel pairs for F16 planes
  const int px_words = px_bytes == 2 ? 1 : px_bytes / 4;
  copy_tiles_kernel<<<dim3(static_cast<unsigned>(n_tiles), static_cast<unsigned>(planes)), 256, 0, stream>>>(
      tiles, planes, static_cast<const uint32_t*>(win), static_cast<uint32_t*>(out), row_bytes / 4, out_rows, win_rows,
      px_words);
  return cuda_status(cudaGetLastError(), "copy_tiles launch");
}

}  // namespace kb2
