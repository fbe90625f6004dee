// Moving tiles of SPAN x2: the copies around the recomputation of the changed tiles (span_tiles.cu).
#pragma once

#include "host_util.h"

namespace kb2 {

// One core tile to write: rows [out_y, out_y + rows) of frame `frame`'s output from rows
// [win_y, win_y + rows) of window `window`'s output, columns [x, x + cols) in units of the output's
// words per pixel (pixel pairs for F16 planes, pixels for display pixels).
struct TileCopy {
  int frame, window, out_y, win_y, x, rows, cols;
};

// out = prev moved by (sx, sy) output pixels, `frames` x `planes` planes of `rows` rows of row_bytes
// (pixels of px_bytes: 2 for F16 planes, 4 or 8 for display pixels); pixels whose source falls
// outside the frame are not written. prev and out must not overlap.
Status shift_frames(cudaStream_t stream, const void* prev, void* out, int frames, int planes, int rows, int row_bytes,
                    int px_bytes, int sx, int sy);

// Writes the listed tiles (device array) from the windows' outputs `win` (planes of win_rows rows)
// into the frames' outputs `out` (planes of out_rows rows), both rows of row_bytes.
Status copy_tiles(cudaStream_t stream, const TileCopy* tiles, int n_tiles, int planes, const void* win, void* out,
                  int row_bytes, int out_rows, int win_rows, int px_bytes);

}  // namespace kb2
