// Stacked-kernel-row 3x3 convolution: the shared constants of the pair kernel (conv3p.cuh) and its
// host side (conv_layer.cu).
//
// A tcgen05.mma of M = 128 costs at least ~45 cycles whatever N is below ~96 (measured on B200; at
// N >= 128 it runs at the tensor rate, N / 2 cycles for K = 16). SPAN's convolutions have 48 output
// channels, so a plain implicit GEMM (conv_tc.cuh) spends half of each instruction idle. A stacked
// conv multiplies every input row once by the three kernel rows at the same time:
//
//     B = [ W(dy = +1) | W(dy = 0) | W(dy = -1) ]      (N = 3 x 48 = 144 rows of weights)
//
// and the three 48-column results land in the accumulators of the three output rows that input row
// feeds (o = t - 2, t - 1, t for input row index t of a band). An output row is complete after its
// third input row; the epilogue then reads it.
//
// Accumulators: output rows cycle through 6 slots; slot s owns the 48-column TMEM block s, and
// slots 0 and 1 also own blocks 6 and 7. The window of input row t starts at the block of
// slot(t - 2), so it never wraps: its third block lands in block 6 or 7 when the ring would wrap,
// and the epilogue adds the two blocks of a slot (8 blocks = 384 columns; 512 at 64 channels).
// When an output row is first touched its block(s) are cleared by an MMA with an all-zero B tile
// and enable-input-d off, so the row's MMAs all accumulate.
#pragma once

#include "conv_tc.cuh"

namespace kb2 {

constexpr int kStackBlocksPerSm = 1;     // one block per SM owning all 512 TMEM columns
constexpr uint32_t kStackTmemCols = 512;
constexpr uint32_t kStackSlots = 6;   // output-row slots (TMEM reuse period, in output rows)
constexpr uint32_t kStackBlocks = 8;  // TMEM blocks: one per slot, plus 6 and 7 for slots 0, 1

// shared memory after the input ring: barriers (128 x 8 B), K-step table, per-channel constants, TMEM
// address, then (at kStackZeroOff) the all-zero B tile of the clearing MMA (48 rows x 32 B)
constexpr uint32_t kStackZeroOff = 2176;
constexpr uint32_t kStackZeroBytes = 48 * 32;
constexpr uint32_t kStackSmemExtra = 1024 + kStackZeroOff + kStackZeroBytes + 64;
static_assert(128 * 8 + (kMaxKSteps + 2) * 8 + 3 * kMaxN * 4 + 4 <= kStackZeroOff, "shared layout");
// kEpiColsBias layers only, after the zero tile: the edge-pixel exchange of the epilogue warps,
// [3 groups][2 buffers][4 lane quadrants][32 floats], and its barriers at bars[kStackXchgBar ..)
constexpr uint32_t kStackXchgOff = kStackZeroOff + kStackZeroBytes;
constexpr uint32_t kStackXchgBytes = 3 * 2 * 4 * 32 * 4;
constexpr uint32_t kStackXchgBar = 64;  // 6 barriers, beyond the ring's 2 x 12 + 9
static_assert(kStackXchgOff % 16 == 0, "exchange rows 16-byte aligned");
// the input ring of kEpiColsBias layers: four 48 KB row slots (four 48-channel sources) beside
// the weights; 4 divides the issuer's 12-row period
constexpr uint32_t kColsRing = 4;
static_assert(((128 + kMaxKSteps + 2) * 8) % 16 == 0, "per-channel constants 16-byte aligned");

}  // namespace kb2
