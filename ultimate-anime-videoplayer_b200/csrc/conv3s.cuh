// 3x3 convolution with the kernel rows stacked along N (sm_100a, tcgen05 + TMEM + TMA).
//
// Why: a tcgen05.mma of M = 128 costs at least ~45 cycles whatever N is below ~96 (measured on
// B200; at N >= 128 it runs at the tensor rate, N / 2 cycles for K = 16). SPAN's convolutions have
// 48 output channels, so the plain implicit GEMM (conv_tc.cuh) spends half of each instruction idle.
// Here every input row is multiplied once by the three kernel rows at the same time:
//
//     B = [ W(dy = +1) | W(dy = 0) | W(dy = -1) ]      (N = 3 x 48 = 144 rows of weights)
//
// and the three 48-column results land in the accumulators of the three output rows that input row
// feeds (o = t - 2, t - 1, t for input row index t of a band). An output row is complete after its
// third input row; the epilogue then reads it.
//
// Issue rate. The single issuing thread is the bottleneck of this kernel: measured on B200, nine
// MMAs issued from one asm block with precomputed descriptors run at the tensor rate (73 cycles
// each for N = 144), while any instruction between two MMAs (a branch, a descriptor update) costs
// ~60 cycles more per MMA. So every input row is exactly n_k MMAs of N = 144 into one contiguous
// 144-column accumulator window (mma_ss_row, one asm block), all accumulating:
//  * output rows cycle through 6 slots; slot s owns the 48-column TMEM block s, and slots 0 and 1
//    also own blocks 6 and 7. The window of input row t starts at the block of slot(t - 2), so it
//    never wraps: its third block lands in block 6 or 7 when the ring would wrap, and the epilogue
//    adds the two blocks of a slot (8 blocks = 384 columns);
//  * when an output row is first touched, its block(s) are cleared by an MMA with an all-zero B tile
//    and enable-input-d off (issued in order just before the row's accumulating MMAs), so the
//    row's n_k MMAs all accumulate;
//  * a slot is reused every 6 output rows, which leaves the epilogue 3 rows of slack;
//  * band edges use the one- or two-block sub-ranges of B (N = 48 / 96) in the same asm block.
//
// Roles: warp 0 = TMA producer (one 128-pixel box of all channel chunks per input row), warp 1 =
// TMEM owner + MMA issuer, warps 2.. = epilogue (4 per kStackEpiCols output channels) with the fused
// epilogues of conv_tc.cuh.
#pragma once

#include "conv_tc.cuh"

namespace kb2 {

// One block per SM owning all 512 TMEM columns, with one epilogue warp per 32 lanes x 8 output
// columns. Measured on 8 x 1080p: two blocks per SM (256 columns and 16-column epilogue warps
// each) made the plain conv 7% faster but the gated conv 55% slower (the wider epilogue warps
// spill and serialise the residual reads), so the single-block shape is kept.
constexpr int kStackBlocksPerSm = 1;
constexpr int kStackEpiCols = 8;
constexpr uint32_t kStackTmemCols = 512;
constexpr uint32_t kStackSlots = 6;   // output-row slots (TMEM reuse period, in output rows)
constexpr uint32_t kStackBlocks = 8;  // 48-column TMEM blocks: one per slot, plus 6 and 7 for slots 0, 1

template <int kCoutPad>
struct StackShape {
  static constexpr int epi_warps = 4 * (kCoutPad / kStackEpiCols);  // 4 quadrants x column groups
  static constexpr int threads = 64 + 32 * epi_warps;
  static constexpr int max_slots = static_cast<int>(kStackSlots);
  static_assert(kStackBlocks * kCoutPad <= kStackTmemCols, "TMEM blocks");
};

constexpr int kRowMaxK = 9;  // K steps per input row (FP16 48 channels: 9; E4M3: 5; conv_1: 2)

// shared memory after the input ring: barriers (128 x 8 B), K-step table, per-channel constants, TMEM
// address, then (at kStackZeroOff) the all-zero B tile of the clearing MMA (48 rows x 32 B)
constexpr uint32_t kStackZeroOff = 2176;
constexpr uint32_t kStackZeroBytes = 48 * 32;
constexpr uint32_t kStackSmemExtra = 1024 + kStackZeroOff + kStackZeroBytes + 64;
static_assert(128 * 8 + (kMaxKSteps + 1) * 8 + 3 * kMaxN * 4 + 4 <= kStackZeroOff, "shared layout");

// ---------------------------------------------------------------- steady-row issue
// A steady input row (band rows 2 .. rows - 1) clears the block(s) of the output row it touches first
// and then multiplies by all three kernel rows. It goes out as two asm blocks: the head tests the
// NEXT row's input and slot barriers (mbarrier.test_wait does not block; the predicates are only
// read after the head's MMAs, so the barrier round trips overlap with MMA issue), clears, and issues
// the first half of the row's MMAs; the tail issues the rest and the row's single commit.
template <bool kFp8, int kNK, int kClears>
__device__ __forceinline__ uint32_t stack_row_head(
    uint32_t d_clear, uint32_t d_clear2, uint64_t zero_desc, uint32_t id_clear, uint32_t d_win, uint32_t idesc,
    uint32_t nf, uint32_t nf_par, uint32_t ns, uint32_t ns_par, const uint64_t (&a)[9], const uint64_t (&b)[9]) {
  static_assert(kNK == 2 || kNK == 5 || kNK == 9, "steady rows: 2, 5 or 9 K steps");
  static_assert(kClears == 1 || kClears == 2, "one or two cleared blocks");
  uint32_t ok;
  if constexpr (kFp8 == false && kNK == 2 && kClears == 1) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%5], %11, %12, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]),
            "l"(b[0])
          : "memory");
  } else if constexpr (kFp8 == false && kNK == 2 && kClears == 2) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%2], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%5], %11, %12, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]),
            "l"(b[0])
          : "memory");
  } else if constexpr (kFp8 == false && kNK == 5 && kClears == 1) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%5], %11, %14, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%5], %12, %15, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%5], %13, %16, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]), "l"(a[2]),
            "l"(b[0]), "l"(b[1]), "l"(b[2])
          : "memory");
  } else if constexpr (kFp8 == false && kNK == 5 && kClears == 2) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%2], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%5], %11, %14, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%5], %12, %15, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%5], %13, %16, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]), "l"(a[2]),
            "l"(b[0]), "l"(b[1]), "l"(b[2])
          : "memory");
  } else if constexpr (kFp8 == false && kNK == 9 && kClears == 1) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%5], %11, %16, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%5], %12, %17, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%5], %13, %18, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%5], %14, %19, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%5], %15, %20, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]),
            "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4])
          : "memory");
  } else if constexpr (kFp8 == false && kNK == 9 && kClears == 2) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%2], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%5], %11, %16, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%5], %12, %17, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%5], %13, %18, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%5], %14, %19, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%5], %15, %20, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]),
            "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 2 && kClears == 1) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%5], %11, %12, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]),
            "l"(b[0])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 2 && kClears == 2) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%2], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%5], %11, %12, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]),
            "l"(b[0])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 5 && kClears == 1) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%5], %11, %14, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%5], %12, %15, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%5], %13, %16, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]), "l"(a[2]),
            "l"(b[0]), "l"(b[1]), "l"(b[2])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 5 && kClears == 2) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%2], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%5], %11, %14, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%5], %12, %15, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%5], %13, %16, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]), "l"(a[2]),
            "l"(b[0]), "l"(b[1]), "l"(b[2])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 9 && kClears == 1) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%5], %11, %16, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%5], %12, %17, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%5], %13, %18, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%5], %14, %19, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%5], %15, %20, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]),
            "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 9 && kClears == 2) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%2], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%5], %11, %16, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%5], %12, %17, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%5], %13, %18, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%5], %14, %19, %6, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%5], %15, %20, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]),
            "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4])
          : "memory");
  }
  return ok;
}

template <bool kFp8, int kNK>
__device__ __forceinline__ void stack_row_tail(uint32_t d_win, uint32_t idesc, uint32_t done,
                                               const uint64_t (&a)[9], const uint64_t (&b)[9]) {
  if constexpr (kFp8 == false && kNK == 2) {
    asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %4, %1, acc;\n\t"
          "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%2];\n\t}\n"
          ::"r"(d_win), "r"(idesc), "r"(done),
            "l"(a[1]),
            "l"(b[1])
          : "memory");
  } else if constexpr (kFp8 == false && kNK == 5) {
    asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %5, %1, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %6, %1, acc;\n\t"
          "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%2];\n\t}\n"
          ::"r"(d_win), "r"(idesc), "r"(done),
            "l"(a[3]), "l"(a[4]),
            "l"(b[3]), "l"(b[4])
          : "memory");
  } else if constexpr (kFp8 == false && kNK == 9) {
    asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %7, %1, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %8, %1, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %5, %9, %1, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %6, %10, %1, acc;\n\t"
          "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%2];\n\t}\n"
          ::"r"(d_win), "r"(idesc), "r"(done),
            "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
            "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 2) {
    asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %3, %4, %1, acc;\n\t"
          "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%2];\n\t}\n"
          ::"r"(d_win), "r"(idesc), "r"(done),
            "l"(a[1]),
            "l"(b[1])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 5) {
    asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %3, %5, %1, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %4, %6, %1, acc;\n\t"
          "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%2];\n\t}\n"
          ::"r"(d_win), "r"(idesc), "r"(done),
            "l"(a[3]), "l"(a[4]),
            "l"(b[3]), "l"(b[4])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 9) {
    asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %3, %7, %1, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %4, %8, %1, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %5, %9, %1, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %6, %10, %1, acc;\n\t"
          "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%2];\n\t}\n"
          ::"r"(d_win), "r"(idesc), "r"(done),
            "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
            "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8])
          : "memory");
  }
}

struct StackIssue {
  const ConvArgs& a;
  uint32_t ring_base, w_base, zero_base, tmem_base;
  const uint64_t* s_k;
  uint64_t* full;
  uint64_t* done;
  uint64_t* slot_free;
};

// The MMA issuer (one thread). kNK: K steps per row when it is one of the steady-row shapes (2, 5,
// 9), else 0 and every row takes the general path.
template <bool kFp8, int kCoutPad, int kNK>
__device__ __forceinline__ void stack_issue(const StackIssue& is) {
  const ConvArgs& a = is.a;
  constexpr int kN = 3 * kCoutPad;
  constexpr uint32_t R = kStackSlots;
  constexpr uint64_t kBStep16 = (2u * kN * 16u) >> 4;   // one K step of B
  constexpr uint64_t kBlock16 = (kCoutPad * 16u) >> 4;  // one kernel-row block of B
  const uint64_t desc_hi = make_sdesc(0, 0, 128);
  const uint64_t b_desc0 = make_sdesc(is.w_base, kN * 16, 128);
  const uint64_t zero_desc = make_sdesc(is.zero_base, kCoutPad * 16, 128);
  const int n_k = kNK > 0 ? kNK : a.n_ksteps;
  uint64_t kd[kRowMaxK];  // per-row K-step deltas of A
  uint64_t bs[kRowMaxK];  // B descriptors of a steady row (all three kernel rows)
#pragma unroll
  for (int j = 0; j < kRowMaxK; ++j) {
    kd[j] = is.s_k[j];
    bs[j] = b_desc0 + static_cast<uint64_t>(j) * kBStep16;
  }
  const uint32_t id_n[3] = {a.idesc_n[0], a.idesc_n[1], a.idesc_n[2]};
  RingPos in{0, 0};
  RingPos acc{0, 0};  // slot (and phase) of output row t, the row first touched by input t
  uint32_t pre = 0;   // next row's barriers found complete by a steady row: 1 = input, 2 = slot
  for (int item = blockIdx.x; item < a.items; item += gridDim.x) {
    const int t0 = item / a.strips;
    const int band = t0 % a.bands;
    const int y0 = band * a.band_rows;
    const int y1 = min(a.H, y0 + a.band_rows);
    const int rows = y1 - y0;
    for (int t = 0; t <= rows + 1; ++t) {
      // blocks [b0, b1) of B feed output rows t - 2 + b0 .. t - 2 + b1 - 1 of the band
      const int b0 = t >= 2 ? 0 : 2 - t;
      const int b1 = t <= rows - 1 ? 3 : (t == rows ? 2 : 1);
      const bool fresh = b1 == 3;  // output row t is touched for the first time
      if (!(pre & 1u) && !wait_bar(&is.full[in.idx], in.phase, a.err, kErrWaitMma)) return;
      // a fresh output row's slot must have been read by the epilogue
      if (fresh && !(pre & 2u) && !wait_bar(&is.slot_free[acc.idx], acc.phase, a.err, kErrWaitMma)) return;
      pre = 0;
      tc_fence_after();
      const uint64_t a_row = desc_hi | static_cast<uint64_t>((is.ring_base + in.idx * a.slot_bytes) >> 4);
      uint64_t ad[kRowMaxK];
#pragma unroll
      for (int j = 0; j < kRowMaxK; ++j) ad[j] = a_row + kd[j];
      // the window starts at the TMEM block of slot(t - 2) = acc.idx - 2 (mod 6); block k of B
      // (output t - 2 + k) lands in TMEM block start + k, never past block 7
      const uint32_t start = acc.idx >= 2 ? acc.idx - 2 : acc.idx + R - 2;
      const uint32_t d_clear = is.tmem_base + acc.idx * kCoutPad;
      const uint32_t d_clear2 = d_clear + 6u * kCoutPad;  // slots 0 and 1 also own block 6 / 7
      if (kNK > 0 && b0 == 0 && fresh) {
        RingPos nin = in;
        nin.advance(a.ring);
        RingPos nacc = acc;
        nacc.advance(R);
        const uint32_t d_win = is.tmem_base + start * kCoutPad;
        const uint32_t nf = smem_u32(&is.full[nin.idx]);
        const uint32_t ns = smem_u32(&is.slot_free[nacc.idx]);
        if constexpr (kNK > 0) {
          if (acc.idx < 2)
            pre = stack_row_head<kFp8, kNK, 2>(d_clear, d_clear2, zero_desc, id_n[0], d_win, id_n[2], nf, nin.phase,
                                               ns, nacc.phase, ad, bs);
          else
            pre = stack_row_head<kFp8, kNK, 1>(d_clear, d_clear2, zero_desc, id_n[0], d_win, id_n[2], nf, nin.phase,
                                               ns, nacc.phase, ad, bs);
          stack_row_tail<kFp8, kNK>(d_win, id_n[2], smem_u32(&is.done[in.idx]), ad, bs);
        }
      } else {
        if (fresh) {  // clear the row's block(s): (any finite A) x (zero B), enable-input-d off
          mma_ss<kFp8>(d_clear, ad[0], zero_desc, id_n[0], 0u);
          if (acc.idx < 2) mma_ss<kFp8>(d_clear2, ad[0], zero_desc, id_n[0], 0u);
        }
        const uint64_t b_first = b_desc0 + static_cast<uint64_t>(b0) * kBlock16;
        uint64_t bd[kRowMaxK];
#pragma unroll
        for (int j = 0; j < kRowMaxK; ++j) bd[j] = b_first + static_cast<uint64_t>(j) * kBStep16;
        const int nb = b1 - b0;
        const uint32_t idesc = nb == 3 ? id_n[2] : (nb == 2 ? id_n[1] : id_n[0]);
        mma_ss_row<kFp8>(is.tmem_base + (start + static_cast<uint32_t>(b0)) * kCoutPad, ad, bd, idesc, n_k);
        mma_commit(&is.done[in.idx]);  // the input row is consumed, its completed output row is ready
      }
      in.advance(a.ring);
      acc.advance(R);  // acc tracks output row t + 1 (virtual past the band's last row)
    }
    // input rows rows and rows + 1 advanced past the band's last output: step back to the next
    // band's first output row
    acc.retreat(R);
    acc.retreat(R);
  }
}

template <bool kFp8, int kCoutPad, int kEpi, int kOut>
__global__ void __launch_bounds__(StackShape<kCoutPad>::threads, kStackBlocksPerSm)
    conv3s_kernel(const __grid_constant__ ConvMaps maps, const __grid_constant__ ConvArgs a) {
  static_assert(kCoutPad == 16 || kCoutPad == 48, "stacked kernel: 16 or 48 output channels");
  constexpr int kEpiWarps = StackShape<kCoutPad>::epi_warps;
  constexpr uint32_t R = kStackSlots;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sw = smem;
  uint8_t* ring = smem + a.w_smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + a.ring * a.slot_bytes);
  uint64_t* full = bars;
  uint64_t* done = bars + a.ring;  // input row consumed = its output rows' MMAs complete
  uint64_t* slot_free = bars + 2 * a.ring;
  uint64_t* wbar = slot_free + R;
  uint64_t* drain = wbar + 1;
  uint64_t* s_k = bars + 128;  // per K step of a row: (a_off >> 4) | (lbo >> 4) << 16
  float* s_bias = reinterpret_cast<float*>(s_k + kMaxKSteps + 1);
  float* s_scale = s_bias + kMaxN;
  float* s_slope = s_scale + kMaxN;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(s_slope + kMaxN);
  uint8_t* zero_b = reinterpret_cast<uint8_t*>(bars) + kStackZeroOff;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  for (uint32_t j = threadIdx.x; j < kStackZeroBytes / 16; j += blockDim.x)
    reinterpret_cast<uint4*>(zero_b)[j] = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();  // the zero tile is read by the tensor core (async proxy)

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < a.ring; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&done[i], 1);
    }
    for (uint32_t i = 0; i < R; ++i) mbar_init(&slot_free[i], kEpiWarps);
    mbar_init(wbar, 1);
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  for (int j = threadIdx.x; j < kMaxN; j += blockDim.x) {
    s_bias[j] = j < kCoutPad ? a.bias[j] : 0.0f;
    s_scale[j] = (a.chan_scale != nullptr && j < kCoutPad) ? a.chan_scale[j] : 1.0f;
    s_slope[j] = (a.slope != nullptr && j < kCoutPad) ? a.slope[j] : 0.0f;
  }
  for (int j = threadIdx.x; j <= kMaxKSteps; j += blockDim.x)
    s_k[j] = j < a.n_ksteps
                 ? (static_cast<uint64_t>(a.ks[j].a_off >> 4) | (static_cast<uint64_t>(a.ks[j].lbo >> 4) << 16))
                 : 0;
  if (warp == 0 && lane == 0) prefetch_tmap(&maps.m[0]);
  if (warp == 1) {
    tmem_alloc(tmem_holder, kStackTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ producer (rows y0-1 .. y1)
      bool ok = true;
      mbar_arrive_expect_tx(wbar, a.wbytes);
      for (uint32_t off = 0; off < a.wbytes; off += 32768u) {
        const uint32_t len = a.wbytes - off < 32768u ? a.wbytes - off : 32768u;
        bulk_load(sw + off, a.wpack + off, len, wbar);
      }
      // ring positions are carried as (slot, phase) counters: an integer division by a runtime
      // divisor costs this single thread hundreds of cycles per row
      RingPos in{0, 0};
      uint32_t issued = 0;
      for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x) {
        const int strip = item % a.strips;
        const int t = item / a.strips;
        const int band = t % a.bands;
        const int n = t / a.bands;
        const int y0 = band * a.band_rows;
        const int y1 = min(a.H, y0 + a.band_rows);
        const int x0 = strip * a.strip_w;
        for (int r = y0 - 1; r <= y1; ++r) {
          if (!wait_bar(&done[in.idx], in.phase ^ 1u, a.err, kErrWaitProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[in.idx], a.slot_bytes);
          // one box: 128 pixels from x0 - 1 (zero fill left of the image), all chunks
          tma_load_4d(ring + in.idx * a.slot_bytes, &maps.m[0], &full[in.idx], (x0 - 1) * 2, 0, r, n);
          in.advance(a.ring);
          ++issued;
        }
      }
      // every copy issued has landed before the block may exit: wait for the last ring's worth
      RingPos back = in;
      for (uint32_t k = 0; k < a.ring && k < issued; ++k) {
        back.retreat(a.ring);
        wait_bar(&full[back.idx], back.phase, a.err, kErrWaitDrain);
      }
      wait_bar(wbar, 0, a.err, kErrWaitDrain);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA issuer
      const bool ok = wait_bar(wbar, 0, a.err, kErrWaitMma);
      if (ok) {
        const StackIssue is{a, smem_u32(ring), smem_u32(sw), smem_u32(zero_b), tmem_base, s_k, full, done, slot_free};
        switch (a.n_ksteps) {
          case 9: stack_issue<kFp8, kCoutPad, 9>(is); break;
          case 5: stack_issue<kFp8, kCoutPad, 5>(is); break;
          case 2: stack_issue<kFp8, kCoutPad, 2>(is); break;
          default: stack_issue<kFp8, kCoutPad, 0>(is); break;
        }
      }
      mma_commit(drain);
      wait_bar(drain, 0, a.err, kErrWaitDrain);
    }
    __syncwarp();
  } else {
    // -------------------------------------------------------------------- epilogue
    const int quad = warp & 3;
    const int col0 = ((warp - 2) >> 2) * kStackEpiCols;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t my_cols = tmem_base + lane_addr + static_cast<uint32_t>(col0);
    // this warp's per-channel constants, held in registers for the whole kernel (reading them from
    // shared memory on every row cost ~9% of the plain conv)
    float r_bias[kStackEpiCols], r_scale[kStackEpiCols], r_slope[kStackEpiCols];
#pragma unroll
    for (int j = 0; j < kStackEpiCols; ++j) {
      r_bias[j] = s_bias[col0 + j];
      r_scale[j] = s_scale[col0 + j];
      r_slope[j] = s_slope[col0 + j];
    }
    // every slot starts free (phase 0 of slot_free)
    if (lane == 0)
      for (uint32_t s = 0; s < R; ++s) mbar_arrive(&slot_free[s]);
    RingPos acc{0, 0};  // TMEM slot of output row y
    RingPos in{0, 0};   // input ring position of the row that completes output row y (y + 2 of the band)
    bool ok = true;
    for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x) {
      const int strip = item % a.strips;
      const int t = item / a.strips;
      const int band = t % a.bands;
      const int n = t / a.bands;
      const int y0 = band * a.band_rows;
      const int y1 = min(a.H, y0 + a.band_rows);
      const int m = quad * 32 + lane;
      const int x = strip * a.strip_w + m;
      const bool store = m < a.strip_w && x < a.W;
      in.advance(a.ring);  // the band's input rows y0 - 1 and y0 complete no output row
      in.advance(a.ring);
      for (int y = y0; y < y1; ++y, acc.advance(R), in.advance(a.ring)) {
        const uint32_t s = acc.idx;
        const bool got = wait_bar(&done[in.idx], in.phase, a.err, kErrWaitEpilogue);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float v[kStackEpiCols];
        tmem_ld8(my_cols + s * kCoutPad, v);
        if (s < 2) {  // slots 0 and 1: the part of the sum that landed in block 6 or 7
          float w[kStackEpiCols];
          tmem_ld8(my_cols + (s + 6) * kCoutPad, w);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < kStackEpiCols; ++j) v[j] += w[j];
        } else {
          tmem_ld_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&slot_free[s]);
        if (store) epilogue_cols<kEpi, kOut, kStackEpiCols>(a, r_bias, r_scale, r_slope, v, 0, n, y, x, col0);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kStackTmemCols);
  }
}

}  // namespace kb2
