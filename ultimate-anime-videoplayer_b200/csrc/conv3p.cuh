// Paired stacked 3x3 convolution: the stacked-kernel-row scheme (stack_common.cuh) with every MMA
// shared by the two SMs of a cluster (sm_100a, tcgen05 cta_group::2, M = 256).
//
// Why: the single issuing thread limits a one-SM stacked conv. Measured on B200, a tcgen05.mma of
// M = 128 costs its issuing thread ~60 cycles whatever else runs, and each instruction between MMAs
// costs more, so a row of 9 MMAs plus its bookkeeping took ~1,400-1,800 cycles against ~820 cycles
// of tensor work. An
// M = 256 MMA (cta_group::2) runs at the same ~72 cycles per instruction (N = 144, measured) but
// feeds both SMs of the pair: the issue cost per output pixel halves.
//
// Layout of the pair: block r of the cluster owns strip 2p + r of its (frame, strip pair) row segments.
//  * A (the input row) is split by rows of M: each block copies its own strip's row into its own
//    ring slot, at the same shared-memory offset in both blocks;
//  * B (the stacked weights, N = 3 x 48 rows per K step) is split by rows of N: block 0 holds rows
//    0 .. N/2 - 1, block 1 rows N/2 .. N - 1, each as [K step][K half][N/2 rows][16 bytes], so one
//    descriptor addresses both halves and D column c is B row c;
//  * D: each block's TMEM holds its own 128 pixels x all N columns (the 6-slot, 8-block dual-location
//    window of stack_common.cuh).
// Block 0's thread issues every MMA; its barriers gather the pair: the input row is "full" when both
// blocks' copies landed (the copies of block 1 complete on block 0's barrier), and an accumulator
// slot is free when both blocks' epilogues read it (block 1 arrives remotely). Commits multicast to
// both blocks' "done" barriers.
//
// Uniform rows. Every input row t of a band (t = 0 .. rows + 1) is issued alike: clear the block(s)
// of output entry t, then n_k MMAs of N = 144 into the window of entries t - 2 .. t. A band of
// `rows` output rows owns rows + 2 consecutive entries; the last two are "virtual" (they collect the
// out-of-band products of the band's first and last input rows) and the epilogue releases them
// without reading. The accumulator ring never steps back, and no band-edge MMA variants exist.
//
// Roles (both blocks): warp 0 = TMA producer, warp 1 = TMEM allocation (pair-wide) and, in block 0,
// the MMA issuer, warps 2.. = epilogue of the block's own pixels (conv_tc.cuh epilogues).
#pragma once

#include <type_traits>

#include <utility>

#include "stack_common.cuh"

namespace kb2 {

constexpr uint16_t kPairMask = 3;  // both blocks of the cluster
constexpr int kPairMaxK = 12;      // K steps per input row: 2, 3 (conv_1), 5, 6 (E4M3), 9, 12 (FP16 64)

// Epilogue shape of the pair kernel: `groups` groups of warps take the accumulator entries in turn
// (entry e goes to group e % groups, so a group owns the slots s with s % groups = g and that many
// rows are in the epilogue at once); a warp covers 32 pixels x warp_cols channels. Measured on
// 8 x 1080p (in-process A/B): without a residual, 3 groups of 4 warps x 48 channels beat 2 groups of
// 12 warps x 16 channels by 5-18 % (fewer epilogue warps disturb the MMA issuer less). The 48-channel
// SPAB gates, which also hold the residual words, take 3 x 4 x 48 too (`wide`, 128 registers): the
// E4M3 gates 10 % and the FP16 gates 2 % faster than on 2 x 12 x 16 with the epilogue's constants in
// the parameter space (before that move, with per-warp register biases, the FP16 gates spilled on
// 3 x 4 x 48 and ran 20-30 % slower). The 64-channel residual shape keeps 2 groups x 8 x 32.
template <int kCoutPad, int kEpi, bool kFp8 = false>
struct PairShape {
  static constexpr bool residual = kEpi == kEpiSpanAttn || kEpi == kEpiResPrelu;
  static constexpr bool wide = residual && kCoutPad == 48;
  static constexpr int groups = residual && !wide ? 2 : 3;
  // 64 channels (the IFNet residual convs): 32 columns a warp, 2 x 8 warps (576 threads)
  static constexpr int cols = wide ? 48 : residual ? (kCoutPad % 32 == 0 ? 32 : 16) : (kCoutPad % 48 == 0 ? 48 : 32);
  static_assert(kStackSlots % groups == 0, "groups divide the accumulator slots");
  static constexpr int warp_cols = kCoutPad < cols ? kCoutPad : cols;
  static_assert(warp_cols % 16 == 0 && kCoutPad % warp_cols == 0, "16-column TMEM loads per warp");
  static constexpr int group_warps = 4 * (kCoutPad / warp_cols);
  static constexpr int epi_warps = groups * group_warps;
  static constexpr int threads = 64 + 32 * epi_warps;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// All threads of both blocks.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Shared::cluster address of the variable at `local` (a shared::cta address) in block `rank`.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// Relaxed arrive: orders nothing before it. For releasing an accumulator slot whose TMEM reads have
// completed (tcgen05.wait::ld): a release at cluster scope would also wait until the epilogue's
// earlier global stores are visible cluster-wide, which cost ~1,000-1,800 cycles per row (measured).
__device__ __forceinline__ void mbar_arrive_remote_relaxed(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// This block's share of a pair copy: its own destination, completion counted on the barrier at
// `cluster_bar` (block 0's). No multicast.
__device__ __forceinline__ void tma_load_4d_pair(void* dst, const CUtensorMap* map, uint32_t cluster_bar, int c0,
                                                 int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(cluster_bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* holder, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(holder)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Arrives on the barrier at this offset in both blocks once every MMA issued so far completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(kPairMask)
      : "memory");
}

// ---------------------------------------------------------------- row issue (two asm blocks)
// The head tests the NEXT row's input and slot barriers (mbarrier.test_wait does not block; its
// predicates are read only after the head's MMAs), clears the fresh entry's block(s) with an MMA of
// a zero B and enable-input-d off, and issues the first half of the row's MMAs; the tail issues the
// rest and the row's commit.
template <bool kFp8, int kNK, int kClears>
__device__ __forceinline__ uint32_t pair_row_head(
    uint32_t d_clear, uint32_t d_clear2, uint64_t zero_desc, uint32_t id_clear, uint32_t d_win, uint32_t idesc,
    uint32_t nf, uint32_t nf_par, uint32_t ns, uint32_t ns_par, const uint64_t (&a)[kNK], const uint64_t (&b)[kNK]) {
  static_assert(kNK == 2 || kNK == 3 || kNK == 5 || kNK == 6 || kNK == 9 || kNK == 12, "rows of 2, 3, 5, 6, 9 or 12 K steps");
  static_assert(kClears == 1 || kClears == 2, "one or two cleared blocks");
  uint32_t ok;
  if constexpr (kFp8 == false && kNK == 2 && kClears == 1) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %11, %12, %6, acc;\n\t"
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
          "tcgen05.mma.cta_group::2.kind::f16 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%2], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %11, %12, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]),
            "l"(b[0])
          : "memory");
  } else if constexpr (kFp8 == false && kNK == 3 && kClears == 1) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %11, %13, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %12, %14, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]),
            "l"(b[0]), "l"(b[1])
          : "memory");
  } else if constexpr (kFp8 == false && kNK == 3 && kClears == 2) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%2], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %11, %13, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %12, %14, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]),
            "l"(b[0]), "l"(b[1])
          : "memory");
  } else if constexpr (kFp8 == false && kNK == 5 && kClears == 1) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %11, %14, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %12, %15, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %13, %16, %6, acc;\n\t"
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
          "tcgen05.mma.cta_group::2.kind::f16 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%2], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %11, %14, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %12, %15, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %13, %16, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]), "l"(a[2]),
            "l"(b[0]), "l"(b[1]), "l"(b[2])
          : "memory");
  } else if constexpr (kFp8 == false && kNK == 6 && kClears == 1) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %11, %14, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %12, %15, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %13, %16, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]), "l"(a[2]),
            "l"(b[0]), "l"(b[1]), "l"(b[2])
          : "memory");
  } else if constexpr (kFp8 == false && kNK == 6 && kClears == 2) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%2], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %11, %14, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %12, %15, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %13, %16, %6, acc;\n\t"
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
          "tcgen05.mma.cta_group::2.kind::f16 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %11, %16, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %12, %17, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %13, %18, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %14, %19, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %15, %20, %6, acc;\n\t"
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
          "tcgen05.mma.cta_group::2.kind::f16 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%2], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %11, %16, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %12, %17, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %13, %18, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %14, %19, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %15, %20, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]),
            "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4])
          : "memory");
  } else if constexpr (kFp8 == false && kNK == 12 && kClears == 1) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %11, %17, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %12, %18, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %13, %19, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %14, %20, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %15, %21, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %16, %22, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]),
            "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5])
          : "memory");
  } else if constexpr (kFp8 == false && kNK == 12 && kClears == 2) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%2], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %11, %17, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %12, %18, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %13, %19, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %14, %20, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %15, %21, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%5], %16, %22, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]),
            "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 2 && kClears == 1) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %11, %12, %6, acc;\n\t"
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
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%2], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %11, %12, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]),
            "l"(b[0])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 3 && kClears == 1) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %11, %13, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %12, %14, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]),
            "l"(b[0]), "l"(b[1])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 3 && kClears == 2) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%2], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %11, %13, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %12, %14, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]),
            "l"(b[0]), "l"(b[1])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 5 && kClears == 1) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %11, %14, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %12, %15, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %13, %16, %6, acc;\n\t"
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
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%2], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %11, %14, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %12, %15, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %13, %16, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]), "l"(a[2]),
            "l"(b[0]), "l"(b[1]), "l"(b[2])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 6 && kClears == 1) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %11, %14, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %12, %15, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %13, %16, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]), "l"(a[2]),
            "l"(b[0]), "l"(b[1]), "l"(b[2])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 6 && kClears == 2) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%2], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %11, %14, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %12, %15, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %13, %16, %6, acc;\n\t"
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
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %11, %16, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %12, %17, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %13, %18, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %14, %19, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %15, %20, %6, acc;\n\t"
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
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%2], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %11, %16, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %12, %17, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %13, %18, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %14, %19, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %15, %20, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]),
            "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 12 && kClears == 1) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %11, %17, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %12, %18, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %13, %19, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %14, %20, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %15, %21, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %16, %22, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]),
            "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 12 && kClears == 2) {
    asm volatile(
          "{\n\t.reg .pred pf, ps, acc, clr;\n\t.reg .b32 t0, t1;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 pf, [%7], %8;\n\t"
          "mbarrier.test_wait.parity.shared::cta.b64 ps, [%9], %10;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "setp.ne.b32 clr, 0, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%1], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%2], %11, %3, %4, clr;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %11, %17, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %12, %18, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %13, %19, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %14, %20, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %15, %21, %6, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%5], %16, %22, %6, acc;\n\t"
          "selp.u32 t0, 1, 0, pf;\n\t"
          "selp.u32 t1, 2, 0, ps;\n\t"
          "or.b32 %0, t0, t1;\n\t}\n"
          : "=r"(ok)
          : "r"(d_clear), "r"(d_clear2), "l"(zero_desc), "r"(id_clear), "r"(d_win), "r"(idesc),
            "r"(nf), "r"(nf_par), "r"(ns), "r"(ns_par),
            "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]),
            "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5])
          : "memory");
  }
  return ok;
}

template <bool kFp8, int kNK>
__device__ __forceinline__ void pair_row_tail(uint32_t d_win, uint32_t idesc, uint32_t done,
                                              const uint64_t (&a)[kNK], const uint64_t (&b)[kNK]) {
  if constexpr (kFp8 == false && kNK == 2) {
    asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %4, %5, %1, acc;\n\t"
          "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%2], %3;\n\t}\n"
          ::"r"(d_win), "r"(idesc), "r"(done), "h"(kPairMask),
            "l"(a[1]),
            "l"(b[1])
          : "memory");
  } else if constexpr (kFp8 == false && kNK == 3) {
    asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %4, %5, %1, acc;\n\t"
          "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%2], %3;\n\t}\n"
          ::"r"(d_win), "r"(idesc), "r"(done), "h"(kPairMask),
            "l"(a[2]),
            "l"(b[2])
          : "memory");
  } else if constexpr (kFp8 == false && kNK == 5) {
    asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %4, %6, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %5, %7, %1, acc;\n\t"
          "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%2], %3;\n\t}\n"
          ::"r"(d_win), "r"(idesc), "r"(done), "h"(kPairMask),
            "l"(a[3]), "l"(a[4]),
            "l"(b[3]), "l"(b[4])
          : "memory");
  } else if constexpr (kFp8 == false && kNK == 6) {
    asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %4, %7, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %5, %8, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %6, %9, %1, acc;\n\t"
          "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%2], %3;\n\t}\n"
          ::"r"(d_win), "r"(idesc), "r"(done), "h"(kPairMask),
            "l"(a[3]), "l"(a[4]), "l"(a[5]),
            "l"(b[3]), "l"(b[4]), "l"(b[5])
          : "memory");
  } else if constexpr (kFp8 == false && kNK == 9) {
    asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %4, %8, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %5, %9, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %6, %10, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %7, %11, %1, acc;\n\t"
          "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%2], %3;\n\t}\n"
          ::"r"(d_win), "r"(idesc), "r"(done), "h"(kPairMask),
            "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
            "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8])
          : "memory");
  } else if constexpr (kFp8 == false && kNK == 12) {
    asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %4, %10, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %5, %11, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %6, %12, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %7, %13, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %8, %14, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %9, %15, %1, acc;\n\t"
          "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%2], %3;\n\t}\n"
          ::"r"(d_win), "r"(idesc), "r"(done), "h"(kPairMask),
            "l"(a[6]), "l"(a[7]), "l"(a[8]), "l"(a[9]), "l"(a[10]), "l"(a[11]),
            "l"(b[6]), "l"(b[7]), "l"(b[8]), "l"(b[9]), "l"(b[10]), "l"(b[11])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 2) {
    asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %4, %5, %1, acc;\n\t"
          "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%2], %3;\n\t}\n"
          ::"r"(d_win), "r"(idesc), "r"(done), "h"(kPairMask),
            "l"(a[1]),
            "l"(b[1])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 3) {
    asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %4, %5, %1, acc;\n\t"
          "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%2], %3;\n\t}\n"
          ::"r"(d_win), "r"(idesc), "r"(done), "h"(kPairMask),
            "l"(a[2]),
            "l"(b[2])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 5) {
    asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %4, %6, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %5, %7, %1, acc;\n\t"
          "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%2], %3;\n\t}\n"
          ::"r"(d_win), "r"(idesc), "r"(done), "h"(kPairMask),
            "l"(a[3]), "l"(a[4]),
            "l"(b[3]), "l"(b[4])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 6) {
    asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %4, %7, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %5, %8, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %6, %9, %1, acc;\n\t"
          "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%2], %3;\n\t}\n"
          ::"r"(d_win), "r"(idesc), "r"(done), "h"(kPairMask),
            "l"(a[3]), "l"(a[4]), "l"(a[5]),
            "l"(b[3]), "l"(b[4]), "l"(b[5])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 9) {
    asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %4, %8, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %5, %9, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %6, %10, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %7, %11, %1, acc;\n\t"
          "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%2], %3;\n\t}\n"
          ::"r"(d_win), "r"(idesc), "r"(done), "h"(kPairMask),
            "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
            "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8])
          : "memory");
  } else if constexpr (kFp8 == true && kNK == 12) {
    asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, 1, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %4, %10, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %5, %11, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %6, %12, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %7, %13, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %8, %14, %1, acc;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %9, %15, %1, acc;\n\t"
          "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%2], %3;\n\t}\n"
          ::"r"(d_win), "r"(idesc), "r"(done), "h"(kPairMask),
            "l"(a[6]), "l"(a[7]), "l"(a[8]), "l"(a[9]), "l"(a[10]), "l"(a[11]),
            "l"(b[6]), "l"(b[7]), "l"(b[8]), "l"(b[9]), "l"(b[10]), "l"(b[11])
          : "memory");
  }
}

// Work split: the output rows of a launch form one row space, unit after unit (unit = frame x strip
// pair, H rows each); cluster c of nc owns the contiguous range [T c / nc, T (c + 1) / nc) of its T
// rows, each end rounded down to a multiple of 6 rows within its unit, and walks it as segments
// inside one unit. A segment of `rows` output rows is issued as rows + 2 + pad input rows and
// entries (uniform rows; the 2 + pad last entries are virtual), pad making the count a multiple of
// the 6 accumulator slots. So every segment starts at slot 0 on a row y = 0 mod 6, output row y
// always lands in slot y mod 6, and the split of its sum between TMEM blocks (slots 0 and 1 use two)
// is the same whatever the batch and the split: results do not depend on them.
__device__ __forceinline__ int pair_pad(int rows) { return (6 - (rows + 2) % 6) % 6; }

struct PairSpan {
  long long r, end;
  __device__ __forceinline__ static long long align6(const ConvArgs& a, long long b) {
    const long long u = b / a.H;
    const long long y = b - u * a.H;
    return u * a.H + (y - y % 6);
  }
  __device__ __forceinline__ PairSpan(const ConvArgs& a, uint32_t c, uint32_t nc) {
    const long long total = static_cast<long long>(a.batch) * a.pairs * a.H;
    r = align6(a, total * c / nc);
    end = c + 1 == nc ? total : align6(a, total * (c + 1) / nc);
  }
  // the next segment: frame n, strip pair `pair`, output rows [y0, y1); false when the range is done
  __device__ __forceinline__ bool next(const ConvArgs& a, int& n, int& pair, int& y0, int& y1) {
    if (r >= end) return false;
    const long long u = r / a.H;
    const long long unit_end = (u + 1) * a.H;
    const long long stop = end < unit_end ? end : unit_end;
    y0 = static_cast<int>(r - u * a.H);
    y1 = static_cast<int>(stop - u * a.H);
    n = static_cast<int>(u / a.pairs);
    pair = static_cast<int>(u % a.pairs);
    r = stop;
    return true;
  }
};

struct PairIssue {
  const ConvArgs& a;
  uint32_t ring_base, w_base, zero_base, tmem_base;
  const uint64_t* s_k;
  uint64_t* full;
  uint64_t* done;
  uint64_t* slot_free;
};

// What every row of the issuer needs, set up once.
template <int kNK>
struct PairRowCtx {
  // The descriptors of a row differ only in their low words (start address and LBO fields), so the
  // context keeps those and one high word each: half the registers of 64-bit arrays (a row of 12 K
  // steps otherwise spills).
  uint32_t a_lo[kNK];  // A descriptors of ring slot 0 (slot k adds k * slot16)
  uint32_t b_lo[kNK];  // B descriptors (all three kernel rows)
  uint32_t a_hi, b_hi;
  uint64_t zero_desc;
  uint32_t slot16;  // one ring slot, in descriptor address units
  uint32_t tmem;
  uint32_t full_u32, done_u32, free_u32;  // shared addresses of full[0], done[0], slot_free[0]
  uint64_t* full;
  uint64_t* slot_free;
  int* err;
};

// Input ring of the pair kernel: 12 row slots, or 6 for rows of 12 K steps (64 FP16 input
// channels: twelve 16 KB slots and the weights do not fit in shared memory).
template <int kNK>
constexpr uint32_t pair_ring() {
  return kNK == 12 ? 6u : 12u;
}

// Input row k of a 12-row period. The accumulator ring has 6 slots and the input ring 12 or 6, so
// within a period every slot index, TMEM address and accumulator phase is a compile-time constant.
// With 12 input slots the input phase is one bit per period (`ph`); with 6 it is 0 for rows 0-5 and
// 1 for rows 6-11 of every period (`ph` stays 0). The issuing thread then executes little besides
// its two asm blocks.
// Input-phase flips over a 12-row period of a ring of kRing slots: the period's rows wrap the ring
// 12 / kRing times, so the phase of slot 0 flips between periods when that count is odd.
template <uint32_t kRing>
constexpr uint32_t pair_period_flip() {
  static_assert(12u % kRing == 0u, "the ring divides the 12-row period");
  return (12u / kRing) & 1u;
}

template <bool kFp8, int kCoutPad, int kNK, uint32_t kRing, int kK>
__device__ __forceinline__ bool pair_row_k(const PairRowCtx<kNK>& c, uint32_t ph, uint32_t& pre) {
  constexpr uint32_t kIn = kK % kRing;
  constexpr uint32_t kInPh = (static_cast<uint32_t>(kK) / kRing) & 1u;
  constexpr uint32_t kSlot = kK % 6;
  constexpr uint32_t kAccPh = kK >= 6 ? 1u : 0u;
  constexpr uint32_t kStart = kSlot >= 2 ? kSlot - 2 : kSlot + 4;
  constexpr uint32_t kNext = (kK + 1) % 12;
  constexpr uint32_t kNextIn = kNext % kRing;
  // the next row's input phase: row 0 of the next period when k = 11
  constexpr uint32_t kNextInPh = kK == 11 ? pair_period_flip<kRing>() : (kNext / kRing) & 1u;
  constexpr uint32_t kNextSlot = kNext % 6;
  constexpr uint32_t kNextAccPh = kNext >= 6 ? 1u : 0u;
  constexpr uint32_t kIdClear = make_idesc(256, kCoutPad);
  constexpr uint32_t kIdWin = make_idesc(256, 3 * kCoutPad);
  if (!(pre & 1u) && !wait_bar(c.full + kIn, ph ^ kInPh, c.err, kErrWaitMma)) return false;
  if (!(pre & 2u) && !wait_bar(c.slot_free + kSlot, kAccPh, c.err, kErrWaitMma)) return false;
  tc_fence_after();
  uint64_t ad[kNK], bd[kNK];
  const uint32_t off = kIn * c.slot16;
#pragma unroll
  for (int j = 0; j < kNK; ++j) {
    ad[j] = (static_cast<uint64_t>(c.a_hi) << 32) | (c.a_lo[j] + off);
    bd[j] = (static_cast<uint64_t>(c.b_hi) << 32) | c.b_lo[j];
  }
  const uint32_t d_clear = c.tmem + kSlot * kCoutPad;
  const uint32_t d_win = c.tmem + kStart * kCoutPad;
  const uint32_t nf = c.full_u32 + kNextIn * 8u;
  const uint32_t nf_par = ph ^ kNextInPh;
  const uint32_t ns = c.free_u32 + kNextSlot * 8u;
  pre = pair_row_head<kFp8, kNK, (kSlot < 2 ? 2 : 1)>(d_clear, d_clear + 6u * kCoutPad, c.zero_desc, kIdClear, d_win,
                                                        kIdWin, nf, nf_par, ns, kNextAccPh, ad, bd);
  pair_row_tail<kFp8, kNK>(d_win, kIdWin, c.done_u32 + kIn * 8u, ad, bd);
  return true;
}

template <bool kFp8, int kCoutPad, int kNK, uint32_t kRing, int... kKs>
__device__ __forceinline__ bool pair_period(const PairRowCtx<kNK>& c, uint32_t ph, uint32_t& pre,
                                            std::integer_sequence<int, kKs...>) {
  return (pair_row_k<kFp8, kCoutPad, kNK, kRing, kKs>(c, ph, pre) && ...);
}

// The MMA issuer of the pair (block 0, one thread), for rows of kNK K steps. Every input row is
// alike (uniform rows), so the issuer only needs the number of input rows of its items. kRing: the
// input ring's slot count (pair_ring, or kColsRing for the four-source kEpiColsBias layers).
template <bool kFp8, int kCoutPad, int kNK, uint32_t kRing = pair_ring<kNK>()>
__device__ __forceinline__ void pair_issue(const PairIssue& is) {
  static_assert(kStackSlots == 6, "the 12-row period assumes 6 accumulator slots");
  const ConvArgs& a = is.a;
  constexpr int kNHalf = 3 * kCoutPad / 2;                  // B rows per block
  constexpr uint64_t kBStep16 = (2u * kNHalf * 16u) >> 4;  // one K step of this block's B
  constexpr uint32_t R = kStackSlots;
  constexpr uint32_t kIdClear = make_idesc(256, kCoutPad);
  constexpr uint32_t kIdWin = make_idesc(256, 3 * kCoutPad);
  PairRowCtx<kNK> c;
  const uint64_t a_base = make_sdesc(0, 0, 128) | static_cast<uint64_t>(is.ring_base >> 4);
  const uint64_t b_desc0 = make_sdesc(is.w_base, kNHalf * 16, 128);
#pragma unroll
  for (int j = 0; j < kNK; ++j) {
    c.a_lo[j] = static_cast<uint32_t>(a_base + is.s_k[j]);
    c.b_lo[j] = static_cast<uint32_t>(b_desc0 + static_cast<uint64_t>(j) * kBStep16);
  }
  c.zero_desc = make_sdesc(is.zero_base, (kCoutPad / 2) * 16, 128);
  c.slot16 = a.slot_bytes >> 4;
  c.a_hi = static_cast<uint32_t>(a_base >> 32);
  c.b_hi = static_cast<uint32_t>(b_desc0 >> 32);
  c.tmem = is.tmem_base;
  c.full_u32 = smem_u32(is.full);
  c.done_u32 = smem_u32(is.done);
  c.free_u32 = smem_u32(is.slot_free);
  c.full = is.full;
  c.slot_free = is.slot_free;
  c.err = a.err;
  // input rows of this cluster's segments: rows + 2 each
  uint32_t total = 0;
  {
    PairSpan sp(a, cluster_id_x(), cluster_count_x());
    int n, pair, y0, y1;
    while (sp.next(a, n, pair, y0, y1)) total += static_cast<uint32_t>(y1 - y0 + 2 + pair_pad(y1 - y0));
  }
  if (a.ring != kRing) return;  // the host sizes the ring by pair_ring / kColsRing
  uint32_t ph = 0;   // input ring phase of slot 0 in the current period
  uint32_t pre = 0;  // next row's barriers found complete by the previous row: 1 = input, 2 = slot
  uint32_t g = 0;
  for (; g + 12u <= total; g += 12u, ph ^= pair_period_flip<kRing>())
    if (!pair_period<kFp8, kCoutPad, kNK, kRing>(c, ph, pre, std::make_integer_sequence<int, 12>{})) return;
  // the last rows (fewer than a period), with run-time positions
  RingPos in{0, ph};
  RingPos acc{0, 0};
  for (; g < total; ++g) {
    if (!(pre & 1u) && !wait_bar(&is.full[in.idx], in.phase, a.err, kErrWaitMma)) return;
    if (!(pre & 2u) && !wait_bar(&is.slot_free[acc.idx], acc.phase, a.err, kErrWaitMma)) return;
    tc_fence_after();
    uint64_t ad[kNK], bd[kNK];
    const uint32_t off = in.idx * c.slot16;
#pragma unroll
    for (int j = 0; j < kNK; ++j) {
      ad[j] = (static_cast<uint64_t>(c.a_hi) << 32) | (c.a_lo[j] + off);
      bd[j] = (static_cast<uint64_t>(c.b_hi) << 32) | c.b_lo[j];
    }
    const uint32_t start = acc.idx >= 2 ? acc.idx - 2 : acc.idx + R - 2;
    const uint32_t d_clear = c.tmem + acc.idx * kCoutPad;
    const uint32_t d_win = c.tmem + start * kCoutPad;
    RingPos nin = in;
    nin.advance(a.ring);
    RingPos nacc = acc;
    nacc.advance(R);
    const uint32_t nf = c.full_u32 + nin.idx * 8u;
    const uint32_t ns = c.free_u32 + nacc.idx * 8u;
    if (acc.idx < 2)
      pre = pair_row_head<kFp8, kNK, 2>(d_clear, d_clear + 6u * kCoutPad, c.zero_desc, kIdClear, d_win, kIdWin, nf,
                                        nin.phase, ns, nacc.phase, ad, bd);
    else
      pre = pair_row_head<kFp8, kNK, 1>(d_clear, d_clear, c.zero_desc, kIdClear, d_win, kIdWin, nf, nin.phase, ns,
                                        nacc.phase, ad, bd);
    pair_row_tail<kFp8, kNK>(d_win, kIdWin, c.done_u32 + in.idx * 8u, ad, bd);
    in.advance(a.ring);
    acc.advance(R);
  }
}

template <bool kFp8, int kCoutPad, int kEpi, int kOut>
__device__ __forceinline__ void conv3p_body(const ConvMaps& maps, const ConvArgs& a) {
  static_assert(kCoutPad == 16 || kCoutPad == 48 || kCoutPad == 64, "paired kernel: 16, 48 or 64 output channels");
  static_assert(kEpi != kEpiColsBias || (kCoutPad == 48 && !kFp8 && (kOut == kOutPixShuf2 || kOut == kOutPixShuf2Display)),
                "columns in N: FP16, 3 kernel columns x 16 channels, a pixel-shuffled output");
  static_assert(kStackBlocks * kCoutPad <= kStackTmemCols, "TMEM blocks");
  constexpr int kGroupWarps = PairShape<kCoutPad, kEpi, kFp8>::group_warps;
  constexpr uint32_t R = kStackSlots;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sw = smem;  // this block's half of B
  uint8_t* ring = smem + a.w_smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + a.ring * a.slot_bytes);
  uint64_t* full = bars;                    // block 0: both copies of an input row landed
  uint64_t* done = bars + a.ring;           // both blocks: the input row is consumed
  uint64_t* slot_free = bars + 2 * a.ring;  // block 0: both epilogues read the slot
  uint64_t* wbar = slot_free + R;           // this block's weights landed
  uint64_t* wpeer = wbar + 1;               // block 0: block 1's weights landed
  uint64_t* drain = wpeer + 1;              // both blocks: every MMA completed
  uint64_t* s_k = bars + 128;               // per K step of a row: (a_off >> 4) | (lbo >> 4) << 16
  // per-channel constants, 16-byte aligned (the epilogue reads them four at a time)
  // PReLU slopes (bias and scale are read from the parameter space, ConvArgs::cbias / cscale)
  float* s_slope = reinterpret_cast<float*>(s_k + kMaxKSteps + 2) + 2 * kMaxN;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(s_slope + kMaxN);
  uint8_t* zero_b = reinterpret_cast<uint8_t*>(bars) + kStackZeroOff;

  const uint32_t rank = cluster_rank();
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
    for (uint32_t i = 0; i < R; ++i) mbar_init(&slot_free[i], 2 * kGroupWarps);  // one group, both blocks
    mbar_init(wbar, 1);
    mbar_init(wpeer, 1);
    mbar_init(drain, 1);
    if constexpr (kEpi == kEpiColsBias)
      for (uint32_t i = 0; i < 6; ++i) mbar_init(&bars[kStackXchgBar + i], 4);  // the 4 warps of a group
    fence_mbar_init();
  }
  for (int j = threadIdx.x; j < kMaxN; j += blockDim.x) {
    s_slope[j] = (a.slope != nullptr && j < kCoutPad) ? a.slope[j] : 0.0f;
  }
  for (int j = threadIdx.x; j <= kMaxKSteps; j += blockDim.x)
    s_k[j] = j < a.n_ksteps
                 ? (static_cast<uint64_t>(a.ks[j].a_off >> 4) | (static_cast<uint64_t>(a.ks[j].lbo >> 4) << 16))
                 : 0;
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&maps.m[0]);
    if constexpr (kEpi == kEpiColsBias)
      for (int src = 1; src < 4; ++src) prefetch_tmap(&maps.m[src]);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, kStackTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  // both blocks' barriers are initialised before any remote arrive, pair copy or multicast commit
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const uint32_t half_w = a.wbytes / 2u;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ producer
      mbar_arrive_expect_tx(wbar, half_w);
      for (uint32_t off = 0; off < half_w; off += 32768u) {
        const uint32_t len = half_w - off < 32768u ? half_w - off : 32768u;
        bulk_load(sw + off, a.wpack + rank * half_w + off, len, wbar);
      }
      const uint32_t full0 = cluster_addr(smem_u32(full), 0);  // block 0's full[0]
      RingPos in{0, 0};
      bool ok = true;
      PairSpan sp(a, cluster_id_x(), cluster_count_x());
      int n, pair, y0, y1;
      while (ok && sp.next(a, n, pair, y0, y1)) {
        const int x0 = (2 * pair + static_cast<int>(rank)) * a.strip_w;
        const int last = y1 + pair_pad(y1 - y0);  // rows past y1: the padding entries' inputs
        for (int r = y0 - 1; r <= last; ++r) {
          if (!wait_bar(&done[in.idx], in.phase ^ 1u, a.err, kErrWaitProducer)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[in.idx], 2u * a.slot_bytes);
          // one box a source: 128 pixels from x0 - 1 (zero fill outside the image), all chunks
          if constexpr (kEpi == kEpiColsBias) {
#pragma unroll
            for (int src = 0; src < 4; ++src)
              tma_load_4d_pair(ring + in.idx * a.slot_bytes + src * a.src_bytes, &maps.m[src], full0 + in.idx * 8u,
                               (x0 - 1) * 2, 0, r, n);
          } else {
            tma_load_4d_pair(ring + in.idx * a.slot_bytes, &maps.m[0], full0 + in.idx * 8u, (x0 - 1) * 2, 0, r, n);
          }
          in.advance(a.ring);
        }
      }
      // every MMA (and so every copy it read) has completed before the pair may exit
      wait_bar(drain, 0, a.err, kErrWaitDrain);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      if (rank == 0) {
        // ---------------------------------------------------------------- MMA issuer (pair)
        if (wait_bar(wbar, 0, a.err, kErrWaitMma) && wait_bar(wpeer, 0, a.err, kErrWaitMma)) {
          const PairIssue is{a, smem_u32(ring), smem_u32(sw), smem_u32(zero_b), tmem_base, s_k, full, done, slot_free};
          // rows of K steps as the host admits them (conv_layer.cu pair_admits): 64 output channels
          // 12 or 3 in FP16, 6 in E4M3 (64 input channels); 48: 12 (FP16), 9, 5, 3 or 2
          if constexpr (kEpi == kEpiColsBias) {
            pair_issue<kFp8, kCoutPad, 12, kColsRing>(is);  // 4 sources x 3 channel pairs
          } else if constexpr (kCoutPad == 64 && kFp8) {
            pair_issue<kFp8, kCoutPad, 6>(is);
          } else if constexpr (kCoutPad == 64) {
            if (a.n_ksteps == 12) pair_issue<kFp8, kCoutPad, 12>(is);
            else pair_issue<kFp8, kCoutPad, 3>(is);
          } else {
            switch (a.n_ksteps) {
              case 12:
                if constexpr (!kFp8 && kCoutPad == 48) pair_issue<kFp8, kCoutPad, 12>(is);
                break;
              case 9: pair_issue<kFp8, kCoutPad, 9>(is); break;
              case 5: pair_issue<kFp8, kCoutPad, 5>(is); break;
              case 3: pair_issue<kFp8, kCoutPad, 3>(is); break;
              default: pair_issue<kFp8, kCoutPad, 2>(is); break;
            }
          }
        }
        mma_commit_pair(drain);
      } else if (wait_bar(wbar, 0, a.err, kErrWaitMma)) {
        mbar_arrive_remote(cluster_addr(smem_u32(wpeer), 0));  // block 1's half of B is in place
      }
    }
    __syncwarp();
  } else {
    // -------------------------------------------------------------------- epilogue
    // The groups of warps take the accumulator entries in turn (PairShape), so that many
    // rows are in the epilogue at once. A warp covers 32 lanes (pixels) x kCols columns of its
    // group's entries in 16-column steps; its residual words are loaded before it waits.
    constexpr int kCols = PairShape<kCoutPad, kEpi, kFp8>::warp_cols;
    constexpr int kSteps = kCols / 16;
    constexpr uint32_t kG = static_cast<uint32_t>(PairShape<kCoutPad, kEpi, kFp8>::groups);
    constexpr bool kResidual = kEpi == kEpiSpanAttn || kEpi == kEpiResPrelu;
    // slots 0 and 1 add their second TMEM block 16 columns at a time on the gated and residual shapes
    // (there a whole second block of live registers beside v and the residual words spilled: ptxas -v;
    // measured 3-9 % faster), and all at once elsewhere (one TMEM wait; 1-2 % faster there)
    constexpr bool kPieceAdd = kResidual || kEpi == kEpiColsBias;  // the column sum holds 48 values too
    const int ew = warp - 2;
    const uint32_t grp = static_cast<uint32_t>(ew / kGroupWarps);
    const int quad = warp & 3;
    const int col0 = ((ew % kGroupWarps) >> 2) * kCols;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t my_cols = tmem_base + lane_addr + static_cast<uint32_t>(col0);
    const uint32_t free0 = cluster_addr(smem_u32(slot_free), 0);  // block 0's slot_free[0]
    // the group's slots start free (phase 0 of slot_free); with the kernel columns in N, slot 4's
    // first phase is group 2's (below)
    if (lane == 0)
      for (uint32_t s = grp; s < R; s += kG)
        if (kEpi != kEpiColsBias || s != 4u) mbar_arrive_remote_relaxed(free0 + s * 8u);
    RingPos acc{0, 0};  // slot of the current entry
    RingPos in{0, 0};   // input ring position of the row that completes output row y (y + 2 of the band)
    uint32_t eg = 0;     // entry index modulo the group count
    bool ok = true;
    // kEpiColsBias: the group's exchange buffer in use (0 / 1) and the phase bit of each one's barrier
    uint32_t xbuf = 0, xph = 0;
    float* xchg = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + kStackXchgOff) + grp * (2u * 4u * 32u);
    // kEpiColsBias: the cluster's input rows (= entries, one each) and the current entry's index.
    // With a ring of 4 input slots a parity wait can pass falsely: waiting for the k-th completion
    // of a slot's `done` succeeds while completion k - 1 is still pending (same parity as "k done").
    // Entry e waits for input row e + 2; every group's previous wait (entry e - 3, row e - 1) has
    // already seen row e - 2, the slot's previous use, complete, except for a group's first entry:
    // group 2 starts at entry 2 (row 4, the second use of slot 0), so it first waits for row 0. That
    // wait could alias too if row 4 had completed as well, so row 4 is held back until it is done:
    // slot 4's first phase (entry 4, issued with row 4) is released by group 2 after the wait.
    uint32_t total_rows = 0, ent = 0;
    if constexpr (kEpi == kEpiColsBias) {
      PairSpan sp0(a, cluster_id_x(), cluster_count_x());
      int n0, p0, r0, r1;
      while (sp0.next(a, n0, p0, r0, r1)) total_rows += static_cast<uint32_t>(r1 - r0 + 2 + pair_pad(r1 - r0));
      static_assert(kColsRing == 4 && kStackSlots == 6, "the start-up order below covers 4 input and 6 accumulator slots");
      if (grp == 2u) {
        if (total_rows > 4u) {
          const bool got0 = wait_bar(&done[0], 0u, a.err, kErrWaitEpilogue);
          if (!__all_sync(0xffffffffu, got0)) ok = false;
        }
        if (lane == 0) mbar_arrive_remote_relaxed(free0 + 4u * 8u);
      }
    }
    PairSpan sp(a, cluster_id_x(), cluster_count_x());
    int n, pair, y0, y1;
    while (ok && sp.next(a, n, pair, y0, y1)) {
      const int m = quad * 32 + lane;
      // the strip column this lane writes: its own pixel, or with the kernel columns in N the pixel
      // of slot position m, one right of the slot's first (x0 - 1): lanes 0 and 127 write nothing
      const int xc = kEpi == kEpiColsBias ? m - 1 : m;
      const int x = (2 * pair + static_cast<int>(rank)) * a.strip_w + xc;
      const bool store = xc >= 0 && xc < a.strip_w && x < a.W;
      in.advance(a.ring);  // the band's input rows y0 - 1 and y0 complete no output row
      in.advance(a.ring);
      for (int y = y0; y < y1; ++y, acc.advance(R), in.advance(a.ring), eg = eg + 1 == kG ? 0 : eg + 1, ++ent) {
        if (eg != grp) continue;
        const uint32_t s = acc.idx;
        uint32_t res[kCols / 2];
        if constexpr (kResidual) {
          if (store) load_residual_words<kCols, kFp8>(a, n, y, x, col0, res);
        }
        const bool got = wait_bar(&done[in.idx], in.phase, a.err, kErrWaitEpilogue);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float v[kCols];
#pragma unroll
        for (int k = 0; k < kSteps; ++k) tmem_ld16(my_cols + s * kCoutPad + 16u * k, v + 16 * k);
        if (s < 2 && kPieceAdd) {  // slots 0 and 1: the part of the sum that landed in block 6 or 7
#pragma unroll
          for (int k = 0; k < kSteps; ++k) {
            float w[16];
            tmem_ld16(my_cols + (s + 6) * kCoutPad + 16u * k, w);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j) v[16 * k + j] += w[j];
          }
        } else if (s < 2) {
          float w[kCols];
#pragma unroll
          for (int k = 0; k < kSteps; ++k) tmem_ld16(my_cols + (s + 6) * kCoutPad + 16u * k, w + 16 * k);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < kCols; ++j) v[j] += w[j];
        } else {
          tmem_ld_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote_relaxed(free0 + s * 8u);
        if constexpr (kEpi == kEpiColsBias) {
          // out[c] = D[m - 1][c] + D[m][16 + c] + D[m + 1][32 + c]: neighbours within the warp by
          // shuffles; lanes 0 and 31 take theirs from the warps of the adjacent lane quadrants, which
          // process the same entry, through a shared buffer (two of them alternate, so a buffer is
          // rewritten only after all four warps passed the barrier of the other one)
          float* xb = xchg + xbuf * (4u * 32u);
          if (lane == 31) {
#pragma unroll
            for (int j = 0; j < 16; ++j) xb[quad * 32 + j] = v[j];
          }
          if (lane == 0) {
#pragma unroll
            for (int j = 0; j < 16; ++j) xb[quad * 32 + 16 + j] = v[32 + j];
          }
          __syncwarp();
          uint64_t* xbar = bars + kStackXchgBar + grp * 2u + xbuf;
          if (lane == 0) mbar_arrive(xbar);
          const bool xok = wait_bar(xbar, (xph >> xbuf) & 1u, a.err, kErrWaitEpilogue);
          if (!__all_sync(0xffffffffu, xok)) {
            ok = false;
            break;
          }
          xph ^= 1u << xbuf;
          xbuf ^= 1u;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float l = __shfl_up_sync(0xffffffffu, v[j], 1);
            float r = __shfl_down_sync(0xffffffffu, v[32 + j], 1);
            if (lane == 0) l = quad > 0 ? xb[(quad - 1) * 32 + j] : 0.0f;
            if (lane == 31) r = quad < 3 ? xb[(quad + 1) * 32 + 16 + j] : 0.0f;
            v[16 + j] += l + r;
          }
          if (store) {
            float* o = v + 16;
            if (y == 0 || y == a.H - 1 || x == 0 || x == a.W - 1) {
              // taps outside the image read zeros in the layer this conv stands for: drop their bias terms
#pragma unroll
              for (int t = 0; t < 9; ++t) {
                const int ky = t / 3, kx = t % 3;
                const bool outside =
                    (ky == 0 && y == 0) || (ky == 2 && y == a.H - 1) || (kx == 0 && x == 0) || (kx == 2 && x == a.W - 1);
                if (outside) {
#pragma unroll
                  for (int j = 0; j < 16; ++j) o[j] -= a.tap_bias[t][j];
                }
              }
            }
            epilogue_cols<kEpiBias, kOut, 16, kConstsBias>(a, a.cbias, a.cscale, s_slope, o, 0, n, y, x, 0, nullptr);
          }
        } else if (store) {
          // Bias and scale come from the parameter space (ConvArgs::cbias / cscale) at the warp's
          // first channel. Where a warp covers every channel that offset is 0; the FP16 48-channel
          // gates (three column groups) dispatch it as a compile-time offset too, so the constants
          // are operands of the epilogue's FMAs, with no loads and no registers held across rows
          // (the other multi-group shapes spill with three copies of the epilogue, and index them).
          // FP16 48- and 16-channel layers use the bias alone (their scale is the constant 1 or 1/2;
          // the 64-channel shapes keep both, which holds their spills to 8 bytes).
          constexpr int kGroups = kCoutPad / kCols;
          constexpr int kConsts = (kFp8 || kCoutPad == 64) ? kConstsAny : kConstsBias;
          auto epi = [&](auto first) {
            constexpr int c0 = decltype(first)::value;
            const int at = c0 < 0 ? col0 : c0;
            epilogue_cols<kEpi, kOut, kCols, kConsts>(a, a.cbias + at, a.cscale + at, s_slope + col0, v, 0, n, y, x,
                                                      col0, kResidual ? res : nullptr);
          };
          static_assert(kGroups >= 1 && kGroups <= 3, "one to three column groups a row");
          if constexpr (kGroups == 1) {
            epi(std::integral_constant<int, 0>{});
          } else if constexpr (kGroups == 3 && !kFp8) {
            if (col0 == 0)
              epi(std::integral_constant<int, 0>{});
            else if (col0 == kCols)
              epi(std::integral_constant<int, kCols>{});
            else
              epi(std::integral_constant<int, 2 * kCols>{});
          } else {
            epi(std::integral_constant<int, -1>{});  // runtime offset
          }
        }
      }
      if (!ok) break;
      // the segment's 2 + pad virtual entries (cleared by its input rows rows .. rows + 1 + pad):
      // nothing to read. The owning group frees each only after that input row is done, i.e. after
      // the issuer took the slot for it: a release before that would complete a second phase of the
      // slot's barrier and leave the issuer waiting on the wrong parity.
      const int virt = 2 + pair_pad(y1 - y0);
      RingPos vin = in;  // input row rows + 2 of the segment
      vin.retreat(a.ring);
      vin.retreat(a.ring);
      for (int k = 0; k < virt - 2; ++k) in.advance(a.ring);  // past the padding rows as well
      for (int k = 0; k < virt; ++k, acc.advance(R), vin.advance(a.ring), eg = eg + 1 == kG ? 0 : eg + 1, ++ent) {
        if (eg != grp) continue;
        bool got;
        if constexpr (kEpi == kEpiColsBias) {
          // With 4 input slots, row e + 4 reuses row e's slot as soon as entry e - 2 (another group)
          // is released, so `done` of row e may have completed twice by now and its parity would
          // alias. Row e + 2 (or the cluster's last row) is safe: its slot is next used by row e + 6,
          // which needs this entry's own slot, released only below.
          const uint32_t r = ent + 2u < total_rows ? ent + 2u : total_rows - 1u;
          got = wait_bar(&done[r % kColsRing], (r / kColsRing) & 1u, a.err, kErrWaitEpilogue);
        } else {
          got = wait_bar(&done[vin.idx], vin.phase, a.err, kErrWaitEpilogue);
        }
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        if (lane == 0) mbar_arrive_remote_relaxed(free0 + acc.idx * 8u);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no block leaves while the other's MMAs, copies or arrives may touch it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kStackTmemCols);
  }
}

// The kernel: one block of a cluster pair per SM, its register budget set by its thread count.
template <bool kFp8, int kCoutPad, int kEpi, int kOut>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairShape<kCoutPad, kEpi, kFp8>::threads, 1)
    conv3p_kernel(const __grid_constant__ ConvMaps maps, const __grid_constant__ ConvArgs a) {
  conv3p_body<kFp8, kCoutPad, kEpi, kOut>(maps, a);
}

}  // namespace kb2
