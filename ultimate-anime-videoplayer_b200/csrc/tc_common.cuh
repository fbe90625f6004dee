// sm_100a building blocks written as inline PTX: mbarriers with bounded waits, TMA tensor and bulk
// copies, TMEM allocation, tcgen05 MMA / commit / load, and the UMMA shared-memory and instruction
// descriptors. Every wait in this library goes through wait_bar(): it gives up after kWaitNs of
// %globaltimer time, records where in the error word and returns false, so a stuck pipeline ends
// the kernel with an error status instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace kb2 {

// Error word codes (device side). The host reads the word after a synchronisation.
enum DeviceError : int {
  kErrNone = 0,
  kErrWaitProducer = 0x100,  // producer waited too long for a free slot
  kErrWaitMma = 0x200,       // MMA issuer waited too long for data or a free accumulator
  kErrWaitEpilogue = 0x300,  // epilogue waited too long for an accumulator
  kErrWaitDrain = 0x400,     // end-of-kernel drain of copies / MMAs in flight timed out
  kErrWaitSelftest = 0x500,  // kb2_selftest_bounded_wait: a wait on a barrier that nothing completes
};

constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase of `parity` to complete. False: timed out (the error word now holds `code`)
// or another block already failed (error word non-zero).
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t spin = 0;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 63u) == 63u) {
      if (*reinterpret_cast<volatile int*>(err) != 0) return false;
      if (globaltimer() - t0 > kWaitNs) {
        atomicCAS(err, 0, code);
        return false;
      }
    }
  }
}

// Position in a ring of mbarrier-guarded slots: index and phase parity, advanced by one slot at a
// time (no integer division on the issuing threads).
struct RingPos {
  uint32_t idx, phase;
  __device__ __forceinline__ void advance(uint32_t n) {
    if (++idx == n) {
      idx = 0;
      phase ^= 1u;
    }
  }
  __device__ __forceinline__ void retreat(uint32_t n) {
    if (idx == 0) {
      idx = n - 1;
      phase ^= 1u;
    } else {
      --idx;
    }
  }
};

// ---------------------------------------------------------------- TMA / bulk copies
__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// Untiled bulk copy global -> shared; both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Makes this thread's generic-proxy shared-memory writes visible to the async proxy (TMA, tensor core).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- TMEM / tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, A: M x K, B: N x K, both K-major.
template <bool kFp8>
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  if constexpr (kFp8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// kN accumulating MMAs into one accumulator, issued from a single asm block: MMA j multiplies A
// descriptor a[j] by B descriptor b[j]. The issuing thread executes nothing between consecutive
// tcgen05.mma instructions; measured on B200 (M = 128, N = 144, K = 16), 9 MMAs issued this way run
// at the tensor rate (73 cycles each), while a loop with one branch per MMA costs 132.
template <bool kFp8, int kN>
__device__ __forceinline__ void mma_ss_block(uint32_t d_tmem, const uint64_t (&a)[9], const uint64_t (&b)[9],
                                             uint32_t idesc) {
  static_assert(kN >= 1 && kN <= 9, "1..9 MMAs");
  if constexpr (kFp8) {
      if constexpr (kN == 1) {
        asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, %20, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %10, %19, acc;\n\t"
          "}\n" ::"r"(d_tmem),
          "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
          "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8]),
          "r"(idesc), "r"(1u)
          : "memory");
      } else if constexpr (kN == 2) {
        asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, %20, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %10, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %2, %11, %19, acc;\n\t"
          "}\n" ::"r"(d_tmem),
          "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
          "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8]),
          "r"(idesc), "r"(1u)
          : "memory");
      } else if constexpr (kN == 3) {
        asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, %20, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %10, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %2, %11, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %3, %12, %19, acc;\n\t"
          "}\n" ::"r"(d_tmem),
          "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
          "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8]),
          "r"(idesc), "r"(1u)
          : "memory");
      } else if constexpr (kN == 4) {
        asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, %20, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %10, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %2, %11, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %3, %12, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %4, %13, %19, acc;\n\t"
          "}\n" ::"r"(d_tmem),
          "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
          "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8]),
          "r"(idesc), "r"(1u)
          : "memory");
      } else if constexpr (kN == 5) {
        asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, %20, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %10, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %2, %11, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %3, %12, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %4, %13, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %5, %14, %19, acc;\n\t"
          "}\n" ::"r"(d_tmem),
          "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
          "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8]),
          "r"(idesc), "r"(1u)
          : "memory");
      } else if constexpr (kN == 6) {
        asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, %20, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %10, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %2, %11, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %3, %12, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %4, %13, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %5, %14, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %6, %15, %19, acc;\n\t"
          "}\n" ::"r"(d_tmem),
          "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
          "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8]),
          "r"(idesc), "r"(1u)
          : "memory");
      } else if constexpr (kN == 7) {
        asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, %20, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %10, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %2, %11, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %3, %12, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %4, %13, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %5, %14, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %6, %15, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %7, %16, %19, acc;\n\t"
          "}\n" ::"r"(d_tmem),
          "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
          "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8]),
          "r"(idesc), "r"(1u)
          : "memory");
      } else if constexpr (kN == 8) {
        asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, %20, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %10, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %2, %11, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %3, %12, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %4, %13, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %5, %14, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %6, %15, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %7, %16, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %8, %17, %19, acc;\n\t"
          "}\n" ::"r"(d_tmem),
          "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
          "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8]),
          "r"(idesc), "r"(1u)
          : "memory");
      } else if constexpr (kN == 9) {
        asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, %20, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %10, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %2, %11, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %3, %12, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %4, %13, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %5, %14, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %6, %15, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %7, %16, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %8, %17, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %9, %18, %19, acc;\n\t"
          "}\n" ::"r"(d_tmem),
          "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
          "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8]),
          "r"(idesc), "r"(1u)
          : "memory");
      }
  } else {
      if constexpr (kN == 1) {
        asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, %20, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %10, %19, acc;\n\t"
          "}\n" ::"r"(d_tmem),
          "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
          "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8]),
          "r"(idesc), "r"(1u)
          : "memory");
      } else if constexpr (kN == 2) {
        asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, %20, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %10, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %11, %19, acc;\n\t"
          "}\n" ::"r"(d_tmem),
          "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
          "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8]),
          "r"(idesc), "r"(1u)
          : "memory");
      } else if constexpr (kN == 3) {
        asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, %20, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %10, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %11, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %12, %19, acc;\n\t"
          "}\n" ::"r"(d_tmem),
          "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
          "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8]),
          "r"(idesc), "r"(1u)
          : "memory");
      } else if constexpr (kN == 4) {
        asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, %20, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %10, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %11, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %12, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %13, %19, acc;\n\t"
          "}\n" ::"r"(d_tmem),
          "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
          "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8]),
          "r"(idesc), "r"(1u)
          : "memory");
      } else if constexpr (kN == 5) {
        asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, %20, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %10, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %11, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %12, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %13, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %5, %14, %19, acc;\n\t"
          "}\n" ::"r"(d_tmem),
          "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
          "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8]),
          "r"(idesc), "r"(1u)
          : "memory");
      } else if constexpr (kN == 6) {
        asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, %20, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %10, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %11, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %12, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %13, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %5, %14, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %6, %15, %19, acc;\n\t"
          "}\n" ::"r"(d_tmem),
          "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
          "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8]),
          "r"(idesc), "r"(1u)
          : "memory");
      } else if constexpr (kN == 7) {
        asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, %20, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %10, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %11, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %12, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %13, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %5, %14, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %6, %15, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %7, %16, %19, acc;\n\t"
          "}\n" ::"r"(d_tmem),
          "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
          "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8]),
          "r"(idesc), "r"(1u)
          : "memory");
      } else if constexpr (kN == 8) {
        asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, %20, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %10, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %11, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %12, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %13, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %5, %14, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %6, %15, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %7, %16, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %8, %17, %19, acc;\n\t"
          "}\n" ::"r"(d_tmem),
          "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
          "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8]),
          "r"(idesc), "r"(1u)
          : "memory");
      } else if constexpr (kN == 9) {
        asm volatile(
          "{\n\t.reg .pred acc;\n\t"
          "setp.ne.b32 acc, %20, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %10, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %11, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %12, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %13, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %5, %14, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %6, %15, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %7, %16, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %8, %17, %19, acc;\n\t"
          "tcgen05.mma.cta_group::1.kind::f16 [%0], %9, %18, %19, acc;\n\t"
          "}\n" ::"r"(d_tmem),
          "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(a[8]),
          "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "l"(b[8]),
          "r"(idesc), "r"(1u)
          : "memory");
      }
  }
}

// n (1..9, runtime) accumulating MMAs: one branch to the matching block, none between MMAs.
template <bool kFp8>
__device__ __forceinline__ void mma_ss_row(uint32_t d_tmem, const uint64_t (&a)[9], const uint64_t (&b)[9],
                                           uint32_t idesc, int n) {
  switch (n) {
    case 1: mma_ss_block<kFp8, 1>(d_tmem, a, b, idesc); break;
    case 2: mma_ss_block<kFp8, 2>(d_tmem, a, b, idesc); break;
    case 3: mma_ss_block<kFp8, 3>(d_tmem, a, b, idesc); break;
    case 4: mma_ss_block<kFp8, 4>(d_tmem, a, b, idesc); break;
    case 5: mma_ss_block<kFp8, 5>(d_tmem, a, b, idesc); break;
    case 6: mma_ss_block<kFp8, 6>(d_tmem, a, b, idesc); break;
    case 7: mma_ss_block<kFp8, 7>(d_tmem, a, b, idesc); break;
    case 8: mma_ss_block<kFp8, 8>(d_tmem, a, b, idesc); break;
    default: mma_ss_block<kFp8, 9>(d_tmem, a, b, idesc); break;
  }
}

// D[tmem] (+)= A[tmem] * B[smem]^T: A (M x K) held in TMEM, lane = row.
template <bool kFp8>
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  if constexpr (kFp8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// Shared memory -> TMEM copy of a 128-row x 32-byte K-major tile (described like an MMA operand)
// into 128 lanes x 8 columns.
__device__ __forceinline__ void tmem_cp_128x256b(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Arrives once on `bar` when every tcgen05 operation issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// 32 lanes x 32 bits, 8 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
// 32 lanes x 32 bits, 16 consecutive columns per thread, all zero.
__device__ __forceinline__ void tmem_st16_zero(uint32_t taddr) {
  const uint32_t z = 0;
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
      "%1, %1};" ::"r"(taddr),
      "r"(z)
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// UMMA shared-memory descriptor, no swizzle (canonical K-major "interleaved" layout): 8-row core
// matrices of 16 bytes per row; `sbo` = byte distance between 8-row groups along M/N, `lbo` =
// byte distance between the two 16-byte K halves of one instruction. Version field = 1 (sm_100).
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  return d;
}

// Instruction descriptor: D = F32, A = B = F16 (kind::f16) or E4M3 (kind::f8f6f4), both K-major.
__host__ __device__ constexpr uint32_t make_idesc(int m, int n) {
  return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// ---------------------------------------------------------------- small numeric helpers
// tanh on the special-function unit (tanh.approx.f32: one MUFU operation, max relative error about
// 2^-11); used through sigmoid(v) = 0.5 * tanh(v / 2) + 0.5 so a sigmoid costs one MUFU operation
// instead of two (exponential + reciprocal). Results are stored as FP16 or E4M3.
__device__ __forceinline__ float tanh_approx(float v) {
  float r;
  asm("tanh.approx.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}
// sigmoid(v) - 0.5
__device__ __forceinline__ float sigmoid_centered(float v) { return 0.5f * tanh_approx(0.5f * v); }
__device__ __forceinline__ float sigmoidf_fast(float v) { return fmaf(0.5f, tanh_approx(0.5f * v), 0.5f); }

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint16_t pack_e4m3x2(float a, float b) {
  return static_cast<uint16_t>(__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3));
}
__device__ __forceinline__ float2 unpack_e4m3x2(uint16_t v) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(v), __NV_E4M3);
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}
__device__ __forceinline__ float2 unpack_half2(uint32_t v) {
  return __half22float2(*reinterpret_cast<const __half2*>(&v));
}

}  // namespace kb2
