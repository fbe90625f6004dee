// Self-test of the bounded device wait (kb2_selftest_bounded_wait): one thread waits on an mbarrier
// that nothing arrives on, through the same wait_bar() every pipeline of this library uses. The wait
// gives up after its %globaltimer limit, records kErrWaitSelftest in the error word and returns;
// the kernel then ends normally, so the context stays usable. No trap, no fault: the failure is a
// flag that nothing sets.
#include "engine.h"
#include "tc_common.cuh"

namespace kb2 {

namespace {

__global__ void selftest_wait_kernel(int* err, unsigned long long* waited_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_mbar_init();
  const unsigned long long t0 = globaltimer();
  const bool ok = wait_bar(&bar, 0, err, kErrWaitSelftest);  // phase 0 never completes
  *waited_ns = globaltimer() - t0;
  if (ok) atomicCAS(err, 0, -1);  // cannot happen: nothing arrived
}

}  // namespace

Status selftest_bounded_wait(int device, int32_t* code, double* waited_s) {
  int count = 0;
  KB2_CUDA(cudaGetDeviceCount(&count));
  if (device < 0 || device >= count) return refuse(KB2_INPUT_MISMATCH, "no such CUDA device");
  KB2_CUDA(cudaSetDevice(device));
  DeviceBuffer words;
  KB2_TRY(words.alloc(16));
  KB2_CUDA(cudaMemset(words.ptr, 0, 16));
  int* err = words.as<int>();
  auto* ns = reinterpret_cast<unsigned long long*>(words.as<uint8_t>() + 8);
  selftest_wait_kernel<<<1, 32>>>(err, ns);
  KB2_CUDA(cudaGetLastError());
  KB2_CUDA(cudaDeviceSynchronize());
  int word = 0;
  unsigned long long t = 0;
  KB2_CUDA(cudaMemcpy(&word, err, sizeof(int), cudaMemcpyDeviceToHost));
  KB2_CUDA(cudaMemcpy(&t, ns, sizeof(t), cudaMemcpyDeviceToHost));
  if (code != nullptr) *code = word;
  if (waited_s != nullptr) *waited_s = static_cast<double>(t) * 1e-9;
  if (word != 0) return refuse(KB2_KERNEL_TIMEOUT, "self-test wait gave up (code " + std::to_string(word) + ")");
  return refuse(KB2_VENDOR_CALL_FAILED, "self-test wait did not give up");
}

}  // namespace kb2
