// Diagnostic kernel of the failure detection: every wait in this library's
// kernels (on an mbarrier, or on a flag another CTA sets) is bounded by
// %globaltimer and, when it runs out, records a code in the device error word
// and lets the kernel return, so a stuck pipeline becomes PKC_ERR_KERNEL on
// the host instead of a hung GPU. This kernel runs those same wait helpers
// (common.cuh: mbar_wait, wait_flag_gpu) on conditions that never come true
// -- an mbarrier nobody arrives on, a global flag nobody sets -- with a short
// limit, so a test can watch the bound expire and the context stay usable.
#include <cuda_runtime.h>

#include <string>

#include "../../../include/pkc.h"
#include "../status.hpp"
#include "common.cuh"

namespace pkc {
namespace {

__global__ void k_bounded_wait_check(int kind, const int* flag, unsigned long long limit_ns, int* err) {
  __shared__ uint64_t bar;
  if (kind == 0) {
    if (threadIdx.x == 0) {
      mbar_init(smem_u32(&bar), 1);
      fence_barrier_init();
    }
    __syncthreads();
    // phase 0 never completes: no thread arrives
    (void)__all_sync(0xffffffffu, mbar_wait(smem_u32(&bar), 0, err, DEV_ERR_TIMEOUT_CHECK, limit_ns) ? 1 : 0);
  } else if (threadIdx.x == 0) {
    wait_flag_gpu(flag, err, DEV_ERR_TIMEOUT_CHECK, limit_ns);  // the flag stays zero
  }
}

}  // namespace
}  // namespace pkc

extern "C" pkc_status pkc_bounded_wait_check(int kind, double limit_ms, int* error_code) {
  using namespace pkc;
  if ((kind != 0 && kind != 1) || !(limit_ms > 0.0) || limit_ms > 2000.0 || !error_code)
    return set_thread_error(PKC_ERR_ARG, "pkc_bounded_wait_check: kind 0 or 1, 0 < limit_ms <= 2000");
  *error_code = 0;
  int* words = nullptr;  // [0] error word, [1] the flag that nobody sets
  if (cudaMalloc(&words, 2 * sizeof(int)) != cudaSuccess)
    return set_thread_error(PKC_ERR_OOM, "pkc_bounded_wait_check: allocation failed");
  cudaError_t e = cudaMemset(words, 0, 2 * sizeof(int));
  if (e == cudaSuccess) {
    k_bounded_wait_check<<<1, 32>>>(kind, words + 1, (unsigned long long)(limit_ms * 1e6), words);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  int code = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&code, words, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(words);
  if (e != cudaSuccess)
    return set_thread_error(PKC_ERR_CUDA, std::string("pkc_bounded_wait_check: ") + cudaGetErrorString(e));
  *error_code = code;
  if (code != 0)
    return set_thread_error(PKC_ERR_KERNEL, "pkc_bounded_wait_check: bounded wait ran out (error word " +
                                                std::to_string(code) + ")");
  return PKC_OK;
}
