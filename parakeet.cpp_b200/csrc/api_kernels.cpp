// Kernel-level C-ABI entry points (device pointers in, device pointers out).
// They exist so the parity tests can drive single kernels through the same
// shared library the encoder uses; the encoder itself calls the launchers
// directly (encoder.cpp).
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/pkc.h"
#include "kernels/gemm.h"
#include "status.hpp"

namespace {

// One device error word per device for the kernel-level entry points.
int* dev_err_word(int dev) {
  static std::mutex mu;
  static int* words[64] = {};
  std::lock_guard<std::mutex> lk(mu);
  if (dev < 0 || dev >= 64) return nullptr;
  if (!words[dev]) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    cudaMemset(p, 0, sizeof(int));
    words[dev] = p;
  }
  return words[dev];
}

}  // namespace

extern "C" pkc_status pkc_gemm(const void* A, int lda, const void* Bw, int ldb, int M, int N,
                               int K, int dtype, int epi, int act, float alpha, const float* bias,
                               void* out, int ldo, void* stream) {
  if (!A || !Bw || !out || M < 0 || N <= 0 || K <= 0 || (dtype != 0 && dtype != 1))
    return pkc::set_thread_error(PKC_ERR_ARG, "pkc_gemm: bad arguments");
  int dev = 0;
  cudaGetDevice(&dev);
  int* err = dev_err_word(dev);
  if (!err) return pkc::set_thread_error(PKC_ERR_CUDA, "pkc_gemm: error word allocation failed");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  pkc::GemmArgs a{};
  a.M = M; a.N = N; a.K = K;
  a.epi = epi; a.act = act; a.alpha = alpha; a.bias = bias;
  a.out = out; a.ldo = ldo; a.err = err;
  cudaError_t e = pkc::gemm_launch(A, lda, Bw, ldb, dtype == 1, a, st);
  if (e != cudaSuccess)
    return pkc::set_thread_error(PKC_ERR_CUDA, std::string("pkc_gemm: ") + cudaGetErrorString(e));
  int h_err = 0;
  if (cudaMemcpyAsync(&h_err, err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return pkc::set_thread_error(PKC_ERR_CUDA, "pkc_gemm: synchronize failed");
  if (h_err != 0) {
    cudaMemsetAsync(err, 0, sizeof(int), st);
    cudaStreamSynchronize(st);
    return pkc::set_thread_error(PKC_ERR_KERNEL,
                                 "pkc_gemm: kernel error word " + std::to_string(h_err));
  }
  return PKC_OK;
}

extern "C" int pkc_abi_version(void) { return PKC_ABI_VERSION; }
