// Kernel-level C-ABI entry points (device pointers in, device pointers out).
// They exist so the parity tests can drive single kernels through the same
// shared library the encoder uses; the encoder itself calls the launchers
// directly (encoder.cpp).
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "../../include/pkc.h"
#include "kernels/gemm.h"
#include "kernels/kernels.h"
#include <vector>
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

// Stream-K workspace for one kernel-level GEMM call, on the call's stream
// (these entry points synchronise before returning, so it is freed there).
struct SplitKScratch {
  float* ws = nullptr;
  int* flags = nullptr;
  cudaStream_t st = nullptr;
  bool attach(pkc::GemmArgs& a, int dev, cudaStream_t stream) {
    st = stream;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return false;
    const int pairs = sms / 2;
    if (cudaMallocAsync(reinterpret_cast<void**>(&ws), pkc::gemm_sk_ws_bytes(pairs), st) != cudaSuccess ||
        cudaMallocAsync(reinterpret_cast<void**>(&flags), pkc::gemm_sk_flag_count(pairs) * sizeof(int), st) !=
            cudaSuccess ||
        cudaMemsetAsync(flags, 0, pkc::gemm_sk_flag_count(pairs) * sizeof(int), st) != cudaSuccess)
      return false;
    a.sk_ws = ws;
    a.sk_flags = flags;
    a.sk_pairs = pairs;
    return true;
  }
  ~SplitKScratch() {
    if (ws) cudaFreeAsync(ws, st);
    if (flags) cudaFreeAsync(flags, st);
  }
};

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
  a.skinny = 1;  // M <= 16: the skinny kernel
  SplitKScratch sks;
  if (!sks.attach(a, dev, st)) return pkc::set_thread_error(PKC_ERR_OOM, "pkc_gemm: workspace allocation failed");
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

// launch, then read and clear the device error word
static pkc_status finish_kernel_call(cudaError_t e, int* err, cudaStream_t st, const char* what) {
  if (e != cudaSuccess) return pkc::set_thread_error(PKC_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  int h_err = 0;
  if (cudaMemcpyAsync(&h_err, err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return pkc::set_thread_error(PKC_ERR_CUDA, std::string(what) + ": synchronize failed");
  if (h_err != 0) {
    cudaMemsetAsync(err, 0, sizeof(int), st);
    cudaStreamSynchronize(st);
    return pkc::set_thread_error(PKC_ERR_KERNEL, std::string(what) + ": kernel error word " + std::to_string(h_err));
  }
  return PKC_OK;
}

extern "C" pkc_status pkc_gemm_split(const void* A, int lda, const void* Bw, int ldb, int M, int N, int Ks, int epi,
                                     int act, float alpha, const float* bias, void* out, int ldo, int ofmt,
                                     int split_ld, void* stream) {
  if (!A || !Bw || !out || M < 0 || N <= 0 || Ks <= 0 || epi < pkc::EPI_STORE_H || epi > pkc::EPI_GLU_H ||
      ofmt < pkc::OUT_H || ofmt > pkc::OUT_SPLIT)
    return pkc::set_thread_error(PKC_ERR_ARG, "pkc_gemm_split: bad arguments");
  int dev = 0;
  cudaGetDevice(&dev);
  int* err = dev_err_word(dev);
  if (!err) return pkc::set_thread_error(PKC_ERR_CUDA, "pkc_gemm_split: error word allocation failed");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  pkc::GemmArgs a{};
  a.M = M; a.N = N; a.K = 3 * Ks;
  a.epi = epi; a.act = act; a.alpha = alpha; a.bias = bias;
  a.out = out; a.ldo = ldo; a.err = err;
  a.split_k = Ks; a.ofmt = ofmt; a.split_ld = split_ld;
  return finish_kernel_call(pkc::gemm_launch(A, lda, Bw, ldb, false, a, st), err, st, "pkc_gemm_split");
}

extern "C" pkc_status pkc_gemm_resid_stats(const void* A, int lda, const void* Bw, int ldb, int M, int N,
                                           int K, int dtype, float alpha, const float* bias, float* x,
                                           int ldx, float* stats, void* stream) {
  if (!A || !Bw || !x || M < 0 || N <= 0 || K <= 0 || (dtype != 0 && dtype != 1) || N % 128 != 0)
    return pkc::set_thread_error(PKC_ERR_ARG, "pkc_gemm_resid_stats: bad arguments");
  int dev = 0;
  cudaGetDevice(&dev);
  int* err = dev_err_word(dev);
  if (!err) return pkc::set_thread_error(PKC_ERR_CUDA, "pkc_gemm_resid_stats: error word allocation failed");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  pkc::GemmArgs a{};
  a.M = M; a.N = N; a.K = K;
  a.epi = pkc::EPI_RESID_F32; a.act = pkc::ACT_NONE; a.alpha = alpha; a.bias = bias;
  a.out = x; a.ldo = ldx; a.err = err; a.stats = stats;
  SplitKScratch sks;
  if (!sks.attach(a, dev, st))
    return pkc::set_thread_error(PKC_ERR_OOM, "pkc_gemm_resid_stats: workspace allocation failed");
  return finish_kernel_call(pkc::gemm_launch(A, lda, Bw, ldb, dtype == 1, a, st), err, st, "pkc_gemm_resid_stats");
}

extern "C" pkc_status pkc_gemm_ln(const float* x, int ldx, const float* stats, const void* Bw, int ldb, int M,
                                  int N, int K, int dtype, int epi, int act, const float* bias, void* out, int ldo,
                                  void* stream) {
  if (!x || !stats || !Bw || !out || M < 0 || N <= 0 || K <= 0 ||
      (dtype != 0 && dtype != 1) || (epi != pkc::EPI_STORE_H && epi != pkc::EPI_GLU_H))
    return pkc::set_thread_error(PKC_ERR_ARG, "pkc_gemm_ln: bad arguments");
  int dev = 0;
  cudaGetDevice(&dev);
  int* err = dev_err_word(dev);
  if (!err) return pkc::set_thread_error(PKC_ERR_CUDA, "pkc_gemm_ln: error word allocation failed");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  pkc::GemmArgs a{};
  a.M = M; a.N = N; a.K = K;
  a.epi = epi; a.act = act; a.alpha = 1.f; a.bias = bias;
  a.out = out; a.ldo = ldo; a.err = err;
  const pkc::LnA la{x, ldx, stats};
  return finish_kernel_call(pkc::gemm_launch_ln(la, Bw, ldb, dtype == 1, a, st), err, st, "pkc_gemm_ln");
}

extern "C" int pkc_abi_version(void) { return PKC_ABI_VERSION; }

// Tables of one kernel-level attention call (offsets, lengths, tiles of `qt`
// query rows, error word) in a temporary device buffer, then the launch.
template <typename L>
static pkc_status attention_call(const char* what, const void* qkv, const void* ptab, int centre,
                                 const float* bias_u, const float* bias_v, const int* lens, int B, int d,
                                 int n_heads, void* ctx, void* stream, int qt, L launch) {
  if (!qkv || !ptab || !bias_u || !bias_v || !lens || B <= 0 || !ctx || n_heads <= 0)
    return pkc::set_thread_error(PKC_ERR_ARG, std::string(what) + ": bad arguments");
  std::vector<int> off(B + 1, 0), len(lens, lens + B), tiles;
  for (int b = 0; b < B; ++b) {
    if (len[b] <= 0 || len[b] > centre)
      return pkc::set_thread_error(PKC_ERR_ARG, std::string(what) + ": lens must be in [1, centre]");
    off[b + 1] = off[b] + len[b];
    for (int q0 = 0; q0 < len[b]; q0 += qt) {
      tiles.push_back(b);
      tiles.push_back(q0);
    }
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  std::vector<int> host;
  host.insert(host.end(), off.begin(), off.end());
  host.insert(host.end(), len.begin(), len.end());
  host.insert(host.end(), tiles.begin(), tiles.end());
  host.push_back(0);  // device error word
  int* dtab = nullptr;
  if (cudaMalloc(&dtab, host.size() * sizeof(int)) != cudaSuccess)
    return pkc::set_thread_error(PKC_ERR_OOM, std::string(what) + ": table allocation failed");
  cudaMemcpyAsync(dtab, host.data(), host.size() * sizeof(int), cudaMemcpyHostToDevice, st);
  int* derr = dtab + host.size() - 1;
  pkc::AttnArgs a{qkv, ptab, 2 * centre - 1, centre, d, bias_u, bias_v, dtab + 2 * B + 1,
                  (int)tiles.size() / 2, dtab, dtab + B + 1, ctx, d, n_heads, off[B], derr};
  cudaError_t e = launch(a, st);
  cudaError_t e2 = cudaStreamSynchronize(st);
  int h_err = 0;
  if (e == cudaSuccess && e2 == cudaSuccess) e2 = cudaMemcpy(&h_err, derr, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(dtab);
  if (e != cudaSuccess || e2 != cudaSuccess)
    return pkc::set_thread_error(PKC_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e != cudaSuccess ? e : e2));
  if (h_err != 0)
    return pkc::set_thread_error(PKC_ERR_KERNEL, std::string(what) + ": kernel error word " + std::to_string(h_err));
  return PKC_OK;
}

extern "C" pkc_status pkc_relpos_attention(const void* qkv, const void* ptab, int centre,
                                           const float* bias_u, const float* bias_v, const int* lens,
                                           int B, int d, int n_heads, int dtype, void* ctx,
                                           void* stream) {
  if (dtype != 0 && dtype != 1) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_relpos_attention: bad dtype");
  return attention_call("pkc_relpos_attention", qkv, ptab, centre, bias_u, bias_v, lens, B, d, n_heads, ctx, stream,
                        pkc::attn_query_tile(),
                        [&](const pkc::AttnArgs& a, cudaStream_t st) { return pkc::attention_launch(a, dtype == 1, st); });
}

extern "C" pkc_status pkc_relpos_attention_f32(const float* qkv, const float* ptab, int centre, const float* bias_u,
                                               const float* bias_v, const int* lens, int B, int d, int n_heads,
                                               void* ctx, void* stream) {
  return attention_call("pkc_relpos_attention_f32", qkv, ptab, centre, bias_u, bias_v, lens, B, d, n_heads, ctx, stream,
                        pkc::attn_f32_query_tile(),
                        [](const pkc::AttnArgs& a, cudaStream_t st) { return pkc::attention_f32_launch(a, st); });
}

extern "C" pkc_status pkc_conv_depthwise(const void* in, const int* lens, int B, int d, int K, const float* w,
                                         const float* bias, const float* scale, const float* shift, int dtype,
                                         void* out, void* stream) {
  if (!in || !lens || B <= 0 || !w || !scale || !shift || !out || (dtype != 0 && dtype != 1))
    return pkc::set_thread_error(PKC_ERR_ARG, "pkc_conv_depthwise: bad arguments");
  std::vector<int> host(2 * B + 1, 0);  // [off | len]
  int max_len = 0;
  for (int b = 0; b < B; ++b) {
    if (lens[b] < 0) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_conv_depthwise: negative length");
    host[b + 1] = host[b] + lens[b];
    host[B + 1 + b] = lens[b];
    max_len = std::max(max_len, lens[b]);
  }
  if (host[B] == 0) return PKC_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int* dtab = nullptr;
  if (cudaMalloc(&dtab, host.size() * sizeof(int)) != cudaSuccess)
    return pkc::set_thread_error(PKC_ERR_OOM, "pkc_conv_depthwise: table allocation failed");
  cudaMemcpyAsync(dtab, host.data(), host.size() * sizeof(int), cudaMemcpyHostToDevice, st);
  cudaError_t e = pkc::dwconv_bn_silu_launch(in, out, d, K, w, bias, scale, shift, dtab, dtab + B + 1, B, max_len,
                                             dtype == 1, st);
  cudaError_t e2 = cudaStreamSynchronize(st);
  cudaFree(dtab);
  if (e != cudaSuccess || e2 != cudaSuccess)
    return pkc::set_thread_error(PKC_ERR_CUDA, std::string("pkc_conv_depthwise: ") +
                                                   cudaGetErrorString(e != cudaSuccess ? e : e2));
  return PKC_OK;
}
