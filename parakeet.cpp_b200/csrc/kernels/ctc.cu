// CTC head on the GPU (reference: CTCDecoder::forward, src/ctc_decoder.cpp:35-116,
// a 1x1 conv d -> V+1 with bias, then log_softmax over the V+1 classes; the
// greedy fold of src/search.cpp:21-90 runs on the host from the per-frame
// argmax and maximum log-probability written here).
//
// The head's weight is f32 in every GGUF (src/ctc_decoder.cpp:78), and the
// greedy decision is an argmax, so the logits are computed to ~22 bits: the
// encoder output x and the weight W are each split into f16 hi + lo parts and
// the tcgen05 GEMM contracts [x_hi | x_hi | x_lo] with [W_hi | W_lo | W_hi]
// (K = 3d), i.e. x_hi W_hi + x_hi W_lo + x_lo W_hi with f32 accumulation.
//
//   k_split3     x f32 [M, d] -> [x_hi | x_hi | x_lo] f16 [M, 3d]
//   (GEMM)       logits f32 [M, Vpad] = A W^T + b (EPI_STORE_F32)
//   k_ctc_rows   per frame: max, argmax (lowest index on ties), log-sum-exp
//                over the V+1 real classes; optionally the log-probabilities
#include "common.cuh"
#include "kernels.h"

namespace pkc {

namespace {

__global__ void k_split3(const float* __restrict__ x, int M, int d, __half* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // one float4 of x
  const int q = d / 4;
  if (i >= (long long)M * q) return;
  const int row = (int)(i / q), c = (int)(i % q) * 4;
  const float4 v = *reinterpret_cast<const float4*>(x + (size_t)row * d + c);
  const __half h0 = __float2half_rn(v.x), h1 = __float2half_rn(v.y), h2 = __float2half_rn(v.z),
               h3 = __float2half_rn(v.w);
  const __half l0 = __float2half_rn(v.x - __half2float(h0)), l1 = __float2half_rn(v.y - __half2float(h1)),
               l2 = __float2half_rn(v.z - __half2float(h2)), l3 = __float2half_rn(v.w - __half2float(h3));
  __half* o = out + (size_t)row * 3 * d + c;
  const __half2 hi01 = __halves2half2(h0, h1), hi23 = __halves2half2(h2, h3);
  const __half2 lo01 = __halves2half2(l0, l1), lo23 = __halves2half2(l2, l3);
  uint2 hi, lo;
  hi.x = *reinterpret_cast<const uint32_t*>(&hi01);
  hi.y = *reinterpret_cast<const uint32_t*>(&hi23);
  lo.x = *reinterpret_cast<const uint32_t*>(&lo01);
  lo.y = *reinterpret_cast<const uint32_t*>(&lo23);
  *reinterpret_cast<uint2*>(o) = hi;
  *reinterpret_cast<uint2*>(o + d) = hi;
  *reinterpret_cast<uint2*>(o + 2 * d) = lo;
}

// One warp per frame. Lane l scans classes l, l+32, ...; the (value, index)
// reduction keeps the larger value and, on equal values, the lower index --
// the first maximum, as the reference's argmax loop (src/search.cpp:57-62).
constexpr int ROWS_PER_CTA = 8;

__global__ void __launch_bounds__(32 * ROWS_PER_CTA)
    k_ctc_rows(const float* __restrict__ logits, int M, int ld, int V1, int* __restrict__ argmax,
               float* __restrict__ maxlp, float* __restrict__ logprobs) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x * ROWS_PER_CTA + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const float* l = logits + (size_t)row * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int v = lane; v < V1; v += 32) {
    const float x = l[v];
    if (x > best) {  // strictly greater: a lane keeps its first maximum
      best = x;
      bi = v;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) {
      best = ob;
      bi = oi;
    }
  }
  float s = 0.f;
  for (int v = lane; v < V1; v += 32) s += __expf(l[v] - best);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float lse = logf(s);  // log-softmax(v) = l[v] - best - lse
  if (lane == 0) {
    argmax[row] = bi;
    maxlp[row] = -lse;
  }
  if (logprobs) {
    float* out = logprobs + (size_t)row * V1;
    for (int v = lane; v < V1; v += 32) out[v] = l[v] - best - lse;
  }
}

}  // namespace

cudaError_t ctc_split3_launch(const float* x, int M, int d, void* out, cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  if (d % 4 != 0) return cudaErrorInvalidValue;
  const long long n = (long long)M * (d / 4);
  return launch_pdl(k_split3, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, x, M, d,
                    static_cast<__half*>(out));
}

cudaError_t ctc_rows_launch(const float* logits, int M, int ld, int V1, int* argmax, float* maxlp, float* logprobs,
                            cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  if (V1 <= 0 || V1 > ld) return cudaErrorInvalidValue;
  return launch_pdl(k_ctc_rows, dim3((M + ROWS_PER_CTA - 1) / ROWS_PER_CTA), dim3(32 * ROWS_PER_CTA), 0, st,
                    logits, M, ld, V1, argmax, maxlp, logprobs);
}

}  // namespace pkc
