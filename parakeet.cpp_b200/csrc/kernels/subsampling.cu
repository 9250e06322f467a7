// dw_striding subsampling convolutions (reference: Subsampling::build_graph_batched,
// src/subsampling.cpp:48-240). The pointwise 1x1 convs and the output linear
// run on the tensor-core GEMM; these kernels are the two spatial convs.
//
// The reference zero-pads every utterance to T_max and multiplies each stage's
// input by a time mask (frames >= the stage's valid length -> 0) so that a
// short utterance equals its standalone run. Here each utterance stores only
// its valid frames, and any read outside [0, valid) x [0, F) is a zero: the
// same values with no padded work.
//
// Activation layout [frames, F, C] with the channel fastest, so that every
// thread moves 8 channels (16 bytes) and the pointwise convs are plain
// [frames*F, C] x [C, C] GEMMs.
#include "common.cuh"
#include "kernels.h"

namespace pkc {

namespace {

// conv.0: 1 -> C channels, 3x3, stride 2, pad 1, + bias, ReLU.
// One CTA = one output frame of one utterance, one thread per channel: the
// thread keeps its 9 taps in registers, the three input mel rows sit in shared
// memory, and each step over f writes C consecutive bf16 (coalesced).
// grid.x = sum of v1 over the batch (row -> utterance by binary search).
__global__ void __launch_bounds__(256)
    k_conv0(const float* __restrict__ logmel, int F, const float* __restrict__ w,
            const float* __restrict__ bias, int C, __nv_bfloat16* __restrict__ out, int F1,
            ItemTables t) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float rows[];  // [3][F + 2], zero padded on both sides
  const int row = blockIdx.x;
  int lo = 0, hi = t.B - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (t.v1_off[mid] <= row) lo = mid; else hi = mid - 1;
  }
  const int b = lo;
  const int tt = row - t.v1_off[b];
  const int valid = t.mel_valid[b];  // masked mel frames past this are zero
  const float* x = logmel + (size_t)t.mel_off[b] * F;
  for (int i = threadIdx.x; i < 3 * (F + 2); i += blockDim.x) {
    const int kh = i / (F + 2), fi = i % (F + 2) - 1;
    const int ti = 2 * tt - 1 + kh;
    rows[i] = (fi >= 0 && fi < F && ti >= 0 && ti < valid) ? x[(size_t)ti * F + fi] : 0.f;
  }
  __syncthreads();
  __nv_bfloat16* o = out + (size_t)row * F1 * C;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float wk[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) wk[k] = w[c * 9 + k];
    const float bc = bias[c];
    for (int f = 0; f < F1; ++f) {
      float s = bc;
#pragma unroll
      for (int kh = 0; kh < 3; ++kh)
#pragma unroll
        for (int kw = 0; kw < 3; ++kw) s = fmaf(wk[kh * 3 + kw], rows[kh * (F + 2) + 2 * f + kw], s);
      o[(size_t)f * C + c] = __float2bfloat16_rn(fmaxf(s, 0.f));
    }
  }
}

// depthwise 3x3 stride 2 pad 1 + bias (no activation: ReLU follows the pointwise conv)
__global__ void __launch_bounds__(256)
    k_dw3x3s2(const __nv_bfloat16* __restrict__ in, int F_in, const int* __restrict__ in_off,
              const int* __restrict__ in_valid, const float* __restrict__ w,
              const float* __restrict__ bias, int C, __nv_bfloat16* __restrict__ out, int F_out,
              const int* __restrict__ out_off, const int* __restrict__ out_valid) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.y;
  const int cg = C / 8;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int vo = out_valid[b];
  if (idx >= (long long)vo * F_out * cg) return;
  const int c0 = (int)(idx % cg) * 8;
  const long long pos = idx / cg;
  const int f = (int)(pos % F_out);
  const int tt = (int)(pos / F_out);
  const int vi = in_valid[b];
  const __nv_bfloat16* x = in + (size_t)in_off[b] * F_in * C;
  uint4 raw[9];
#pragma unroll
  for (int kh = 0; kh < 3; ++kh) {
    const int ti = 2 * tt - 1 + kh;
#pragma unroll
    for (int kw = 0; kw < 3; ++kw) {
      const int fi = 2 * f - 1 + kw;
      raw[kh * 3 + kw] = (ti >= 0 && ti < vi && fi >= 0 && fi < F_in)
                             ? *reinterpret_cast<const uint4*>(x + ((size_t)ti * F_in + fi) * C + c0)
                             : make_uint4(0, 0, 0, 0);
    }
  }
  const float4 b0 = *reinterpret_cast<const float4*>(bias + c0), b1 = *reinterpret_cast<const float4*>(bias + c0 + 4);
  float acc[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
  for (int k = 0; k < 9; ++k) {
    const float4 wa = *reinterpret_cast<const float4*>(w + k * C + c0);
    const float4 wb = *reinterpret_cast<const float4*>(w + k * C + c0 + 4);
    const float wk[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
    const __nv_bfloat16* hv = reinterpret_cast<const __nv_bfloat16*>(&raw[k]);
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = fmaf(wk[c], __bfloat162float(hv[c]), acc[c]);
  }
  uint4 o;
  o.x = pack2<__nv_bfloat16>(acc[0], acc[1]);
  o.y = pack2<__nv_bfloat16>(acc[2], acc[3]);
  o.z = pack2<__nv_bfloat16>(acc[4], acc[5]);
  o.w = pack2<__nv_bfloat16>(acc[6], acc[7]);
  *reinterpret_cast<uint4*>(out + (((size_t)out_off[b] + tt) * F_out + f) * C + c0) = o;
}

}  // namespace

cudaError_t sub_conv0_launch(const float* logmel, int F, const float* w, const float* b, int C,
                             __nv_bfloat16* out, int F1, const ItemTables& t, int total_v1,
                             cudaStream_t st) {
  if (t.B <= 0 || total_v1 <= 0) return cudaSuccess;
  const size_t smem = (size_t)3 * (F + 2) * sizeof(float);
  return launch_pdl(k_conv0, dim3(total_v1), dim3(256), smem, st, logmel, F, w, b, C, out, F1, t);
}

cudaError_t sub_dw_launch(const __nv_bfloat16* in, int F_in, const int* in_off, const int* in_valid,
                          const float* w, const float* b, int C, __nv_bfloat16* out, int F_out,
                          const int* out_off, const int* out_valid, int B, int max_out,
                          cudaStream_t st) {
  if (B <= 0 || max_out <= 0) return cudaSuccess;
  if (C % 8) return cudaErrorInvalidValue;
  const long long n = (long long)max_out * F_out * (C / 8);
  return launch_pdl(k_dw3x3s2, dim3((unsigned)((n + 255) / 256), B), dim3(256), 0, st, in, F_in, in_off, in_valid,
                    w, b, C, out, F_out, out_off, out_valid);
}

}  // namespace pkc
