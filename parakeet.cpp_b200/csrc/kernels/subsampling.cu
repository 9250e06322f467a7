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
#include "per_device.h"

namespace pkc {

namespace {

// conv.0: 1 -> C channels, 3x3, stride 2, pad 1, + bias, ReLU.
// One CTA = one output frame of one utterance, one thread per channel: the
// thread keeps its 9 taps in registers, the three input mel rows sit in shared
// memory, and each step over f writes C consecutive bf16 (coalesced).
// grid.x = sum of v1 over the batch (row -> utterance by binary search).
__device__ __forceinline__ void store_act(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
__device__ __forceinline__ void store_act(float* p, float v) { *p = v; }

// O: bf16 (the f16 / bf16 compute path) or f32 (the f32-accurate path)
template <typename O>
__global__ void __launch_bounds__(256)
    k_conv0(const float* __restrict__ logmel, int F, const float* __restrict__ w,
            const float* __restrict__ bias, int C, O* __restrict__ out, int F1,
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
  O* o = out + (size_t)row * F1 * C;
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
      store_act(o + (size_t)f * C + c, fmaxf(s, 0.f));
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

// ---------------------------------------------------------------------------
// Stage 1 fused: conv.0 (1 -> C, 3x3, s2, p1) + bias + ReLU, then the first
// depthwise 3x3 s2 p1 + bias, without the C-channel conv.0 map (v1 x F1 x C,
// the largest tensor of the encoder) ever reaching memory.
//
// One CTA = S1_T2 consecutive stage-2 frames of one utterance x S1_CG
// channels. It needs conv.0 rows t1 = 2 t2_0 - 1 ... 2 (t2_0 + S1_T2) - 1
// (S1_ROWS of them) and mel rows 4 t2_0 - 3 ... (S1_MROWS):
//  1. the mel rows go to shared memory (zeros outside the utterance's valid
//     frames and outside [0, F));
//  2. conv.0 runs on the tensor cores as [positions x 16] x [16 x channels]
//     (the 9 taps, zero-padded to K = 16; f16 operands, f32 accumulation,
//     mma.sync m16n8k16 -- K = 9 is far too small for a tcgen05 tile), and
//     bias + ReLU go into a bf16 tile in shared memory: rows outside
//     [0, v1) are zero, which is the reference's stage-2 input mask;
//  3. the depthwise conv reads that tile and writes stage-2 frames (bf16).
// The bf16 tile matches the rounding of the unfused path, where the conv.0
// map is stored in bf16.
constexpr int S1_T2 = 4;
constexpr int S1_CG = 64;
constexpr int S1_ROWS = 2 * S1_T2 + 1;
constexpr int S1_MROWS = 4 * S1_T2 + 3;
constexpr int S1_THREADS = 256;

// relu(a), relu(b) rounded to bf16 and packed (a in the low half), one instruction
__device__ __forceinline__ uint32_t pack_relu_bf16(float a, float b) {
  uint32_t d;
  asm("cvt.rn.relu.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(b), "f"(a));
  return d;
}
// two bf16 (low, high halves of u) as the two f32 lanes of a 64-bit register
__device__ __forceinline__ uint64_t bf2_to_f2(uint32_t u) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(u << 16), "r"(u & 0xffff0000u));
  return d;
}
__device__ __forceinline__ uint32_t f2_to_bf2(uint64_t v) {
  const float2 f = f2_unpack(v);
  return pack2<__nv_bfloat16>(f.x, f.y);
}

__device__ __forceinline__ void mma16816_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int F1>
__global__ void __launch_bounds__(S1_THREADS)
    k_sub_stage1(const float* __restrict__ logmel, int F, const float* __restrict__ w0,
                 const float* __restrict__ b0, const float* __restrict__ w1, const float* __restrict__ b1,
                 int C, __nv_bfloat16* __restrict__ out, ItemTables t) {
  constexpr int F2 = (F1 - 1) / 2 + 1;
  constexpr int NP = S1_ROWS * F1;          // conv.0 positions in the tile
  constexpr int MT = (NP + 15) / 16;        // 16-position MMA tiles
  constexpr int NT = S1_CG / 8;             // 8-channel MMA tiles
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int b = blockIdx.y;
  const int t2_0 = blockIdx.x * S1_T2;
  const int v2b = t.v2[b];
  if (t2_0 >= v2b) return;
  const int cg0 = blockIdx.z * S1_CG;
  const int v1b = t.v1[b], mvalid = t.mel_valid[b];
  const float* mel = logmel + (size_t)t.mel_off[b] * F;
  const int t1_0 = 2 * t2_0 - 1;
  const int tm_0 = 2 * t1_0 - 1;
  const int FP = F + 2;                      // padded mel row
  float* melt = reinterpret_cast<float*>(smem_raw);                              // [S1_MROWS][FP]
  uint8_t* s1 = smem_raw + (((size_t)S1_MROWS * FP * 4 + 127) / 128) * 128;      // [S1_ROWS*F1][S1_CG] bf16
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // 1. mel rows: thread tid owns padded column tid (FP <= S1_THREADS, checked
  //    at launch), its S1_MROWS loads in flight together
  if (tid < FP) {
    const int col = tid - 1;
    const bool col_ok = col >= 0 && col < F;
    float v[S1_MROWS];
#pragma unroll
    for (int r = 0; r < S1_MROWS; ++r) {
      const int tm = tm_0 + r;
      v[r] = (col_ok && tm >= 0 && tm < mvalid) ? mel[(size_t)tm * F + col] : 0.f;
    }
#pragma unroll
    for (int r = 0; r < S1_MROWS; ++r) melt[r * FP + tid] = v[r];
  }
  __syncthreads();

  // 2. conv.0 on the tensor cores
  {
    const int g = lane >> 2, t4 = lane & 3;
    uint32_t bf[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const float* wc = w0 + (size_t)(cg0 + nt * 8 + g) * 9;
      const int k0 = 2 * t4, k2 = 2 * t4 + 8;
      bf[nt][0] = pack2<__half>(wc[k0], wc[k0 + 1]);  // k0 + 1 <= 7
      bf[nt][1] = pack2<__half>(k2 < 9 ? wc[k2] : 0.f, 0.f);
    }
    float bias[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      bias[nt][0] = b0[cg0 + nt * 8 + 2 * t4];
      bias[nt][1] = b0[cg0 + nt * 8 + 2 * t4 + 1];
    }
    // tap k of position p = (r1, f1) reads melt[(2 r1 + k / 3) FP + 2 f1 + k % 3]:
    // a position's base plus a tap offset. This thread's taps are 2 t4,
    // 2 t4 + 1 (always < 9) and 2 t4 + 8 (< 9 only for t4 = 0); 2 t4 + 9 is
    // past the 9 taps (the zero K padding).
    auto toff = [&](int k) { return (k / 3) * FP + k % 3; };
    const int o0 = toff(2 * t4), o1 = toff(2 * t4 + 1), o2 = toff(8);
    const bool has8 = t4 == 0;
    auto base = [&](int p) { return 2 * (p / F1) * FP + 2 * (p % F1); };
    for (int mt = warp; mt < MT; mt += S1_THREADS / 32) {
      const int p0 = mt * 16 + g, p1 = p0 + 8;
      const bool in0 = p0 < NP, in1 = p1 < NP;
      const float* m0 = melt + base(p0);
      const float* m1 = melt + base(p1);
      uint32_t a[4];
      a[0] = pack2<__half>(in0 ? m0[o0] : 0.f, in0 ? m0[o1] : 0.f);
      a[1] = pack2<__half>(in1 ? m1[o0] : 0.f, in1 ? m1[o1] : 0.f);
      a[2] = pack2<__half>(in0 && has8 ? m0[o2] : 0.f, 0.f);
      a[3] = pack2<__half>(in1 && has8 ? m1[o2] : 0.f, 0.f);
      // rows of this tile's positions outside [0, v1) are zero (stage-2 input mask)
      const bool live0 = p0 < NP && t1_0 + p0 / F1 >= 0 && t1_0 + p0 / F1 < v1b;
      const bool live1 = p1 < NP && t1_0 + p1 / F1 >= 0 && t1_0 + p1 / F1 < v1b;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        // the bias is the accumulator's starting value (as in the CUDA-core
        // conv.0, which starts its sum at the bias); ReLU in the bf16 rounding
        float acc[4] = {bias[nt][0], bias[nt][1], bias[nt][0], bias[nt][1]};
        mma16816_f16(acc, a, bf[nt][0], bf[nt][1]);
        // (position, 8-channel chunk nt) at chunk slot nt ^ (f1 & 7) of the position's 128-byte row
        if (p0 < NP) {
          const uint32_t v = live0 ? pack_relu_bf16(acc[0], acc[1]) : 0u;
          *reinterpret_cast<uint32_t*>(s1 + (size_t)p0 * (S1_CG * 2) + ((nt ^ ((p0 % F1) & 7)) << 4) + 4 * t4) = v;
        }
        if (p1 < NP) {
          const uint32_t v = live1 ? pack_relu_bf16(acc[2], acc[3]) : 0u;
          *reinterpret_cast<uint32_t*>(s1 + (size_t)p1 * (S1_CG * 2) + ((nt ^ ((p1 % F1) & 7)) << 4) + 4 * t4) = v;
        }
      }
    }
  }
  __syncthreads();

  // 3. depthwise 3x3 s2 p1 + bias: thread = 8 channels (chunk ch) of positions
  //    (frame tt, f2) = pos, pos + 32, ...
  // taps and bias as channel pairs: the sums run two channels per
  // instruction (fma.rn.f32x2), each lane exactly as fmaf
  const int ch = tid & 7;
  const int c = cg0 + ch * 8;
  uint64_t wk[9][4], bi[4];
#pragma unroll
  for (int k = 0; k < 9; ++k) {
    const float4 wa = __ldg(reinterpret_cast<const float4*>(w1 + (size_t)k * C + c));
    const float4 wb = __ldg(reinterpret_cast<const float4*>(w1 + (size_t)k * C + c + 4));
    wk[k][0] = f2_pack(wa.x, wa.y); wk[k][1] = f2_pack(wa.z, wa.w);
    wk[k][2] = f2_pack(wb.x, wb.y); wk[k][3] = f2_pack(wb.z, wb.w);
  }
  {
    const float4 ba = __ldg(reinterpret_cast<const float4*>(b1 + c));
    const float4 bb = __ldg(reinterpret_cast<const float4*>(b1 + c + 4));
    bi[0] = f2_pack(ba.x, ba.y); bi[1] = f2_pack(ba.z, ba.w); bi[2] = f2_pack(bb.x, bb.y); bi[3] = f2_pack(bb.z, bb.w);
  }
  __nv_bfloat16* ob = out + (size_t)t.v2_off[b] * F2 * C;
  for (int pos = tid >> 3; pos < S1_T2 * F2; pos += S1_THREADS / 8) {
    const int tt = pos / F2, f2 = pos % F2;
    if (t2_0 + tt >= v2b) break;
    uint64_t acc[4] = {bi[0], bi[1], bi[2], bi[3]};
#pragma unroll
    for (int kh = 0; kh < 3; ++kh) {
#pragma unroll
      for (int kw = 0; kw < 3; ++kw) {
        const int f1 = 2 * f2 - 1 + kw;
        if (f1 < 0 || f1 >= F1) continue;
        const int p = (2 * tt + kh) * F1 + f1;
        const uint4 raw = *reinterpret_cast<const uint4*>(s1 + (size_t)p * (S1_CG * 2) + ((ch ^ (f1 & 7)) << 4));
        const uint32_t rv[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[e] = ffma2(wk[kh * 3 + kw][e], bf2_to_f2(rv[e]), acc[e]);
      }
    }
    uint4 o;
    o.x = f2_to_bf2(acc[0]);
    o.y = f2_to_bf2(acc[1]);
    o.z = f2_to_bf2(acc[2]);
    o.w = f2_to_bf2(acc[3]);
    *reinterpret_cast<uint4*>(ob + ((size_t)(t2_0 + tt) * F2 + f2) * C + c) = o;
  }
}

}  // namespace

size_t sub_stage1_smem(int F, int F1) {
  return (((size_t)S1_MROWS * (F + 2) * 4 + 127) / 128) * 128 + (size_t)S1_ROWS * F1 * S1_CG * 2;
}

cudaError_t sub_stage1_launch(const float* logmel, int F, const float* w0, const float* b0, const float* w1,
                              const float* b1, int C, __nv_bfloat16* out, int F1, const ItemTables& t,
                              int max_v2, cudaStream_t st) {
  if (t.B <= 0 || max_v2 <= 0) return cudaSuccess;
  if (C % S1_CG != 0 || F + 2 > S1_THREADS) return cudaErrorInvalidValue;
  const size_t smem = sub_stage1_smem(F, F1);
  const dim3 grid((max_v2 + S1_T2 - 1) / S1_T2, t.B, C / S1_CG);
  // the largest dynamic shared memory this kernel has been allowed, per device
#define PKC_S1(FF)                                                                                   \
  {                                                                                                  \
    static PerDevice attr;                                                                           \
    const cudaError_t e = allow_smem(attr, k_sub_stage1<FF>, (int)smem);                             \
    if (e != cudaSuccess) return e;                                                                  \
    return launch_pdl(k_sub_stage1<FF>, grid, dim3(S1_THREADS), smem, st, logmel, F, w0, b0, w1, b1, C, out, t); \
  }
  switch (F1) {
    case 64: PKC_S1(64)
    case 40: PKC_S1(40)
    default: return cudaErrorInvalidValue;
  }
#undef PKC_S1
}

cudaError_t sub_conv0_launch(const float* logmel, int F, const float* w, const float* b, int C,
                             __nv_bfloat16* out, int F1, const ItemTables& t, int total_v1,
                             cudaStream_t st) {
  if (t.B <= 0 || total_v1 <= 0) return cudaSuccess;
  const size_t smem = (size_t)3 * (F + 2) * sizeof(float);
  return launch_pdl(k_conv0<__nv_bfloat16>, dim3(total_v1), dim3(256), smem, st, logmel, F, w, b, C, out, F1, t);
}

cudaError_t sub_conv0_f32_launch(const float* logmel, int F, const float* w, const float* b, int C, float* out,
                                 int F1, const ItemTables& t, int total_v1, cudaStream_t st) {
  if (t.B <= 0 || total_v1 <= 0) return cudaSuccess;
  const size_t smem = (size_t)3 * (F + 2) * sizeof(float);
  return launch_pdl(k_conv0<float>, dim3(total_v1), dim3(256), smem, st, logmel, F, w, b, C, out, F1, t);
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
