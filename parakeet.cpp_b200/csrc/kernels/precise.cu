// Kernels of the f32-accurate path (f32 GGUF weights). The reference runs an
// f32 model with f32 arithmetic (its ggml mul_mat nodes consume F32 weights:
// src/conformer.cpp:319-324, src/relpos_attention.cpp:191-194,305). Here the
// contractions stay on the tcgen05 tensor cores as split-f16 products: an f32
// value v is carried as hi = f16(v), lo = f16(v - hi), and A B^T is
// accumulated as A_hi B_hi + A_hi B_lo + A_lo B_hi in f32 (~22 significant
// bits per product; the GEMM's split_k mode). So every GEMM operand is
// written as an f16 row pair [hi | lo] of width 2K, and everything between
// the GEMMs runs in f32:
//   split_rows      f32 rows -> [hi | lo] rows (the subsampling output linear's
//                   operand, which the pointwise GEMM writes as f32 first)
//   pos_table_split rel_pos_encoding sinusoids (src/pos_enc.cpp:10-34) -> [hi | lo]
//   sub_dw_f32split subsampling depthwise 3x3 s2 + bias, f32 in, [hi | lo] out
//                   (the next pointwise GEMM's operand)
//   dwconv_f32split conv module depthwise + BatchNorm + SiLU, f32 in, [hi | lo] out
//   attention_f32   rel-pos attention in f32 on the CUDA cores (scores, softmax,
//                   P V), [hi | lo] out for the output projection
#include "common.cuh"
#include "kernels.h"

namespace pkc {

namespace {

__device__ __forceinline__ void split1(float v, __half& hi, __half& lo) {
  hi = __float2half_rn(v);
  lo = __float2half_rn(v - __half2float(hi));
}

__device__ __forceinline__ uint2 pack4(const __half* h) {
  uint2 r;
  r.x = (uint32_t)__half_as_ushort(h[0]) | ((uint32_t)__half_as_ushort(h[1]) << 16);
  r.y = (uint32_t)__half_as_ushort(h[2]) | ((uint32_t)__half_as_ushort(h[3]) << 16);
  return r;
}

// one thread = 4 consecutive values of a row
__global__ void __launch_bounds__(256)
    k_split_rows(const float* __restrict__ x, long long rows, int K, int ldx, __half* __restrict__ out, int ldo) {
  pdl_wait();
  pdl_trigger();
  const int q = K / 4;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * q) return;
  const long long r = idx / q;
  const int c = (int)(idx - r * q) * 4;
  const float4 v = *reinterpret_cast<const float4*>(x + r * ldx + c);
  __half hi[4], lo[4];
  split1(v.x, hi[0], lo[0]);
  split1(v.y, hi[1], lo[1]);
  split1(v.z, hi[2], lo[2]);
  split1(v.w, hi[3], lo[3]);
  *reinterpret_cast<uint2*>(out + r * ldo + c) = pack4(hi);
  *reinterpret_cast<uint2*>(out + r * ldo + K + c) = pack4(lo);
}

// sinusoid of relative position centre-1-r at column pair (2i, 2i+1), f64
// arguments as the reference's rel_pos_encoding computes them
__global__ void k_pos_table_split(__half* out, int centre, int d) {
  pdl_wait();
  pdl_trigger();
  const int half = d / 2;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int rows = 2 * centre - 1;
  if (idx >= (long long)rows * half) return;
  const int r = (int)(idx / half);
  const int i = (int)(idx % half);
  const double factor = -(log(10000.0) / (double)d);
  const double div = exp((double)(2 * i) * factor);
  const double arg = (double)(centre - 1 - r) * div;
  __half h0, l0, h1, l1;
  split1((float)sin(arg), h0, l0);
  split1((float)cos(arg), h1, l1);
  __half* o = out + (size_t)r * 2 * d;
  o[2 * i] = h0;
  o[2 * i + 1] = h1;
  o[d + 2 * i] = l0;
  o[d + 2 * i + 1] = l1;
}

// Depthwise Conv2d(C, 3x3, stride 2, pad 1) + bias over [frames, F, C]
// (channel fastest) f32 input; one thread = 8 channels of one output
// position; zeros outside the utterance's valid frames and the F axis.
__global__ void __launch_bounds__(256)
    k_sub_dw_f32split(const float* __restrict__ in, int F_in, const int* __restrict__ in_off,
                      const int* __restrict__ in_valid, const float* __restrict__ w, const float* __restrict__ bias,
                      int C, __half* __restrict__ out, int F_out, const int* __restrict__ out_off,
                      const int* __restrict__ out_valid) {
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
  const float* x = in + (size_t)in_off[b] * F_in * C;
  float acc[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) acc[c] = bias[c0 + c];
#pragma unroll
  for (int kh = 0; kh < 3; ++kh) {
    const int ti = 2 * tt - 1 + kh;
#pragma unroll
    for (int kw = 0; kw < 3; ++kw) {
      const int fi = 2 * f - 1 + kw;
      if (ti < 0 || ti >= vi || fi < 0 || fi >= F_in) continue;
      const float* xp = x + ((size_t)ti * F_in + fi) * C + c0;
      const float4 a = *reinterpret_cast<const float4*>(xp), bq = *reinterpret_cast<const float4*>(xp + 4);
      const float xv[8] = {a.x, a.y, a.z, a.w, bq.x, bq.y, bq.z, bq.w};
      const float* wk = w + (kh * 3 + kw) * C + c0;
#pragma unroll
      for (int c = 0; c < 8; ++c) acc[c] = fmaf(wk[c], xv[c], acc[c]);
    }
  }
  __half hi[8], lo[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) split1(acc[c], hi[c], lo[c]);
  __half* o = out + (((size_t)out_off[b] + tt) * F_out + f) * 2 * C;
  *reinterpret_cast<uint2*>(o + c0) = pack4(hi);
  *reinterpret_cast<uint2*>(o + c0 + 4) = pack4(hi + 4);
  *reinterpret_cast<uint2*>(o + C + c0) = pack4(lo);
  *reinterpret_cast<uint2*>(o + C + c0 + 4) = pack4(lo + 4);
}

// Conv module depthwise Conv1d(K, pad (K-1)/2) + bias -> BatchNorm (folded
// scale / shift) -> SiLU on f32 [M, d] rows; one thread = 2 channels x
// DWF frames of one utterance, zeros outside its frames (the reference's
// pre-depthwise time mask, src/conformer.cpp:63-79).
constexpr int DWF = 16;
template <int K>
__global__ void __launch_bounds__(256)
    k_dwconv_f32split(const float* __restrict__ in, __half* __restrict__ out, int d, const float* __restrict__ w,
                      const float* __restrict__ bias, const float* __restrict__ scale,
                      const float* __restrict__ shift, const int* __restrict__ item_off,
                      const int* __restrict__ item_len) {
  const int t0 = blockIdx.x * DWF;
  const int c0 = blockIdx.z * 512 + threadIdx.x * 2;
  float2 wk[K], sc = make_float2(0.f, 0.f), sh = make_float2(0.f, 0.f), bi = make_float2(0.f, 0.f);
  if (c0 < d) {
#pragma unroll
    for (int k = 0; k < K; ++k) wk[k] = __ldg(reinterpret_cast<const float2*>(w + (size_t)k * d + c0));
    sc = __ldg(reinterpret_cast<const float2*>(scale + c0));
    sh = __ldg(reinterpret_cast<const float2*>(shift + c0));
    if (bias) bi = __ldg(reinterpret_cast<const float2*>(bias + c0));
  }
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.y;
  const int T = item_len[b];
  if (t0 >= T || c0 >= d) return;
  constexpr int pad = (K - 1) / 2;
  constexpr int NR = DWF + K - 1;
  const float* x = in + (size_t)item_off[b] * d + c0;
  float2 xf[NR];
#pragma unroll
  for (int r = 0; r < NR; ++r) {
    const int ti = t0 - pad + r;
    xf[r] = (ti >= 0 && ti < T) ? __ldg(reinterpret_cast<const float2*>(x + (size_t)ti * d)) : make_float2(0.f, 0.f);
  }
  __half* y = out + (size_t)item_off[b] * 2 * d + c0;
  const int nf = min(DWF, T - t0);
#pragma unroll
  for (int f = 0; f < DWF; ++f) {
    if (f >= nf) break;
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      a0 = fmaf(wk[k].x, xf[f + k].x, a0);
      a1 = fmaf(wk[k].y, xf[f + k].y, a1);
    }
    // ((acc + bias) * scale + shift), then SiLU with an accurate exponential
    const float z0 = (a0 + bi.x) * sc.x + sh.x, z1 = (a1 + bi.y) * sc.y + sh.y;
    const float s0 = z0 / (1.0f + expf(-z0)), s1 = z1 / (1.0f + expf(-z1));
    __half h0, l0, h1, l1;
    split1(s0, h0, l0);
    split1(s1, h1, l1);
    __half* yr = y + (size_t)(t0 + f) * 2 * d;
    *reinterpret_cast<__half2*>(yr) = __halves2half2(h0, h1);
    *reinterpret_cast<__half2*>(yr + d) = __halves2half2(l0, l1);
  }
}

// ---------------------------------------------------------------------------
// Rel-pos attention in f32 (reference: RelPosAttention::build_graph_batched,
// src/relpos_attention.cpp:162-306): s = (q + u) k^T + rel_shift((q + v) p^T),
// keys past the utterance masked, softmax(s / sqrt(dk)), ctx = P v, in f32
// with expf; output rows [hi | lo] for the split-f16 output projection.
// rel_shift as an index: score (i, j) uses positional row centre - 1 - (i - j)
// (the row of relative position i - j). One CTA = (one head, QT query rows of
// one utterance); keys in tiles of KT; online softmax.
constexpr int QT = 32;
constexpr int KT = 64;
constexpr int PW = QT + KT - 1;  // positional rows per key tile
constexpr int PWP = PW + 2;      // padded row of the transposed window (odd stride)
constexpr int ATHREADS = 256;

template <int DK>
struct F32Smem {
  float qu[QT][DK + 1];   // odd row stride: rows 2 apart hit different banks
  float qv[QT][DK + 1];
  float kt[DK][KT + 1];   // keys, transposed
  float pt[DK][PWP];      // positional window, transposed
  float vs[KT][DK];
  float sp[QT][KT + 1];   // scores, then probabilities
  float m[QT], l[QT], corr[QT];
};

template <int DK>
__global__ void __launch_bounds__(ATHREADS)
    k_relpos_attn_f32(const float* __restrict__ qkv, const float* __restrict__ ptab, int ptab_rows, int ptab_ld,
                      int centre, const float* __restrict__ bias_u, const float* __restrict__ bias_v,
                      const int* __restrict__ tiles, const int* __restrict__ item_off,
                      const int* __restrict__ item_len, __half* __restrict__ ctx, int d, float scale) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  F32Smem<DK>& S = *reinterpret_cast<F32Smem<DK>*>(smem_raw);
  pdl_wait();
  pdl_trigger();
  const int h = blockIdx.y;
  const int item = tiles[2 * blockIdx.x], q0 = tiles[2 * blockIdx.x + 1];
  const int T = item_len[item];
  const size_t off = (size_t)item_off[item];
  const int tid = threadIdx.x;
  const int ld = 3 * d;
  const int hc = h * DK;
  // q + u, q + v (rows past the utterance: zero)
  for (int i = tid; i < QT * DK; i += ATHREADS) {
    const int r = i / DK, k = i % DK;
    const float q = (q0 + r < T) ? qkv[(off + q0 + r) * ld + hc + k] : 0.f;
    S.qu[r][k] = q + bias_u[hc + k];
    S.qv[r][k] = q + bias_v[hc + k];
  }
  if (tid < QT) {
    S.m[tid] = -INFINITY;
    S.l[tid] = 0.f;
  }
  const int ty = tid / 16, tx = tid % 16;  // score / output block: rows 2ty, 2ty+1
  constexpr int OC = DK / 16;               // output columns tx + 16 c per thread
  float o[2][OC];
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int c = 0; c < OC; ++c) o[r][c] = 0.f;

  for (int k0 = 0; k0 < T; k0 += KT) {
    __syncthreads();  // previous tile's smem reads done
    // keys and values of this tile (zero past the utterance)
    for (int i = tid; i < KT * DK; i += ATHREADS) {
      const int j = i / DK, k = i % DK;
      const bool ok = k0 + j < T;
      const float* row = qkv + (off + k0 + j) * ld + hc + k;
      S.kt[k][j] = ok ? row[d] : 0.f;
      S.vs[j][k] = ok ? row[2 * d] : 0.f;
    }
    // positional rows rb .. rb + PW - 1, rb = centre - 1 - (q0 + QT - 1) + k0
    const int rb = centre - 1 - (q0 + QT - 1) + k0;
    for (int i = tid; i < PW * DK; i += ATHREADS) {
      const int w = i / DK, k = i % DK;
      const int r = rb + w;
      S.pt[k][w] = (r >= 0 && r < ptab_rows) ? ptab[(size_t)r * ptab_ld + hc + k] : 0.f;
    }
    __syncthreads();
    // scores of rows 2ty + {0,1}, keys tx + 16 c; the window column of (i, j) is QT - 1 - i + j
    float s[2][4];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[r][c] = 0.f;
    const int i0 = 2 * ty;
#pragma unroll 4
    for (int k = 0; k < DK; ++k) {
      const float a0 = S.qu[i0][k], a1 = S.qu[i0 + 1][k];
      const float b0 = S.qv[i0][k], b1 = S.qv[i0 + 1][k];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int j = tx + 16 * c;
        const float kv = S.kt[k][j];
        const int w = QT - 1 - i0 + j;
        s[0][c] = fmaf(a0, kv, fmaf(b0, S.pt[k][w], s[0][c]));
        s[1][c] = fmaf(a1, kv, fmaf(b1, S.pt[k][w - 1], s[1][c]));
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int j = tx + 16 * c;
        S.sp[i0 + r][j] = (k0 + j < T) ? s[r][c] : -INFINITY;
      }
    __syncthreads();
    // online softmax: 8 threads per row, 8 keys each
    {
      const int r = tid / 8, part = tid % 8;
      float mx = -INFINITY;
#pragma unroll
      for (int e = 0; e < 8; ++e) mx = fmaxf(mx, S.sp[r][part + 8 * e]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      const float m_old = S.m[r];
      const float m_new = fmaxf(m_old, mx);  // finite: the tile holds at least one key
      float sum = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int j = part + 8 * e;
        const float p = expf((S.sp[r][j] - m_new) * scale);  // exp(-inf) = 0 for masked keys
        S.sp[r][j] = p;
        sum += p;
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      sum += __shfl_xor_sync(0xffffffffu, sum, 4);
      __syncwarp();
      if (part == 0) {
        const float cr = m_old == -INFINITY ? 0.f : expf((m_old - m_new) * scale);
        S.corr[r] = cr;
        S.l[r] = S.l[r] * cr + sum;
        S.m[r] = m_new;
      }
    }
    __syncthreads();
    // O = O * corr + P V
    const float c0r = S.corr[i0], c1r = S.corr[i0 + 1];
#pragma unroll
    for (int c = 0; c < OC; ++c) {
      o[0][c] *= c0r;
      o[1][c] *= c1r;
    }
#pragma unroll 4
    for (int j = 0; j < KT; ++j) {
      const float p0 = S.sp[i0][j], p1 = S.sp[i0 + 1][j];
#pragma unroll
      for (int c = 0; c < OC; ++c) {
        const float v = S.vs[j][tx + 16 * c];
        o[0][c] = fmaf(p0, v, o[0][c]);
        o[1][c] = fmaf(p1, v, o[1][c]);
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int i = 2 * ty + r;
    if (q0 + i >= T) continue;
    const float inv = 1.0f / S.l[i];
    __half* dst = ctx + (off + q0 + i) * 2 * (size_t)d + hc;
#pragma unroll
    for (int c = 0; c < OC; ++c) {
      __half hi, lo;
      split1(o[r][c] * inv, hi, lo);
      dst[tx + 16 * c] = hi;
      dst[d + tx + 16 * c] = lo;
    }
  }
}

template <int DK>
cudaError_t launch_attn_f32(const AttnArgs& a, cudaStream_t st) {
  const int smem = (int)sizeof(F32Smem<DK>);
  const cudaError_t e = cudaFuncSetAttribute(k_relpos_attn_f32<DK>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(k_relpos_attn_f32<DK>, dim3(a.n_tiles, a.n_heads), dim3(ATHREADS), smem, st,
                    static_cast<const float*>(a.qkv), static_cast<const float*>(a.ptab), a.ptab_rows,
                    a.ptab_ld > 0 ? a.ptab_ld : a.d, a.centre, a.bias_u, a.bias_v, a.tiles, a.item_off, a.item_len,
                    static_cast<__half*>(a.ctx), a.d, 1.0f / sqrtf((float)DK));
}

}  // namespace

cudaError_t split_rows_launch(const float* x, long long rows, int K, int ldx, __half* out, int ldo,
                              cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (K % 4 || ldx % 4 || ldo % 4 || ldo < 2 * K) return cudaErrorInvalidValue;
  const long long n = rows * (K / 4);
  return launch_pdl(k_split_rows, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, x, rows, K, ldx, out, ldo);
}

cudaError_t pos_table_split_launch(__half* out, int centre, int d, cudaStream_t st) {
  const long long n = (long long)(2 * centre - 1) * (d / 2);
  if (n <= 0) return cudaSuccess;
  return launch_pdl(k_pos_table_split, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, out, centre, d);
}

cudaError_t sub_dw_f32split_launch(const float* in, int F_in, const int* in_off, const int* in_valid, const float* w,
                                   const float* b, int C, __half* out, int F_out, const int* out_off,
                                   const int* out_valid, int B, int max_out, cudaStream_t st) {
  if (B <= 0 || max_out <= 0) return cudaSuccess;
  if (C % 8) return cudaErrorInvalidValue;
  const long long n = (long long)max_out * F_out * (C / 8);
  return launch_pdl(k_sub_dw_f32split, dim3((unsigned)((n + 255) / 256), B), dim3(256), 0, st, in, F_in, in_off,
                    in_valid, w, b, C, out, F_out, out_off, out_valid);
}

cudaError_t dwconv_f32split_launch(const float* in, __half* out, int d, int K, const float* w, const float* bias,
                                   const float* scale, const float* shift, const int* item_off, const int* item_len,
                                   int B, int max_len, cudaStream_t st) {
  if (B <= 0 || max_len <= 0) return cudaSuccess;
  if (d % 2) return cudaErrorInvalidValue;
  const dim3 grid((max_len + DWF - 1) / DWF, B, (d + 511) / 512);
  switch (K) {
#define PKC_DWF(KK) \
  case KK:          \
    return launch_pdl(k_dwconv_f32split<KK>, grid, dim3(256), 0, st, in, out, d, w, bias, scale, shift, item_off, item_len);
    PKC_DWF(9)
    PKC_DWF(7)
    PKC_DWF(5)
    PKC_DWF(3)
#undef PKC_DWF
    default:
      return cudaErrorInvalidValue;
  }
}

int attn_f32_query_tile() { return QT; }

cudaError_t attention_f32_launch(const AttnArgs& a, cudaStream_t st) {
  if (a.n_tiles <= 0) return cudaSuccess;
  if (a.d % a.n_heads != 0) return cudaErrorInvalidValue;
  if (a.n_heads > 65535) return cudaErrorInvalidValue;
  const int dk = a.d / a.n_heads;
  if (dk == 64) return launch_attn_f32<64>(a, st);
  if (dk == 128) return launch_attn_f32<128>(a, st);
  return cudaErrorInvalidValue;
}

}  // namespace pkc
