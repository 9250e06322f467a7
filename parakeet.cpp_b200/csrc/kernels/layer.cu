// Per-layer memory-bound kernels of the conformer block:
//   k_layernorm     ggml_norm(x, 1e-5) * gamma + beta (src/conformer.cpp:300-307),
//                   optionally two in a row (norm_out of layer i, then
//                   norm_feed_forward1 of layer i+1) in one pass over the row
//   k_pos_table     rel_pos_encoding sinusoids (src/pos_enc.cpp:10-34), f64 math
//   k_dwconv        conv module depthwise Conv1d(K, pad (K-1)/2) + bias ->
//                   BatchNorm (host-folded scale/shift, src/conformer.cpp:134-154)
//                   -> SiLU, with zeros outside each utterance's frames (the
//                   reference's pre-depthwise time mask, :63-79)
//   k_to_chfirst    packed time-major -> per-utterance channels-first output
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "per_device.h"

namespace pkc {

namespace {

// One warp per row, each lane holding d/32 values (NV float4 chunks); the
// grid is at most a few CTAs per SM and every warp walks rows with a stride,
// loading its next row while it normalises the current one. gamma / beta of
// both norms are staged once per CTA in shared memory (they are weights:
// before the dependency wait) instead of 2 d floats of registers per lane,
// which left room for two rows per SM sub-partition at d = 1024.
// SPLIT (f32-accurate path, H = f16): out_h rows are [hi | lo] of width 2d,
// hi = f16(y), lo = f16(y - hi).
constexpr int LN_THREADS = 256;
constexpr int LN_WARPS = LN_THREADS / 32;

template <int NV, typename H, bool SPLIT>
__global__ void __launch_bounds__(LN_THREADS)
    k_layernorm(float* __restrict__ x, int M, const float* __restrict__ g, const float* __restrict__ b,
                H* __restrict__ out_h, const float* __restrict__ g2, const float* __restrict__ b2,
                int write_x) {
  constexpr int D = NV * 128;
  __shared__ float4 s_g[2][D / 4], s_b[2][D / 4];
  for (int i = threadIdx.x; i < D / 4; i += LN_THREADS) {
    s_g[0][i] = __ldg(reinterpret_cast<const float4*>(g) + i);
    s_b[0][i] = __ldg(reinterpret_cast<const float4*>(b) + i);
    if (g2) {
      s_g[1][i] = __ldg(reinterpret_cast<const float4*>(g2) + i);
      s_b[1][i] = __ldg(reinterpret_cast<const float4*>(b2) + i);
    }
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int stride = gridDim.x * LN_WARPS;
  int row = blockIdx.x * LN_WARPS + (threadIdx.x >> 5);
  float4 nx[NV];
  if (row < M) {
    const float* xr = x + (size_t)row * D;
#pragma unroll
    for (int i = 0; i < NV; ++i) nx[i] = *reinterpret_cast<const float4*>(xr + (i * 32 + lane) * 4);
  }
  for (; row < M; row += stride) {
    float v[NV * 4];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      v[4 * i] = nx[i].x; v[4 * i + 1] = nx[i].y; v[4 * i + 2] = nx[i].z; v[4 * i + 3] = nx[i].w;
    }
    // the warp's next row in flight while this one is normalised
    if (row + stride < M) {
      const float* xn = x + (size_t)(row + stride) * D;
#pragma unroll
      for (int i = 0; i < NV; ++i) nx[i] = *reinterpret_cast<const float4*>(xn + (i * 32 + lane) * 4);
    }
    float* xr = x + (size_t)row * D;
    auto norm = [&](int w) {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < NV * 4; ++i) s += v[i];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      const float mean = s / (float)D;
      float s2 = 0.f;
#pragma unroll
      for (int i = 0; i < NV * 4; ++i) {
        v[i] -= mean;
        s2 += v[i] * v[i];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
      const float scale = 1.0f / sqrtf(s2 / (float)D + 1e-5f);
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const float4 g4 = s_g[w][i * 32 + lane], b4 = s_b[w][i * 32 + lane];
        v[4 * i] = v[4 * i] * scale * g4.x + b4.x;
        v[4 * i + 1] = v[4 * i + 1] * scale * g4.y + b4.y;
        v[4 * i + 2] = v[4 * i + 2] * scale * g4.z + b4.z;
        v[4 * i + 3] = v[4 * i + 3] * scale * g4.w + b4.w;
      }
    };
    norm(0);
    if (write_x) {
#pragma unroll
      for (int i = 0; i < NV; ++i)
        *reinterpret_cast<float4*>(xr + (i * 32 + lane) * 4) =
            make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
    if (g2) norm(1);
    if (out_h) {
      H* o = out_h + (size_t)row * D * (SPLIT ? 2 : 1);
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        if constexpr (SPLIT) {
          float hi[4], lo[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            hi[e] = from_h(to_h<H>(v[4 * i + e]));
            lo[e] = v[4 * i + e] - hi[e];
          }
          *reinterpret_cast<uint2*>(o + (i * 32 + lane) * 4) =
              make_uint2(pack2<H>(hi[0], hi[1]), pack2<H>(hi[2], hi[3]));
          *reinterpret_cast<uint2*>(o + D + (i * 32 + lane) * 4) =
              make_uint2(pack2<H>(lo[0], lo[1]), pack2<H>(lo[2], lo[3]));
        } else {
          uint2 w;
          w.x = pack2<H>(v[4 * i], v[4 * i + 1]);
          w.y = pack2<H>(v[4 * i + 2], v[4 * i + 3]);
          *reinterpret_cast<uint2*>(o + (i * 32 + lane) * 4) = w;
        }
      }
    }
  }
}

template <typename H>
__global__ void k_pos_table(H* out, int centre, int d) {
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
  out[(size_t)r * d + 2 * i] = to_h<H>((float)sin(arg));
  out[(size_t)r * d + 2 * i + 1] = to_h<H>((float)cos(arg));
}

// Depthwise Conv1d over each utterance's frames + bias -> BatchNorm -> SiLU.
// One CTA = DW_CHUNKS x DW_FRAMES consecutive frames of one utterance x DW_CH
// channels; a thread owns 2 channels (one 4-byte load per row: a warp reads
// 128 contiguous bytes). The thread keeps a window of DW_FRAMES + K - 1 input
// rows in f32 registers and walks its frames chunk by chunk, the next
// chunk's DW_FRAMES rows in flight while the current chunk is computed, so
// the taps and the folded BatchNorm (weights, loaded before the dependency
// wait) are read once per DW_CHUNKS chunks. A CTA past its utterance's end
// returns before loading anything (the length tables do not come from the
// kernel before this one). grid (ceil(max_len / (DW_CHUNKS DW_FRAMES)), B,
// ceil(d / DW_CH)). Measured at M = 14k frames, d = 1024: one chunk per CTA
// 0.77 ms per step (0.81 before the early return), two chunks 0.92, four
// 0.94 (fewer CTAs left to hide each one's load latency); the kernel is
// latency-bound, not limited by the weight reloads.
constexpr int DW_FRAMES = 16;
constexpr int DW_CHUNKS = 1;
constexpr int DW_THREADS = 256;
constexpr int DW_CH = DW_THREADS * 2;

template <typename H> struct H2;
template <> struct H2<__half> {
  static __device__ __forceinline__ float2 to_f2(uint32_t v) { return __half22float2(*reinterpret_cast<const __half2*>(&v)); }
};
template <> struct H2<__nv_bfloat16> {
  static __device__ __forceinline__ float2 to_f2(uint32_t v) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
  }
};

template <typename H, int K>
__global__ void __launch_bounds__(DW_THREADS)
    k_dwconv_bn_silu(const H* __restrict__ in, H* __restrict__ out, int d,
                     const float* __restrict__ w, const float* __restrict__ bias,
                     const float* __restrict__ scale, const float* __restrict__ shift,
                     const int* __restrict__ item_off, const int* __restrict__ item_len) {
  const int t0 = blockIdx.x * (DW_CHUNKS * DW_FRAMES);
  const int c0 = blockIdx.z * DW_CH + threadIdx.x * 2;
  const int b = blockIdx.y;
  const int T = item_len[b];
  if (t0 >= T || c0 >= d) {
    pdl_trigger();
    return;
  }
  // the taps and the folded BatchNorm: before the dependency wait. The
  // thread's two channels ride in the two lanes of the packed FMA
  // (fma.rn.f32x2: each lane rounded as fmaf), half the FMA instructions.
  uint64_t wk[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const float2 v = __ldg(reinterpret_cast<const float2*>(w + (size_t)k * d + c0));
    wk[k] = f2_pack(v.x, v.y);
  }
  const float2 scf = __ldg(reinterpret_cast<const float2*>(scale + c0));
  float2 shf = __ldg(reinterpret_cast<const float2*>(shift + c0));
  if (bias) {
    // (acc + bias) * scale + shift = acc * scale + (bias * scale + shift)
    const float2 bi = __ldg(reinterpret_cast<const float2*>(bias + c0));
    shf.x = fmaf(bi.x, scf.x, shf.x);
    shf.y = fmaf(bi.y, scf.y, shf.y);
  }
  const uint64_t sc = f2_pack(scf.x, scf.y), sh = f2_pack(shf.x, shf.y);
  pdl_wait();
  pdl_trigger();
  constexpr int pad = (K - 1) / 2;
  constexpr int NR = DW_FRAMES + K - 1;
  const H* x = in + (size_t)item_off[b] * d + c0;
  H* y = out + (size_t)item_off[b] * d + c0;
  auto row = [&](int ti) -> uint32_t {
    return (ti >= 0 && ti < T) ? __ldg(reinterpret_cast<const uint32_t*>(x + (size_t)ti * d)) : 0u;
  };
  // window rows: frames t - pad .. t - pad + NR - 1 of the chunk starting at t
  uint64_t xf[NR];
  {
    uint32_t raw[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) raw[r] = row(t0 - pad + r);
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      const float2 v = H2<H>::to_f2(raw[r]);
      xf[r] = f2_pack(v.x, v.y);
    }
  }
#pragma unroll 1
  for (int c = 0; c < DW_CHUNKS; ++c) {
    const int tc = t0 + c * DW_FRAMES;
    if (tc >= T) break;
    // the next chunk's new rows (frames tc + DW_FRAMES + pad ..) in flight
    uint32_t nraw[DW_FRAMES];
    const bool more = c + 1 < DW_CHUNKS && tc + DW_FRAMES < T;
    if (more) {
#pragma unroll
      for (int r = 0; r < DW_FRAMES; ++r) nraw[r] = row(tc + DW_FRAMES - pad + (K - 1) + r);
    }
    const int nf = min(DW_FRAMES, T - tc);
#pragma unroll
    for (int f = 0; f < DW_FRAMES; ++f) {
      if (f >= nf) break;
      uint64_t a = 0ull;  // (+0, +0)
#pragma unroll
      for (int k = 0; k < K; ++k) a = ffma2(wk[k], xf[f + k], a);
      const float2 v = f2_unpack(ffma2(a, sc, sh));
      *reinterpret_cast<uint32_t*>(y + (size_t)(tc + f) * d) = pack2<H>(siluf_(v.x), siluf_(v.y));
    }
    if (more) {
#pragma unroll
      for (int r = 0; r < K - 1; ++r) xf[r] = xf[r + DW_FRAMES];
#pragma unroll
      for (int r = 0; r < DW_FRAMES; ++r) {
        const float2 v = H2<H>::to_f2(nraw[r]);
        xf[K - 1 + r] = f2_pack(v.x, v.y);
      }
    }
  }
}

// 32x32 tiled transpose per item: out[off*d + c*T + t] = x[(off + t)*d + c]
__global__ void k_to_chfirst(const float* __restrict__ x, float* __restrict__ out, int d,
                             const int* __restrict__ item_off, const int* __restrict__ item_len) {
  pdl_wait();
  pdl_trigger();
  __shared__ float tile[32][33];
  const int b = blockIdx.z;
  const int T = item_len[b];
  const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  if (t0 >= T) return;
  const size_t off = (size_t)item_off[b];
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int t = t0 + r, c = c0 + threadIdx.x;
    tile[r][threadIdx.x] = (t < T) ? x[(off + t) * d + c] : 0.f;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int c = c0 + r, t = t0 + threadIdx.x;
    if (t < T) out[off * d + (size_t)c * T + t] = tile[threadIdx.x][r];
  }
}

}  // namespace

namespace {
// one launch of k_layernorm<NV, H, SPLIT>: rows stride over one wave (the
// CTAs resident on all SMs at once, from the occupancy of this instantiation)
template <int NV, typename H, bool SPLIT>
cudaError_t ln_go(float* x, int M, const float* g, const float* b, H* out, const float* g2, const float* b2,
                  int wx, cudaStream_t st) {
  auto kern = k_layernorm<NV, H, SPLIT>;
  static PerDevice wave;
  int w = 0;
  const cudaError_t we = per_device(wave, &w, [&](int dev, int& v) {
    int n_sm = 0, per_sm = 0;
    cudaError_t r = cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    if (r == cudaSuccess) r = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, LN_THREADS, 0);
    v = std::max(1, per_sm) * n_sm;
    return r;
  });
  if (we != cudaSuccess) return we;
  const int need = (M + LN_WARPS - 1) / LN_WARPS;
  return launch_pdl(kern, dim3(std::min(need, w)), dim3(LN_THREADS), 0, st, x, M, g, b, out, g2, b2, wx);
}
}  // namespace

cudaError_t layernorm_launch(float* x, int M, int d, const float* g, const float* b, void* out_h,
                             bool bf16, const float* g2, const float* b2, bool write_x,
                             cudaStream_t st, bool split) {
  if (M <= 0) return cudaSuccess;
  if (split && bf16) return cudaErrorInvalidValue;
  const int wx = write_x ? 1 : 0;
  cudaError_t e = cudaSuccess;
#define PKC_LN(NV)                                                                                   \
  if (split)                                                                                         \
    e = ln_go<NV, __half, true>(x, M, g, b, (__half*)out_h, g2, b2, wx, st);                         \
  else if (bf16)                                                                                     \
    e = ln_go<NV, __nv_bfloat16, false>(x, M, g, b, (__nv_bfloat16*)out_h, g2, b2, wx, st);          \
  else                                                                                               \
    e = ln_go<NV, __half, false>(x, M, g, b, (__half*)out_h, g2, b2, wx, st);
  switch (d) {
    case 256: PKC_LN(2) break;
    case 512: PKC_LN(4) break;
    case 768: PKC_LN(6) break;
    case 1024: PKC_LN(8) break;
    default: return cudaErrorInvalidValue;
  }
#undef PKC_LN
  return e;
}

cudaError_t pos_table_launch(void* out, int centre, int d, bool bf16, cudaStream_t st) {
  const long long n = (long long)(2 * centre - 1) * (d / 2);
  if (n <= 0) return cudaSuccess;
  const unsigned grid = (unsigned)((n + 255) / 256);
  if (bf16) return launch_pdl(k_pos_table<__nv_bfloat16>, dim3(grid), dim3(256), 0, st, (__nv_bfloat16*)out, centre, d);
  return launch_pdl(k_pos_table<__half>, dim3(grid), dim3(256), 0, st, (__half*)out, centre, d);
}

cudaError_t dwconv_bn_silu_launch(const void* in, void* out, int d, int K, const float* w,
                                  const float* bias, const float* scale, const float* shift,
                                  const int* item_off, const int* item_len, int B, int max_len,
                                  bool bf16, cudaStream_t st) {
  if (B <= 0 || max_len <= 0) return cudaSuccess;
  if (d % 8) return cudaErrorInvalidValue;
  const dim3 grid((max_len + DW_CHUNKS * DW_FRAMES - 1) / (DW_CHUNKS * DW_FRAMES), B, (d + DW_CH - 1) / DW_CH);
  const int threads = DW_THREADS;
  cudaError_t e = cudaSuccess;
#define PKC_DW(KK)                                                                                 \
  if (bf16)                                                                                        \
    e = launch_pdl(k_dwconv_bn_silu<__nv_bfloat16, KK>, grid, dim3(threads), 0, st,                \
        (const __nv_bfloat16*)in, (__nv_bfloat16*)out, d, w, bias, scale, shift, item_off, item_len); \
  else                                                                                             \
    e = launch_pdl(k_dwconv_bn_silu<__half, KK>, grid, dim3(threads), 0, st, (const __half*)in, (__half*)out, d, \
                   w, bias, scale, shift, item_off, item_len);
  switch (K) {
    case 9: PKC_DW(9) break;
    case 7: PKC_DW(7) break;
    case 5: PKC_DW(5) break;
    case 3: PKC_DW(3) break;
    default: return cudaErrorInvalidValue;
  }
#undef PKC_DW
  return e;
}

cudaError_t to_channels_first_launch(const float* x, float* out, int d, const int* item_off,
                                     const int* item_len, int B, int max_len, cudaStream_t st) {
  if (B <= 0 || max_len <= 0) return cudaSuccess;
  if (d % 32) return cudaErrorInvalidValue;
  return launch_pdl(k_to_chfirst, dim3((max_len + 31) / 32, d / 32, B), dim3(32, 8), 0, st, x, out, d, item_off, item_len);
}

}  // namespace pkc
