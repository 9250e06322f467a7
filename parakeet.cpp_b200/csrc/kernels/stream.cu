// Cache-aware streaming encoder kernels (reference: StreamingEncoder,
// src/streaming_encoder.cpp, and the causal branches of the subsampling and
// conv module). S streams step together: their windows and chunk frames are
// stacked along the rows, and their caches are reached through device tables
// of per-stream pointers. A chunk is a few frames per stream, so these kernels
// are sized for latency; the projections around them are the library's GEMMs.
//
//   k_causal_conv0   Conv2d(1 -> C, 3x3, stride 2) over each mel window, both
//                    axes padded 2 before and 1 after (NeMo CausalConv2D,
//                    src/subsampling.cpp:283-295), + bias + ReLU
//   k_causal_dw      depthwise Conv2d(C, 3x3, stride 2), same padding, + bias
//   k_stream_attn    rel-pos attention of a stream's chunk queries over its
//                    [attention cache | chunk] keys with the chunked-limited
//                    and empty-cache mask (src/streaming_encoder.cpp:170-284)
//   k_stream_dwconv  causal depthwise Conv1d over [conv cache | GLU rows],
//                    + bias, LayerNorm over channels or folded BatchNorm, SiLU
//                    (src/streaming_encoder.cpp:286-338, src/conformer.cpp:102-154)
//   k_stream_roll    every layer's next attention and conv caches
//   k_stream_advance the attention-cache fill counts
// Every kernel is a programmatic dependent launch: it waits for its
// predecessor before touching what that wrote.
#include <algorithm>
#include <utility>

#include "common.cuh"
#include "kernels.h"

namespace pkc {

namespace {

template <typename H>
__device__ __forceinline__ float ld_h(const H* p) {
  if constexpr (std::is_same<H, __half>::value) return __half2float(*p);
  else return __bfloat162float(*p);
}
template <typename H>
__device__ __forceinline__ H to_h(float v) {
  if constexpr (std::is_same<H, __half>::value) return __float2half_rn(v);
  else return __float2bfloat16_rn(v);
}

// mel [S][F][n] (feature-major windows); frames >= valid are zero (the
// reference's per-stage time mask). Output [S][T1][F1][C] bf16.
__global__ void k_causal_conv0(const float* __restrict__ mel, int S, int F, int n, int valid,
                               const float* __restrict__ w, const float* __restrict__ b, int C, int T1, int F1,
                               __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long per = (long long)T1 * F1 * C;
  if (i >= per * S) return;
  const int s = (int)(i / per);
  const long long r = i - s * per;
  const int c = (int)(r % C), f1 = (int)((r / C) % F1), t1 = (int)(r / ((long long)C * F1));
  const float* m = mel + (size_t)s * F * n;
  float acc = b[c];
#pragma unroll
  for (int kh = 0; kh < 3; ++kh) {
    const int t = 2 * t1 + kh - 2;
    if (t < 0 || t >= n || t >= valid) continue;
#pragma unroll
    for (int kw = 0; kw < 3; ++kw) {
      const int f = 2 * f1 + kw - 2;
      if (f < 0 || f >= F) continue;
      acc = fmaf(w[c * 9 + kh * 3 + kw], m[(size_t)f * n + t], acc);
    }
  }
  out[i] = __float2bfloat16_rn(fmaxf(acc, 0.f));
}

// in [S][Ti][Fi][C], rows >= valid zero; w tap-major [9][C]. Out [S][To][Fo][C].
__global__ void k_causal_dw(const __nv_bfloat16* __restrict__ in, int S, int Ti, int Fi, int valid,
                            const float* __restrict__ w, const float* __restrict__ b, int C, int To, int Fo,
                            __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long per = (long long)To * Fo * C;
  if (i >= per * S) return;
  const int s = (int)(i / per);
  const long long r = i - s * per;
  const int c = (int)(r % C), fo = (int)((r / C) % Fo), to = (int)(r / ((long long)C * Fo));
  const __nv_bfloat16* src = in + (size_t)s * Ti * Fi * C;
  float acc = b[c];
#pragma unroll
  for (int kh = 0; kh < 3; ++kh) {
    const int t = 2 * to + kh - 2;
    if (t < 0 || t >= Ti || t >= valid) continue;
#pragma unroll
    for (int kw = 0; kw < 3; ++kw) {
      const int f = 2 * fo + kw - 2;
      if (f < 0 || f >= Fi) continue;
      acc = fmaf(w[(kh * 3 + kw) * C + c], __bfloat162float(src[((size_t)t * Fi + f) * C + c]), acc);
    }
  }
  out[i] = __float2bfloat16_rn(acc);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();  // red is reused
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  for (int w = 0; w < nw; ++w) s += red[w];
  return s;
}
__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = -INFINITY;
  for (int w = 0; w < nw; ++w) m = fmaxf(m, red[w]);
  return m;
}

constexpr int SA_THREADS = 128;

// One CTA per (head, query, stream). Keys / values j < cache_len come from
// the stream's cache of projected k | v rows, j >= cache_len from its chunk's
// qkv rows; ptab rows 0 .. 2 Tk - 2 hold the projected positions Tk - 1 ...
// -(Tk - 1) (row stride ldp). The head's key, value and position rows the
// query reads are first staged in shared memory with coalesced 16-byte loads
// (f32 there), so the dot products run from shared memory instead of chains of
// dependent global loads. No kernel of a chunk step writes the live cache
// (the roll writes the other buffer), the positional rows (made before the
// step) or the fill count (updated by the step's last kernel), so those are
// staged before the dependency wait, while the QKV GEMM before this kernel
// still runs; only the chunk's own rows wait for it.
template <typename H>
__global__ void __launch_bounds__(SA_THREADS) k_stream_attn(StreamAttnArgs a) {
  extern __shared__ float sa_sm[];
  __shared__ float qu[128], qv[128], red[SA_THREADS / 32];
  const int head = blockIdx.x, i = blockIdx.y, s = blockIdx.z;
  const int d = a.d, dk = d / a.n_heads, Tk = a.cache_len + a.Tc;
  const int ld = dk + 1;  // padded row stride: lanes of a key loop hit distinct banks
  float* sK = sa_sm;                   // [Tk][ld]
  float* sV = sK + (size_t)Tk * ld;    // [Tk][ld]
  float* sP = sV + (size_t)Tk * ld;    // [Tk][ld]: position row of key j for this query
  float* prob = sP + (size_t)Tk * ld;  // [Tk]
  const H* qkv = static_cast<const H*>(a.qkv) + (size_t)s * a.Tc * 3 * d;  // this stream's chunk rows
  const H* kvc = a.cache_len ? static_cast<const H*>(a.kv_cache[s]) + a.kv_layer_off : nullptr;
  const H* ptab = static_cast<const H*>(a.ptab);
  const int qrow = a.cache_len + i;  // the query's frame among [cache | chunk]
  // stage: 8 elements (16 bytes) per load, 4 loads in flight per thread
  // before their stores (a load cannot pass an earlier store it may alias);
  // at(e) gives element group e's source and its f32 destination
  const int v8 = dk / 8;
  auto stage = [&](int total, auto at) {
    for (int e0 = threadIdx.x; e0 < total; e0 += 4 * SA_THREADS) {
      uint4 raw[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int e = e0 + u * SA_THREADS;
        raw[u] = e < total ? *reinterpret_cast<const uint4*>(at(e).first) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int e = e0 + u * SA_THREADS;
        if (e >= total) break;
        const H* hv = reinterpret_cast<const H*>(&raw[u]);
        float* dst = at(e).second;
#pragma unroll
        for (int q = 0; q < 8; ++q) dst[q] = ld_h(hv + q);
      }
    }
  };
  using Src = std::pair<const H*, float*>;
  // before the wait: the cache's k | v rows, then the position row of every key
  const int n_cache = 2 * a.cache_len * v8;
  stage(n_cache + Tk * v8, [&](int e) -> Src {
    if (e < n_cache) {
      const int which = e / (a.cache_len * v8), r = (e / v8) % a.cache_len, c8 = (e % v8) * 8;
      return {kvc + (size_t)r * 2 * d + which * d + head * dk + c8, (which ? sV : sK) + (size_t)r * ld + c8};
    }
    const int f = e - n_cache, r = f / v8, c8 = (f % v8) * 8;
    return {ptab + (size_t)(r + a.Tc - 1 - i) * a.ldp + head * dk + c8, sP + (size_t)r * ld + c8};
  });
  for (int e = threadIdx.x; e < dk; e += SA_THREADS) {
    qu[e] = a.bias_u[head * dk + e];
    qv[e] = a.bias_v[head * dk + e];
  }
  const int filled_now = *a.filled[s];
  pdl_wait();
  pdl_trigger();
  // after it: the chunk's k | v rows and the query, from this layer's QKV GEMM
  stage(2 * a.Tc * v8, [&](int e) -> Src {
    const int which = e / (a.Tc * v8), r = (e / v8) % a.Tc, c8 = (e % v8) * 8;
    return {qkv + (size_t)r * 3 * d + (which + 1) * d + head * dk + c8,
            (which ? sV : sK) + (size_t)(a.cache_len + r) * ld + c8};
  });
  for (int e = threadIdx.x; e < dk; e += SA_THREADS) {
    const float q = ld_h(qkv + (size_t)i * 3 * d + head * dk + e);
    qu[e] = q + qu[e];
    qv[e] = q + qv[e];
  }
  __syncthreads();
  // chunked-limited: chunk = att_right + 1, visible iff 0 <= gq/chunk - gk/chunk <= att_left/chunk;
  // the cache's first cache_len - filled columns are not filled yet
  const int chunk = a.att_right + 1;
  const int left_chunks = chunk > 0 ? a.att_left / chunk : 0;
  const int filled = min(max(filled_now, 0), a.cache_len);
  const int gq = qrow, first_filled = a.cache_len - filled;
  const float scale = rsqrtf((float)dk);
  float mx = -INFINITY;
  for (int j = threadIdx.x; j < Tk; j += SA_THREADS) {
    const int diff = gq / chunk - j / chunk;
    float sc = -INFINITY;
    if (j >= first_filled && diff >= 0 && diff <= left_chunks) {
      const float* kr = sK + (size_t)j * ld;
      const float* pr = sP + (size_t)j * ld;  // relative position gq - j
      float ac = 0.f, bd = 0.f;
#pragma unroll 8
      for (int e = 0; e < dk; ++e) {
        ac = fmaf(qu[e], kr[e], ac);
        bd = fmaf(qv[e], pr[e], bd);
      }
      sc = (ac + bd) * scale;
    }
    prob[j] = sc;
    mx = fmaxf(mx, sc);
  }
  mx = block_max(mx, red);
  float sum = 0.f;
  for (int j = threadIdx.x; j < Tk; j += SA_THREADS) {
    const float p = prob[j] == -INFINITY ? 0.f : __expf(prob[j] - mx);
    prob[j] = p;
    sum += p;
  }
  sum = block_sum(sum, red);  // ends with a barrier: prob[] is complete
  const float inv = 1.0f / sum;
  H* ctx = static_cast<H*>(a.ctx) + ((size_t)s * a.Tc + i) * d;
  for (int e = threadIdx.x; e < dk; e += SA_THREADS) {
    float acc = 0.f;
#pragma unroll 4
    for (int j = 0; j < Tk; ++j) acc = fmaf(prob[j], sV[(size_t)j * ld + e], acc);
    ctx[head * dk + e] = to_h<H>(acc * inv);
  }
}

size_t stream_attn_smem(int Tk, int dk) { return ((size_t)3 * Tk * (dk + 1) + Tk) * sizeof(float); }

constexpr int SD_THREADS = 256;

// One CTA per (output frame t, stream): row r of [conv cache | GLU rows] is
// cache row r (r < K - 1) or GLU row r - (K - 1) of the stream's chunk. The
// live conv cache is not written during a chunk step, so its taps are summed
// before the dependency wait and the GLU rows' taps after it (the same
// ascending tap order as one loop).
template <typename H, int CPT>
__global__ void __launch_bounds__(SD_THREADS) k_stream_dwconv(StreamConvArgs a) {
  __shared__ float red[SD_THREADS / 32];
  const int t = blockIdx.x, s = blockIdx.y, d = a.d, lp = a.K - 1;
  const H* cache = lp ? static_cast<const H*>(a.cv_cache[s]) + a.cv_layer_off : nullptr;
  const H* glu = static_cast<const H*>(a.glu) + (size_t)s * a.Tc * d;
  const int k_glu = max(0, lp - t);  // taps k >= k_glu read GLU rows
  float v[CPT];
#pragma unroll
  for (int u = 0; u < CPT; ++u) {
    const int c = threadIdx.x + u * SD_THREADS;
    float acc = 0.f;
    if (c < d) {
      acc = a.bias ? a.bias[c] : 0.f;
      for (int k = 0; k < min(k_glu, a.K); ++k) acc = fmaf(a.w[k * d + c], ld_h(cache + (size_t)(t + k) * d + c), acc);
    }
    v[u] = acc;
  }
  pdl_wait();
  pdl_trigger();
  float sm = 0.f;
#pragma unroll
  for (int u = 0; u < CPT; ++u) {
    const int c = threadIdx.x + u * SD_THREADS;
    float acc = v[u];
    if (c < d)
      for (int k = k_glu; k < a.K; ++k) acc = fmaf(a.w[k * d + c], ld_h(glu + (size_t)(t + k - lp) * d + c), acc);
    v[u] = acc;
    sm += acc;
  }
  if (a.layer_norm) {  // ggml_norm over channels (population variance, eps 1e-5) * gamma + beta
    const float mean = block_sum(sm, red) / (float)d;
    float q = 0.f;
#pragma unroll
    for (int u = 0; u < CPT; ++u)
      if (threadIdx.x + u * SD_THREADS < d) q += (v[u] - mean) * (v[u] - mean);
    const float rstd = rsqrtf(block_sum(q, red) / (float)d + 1e-5f);
#pragma unroll
    for (int u = 0; u < CPT; ++u) {
      const int c = threadIdx.x + u * SD_THREADS;
      if (c < d) v[u] = (v[u] - mean) * rstd * a.g[c] + a.b[c];
    }
  } else {
#pragma unroll
    for (int u = 0; u < CPT; ++u) {
      const int c = threadIdx.x + u * SD_THREADS;
      if (c < d) v[u] = v[u] * a.g[c] + a.b[c];
    }
  }
  H* out = static_cast<H*>(a.out) + ((size_t)s * a.Tc + t) * d;
#pragma unroll
  for (int u = 0; u < CPT; ++u) {
    const int c = threadIdx.x + u * SD_THREADS;
    if (c < d) out[c] = to_h<H>(v[u] / (1.0f + __expf(-v[u])));
  }
}

__global__ void k_stream_advance(int* const* filled, int n_streams, int Tc, int cache_len) {
  pdl_wait();
  pdl_trigger();
  for (int s = threadIdx.x; s < n_streams; s += blockDim.x) *filled[s] = min(cache_len, *filled[s] + Tc);
}

// grid (chunks, layers, streams). 16-byte copies.
__global__ void k_stream_roll(StreamRollArgs a) {
  pdl_wait();
  pdl_trigger();
  const int l = blockIdx.y, s = blockIdx.z;
  const int d8 = a.d / 8;  // 16-byte chunks per d elements
  const uint4* q = static_cast<const uint4*>(a.qkv) + ((size_t)l * a.layer_rows + (size_t)s * a.Tc) * 3 * d8;
  const uint4* gl = static_cast<const uint4*>(a.glu) + ((size_t)l * a.layer_rows + (size_t)s * a.Tc) * d8;
  const uint4* kvc = a.cache_len ? static_cast<const uint4*>(a.kv_cur[s]) + (size_t)l * a.cache_len * 2 * d8 : nullptr;
  uint4* kvn = a.cache_len ? static_cast<uint4*>(a.kv_next[s]) + (size_t)l * a.cache_len * 2 * d8 : nullptr;
  const uint4* cvc = a.lp ? static_cast<const uint4*>(a.cv_cur[s]) + (size_t)l * a.lp * d8 : nullptr;
  uint4* cvn = a.lp ? static_cast<uint4*>(a.cv_next[s]) + (size_t)l * a.lp * d8 : nullptr;
  const int keep = max(0, a.cache_len - a.Tc), fresh = a.cache_len - keep;
  const int ckeep = max(0, a.lp - a.Tc), cfresh = a.lp - ckeep;
  const int n_kv = a.cache_len * 2 * d8, n_cv = a.lp * d8;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n_kv + n_cv; e += gridDim.x * blockDim.x) {
    if (e < n_kv) {
      const int r = e / (2 * d8), c = e % (2 * d8);
      kvn[e] = r < keep ? kvc[(size_t)(r + a.Tc) * 2 * d8 + c]
                        : q[(size_t)(a.Tc - fresh + (r - keep)) * 3 * d8 + d8 + c];
    } else {
      const int f = e - n_kv, r = f / d8, c = f % d8;  // row r of the last lp of [cache | GLU]
      cvn[f] = r < ckeep ? cvc[(size_t)(r + a.Tc) * d8 + c] : gl[(size_t)(a.Tc - cfresh + (r - ckeep)) * d8 + c];
    }
  }
}

}  // namespace

cudaError_t causal_conv0_launch(const float* mel, int S, int F, int n, int valid, const float* w, const float* b,
                                int C, int T1, int F1, __nv_bfloat16* out, cudaStream_t st) {
  const long long total = (long long)S * T1 * F1 * C;
  if (total <= 0) return cudaSuccess;
  return launch_pdl(k_causal_conv0, dim3((unsigned)((total + 255) / 256)), dim3(256), 0, st, mel, S, F, n, valid, w, b,
                    C, T1, F1, out);
}

cudaError_t causal_dw_launch(const __nv_bfloat16* in, int S, int Ti, int Fi, int valid, const float* w,
                             const float* b, int C, int To, int Fo, __nv_bfloat16* out, cudaStream_t st) {
  const long long total = (long long)S * To * Fo * C;
  if (total <= 0) return cudaSuccess;
  return launch_pdl(k_causal_dw, dim3((unsigned)((total + 255) / 256)), dim3(256), 0, st, in, S, Ti, Fi, valid, w, b,
                    C, To, Fo, out);
}

cudaError_t stream_attention_launch(const StreamAttnArgs& a, bool bf16, cudaStream_t st) {
  if (a.Tc <= 0 || a.n_streams <= 0) return cudaSuccess;
  const int dk = a.n_heads > 0 ? a.d / a.n_heads : 0;
  const int Tk = a.cache_len + a.Tc;
  const size_t smem = stream_attn_smem(Tk, dk);
  if (dk <= 0 || dk > 128 || dk % 8 || a.d % 8 || a.ldp % 8 || !a.filled || a.att_right < 0 || smem > 200 * 1024 ||
      a.n_streams > 65535 || a.Tc > 65535)
    return cudaErrorInvalidValue;
  const dim3 grid(a.n_heads, a.Tc, a.n_streams);
  cudaError_t e;
  if (bf16) {
    e = cudaFuncSetAttribute(k_stream_attn<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(k_stream_attn<__nv_bfloat16>, grid, dim3(SA_THREADS), smem, st, a);
  }
  e = cudaFuncSetAttribute(k_stream_attn<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(k_stream_attn<__half>, grid, dim3(SA_THREADS), smem, st, a);
}

cudaError_t stream_dwconv_launch(const StreamConvArgs& a, bool bf16, cudaStream_t st) {
  if (a.Tc <= 0 || a.n_streams <= 0) return cudaSuccess;
  if (a.d > 4 * SD_THREADS || a.K < 1 || a.n_streams > 65535) return cudaErrorInvalidValue;
  const dim3 grid(a.Tc, a.n_streams);
  if (bf16) return launch_pdl(k_stream_dwconv<__nv_bfloat16, 4>, grid, dim3(SD_THREADS), 0, st, a);
  return launch_pdl(k_stream_dwconv<__half, 4>, grid, dim3(SD_THREADS), 0, st, a);
}

cudaError_t stream_advance_launch(int* const* filled, int n_streams, int Tc, int cache_len, cudaStream_t st) {
  if (n_streams <= 0) return cudaSuccess;
  return launch_pdl(k_stream_advance, dim3(1), dim3(256), 0, st, filled, n_streams, Tc, cache_len);
}

cudaError_t stream_roll_launch(const StreamRollArgs& a, cudaStream_t st) {
  if (a.d % 8 || a.layers <= 0 || a.n_streams <= 0 || a.n_streams > 65535 || a.layers > 65535)
    return cudaErrorInvalidValue;
  const long long n = (long long)a.cache_len * 2 * (a.d / 8) + (long long)a.lp * (a.d / 8);
  if (n <= 0) return cudaSuccess;
  const unsigned gx = (unsigned)std::min<long long>((n + 255) / 256, 32);
  return launch_pdl(k_stream_roll, dim3(gx, a.layers, a.n_streams), dim3(256), 0, st, a);
}

}  // namespace pkc
