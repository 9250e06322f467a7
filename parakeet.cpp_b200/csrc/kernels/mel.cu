// Log-mel front end (reference: GpuMel::compute, src/mel_gpu.cpp:34-162, whose
// numerics follow MelFrontend::compute, src/mel.cpp:95-176).
//
//   k_mel_frames  pre-emphasis (f64) + centre zero-pad + framing + window
//                 -> the DFT GEMM operand [Xhi | Xhi | Xlo] in f16, and the
//                 Nyquist bin's power (its basis row is (-1)^n, summed in f64)
//   (GEMM)        bins 0..n_fft/2-1 on the tensor cores: the basis is split
//                 the same way, [Bhi | Blo | Bhi], so one K = 3*n_fft GEMM sums
//                 Xhi*Bhi + Xhi*Blo + Xlo*Bhi (~22-bit products, f32
//                 accumulate); its POWER epilogue writes re^2 + im^2
//   k_mel_fb_log  mel filterbank (sparse rows) + log(mel + guard)
//   k_mel_norm    per-feature mean / unbiased std over the valid frames in
//                 f64, frames past them zeroed
#include "common.cuh"
#include "kernels.h"

namespace pkc {

namespace {

__device__ __forceinline__ int find_item(const int* off, int B, int row) {
  int lo = 0, hi = B - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (off[mid] <= row) lo = mid; else hi = mid - 1;
  }
  return lo;
}

constexpr int FR_THREADS = 128;

__global__ void __launch_bounds__(FR_THREADS)
    k_mel_frames(MelArgs a, ItemTables t) {
  pdl_wait();
  pdl_trigger();
  const int row = a.row0 + (int)blockIdx.x;
  if (row >= a.row0 + a.total_frames) return;
  const int b = find_item(t.mel_off, t.B, row);
  const int fr = row - t.mel_off[b];
  const float* s = a.pcm + t.pcm_off[b];
  const int S = t.n_samples[b];
  const int N = a.n_fft;
  const int pad = N / 2;
  const double pre = (double)a.preemph;
  __half* dst = a.dft_a + (size_t)row * (3 * N);
  double nyq = 0.0;
  for (int i = threadIdx.x; i < N; i += FR_THREADS) {
    const int pos = fr * a.hop + i - pad;
    double x = 0.0;
    if (pos >= 0 && pos < S) {
      x = (double)s[pos];
      if (pre > 0.0 && pos > 0) x -= pre * (double)s[pos - 1];
    }
    const float xw = (float)(x * (double)a.window[i]);
    const __half hi = __float2half_rn(xw);
    const __half lo = __float2half_rn(xw - __half2float(hi));
    dst[i] = hi;
    dst[N + i] = hi;
    dst[2 * N + i] = lo;
    nyq += (i & 1) ? -(double)xw : (double)xw;
  }
  __shared__ double red[FR_THREADS / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) nyq += __shfl_xor_sync(0xffffffffu, nyq, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = nyq;
  __syncthreads();
  if (threadIdx.x == 0) {
    double tot = 0.0;
    for (int w = 0; w < FR_THREADS / 32; ++w) tot += red[w];
    const float re = (float)tot;
    a.power[(size_t)row * a.power_ld + N / 2] = re * re;
  }
}

__global__ void k_mel_fb_log(FbArgs a) {
  pdl_wait();
  pdl_trigger();
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)a.total_frames * a.n_mels) return;
  const int row = (int)(idx / a.n_mels);
  const int m = (int)(idx % a.n_mels);
  const float* p = a.power + (size_t)row * a.power_ld + a.fb_start[m];
  const float* w = a.fb_w + a.fb_off[m];
  const int n = a.fb_len[m];
  float acc = 0.f;
  for (int k = 0; k < n; ++k) acc = fmaf(w[k], p[k], acc);
  a.logmel[(size_t)row * a.n_mels + m] = logf(acc + a.log_guard);
}

// block (32 mel bins) x (32 frame lanes); grid (ceil(F/32), B)
constexpr int NORM_LANES = 32;
__global__ void __launch_bounds__(1024) k_mel_norm(float* logmel, int F, ItemTables t) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.y;
  const int m = blockIdx.x * 32 + threadIdx.x;
  const int T = t.mel_T[b];
  const int valid = min(t.mel_valid[b], T);
  float* base = logmel + (size_t)t.mel_off[b] * F;
  __shared__ double red[NORM_LANES][33];
  __shared__ double stat[2][32];
  double acc = 0.0;
  if (m < F)
    for (int f = threadIdx.y; f < valid; f += NORM_LANES) acc += (double)base[(size_t)f * F + m];
  red[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y == 0) {
    double s = 0.0;
    for (int k = 0; k < NORM_LANES; ++k) s += red[k][threadIdx.x];
    stat[0][threadIdx.x] = valid > 0 ? s / (double)valid : 0.0;
  }
  __syncthreads();
  const double mean = stat[0][threadIdx.x];
  acc = 0.0;
  if (m < F)
    for (int f = threadIdx.y; f < valid; f += NORM_LANES) {
      const double dlt = (double)base[(size_t)f * F + m] - mean;
      acc += dlt * dlt;
    }
  red[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y == 0) {
    double s = 0.0;
    for (int k = 0; k < NORM_LANES; ++k) s += red[k][threadIdx.x];
    const double var = valid > 1 ? s / (double)(valid - 1) : 0.0;
    stat[1][threadIdx.x] = sqrt(var) + 1e-5;
  }
  __syncthreads();
  const double sd = stat[1][threadIdx.x];
  if (m < F)
    for (int f = threadIdx.y; f < T; f += NORM_LANES) {
      float* p = base + (size_t)f * F + m;
      *p = f < valid ? (float)(((double)*p - mean) / sd) : 0.0f;
    }
}

__global__ void k_mel_to_batch(const float* logmel, int F, int Tmax, float* out, ItemTables t) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.z;
  const int m = blockIdx.y;
  const int f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= Tmax) return;
  const int T = t.mel_T[b];
  out[((size_t)b * F + m) * Tmax + f] = f < T ? logmel[(size_t)(t.mel_off[b] + f) * F + m] : 0.0f;
}

__global__ void k_batch_to_packed(const float* in, int F, int Tmax, float* logmel, ItemTables t) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.z;
  const int m = blockIdx.y;
  const int f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= t.mel_T[b]) return;
  logmel[(size_t)(t.mel_off[b] + f) * F + m] = in[((size_t)b * F + m) * Tmax + f];
}

}  // namespace

cudaError_t mel_frames_launch(const MelArgs& a, const ItemTables& t, cudaStream_t st) {
  if (a.total_frames <= 0) return cudaSuccess;
  return launch_pdl(k_mel_frames, dim3(a.total_frames), dim3(FR_THREADS), 0, st, a, t);
}

cudaError_t mel_fb_log_launch(const FbArgs& a, cudaStream_t st) {
  const long long n = (long long)a.total_frames * a.n_mels;
  if (n <= 0) return cudaSuccess;
  return launch_pdl(k_mel_fb_log, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, a);
}

cudaError_t mel_norm_launch(float* logmel, int n_mels, const ItemTables& t, cudaStream_t st) {
  if (t.B <= 0) return cudaSuccess;
  return launch_pdl(k_mel_norm, dim3((n_mels + 31) / 32, t.B), dim3(32, NORM_LANES), 0, st, logmel, n_mels, t);
}

cudaError_t mel_to_batch_launch(const float* logmel, int n_mels, int T_max, float* out,
                                const ItemTables& t, cudaStream_t st) {
  if (t.B <= 0 || T_max <= 0) return cudaSuccess;
  k_mel_to_batch<<<dim3((T_max + 127) / 128, n_mels, t.B), 128, 0, st>>>(logmel, n_mels, T_max, out, t);
  return cudaGetLastError();
}

cudaError_t batch_to_packed_launch(const float* in, int n_mels, int T_max, float* logmel,
                                   const ItemTables& t, int max_T, cudaStream_t st) {
  if (t.B <= 0 || max_T <= 0) return cudaSuccess;
  k_batch_to_packed<<<dim3((max_T + 127) / 128, n_mels, t.B), 128, 0, st>>>(in, n_mels, T_max, logmel, t);
  return cudaGetLastError();
}

}  // namespace pkc
