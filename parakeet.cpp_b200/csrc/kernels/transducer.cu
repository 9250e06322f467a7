// Greedy transducer decode on the GPU, all utterances of a batch in lockstep.
//
// Reference: tdt_greedy (src/tdt.cpp:8-126) and rnnt_decode_frames /
// rnnt_greedy (src/rnnt.cpp:17-122), driving PredictionNet::step
// (src/prediction.cpp: embedding, stacked LSTM, PyTorch gate order i f g o)
// and Joint::step_logits (src/joint.hpp: ReLU(enc_proj[t] + W_pred g + b_pred)
// -> W_out . + b_out). The encoder projection enc_proj = W_enc enc + b_enc of
// every frame is one split-f16 GEMM before this kernel (as the reference's
// precompute_enc_proj).
//
// One persistent grid (cooperative launch: every CTA resident), one joint
// evaluation per utterance per iteration:
//   P  (only when some utterance needs its prediction output recomputed)
//      LSTM layer by layer, then the pred projection; each CTA owns a slice of
//      hidden units (all four gate rows of a unit, so the cell update is local)
//      and of projection rows, for every pending utterance
//   J  joint: each CTA owns a slice of the V+1(+D) output rows; per utterance a
//      partial (max, first argmax, sum of exp) of the token part and (max,
//      first argmax) of the duration part
//   D  CTA 0 merges the partials, applies the reference's per-utterance state
//      machine, appends tokens, marks utterances that need a new prediction
// Phases are separated by a grid barrier whose wait is bounded (kWaitLimitNs):
// on a timeout the kernel records DEV_ERR_TIMEOUT_DECODE and every CTA leaves.
// All arithmetic is f32 on f32 weights (the decoder weights are f32 in GGUF).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace pkc {

namespace {

constexpr int TD_THREADS = 256;
constexpr int TD_WARPS = TD_THREADS / 32;
constexpr int TD_CHUNK = 8;  // utterances whose vectors sit in shared memory at once
constexpr int TD_KV = 8;     // float4 per lane of one weight row: rows up to 8 * 128 = 1024 wide
constexpr int TD_STG = 4;    // staged elements per thread and vector: vectors up to 4 * 256 = 1024 long

struct Partial {
  float tmax, tsum, dmax;
  int targ, darg;
};

__device__ __forceinline__ bool grid_sync(unsigned int* bar_count, unsigned int* bar_gen, int* err, int* smem_ok) {
  __syncthreads();
  if (threadIdx.x == 0) {
    bool ok = true;
    unsigned int g;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(g) : "l"(bar_gen) : "memory");
    __threadfence();
    const unsigned int arrived = atomicAdd(bar_count, 1u) + 1u;
    if (arrived == gridDim.x) {
      *bar_count = 0u;
      __threadfence();
      asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(bar_gen), "r"(g + 1u) : "memory");
    } else {
      const unsigned long long t0 = globaltimer_ns();
      for (uint32_t it = 0;; ++it) {
        unsigned int cur;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(cur) : "l"(bar_gen) : "memory");
        if (cur != g) break;
        if ((it & 255u) == 255u && globaltimer_ns() - t0 > kWaitLimitNs) {
          report_error(err, DEV_ERR_TIMEOUT_DECODE);
          ok = false;
          break;
        }
        if (it > 4096u) __nanosleep(128);  // spin first: phases are a few microseconds
      }
    }
    __threadfence();
    *smem_ok = ok ? 1 : 0;
  }
  __syncthreads();
  return *smem_ok != 0;
}

__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + __expf(-x)); }

// Weight-row slice of this lane, loaded as one block of independent loads
// (volatile, so the compiler cannot sink them one by one next to their uses
// under register pressure: each would then cost a full L2 round trip).
__device__ __forceinline__ void load_row(float4 (&w)[8], const float* row, int n) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int k = lane * 4 + 128 * u;
    if (k < n) {
      asm volatile("ld.global.nc.v4.f32 {%0,%1,%2,%3}, [%4];"
                   : "=f"(w[u].x), "=f"(w[u].y), "=f"(w[u].z), "=f"(w[u].w)
                   : "l"(row + k));
    } else {
      w[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
}

// dot of a weight row (n floats, n % 4 == 0, 16-byte aligned) with a vector
__device__ __forceinline__ float warp_dot(const float* __restrict__ w, const float* __restrict__ x, int n) {
  const int lane = threadIdx.x & 31;
  float s = 0.f;
  for (int k = lane * 4; k < n; k += 128) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(w + k));
    const float4 b = *reinterpret_cast<const float4*>(x + k);
    s = fmaf(a.x, b.x, s);
    s = fmaf(a.y, b.y, s);
    s = fmaf(a.z, b.z, s);
    s = fmaf(a.w, b.w, s);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

// Merge partial q into p (max with first index on ties; sum of exp rescaled).
__device__ __forceinline__ void merge_partial(Partial& p, const Partial& q) {
  if (q.tmax > p.tmax || (q.tmax == p.tmax && q.targ < p.targ)) {
    p.tsum = (p.tmax == -INFINITY ? 0.f : p.tsum * __expf(p.tmax - q.tmax)) + q.tsum;
    p.tmax = q.tmax;
    p.targ = q.targ;
  } else if (q.tmax != -INFINITY) {
    p.tsum += q.tsum * __expf(q.tmax - p.tmax);
  }
  if (q.dmax > p.dmax || (q.dmax == p.dmax && q.darg < p.darg)) {
    p.dmax = q.dmax;
    p.darg = q.darg;
  }
}

__global__ void __launch_bounds__(TD_THREADS, 1) k_transducer_greedy(TransducerArgs a) {
  extern __shared__ float sh[];  // [TD_CHUNK][J] joint hidden vectors, then the utterance state
  __shared__ int s_ok, s_pending, s_done;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  const int H = a.H, J = a.J, L = a.L, V1 = a.V1, VP = a.V1 + a.D, B = a.B;
  // Every CTA keeps its own copy of the per-utterance state and makes the
  // (deterministic) decisions itself, so no barrier follows the decisions;
  // CTA 0 alone writes the tokens.
  int* st_t = reinterpret_cast<int*>(sh + TD_CHUNK * max(2 * H, J));
  int* st_sym = st_t + B;
  int* st_cur = st_sym + B;
  int* st_have = st_cur + B;
  int* st_last = st_have + B;
  int* st_pend = st_last + B;
  int* st_done = st_pend + B;
  for (int b = threadIdx.x; b < B; b += TD_THREADS) {
    st_t[b] = a.t[b];
    st_sym[b] = a.sym[b];
    st_cur[b] = a.cur[b];
    st_have[b] = a.have_token[b];
    st_last[b] = a.last_token[b];
    st_pend[b] = a.pending[b];
    st_done[b] = a.done[b];
  }
  if (threadIdx.x == 0) s_pending = *a.n_pending;
  __syncthreads();

  for (int iter = 0;; ++iter) {
    Partial* parts = reinterpret_cast<Partial*>(a.partials) + (size_t)(iter & 1) * G * B;
    // ---- P: prediction network for utterances whose output is stale. The
    // chunk's input / hidden vectors are staged in shared memory by one
    // coalesced pass; a warp owns one hidden unit, holds each of its gate rows
    // in registers (one round trip per row pair) and applies it to the chunk.
    if (s_pending > 0) {
      for (int l = 0; l < L; ++l) {
        const float* wi = a.w_ih + (size_t)l * 4 * H * H;
        const float* wh = a.w_hh + (size_t)l * 4 * H * H;
        const float* bb = a.b_lstm + (size_t)l * 4 * H;
        for (int b0 = 0; b0 < B; b0 += TD_CHUNK) {
          bool any = false;
          for (int bi = 0; bi < TD_CHUNK && b0 + bi < B; ++bi) any |= st_pend[b0 + bi] != 0;
          if (!any) continue;  // uniform across the CTA
          __syncthreads();
          {
            // every load of this thread first (global space, L2-coherent: the
            // vectors were written by other CTAs in this launch), then the stores
            float xv[TD_CHUNK][TD_STG], hv[TD_CHUNK][TD_STG];
#pragma unroll
            for (int bi = 0; bi < TD_CHUNK; ++bi) {
              const int b = b0 + bi;
              const bool act = b < B && st_pend[b];
              const int cur = act ? st_cur[b] : 0;
              const float* hp = a.h + (((size_t)cur * L + l) * B + (act ? b : 0)) * H;
              const float* xp = !act ? nullptr
                                : l > 0 ? a.h + (((size_t)(1 - cur) * L + (l - 1)) * B + b) * H
                                : st_have[b] ? a.embed + (size_t)st_last[b] * H
                                             : nullptr;  // SOS: zero input
#pragma unroll
              for (int r = 0; r < TD_STG; ++r) {
                const int k = threadIdx.x + TD_THREADS * r;
                xv[bi][r] = (xp && k < H) ? __ldcg(xp + k) : 0.f;
                hv[bi][r] = (act && k < H) ? __ldcg(hp + k) : 0.f;
              }
            }
#pragma unroll
            for (int bi = 0; bi < TD_CHUNK; ++bi)
#pragma unroll
              for (int r = 0; r < TD_STG; ++r) {
                const int k = threadIdx.x + TD_THREADS * r;
                if (k < H) {
                  sh[bi * 2 * H + k] = xv[bi][r];
                  sh[bi * 2 * H + H + k] = hv[bi][r];
                }
              }
          }
          __syncthreads();
          for (int j = cta * TD_WARPS + warp; j < H; j += G * TD_WARPS) {
            float acc[4][TD_CHUNK];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float4 w1[TD_KV], w2[TD_KV];
              load_row(w1, wi + (size_t)(q * H + j) * H, H);
              load_row(w2, wh + (size_t)(q * H + j) * H, H);
#pragma unroll
              for (int bi = 0; bi < TD_CHUNK; ++bi) {
                float s = 0.f;
#pragma unroll
                for (int u = 0; u < TD_KV; ++u) {
                  const int k = lane * 4 + 128 * u;
                  if (k < H) {
                    const float4 x = *reinterpret_cast<const float4*>(sh + bi * 2 * H + k);
                    const float4 h = *reinterpret_cast<const float4*>(sh + bi * 2 * H + H + k);
                    s = fmaf(w1[u].x, x.x, s); s = fmaf(w1[u].y, x.y, s); s = fmaf(w1[u].z, x.z, s); s = fmaf(w1[u].w, x.w, s);
                    s = fmaf(w2[u].x, h.x, s); s = fmaf(w2[u].y, h.y, s); s = fmaf(w2[u].z, h.z, s); s = fmaf(w2[u].w, h.w, s);
                  }
                }
                acc[q][bi] = s;
              }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
              for (int bi = 0; bi < TD_CHUNK; ++bi)
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc[q][bi] += __shfl_xor_sync(0xffffffffu, acc[q][bi], o);
            if (lane < TD_CHUNK) {
              // lane bi finishes utterance b0 + bi (values are warp-uniform)
              float z[4];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                float v = acc[q][0];
#pragma unroll
                for (int bi = 1; bi < TD_CHUNK; ++bi) v = lane == bi ? acc[q][bi] : v;
                z[q] = v + bb[q * H + j];
              }
              const int b = b0 + lane;
              if (b < B && st_pend[b]) {
                const int cur = st_cur[b];
                const float cin = a.c[(((size_t)cur * L + l) * B + b) * H + j];
                const float ig = sigm(z[0]), fg = sigm(z[1]), gg = tanhf(z[2]), og = sigm(z[3]);
                const float cn = fmaf(fg, cin, ig * gg);
                a.c[(((size_t)(1 - cur) * L + l) * B + b) * H + j] = cn;
                a.h[(((size_t)(1 - cur) * L + l) * B + b) * H + j] = og * tanhf(cn);
              }
            }
          }
        }
        if (!grid_sync(a.bar_count, a.bar_gen, a.err, &s_ok)) return;
      }
      // pred projection of the new top-layer output: g vectors staged, a warp per row
      for (int b0 = 0; b0 < B; b0 += TD_CHUNK) {
        bool any = false;
        for (int bi = 0; bi < TD_CHUNK && b0 + bi < B; ++bi) any |= st_pend[b0 + bi] != 0;
        if (!any) continue;
        __syncthreads();
        {
          float gv[TD_CHUNK][TD_STG];
#pragma unroll
          for (int bi = 0; bi < TD_CHUNK; ++bi) {
            const int b = b0 + bi;
            const bool act = b < B && st_pend[b];
            const float* gp = act ? a.h + (((size_t)(1 - st_cur[b]) * L + (L - 1)) * B + b) * H : nullptr;
#pragma unroll
            for (int r = 0; r < TD_STG; ++r) {
              const int k = threadIdx.x + TD_THREADS * r;
              gv[bi][r] = (act && k < H) ? __ldcg(gp + k) : 0.f;
            }
          }
#pragma unroll
          for (int bi = 0; bi < TD_CHUNK; ++bi)
#pragma unroll
            for (int r = 0; r < TD_STG; ++r) {
              const int k = threadIdx.x + TD_THREADS * r;
              if (k < H) sh[bi * H + k] = gv[bi][r];
            }
        }
        __syncthreads();
        for (int jj = cta * TD_WARPS + warp; jj < J; jj += G * TD_WARPS) {
          float4 w[TD_KV];
          load_row(w, a.w_pred + (size_t)jj * H, H);
          float acc[TD_CHUNK];
#pragma unroll
          for (int bi = 0; bi < TD_CHUNK; ++bi) {
            float s = 0.f;
#pragma unroll
            for (int u = 0; u < TD_KV; ++u) {
              const int k = lane * 4 + 128 * u;
              if (k < H) {
                const float4 g = *reinterpret_cast<const float4*>(sh + bi * H + k);
                s = fmaf(w[u].x, g.x, fmaf(w[u].y, g.y, fmaf(w[u].z, g.z, fmaf(w[u].w, g.w, s))));
              }
            }
            acc[bi] = s;
          }
#pragma unroll
          for (int bi = 0; bi < TD_CHUNK; ++bi)
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[bi] += __shfl_xor_sync(0xffffffffu, acc[bi], o);
          if (lane < TD_CHUNK) {
            float v = acc[0];
#pragma unroll
            for (int bi = 1; bi < TD_CHUNK; ++bi) v = lane == bi ? acc[bi] : v;
            const int b = b0 + lane;
            if (b < B && st_pend[b]) a.pred_proj[(size_t)b * J + jj] = v + a.b_pred[jj];
          }
        }
      }
      if (!grid_sync(a.bar_count, a.bar_gen, a.err, &s_ok)) return;
    }

    // ---- J: joint output rows of this CTA for every active utterance; a warp
    // reads each of its rows once and applies it to TD_CHUNK utterances
    const int r0 = (int)((long long)VP * cta / G), r1 = (int)((long long)VP * (cta + 1) / G);
    for (int b0 = 0; b0 < B; b0 += TD_CHUNK) {
      const int nb = min(TD_CHUNK, B - b0);
      bool any = false;
      for (int bi = 0; bi < nb; ++bi) any |= !st_done[b0 + bi];
      if (!any) continue;  // uniform across the CTA
      __syncthreads();
      {
        float fv[TD_CHUNK][TD_STG];
#pragma unroll
        for (int bi = 0; bi < TD_CHUNK; ++bi) {
          const int b = b0 + bi;
          const bool act = bi < nb && !st_done[b];
          const float* ep = act ? a.enc_proj + (size_t)(a.item_off[b] + st_t[b]) * a.ld_enc : nullptr;
          const float* pp = act ? a.pred_proj + (size_t)b * J : nullptr;
#pragma unroll
          for (int r = 0; r < TD_STG; ++r) {
            const int j = threadIdx.x + TD_THREADS * r;
            fv[bi][r] = (act && j < J) ? fmaxf(__ldg(ep + j) + __ldcg(pp + j), 0.f) : 0.f;
          }
        }
#pragma unroll
        for (int bi = 0; bi < TD_CHUNK; ++bi)
#pragma unroll
          for (int r = 0; r < TD_STG; ++r) {
            const int j = threadIdx.x + TD_THREADS * r;
            if (j < J) sh[bi * J + j] = fv[bi][r];
          }
      }
      __syncthreads();
      float tmax[TD_CHUNK], tsum[TD_CHUNK], dmax[TD_CHUNK];
      int targ[TD_CHUNK], darg[TD_CHUNK];
#pragma unroll
      for (int bi = 0; bi < TD_CHUNK; ++bi) {
        tmax[bi] = -INFINITY; tsum[bi] = 0.f; dmax[bi] = -INFINITY;
        targ[bi] = 0x7fffffff; darg[bi] = 0x7fffffff;
      }
      for (int v = r0 + warp; v < r1; v += TD_WARPS) {
        float4 w[TD_KV];
        load_row(w, a.w_out + (size_t)v * J, J);
        float acc[TD_CHUNK];
#pragma unroll
        for (int bi = 0; bi < TD_CHUNK; ++bi) {
          float s = 0.f;
#pragma unroll
          for (int u = 0; u < TD_KV; ++u) {
            const int k = lane * 4 + 128 * u;
            if (k < J) {
              const float4 f = *reinterpret_cast<const float4*>(sh + bi * J + k);
              s = fmaf(w[u].x, f.x, fmaf(w[u].y, f.y, fmaf(w[u].z, f.z, fmaf(w[u].w, f.w, s))));
            }
          }
          acc[bi] = s;
        }
        const float bo = a.b_out[v];
#pragma unroll
        for (int bi = 0; bi < TD_CHUNK; ++bi) {
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) acc[bi] += __shfl_xor_sync(0xffffffffu, acc[bi], o);
          const float lg = acc[bi] + bo;
          if (v < V1) {
            if (lg > tmax[bi]) {
              tsum[bi] = tsum[bi] * __expf(tmax[bi] - lg) + 1.f;
              tmax[bi] = lg;
              targ[bi] = v;
            } else {
              tsum[bi] += __expf(lg - tmax[bi]);
            }
          } else if (lg > dmax[bi]) {
            dmax[bi] = lg;
            darg[bi] = v - V1;
          }
        }
      }
      // merge the warps of this CTA per utterance (lane 0 of each holds the values)
      __shared__ Partial wp[TD_WARPS][TD_CHUNK];
      if (lane == 0)
#pragma unroll
        for (int bi = 0; bi < TD_CHUNK; ++bi) wp[warp][bi] = Partial{tmax[bi], tsum[bi], dmax[bi], targ[bi], darg[bi]};
      __syncthreads();
      if (threadIdx.x < nb) {
        const int bi = threadIdx.x, b = b0 + bi;
        if (!st_done[b]) {
          Partial p = wp[0][bi];
          for (int w = 1; w < TD_WARPS; ++w) merge_partial(p, wp[w][bi]);
          parts[(size_t)cta * B + b] = p;
        }
      }
      __syncthreads();
    }
    if (!grid_sync(a.bar_count, a.bar_gen, a.err, &s_ok)) return;

    // ---- D: decisions, in every CTA (one warp per utterance)
    for (int b = warp; b < B; b += TD_WARPS) {
      if (st_done[b]) continue;
      Partial p{-INFINITY, 0.f, -INFINITY, 0x7fffffff, 0x7fffffff};
      for (int c0 = 0; c0 < G; c0 += 32 * 8) {
        Partial q[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {  // all loads first
          const int c = c0 + 32 * u + lane;
          if (c < G) {
            const float* pf = reinterpret_cast<const float*>(parts + (size_t)c * B + b);
            q[u] = Partial{__ldcg(pf), __ldcg(pf + 1), __ldcg(pf + 2), __float_as_int(__ldcg(pf + 3)),
                           __float_as_int(__ldcg(pf + 4))};
          } else {
            q[u] = Partial{-INFINITY, 0.f, -INFINITY, 0x7fffffff, 0x7fffffff};
          }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) merge_partial(p, q[u]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        Partial q;
        q.tmax = __shfl_xor_sync(0xffffffffu, p.tmax, o);
        q.tsum = __shfl_xor_sync(0xffffffffu, p.tsum, o);
        q.targ = __shfl_xor_sync(0xffffffffu, p.targ, o);
        q.dmax = __shfl_xor_sync(0xffffffffu, p.dmax, o);
        q.darg = __shfl_xor_sync(0xffffffffu, p.darg, o);
        merge_partial(p, q);
      }
      if (lane == 0) {
        const int k = p.targ;
        int t = st_t[b];
        const bool emit = k != a.blank;
        const int skip = a.D > 0 ? a.durations[p.darg] : 1;
        if (emit) {
          if (cta == 0) {
            // max_prob confidence over the token part: (N p_max - 1) / (N - 1)
            const float conf = ((float)V1 * (1.0f / p.tsum) - 1.0f) / ((float)V1 - 1.0f);
            const int n = a.ntok[b];
            if (n < a.tok_cap[b]) {
              int* tk = a.tokens + ((size_t)a.tok_off[b] + n) * 4;
              tk[0] = k;
              tk[1] = t;
              tk[2] = __float_as_int(conf);
              tk[3] = a.D > 0 ? skip : 1;
              a.ntok[b] = n + 1;
            } else {
              report_error(a.err, DEV_ERR_BAD_SHAPE);
            }
          }
          st_last[b] = k;
          st_have[b] = 1;
          st_cur[b] = 1 - st_cur[b];  // commit the step's (h', c')
        }
        int sym = st_sym[b] + 1;
        if (a.D > 0) {
          // tdt_greedy: symbols_added += 1; t += skip; stay while skip == 0
          t += skip;
          if (!(skip == 0 && sym < a.max_symbols)) {
            if (sym == a.max_symbols) t += 1;
            sym = 0;
          }
        } else if (!emit || sym >= a.max_symbols) {
          // rnnt: blank -> next frame; max_symbols emissions -> next frame
          t += 1;
          sym = 0;
        }
        st_t[b] = t;
        st_sym[b] = sym;
        st_pend[b] = emit ? 1 : 0;  // a new committed state needs a new prediction
        if (t >= a.item_len[b]) {
          st_done[b] = 1;
          st_pend[b] = 0;
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int np = 0, nd = 0;
      for (int b = 0; b < B; ++b) {
        np += st_pend[b];
        nd += st_done[b];
      }
      if (iter + 1 >= a.max_iters && nd < B) {
        if (cta == 0) report_error(a.err, DEV_ERR_BAD_SHAPE);
        nd = B;  // stop
      }
      s_pending = np;
      s_done = nd;
    }
    __syncthreads();
    if (s_done >= B) return;
  }
}

}  // namespace

size_t transducer_smem_bytes(int H, int J, int B) {
  return (size_t)TD_CHUNK * std::max(2 * H, J) * sizeof(float) + (size_t)7 * B * sizeof(int);
}
size_t transducer_partial_bytes(int grid, int B) { return (size_t)2 * grid * B * sizeof(Partial); }

cudaError_t transducer_greedy_launch(const TransducerArgs& a, int grid, cudaStream_t st) {
  if (a.B <= 0) return cudaSuccess;
  if (a.H % 4 || a.J % 4 || a.H > TD_KV * 128 || a.J > TD_KV * 128 || a.L < 1 || grid < 1 || a.B > 4096)
    return cudaErrorInvalidValue;
  const size_t smem = transducer_smem_bytes(a.H, a.J, a.B);
  cudaError_t e = cudaFuncSetAttribute(k_transducer_greedy, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  TransducerArgs ka = a;
  void* params[] = {&ka};
  return cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(&k_transducer_greedy), dim3(grid),
                                     dim3(TD_THREADS), params, smem, st);
}

// One CTA per SM: the cooperative launch guarantees they are all resident,
// which the grid barrier needs.
int transducer_grid() {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

}  // namespace pkc
