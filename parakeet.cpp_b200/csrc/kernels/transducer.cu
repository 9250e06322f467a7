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
// One persistent grid (cooperative launch: every CTA resident). Iteration =
// one joint evaluation per live utterance:
//   P  (only when some utterance emitted, so its prediction output is stale)
//      LSTM layer by layer, then the pred projection
//   J  joint: each CTA evaluates its slice of the V+1(+D) output rows and
//      folds its best token and best duration into one packed 64-bit key per
//      utterance with atomicMax (ordered value bits above the inverted row
//      index, so the largest value and on ties the lowest index wins -- the
//      reference's first-maximum argmax), plus a (max, sum of exp) partial of
//      the token part for the confidence
//   D  every CTA reads the two keys of each utterance and applies the
//      reference's state machine to its own shared-memory copy of the state
//      (all CTAs decide identically); CTA 0 appends the tokens
// Layer 0's input part W_ih0 embed[token] + b0 is a table over the vocabulary
// computed at load (transducer_gate0_launch), so layer 0 contracts only
// W_hh0 h; deeper layers contract [W_ih | W_hh] [x | h].
// Each CTA owns a contiguous slice of hidden units (all four gate rows of a
// unit, so the cell update is local), of pred rows and of joint rows. Those
// weight rows are copied into its shared memory once, by bulk copies, and stay
// there for the whole decode (the LSTM rows of all layers when they fit, else
// one layer at a time, the next layer's copy overlapping the grid barrier).
// Per phase the CTA bulk-copies the input vectors of 16 utterances into shared
// memory and its 8 warps split K of the 8-row x 16-utterance dot products.
// Confidences (max_prob, ((V+1) p_max - 1) / V) of the tokens emitted in one
// iteration are merged from the per-CTA partials during the next one, by the
// CTA the utterance maps to.
// Phases are separated by a grid barrier (monotonic arrival counter) whose
// wait, like every mbarrier wait, is bounded (kWaitLimitNs): on a timeout the
// kernel records DEV_ERR_TIMEOUT_DECODE and every CTA leaves.
// All arithmetic is f32 on f32 weights (the decoder weights are f32 in GGUF).
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"

namespace pkc {

namespace {

constexpr int TD_THREADS = 256;
constexpr int TD_WARPS = TD_THREADS / 32;
constexpr int TD_CB = 16;  // utterances per staged chunk (one per lane of a half-warp)
constexpr int TD_RG = 8;   // weight rows per dot-product pass (two LSTM units x four gates)
constexpr int TD_MAX_DUR = 32;
constexpr int TD_STATE_INTS = 13;  // per-utterance ints in each CTA's shared memory
constexpr size_t TD_SMEM_LIMIT = 227 * 1024 - 1024;  // dynamic part (the static part is < 1 KB)

// Shared-memory layout of one CTA (offsets in floats from the dynamic base).
struct TdLayout {
  int ldk;         // sX row stride: max(2H, 2J) + 4
  int nu, nj, nv;  // most hidden units / pred rows / joint rows any CTA owns
  int held;        // LSTM layers resident at once (L, or 1 when all do not fit)
  int jres;        // joint rows resident (1), or streamed through a two-slot ring of TD_RG-row groups (0)
  int o_x, o_wl, o_wp, o_wj, o_bl, o_bp, o_bj, o_r, o_z, o_c, o_e, o_st;
  int wl_l0, wl_l;  // floats of the layer-0 slot ([4 nu][H]) and of a deeper layer's ([4 nu][2H])
  size_t bytes;
};

__host__ __device__ inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

__host__ __device__ inline TdLayout td_layout(int H, int J, int L, int VP, int G, int B, int held, int jres) {
  TdLayout t;
  t.ldk = (2 * H > 2 * J ? 2 * H : 2 * J) + 4;
  t.nu = ceil_div(H, G);
  t.nj = ceil_div(J, G);
  t.nv = ceil_div(VP, G);
  t.held = held;
  t.jres = jres;
  int o = 0;
  auto take = [&](int n) {
    const int r = o;
    o += (n + 3) & ~3;
    return r;
  };
  t.wl_l0 = 4 * t.nu * H;
  t.wl_l = 4 * t.nu * 2 * H;
  t.o_x = take(TD_CB * t.ldk);
  // held == L: layer 0, then layers 1.. in turn; held == 1: one slot of the larger size
  t.o_wl = take(held == L ? t.wl_l0 + (L - 1) * t.wl_l : (L > 1 ? t.wl_l : t.wl_l0));
  t.o_wp = take(t.nj * H);
  t.o_wj = take(jres ? t.nv * J : 2 * TD_RG * J);
  t.o_bl = take(L * 4 * t.nu);
  t.o_bp = take(t.nj);
  t.o_bj = take(t.nv);
  t.o_r = take(TD_WARPS * TD_RG * TD_CB);
  t.o_z = take(TD_RG * TD_CB);
  t.o_c = take(t.nu * TD_CB);
  t.o_e = take(t.nu * TD_CB * 4);
  t.o_st = take(TD_STATE_INTS * B);
  t.bytes = (size_t)o * sizeof(float);
  return t;
}

// The layout the launch uses: the first that fits of every LSTM layer
// resident / one resident layer, each first with the joint rows resident,
// then streamed (large vocabularies: 8 K classes are ~56 rows of J per CTA).
inline TdLayout td_layout_for(int H, int J, int L, int VP, int G, int B) {
  TdLayout t = td_layout(H, J, L, VP, G, B, L, 1);
  if (t.bytes > TD_SMEM_LIMIT && L > 1) t = td_layout(H, J, L, VP, G, B, 1, 1);
  if (t.bytes > TD_SMEM_LIMIT) t = td_layout(H, J, L, VP, G, B, L, 0);
  if (t.bytes > TD_SMEM_LIMIT && L > 1) t = td_layout(H, J, L, VP, G, B, 1, 0);
  return t;
}

// ---------------------------------------------------------------- bulk copies
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Global -> this CTA's shared memory, completing `bytes` on the mbarrier.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// Generic-proxy writes to global memory before async-proxy reads of them.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// One copy per calling lane (src null: none), then one arrival: the calling
// warp must be converged.
__device__ __forceinline__ void warp_copy(uint32_t bar, uint32_t dst, const void* src, uint32_t bytes) {
  if (src) {
    mbar_expect_tx(bar, bytes);
    bulk_g2s(dst, src, bytes, bar);
  }
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

// Every thread waits for the phase; false in every thread if any timed out
// (the phase then stays outstanding).
__device__ __forceinline__ bool cta_wait(uint32_t bar, uint32_t& parity, bool& outstanding, int* err) {
  const bool ok = __syncthreads_and(mbar_wait(bar, parity, err, DEV_ERR_TIMEOUT_DECODE)) != 0;
  if (ok) {
    parity ^= 1u;
    outstanding = false;
  }
  return ok;
}

// ---------------------------------------------------------------- grid barrier
// Barrier k of the launch completes when the arrival counter (zeroed by the
// host before the launch) reaches k * gridDim.x. The CTA's writes are ordered
// before the release-add by the CTA barrier, and the acquire-load orders the
// reads after it.
__device__ __forceinline__ bool grid_sync(unsigned int* count, unsigned int& target, int* err, int* smem_ok) {
  target += gridDim.x;
  __syncthreads();
  if (threadIdx.x == 0) {
    bool ok = true;
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(count) : "memory");
    const unsigned long long t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
      unsigned int cur;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(cur) : "l"(count) : "memory");
      if ((int)(cur - target) >= 0) break;
      if ((it & 255u) == 255u && globaltimer_ns() - t0 > kWaitLimitNs) {
        report_error(err, DEV_ERR_TIMEOUT_DECODE);
        ok = false;
        break;
      }
      if (it > 4096u) __nanosleep(128);  // spin first: phases are a few microseconds
    }
    *smem_ok = ok ? 1 : 0;
  }
  __syncthreads();
  return *smem_ok != 0;
}

__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + __expf(-x)); }

// Order-preserving map of a float onto 32 unsigned bits; NaN ranks below
// every number.
__device__ __forceinline__ uint32_t ord_bits(float x) {
  if (x != x) return 0u;
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  return ((unsigned long long)ord_bits(v) << 32) | (unsigned long long)(~(uint32_t)idx);
}

// sZ[r][i] = sum_k W[min(r, nr - 1)][k] * X[i][k] for r < TD_RG, i < TD_CB.
// W rows at stride ldw, X rows at stride ldx (both in shared memory). All
// threads call it; it ends with sZ visible to the CTA.
__device__ __forceinline__ void cta_gemv(const float* W, int ldw, int nr, const float* X, int ldx, int K, float* sR,
                                         float* sZ) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = ((K + TD_WARPS - 1) / TD_WARPS + 3) & ~3;  // k slice per warp, multiple of 4
  const int kb = warp * ks, ke = min(K, kb + ks);
  const int i = lane & (TD_CB - 1), rb = (lane >> 4) * 4;
  const float* w[4];
#pragma unroll
  for (int rr = 0; rr < 4; ++rr) w[rr] = W + min(rb + rr, nr - 1) * ldw;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const float* xr = X + i * ldx;
#pragma unroll 4
  for (int k = kb; k < ke; k += 4) {
    const float4 x = *reinterpret_cast<const float4*>(xr + k);
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) {
      const float4 v = *reinterpret_cast<const float4*>(w[rr] + k);
      acc[rr] = fmaf(v.x, x.x, fmaf(v.y, x.y, fmaf(v.z, x.z, fmaf(v.w, x.w, acc[rr]))));
    }
  }
#pragma unroll
  for (int rr = 0; rr < 4; ++rr) sR[(warp * TD_RG + rb + rr) * TD_CB + i] = acc[rr];
  __syncthreads();
  if (threadIdx.x < TD_RG * TD_CB) {
    float s = 0.f;
#pragma unroll
    for (int w2 = 0; w2 < TD_WARPS; ++w2) s += sR[w2 * TD_RG * TD_CB + threadIdx.x];
    sZ[threadIdx.x] = s;
  }
  __syncthreads();
}

// Confidence of one stored token from the per-CTA (max, sum of exp) partials
// of its iteration (one warp): max_prob over the token part,
// (N p_max - 1) / (N - 1) with N = V + 1 and p_max = 1 / (sum of exp(l - max)).
__device__ __noinline__ void merge_conf(const float2* parts, int G, int B, int b, int V1, int* out) {
  const int lane = threadIdx.x & 31;
  float m = -INFINITY, s = 0.f;
  for (int c = lane; c < G; c += 32) {
    const float2 q = __ldcg(parts + (size_t)c * B + b);
    if (q.x > m) {
      s = (m == -INFINITY ? 0.f : s * __expf(m - q.x)) + q.y;
      m = q.x;
    } else if (q.x != -INFINITY) {
      s += q.y * __expf(q.x - m);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, s, o);
    const float nm = fmaxf(m, om);
    s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
    m = nm;
  }
  if (lane == 0) *out = __float_as_int(((float)V1 * (1.0f / s) - 1.0f) / ((float)V1 - 1.0f));
}

__global__ void __launch_bounds__(TD_THREADS, 1) k_transducer_greedy(TransducerArgs a) {
  extern __shared__ __align__(16) float sm[];
  __shared__ __align__(8) unsigned long long s_bar[4];  // 0: weights, 1: inputs, 2 / 3: joint ring slots
  __shared__ int s_ok, s_np, s_nd;
  __shared__ int s_dur[TD_MAX_DUR];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  const int H = a.H, J = a.J, L = a.L, V1 = a.V1, VP = a.V1 + a.D, B = a.B;
  const TdLayout lay = td_layout(H, J, L, VP, G, B, a.held, a.jres);
  const int ldk = lay.ldk;
  float* sX = sm + lay.o_x;
  float* sWl = sm + lay.o_wl;
  float* sWp = sm + lay.o_wp;
  float* sWj = sm + lay.o_wj;
  float* sBl = sm + lay.o_bl;
  float* sBp = sm + lay.o_bp;
  float* sBj = sm + lay.o_bj;
  float* sR = sm + lay.o_r;
  float* sZ = sm + lay.o_z;
  float* sC = sm + lay.o_c;
  float* sE = sm + lay.o_e;  // layer-0 input gates of the chunk [unit][item][gate]
  // per-utterance state (this CTA's copy) and constants
  int* st_t = reinterpret_cast<int*>(sm + lay.o_st);
  int* st_sym = st_t + B;
  int* st_cur = st_sym + B;
  int* st_have = st_cur + B;
  int* st_last = st_have + B;
  int* st_pend = st_last + B;
  int* st_done = st_pend + B;
  int* st_ntok = st_done + B;
  int* st_off = st_ntok + B;
  int* st_len = st_off + B;
  int* st_toff = st_len + B;
  int* st_tcap = st_toff + B;
  int* st_emit = st_tcap + B;  // stored a token in the last iteration
  const uint32_t bar_w = smem_u32(&s_bar[0]), bar_x = smem_u32(&s_bar[1]);
  const uint32_t bar_j[2] = {smem_u32(&s_bar[2]), smem_u32(&s_bar[3])};
  uint32_t par_j[2] = {0, 0};
  bool j_out[2] = {false, false};
  uint32_t par_w = 0, par_x = 0;
  bool w_out = false, x_out = false;  // a phase of bar_w / bar_x with copies not yet waited for
  unsigned int bar_target = 0;
  unsigned long long* tok_key = a.keys;          // [3][B]
  unsigned long long* dur_key = a.keys + 3 * B;  // [3][B]
  float2* parts_all = reinterpret_cast<float2*>(a.keys + 6 * B);  // [2][G][B] (max, sum of exp)

  // this CTA's rows: hidden units [u0, u1), pred rows [j0, j1), joint rows [v0, v1)
  const int u0 = (int)((long long)H * cta / G), u1 = (int)((long long)H * (cta + 1) / G);
  const int j0 = (int)((long long)J * cta / G), j1 = (int)((long long)J * (cta + 1) / G);
  const int v0 = (int)((long long)VP * cta / G), v1 = (int)((long long)VP * (cta + 1) / G);
  const int nu = u1 - u0, nj = j1 - j0, nv = v1 - v0;
  // resident LSTM rows of layer l: layer 0 as [4 nu][H] (W_hh), deeper layers [4 nu][2H] ([W_ih | W_hh])
  auto wl_of = [&](int l) -> float* {
    if (a.held < L) return sWl;
    return sWl + (l == 0 ? 0 : (size_t)lay.wl_l0 + (size_t)(l - 1) * lay.wl_l);
  };

  if (threadIdx.x == 0) {
    mbar_init(bar_w, 1);
    mbar_init(bar_x, 1);
    mbar_init(bar_j[0], 1);
    mbar_init(bar_j[1], 1);
    fence_barrier_init();
  }
  for (int b = threadIdx.x; b < B; b += TD_THREADS) {
    st_t[b] = a.t[b];
    st_sym[b] = a.sym[b];
    st_cur[b] = a.cur[b];
    st_have[b] = a.have_token[b];
    st_last[b] = a.last_token[b];
    st_pend[b] = a.pending[b];
    st_done[b] = a.done[b];
    st_ntok[b] = a.ntok[b];
    st_off[b] = a.item_off[b];
    st_len[b] = a.item_len[b];
    st_toff[b] = a.tok_off[b];
    st_tcap[b] = a.tok_cap[b];
    st_emit[b] = 0;
  }
  for (int i = threadIdx.x; i < a.D; i += TD_THREADS) s_dur[i] = a.durations[i];
  for (int i = threadIdx.x; i < L * 4 * nu; i += TD_THREADS) {  // [l][unit][gate] (layer 0's is in gate0)
    const int l = i / (4 * nu), r = i % (4 * nu);
    sBl[(l * lay.nu + (r >> 2)) * 4 + (r & 3)] = a.b_lstm[(size_t)l * 4 * H + (r & 3) * H + u0 + (r >> 2)];
  }
  for (int i = threadIdx.x; i < nj; i += TD_THREADS) sBp[i] = a.b_pred[j0 + i];
  for (int i = threadIdx.x; i < nv; i += TD_THREADS) sBj[i] = a.b_out[v0 + i];
  __syncthreads();

  // copies of LSTM layer l's rows (row 4 u + q = gate q of unit u0 + u): layer
  // 0 the W_hh rows, deeper layers [W_ih row | W_hh row]; lanes of warp 0 split them
  auto lstm_bytes = [&](int l) { return (uint32_t)((l == 0 ? 4 : 8) * nu * H * 4); };
  auto copy_lstm = [&](int l) {
    const float* wi = a.w_ih + (size_t)l * 4 * H * H;
    const float* wh = a.w_hh + (size_t)l * 4 * H * H;
    float* dst = wl_of(l);
    const int parts = l == 0 ? 1 : 2;
    for (int c = lane; c < 4 * nu * parts; c += 32) {
      const int r = c / parts, half = parts == 1 ? 1 : c % parts;
      const size_t row = (size_t)((r & 3) * H + u0 + (r >> 2)) * H;
      bulk_g2s(smem_u32(dst + (size_t)r * parts * H + (parts == 1 ? 0 : half * H)), (half ? wh : wi) + row,
               (uint32_t)(H * 4), bar_w);
    }
  };

  // resident weights: LSTM layers [0, held), pred rows, joint rows
  if (warp == 0) {
    if (lane == 0) {
      uint32_t bytes = (uint32_t)((nj * H + (lay.jres ? nv : 0) * J) * 4);
      for (int l = 0; l < a.held; ++l) bytes += lstm_bytes(l);
      mbar_expect_tx(bar_w, bytes);
    }
    __syncwarp();
    for (int l = 0; l < a.held; ++l) copy_lstm(l);
    for (int r = lane; r < nj; r += 32)
      bulk_g2s(smem_u32(sWp + (size_t)r * H), a.w_pred + (size_t)(j0 + r) * H, (uint32_t)(H * 4), bar_w);
    for (int r = lane; r < (lay.jres ? nv : 0); r += 32)
      bulk_g2s(smem_u32(sWj + (size_t)r * J), a.w_out + (size_t)(v0 + r) * J, (uint32_t)(J * 4), bar_w);
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_w);
  }
  w_out = true;
  // before leaving: give copies still in flight their (bounded) time to land
  auto drain = [&]() {
    if (w_out) mbar_wait(bar_w, par_w, nullptr, 0);
    if (x_out) mbar_wait(bar_x, par_x, nullptr, 0);
    for (int q = 0; q < 2; ++q)
      if (j_out[q]) mbar_wait(bar_j[q], par_j[q], nullptr, 0);
    __syncthreads();
  };
  // streamed joint rows: group g (rows v0 + 8g ..) into ring slot g & 1, one row per lane of warp 0
  auto issue_joint = [&](int g) {
    const int q = g & 1, r0 = g * TD_RG, nr = min(TD_RG, nv - r0);
    if (warp == 0) {
      fence_proxy_async_smem();
      if (lane == 0) mbar_expect_tx(bar_j[q], (uint32_t)(nr * J * 4));
      __syncwarp();
      if (lane < nr)
        bulk_g2s(smem_u32(sWj + (size_t)(q * TD_RG + lane) * J), a.w_out + (size_t)(v0 + r0 + lane) * J,
                 (uint32_t)(J * 4), bar_j[q]);
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_j[q]);
    }
    j_out[q] = true;
  };
  const bool stream_lstm = a.held < L;  // one resident layer: the next one is copied during the barrier
  if (!stream_lstm && !cta_wait(bar_w, par_w, w_out, a.err)) return drain();

  auto chunk_has = [&](int c0, const int* flags, int want) {
    bool any = false;
    for (int i = 0; i < TD_CB && c0 + i < B; ++i) any |= flags[c0 + i] == want;
    return any;
  };
  auto merge_confs = [&](int it) {
    const float2* pp = parts_all + (size_t)(it & 1) * G * B;
    for (int b = cta; b < B; b += G)
      if (st_emit[b]) merge_conf(pp, G, B, b, V1, a.tokens + ((size_t)st_toff[b] + st_ntok[b] - 1) * 4 + 2);
  };

  int n_pending = 0;
  for (int b = 0; b < B; ++b) n_pending += st_pend[b];
  int iter = 0;
  for (;; ++iter) {
    // ---- P: prediction network (utterances whose output is stale)
    if (n_pending > 0) {
      for (int l = 0; l < L; ++l) {
        if (stream_lstm && !cta_wait(bar_w, par_w, w_out, a.err)) return drain();  // this layer's rows
        const float* wl = wl_of(l);
        const int K = l == 0 ? H : 2 * H;  // layer 0: h only (its input part is in gate0)
        for (int c0 = 0; c0 < B; c0 += TD_CB) {
          if (nu == 0 || !chunk_has(c0, st_pend, 1)) continue;  // uniform across the CTA
          __syncthreads();  // earlier readers of sX / sC are done
          if (warp == 0) {
            // inputs per pending utterance: layer 0 [h], deeper layers [x | h]
            // with x the new output of the layer below; h = the committed state
            fence_proxy_async_smem();
            fence_proxy_async_global();
            const int i = lane & (TD_CB - 1), b = c0 + i;
            const float* src = nullptr;
            if (b < B && st_pend[b] && (l > 0 || lane >= TD_CB)) {
              const int cur = st_cur[b];
              src = lane < TD_CB ? a.h + (((size_t)(1 - cur) * L + (l - 1)) * B + b) * H
                                 : a.h + (((size_t)cur * L + l) * B + b) * H;
            }
            warp_copy(bar_x, smem_u32(sX + i * ldk + (lane < TD_CB || l == 0 ? 0 : H)), src, (uint32_t)(H * 4));
          }
          x_out = true;
          for (int e = threadIdx.x; e < nu * TD_CB; e += TD_THREADS) {  // committed cells [unit][item]
            const int u = e / TD_CB, i = e % TD_CB, b = c0 + i;
            const bool act = b < B && st_pend[b];
            sC[e] = act ? __ldcg(a.c + (((size_t)st_cur[b] * L + l) * B + b) * H + u0 + u) : 0.f;
            if (l == 0) {  // input gates of the last token (row V1: the SOS step)
              const float* g = a.gate0 + (size_t)(act && st_have[b] ? st_last[b] : V1) * 4 * H + u0 + u;
#pragma unroll
              for (int q = 0; q < 4; ++q) sE[e * 4 + q] = __ldg(g + (size_t)q * H);
            }
          }
          if (!cta_wait(bar_x, par_x, x_out, a.err)) return drain();
          for (int ug = 0; ug < nu; ug += 2) {
            cta_gemv(wl + (size_t)ug * 4 * K, K, min(TD_RG, 4 * (nu - ug)), sX, ldk, K, sR, sZ);
            if (threadIdx.x < 2 * TD_CB) {
              const int uu = threadIdx.x / TD_CB, i = threadIdx.x % TD_CB, b = c0 + i, u = ug + uu;
              if (u < nu && b < B && st_pend[b]) {
                const int cur = st_cur[b];
                const float* bl = l == 0 ? sE + (u * TD_CB + i) * 4 : sBl + (l * lay.nu + u) * 4;
                const float zi = sZ[(uu * 4 + 0) * TD_CB + i] + bl[0];
                const float zf = sZ[(uu * 4 + 1) * TD_CB + i] + bl[1];
                const float zg = sZ[(uu * 4 + 2) * TD_CB + i] + bl[2];
                const float zo = sZ[(uu * 4 + 3) * TD_CB + i] + bl[3];
                const float cn = fmaf(sigm(zf), sC[u * TD_CB + i], sigm(zi) * tanhf(zg));
                const size_t o = (((size_t)(1 - cur) * L + l) * B + b) * H + u0 + u;
                a.c[o] = cn;
                a.h[o] = sigm(zo) * tanhf(cn);
              }
            }
          }
        }
        if (threadIdx.x < 2 * TD_CB) fence_proxy_async_global();  // h is read by bulk copies next
        if (stream_lstm) {  // the slot is free: copy the next layer (of this step or the next)
          __syncthreads();
          if (warp == 0) {
            fence_proxy_async_smem();
            if (lane == 0) mbar_expect_tx(bar_w, lstm_bytes((l + 1) % L));
            __syncwarp();
            copy_lstm((l + 1) % L);
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_w);
          }
          w_out = true;
        }
        if (!grid_sync(a.bar_count, bar_target, a.err, &s_ok)) return drain();
      }
      // pred projection of the new top-layer output
      for (int c0 = 0; c0 < B; c0 += TD_CB) {
        if (nj == 0 || !chunk_has(c0, st_pend, 1)) continue;
        __syncthreads();
        if (warp == 0) {
          fence_proxy_async_smem();
          fence_proxy_async_global();
          const int b = c0 + lane;
          const float* src = (lane < TD_CB && b < B && st_pend[b])
                                 ? a.h + (((size_t)(1 - st_cur[b]) * L + (L - 1)) * B + b) * H
                                 : nullptr;
          warp_copy(bar_x, smem_u32(sX + (lane & (TD_CB - 1)) * ldk), src, (uint32_t)(H * 4));
        }
        x_out = true;
        if (!cta_wait(bar_x, par_x, x_out, a.err)) return drain();
        for (int r0 = 0; r0 < nj; r0 += TD_RG) {
          const int nr = min(TD_RG, nj - r0);
          cta_gemv(sWp + (size_t)r0 * H, H, nr, sX, ldk, H, sR, sZ);
          if (threadIdx.x < TD_RG * TD_CB) {
            const int r = threadIdx.x / TD_CB, i = threadIdx.x % TD_CB, b = c0 + i;
            if (r < nr && b < B && st_pend[b]) a.pred_proj[(size_t)b * J + j0 + r0 + r] = sZ[threadIdx.x] + sBp[r0 + r];
          }
        }
      }
      if (threadIdx.x < TD_RG * TD_CB) fence_proxy_async_global();  // pred_proj is read by bulk copies next
      if (!grid_sync(a.bar_count, bar_target, a.err, &s_ok)) return drain();
    }

    // ---- J: joint rows [v0, v1) of this CTA for every live utterance
    const int kb = iter % 3;
    float2* parts = parts_all + (size_t)(iter & 1) * G * B;
    bool conf_done = iter == 0;
    for (int c0 = 0; c0 < B; c0 += TD_CB) {
      if (!chunk_has(c0, st_done, 0)) continue;
      __syncthreads();
      if (warp == 0) {  // [enc_proj row of the utterance's frame | pred_proj]
        fence_proxy_async_smem();
        fence_proxy_async_global();
        const int i = lane & (TD_CB - 1), b = c0 + i;
        const float* src = nullptr;
        if (b < B && !st_done[b])
          src = lane < TD_CB ? a.enc_proj + (size_t)(st_off[b] + st_t[b]) * a.ld_enc : a.pred_proj + (size_t)b * J;
        warp_copy(bar_x, smem_u32(sX + i * ldk + (lane < TD_CB ? 0 : J)), src, (uint32_t)(J * 4));
      }
      x_out = true;
      if (!lay.jres) {  // the first two row groups of the streamed joint weight
        for (int g = 0; g < 2 && g * TD_RG < nv; ++g) issue_joint(g);
      }
      if (!conf_done && warp == 1) merge_confs(iter - 1);  // overlaps the copies
      conf_done = true;
      if (!cta_wait(bar_x, par_x, x_out, a.err)) return drain();
      for (int e = threadIdx.x; e < TD_CB * (J / 4); e += TD_THREADS) {  // sX[i] = ReLU(enc + pred)
        const int i = e / (J / 4), k = (e % (J / 4)) * 4;
        float4* x = reinterpret_cast<float4*>(sX + i * ldk + k);
        const float4 e4 = *x, p4 = *reinterpret_cast<const float4*>(sX + i * ldk + J + k);
        *x = make_float4(fmaxf(e4.x + p4.x, 0.f), fmaxf(e4.y + p4.y, 0.f), fmaxf(e4.z + p4.z, 0.f),
                         fmaxf(e4.w + p4.w, 0.f));
      }
      __syncthreads();
      // thread i < TD_CB: running (token max, first arg, sum of exp) and (duration max, first arg)
      float tmax = -INFINITY, tsum = 0.f, dmax = -INFINITY;
      int targ = -1, darg = -1;
      for (int r0 = 0, g = 0; r0 < nv; r0 += TD_RG, ++g) {
        const int nr = min(TD_RG, nv - r0);
        const float* wj = sWj + (size_t)r0 * J;
        if (!lay.jres) {
          if (!cta_wait(bar_j[g & 1], par_j[g & 1], j_out[g & 1], a.err)) return drain();
          wj = sWj + (size_t)(g & 1) * TD_RG * J;
        }
        cta_gemv(wj, J, nr, sX, ldk, J, sR, sZ);  // ends with a CTA barrier: the slot is free again
        if (!lay.jres && r0 + 2 * TD_RG < nv) issue_joint(g + 2);
        if (threadIdx.x < TD_CB) {
          for (int r = 0; r < nr; ++r) {  // rows in increasing order: the first maximum wins on ties
            const int v = v0 + r0 + r;
            const float lg = sZ[r * TD_CB + threadIdx.x] + sBj[r0 + r];
            if (v < V1) {
              if (targ < 0 || lg > tmax) {
                tsum = (targ < 0 ? 0.f : tsum * __expf(tmax - lg)) + 1.f;
                tmax = lg;
                targ = v;
              } else {
                tsum += __expf(lg - tmax);
              }
            } else if (darg < 0 || lg > dmax) {
              dmax = lg;
              darg = v - V1;
            }
          }
        }
      }
      if (threadIdx.x < TD_CB) {
        const int b = c0 + threadIdx.x;
        if (b < B && !st_done[b]) {
          if (targ >= 0) atomicMax(tok_key + kb * B + b, argmax_key(tmax, targ));
          if (darg >= 0) atomicMax(dur_key + kb * B + b, argmax_key(dmax, darg));
          parts[(size_t)cta * B + b] = targ >= 0 ? make_float2(tmax, tsum) : make_float2(-INFINITY, 0.f);
        }
      }
    }
    if (!conf_done && warp == 1) merge_confs(iter - 1);  // no live utterance left in any chunk
    if (!grid_sync(a.bar_count, bar_target, a.err, &s_ok)) return drain();

    // ---- D: decisions, in every CTA (a thread per utterance)
    if (threadIdx.x == 0) {
      s_np = 0;
      s_nd = 0;
    }
    __syncthreads();
    int np = 0, nd = 0;
    for (int b = threadIdx.x; b < B; b += TD_THREADS) {
      int emitted = 0;
      if (!st_done[b]) {
        const unsigned long long tk = __ldcg(tok_key + kb * B + b);
        const unsigned long long dk = a.D > 0 ? __ldcg(dur_key + kb * B + b) : 0ull;
        const int k = (int)~(uint32_t)tk, da = (int)~(uint32_t)dk;
        if (tk == 0ull || k < 0 || k >= V1 || (a.D > 0 && (dk == 0ull || da < 0 || da >= a.D))) {
          // no CTA produced a maximum: no token or duration to follow
          if (cta == 0) report_error(a.err, DEV_ERR_NONFINITE);
          st_done[b] = 1;
          st_pend[b] = 0;
        } else {
          int t = st_t[b];
          const bool emit = k != a.blank;
          const int skip = a.D > 0 ? s_dur[da] : 1;
          if (emit) {
            const int n = st_ntok[b];
            if (n < st_tcap[b]) {
              if (cta == 0) {
                int* tk4 = a.tokens + ((size_t)st_toff[b] + n) * 4;
                tk4[0] = k;
                tk4[1] = t;  // tk4[2], the confidence, is merged during the next iteration
                tk4[3] = a.D > 0 ? skip : 1;
                a.ntok[b] = n + 1;
              }
              st_ntok[b] = n + 1;
              emitted = 1;
            } else if (cta == 0) {
              report_error(a.err, DEV_ERR_BAD_SHAPE);
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
          if (t >= st_len[b]) {
            st_done[b] = 1;
            st_pend[b] = 0;
          }
        }
      }
      st_emit[b] = emitted;
      np += st_pend[b];
      nd += st_done[b];
      if (cta == 0) {  // keys of iteration iter + 2 (all CTAs last read them in iteration iter - 1)
        tok_key[((iter + 2) % 3) * B + b] = 0ull;
        dur_key[((iter + 2) % 3) * B + b] = 0ull;
      }
    }
    if (np) atomicAdd(&s_np, np);
    if (nd) atomicAdd(&s_nd, nd);
    __syncthreads();
    n_pending = s_np;
    bool stop = s_nd >= B;
    if (!stop && iter + 1 >= a.max_iters) {
      if (cta == 0 && threadIdx.x == 0) report_error(a.err, DEV_ERR_BAD_SHAPE);
      stop = true;
    }
    if (stop) break;
  }
  // confidences of the final iteration's tokens (no later iteration overwrites them)
  if (warp == 1) merge_confs(iter);
  drain();  // a streamed layer copy may still be in flight
}

// out[v][r] = sum_k embed[v][k] w[r][k] + b[r] (v < V1), out[V1][r] = b[r]:
// 64 x 64 output tiles, 16-deep k slabs in shared memory, 4 x 4 per thread.
__global__ void __launch_bounds__(256) k_gate0(const float* __restrict__ embed, const float* __restrict__ w,
                                               const float* __restrict__ b, int V1, int N, int K,
                                               float* __restrict__ out) {
  __shared__ float sa[16][64 + 4], sb[16][64 + 4];  // [k][row] of embed / w
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int r0 = blockIdx.x * 64, v0 = blockIdx.y * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int e = threadIdx.x; e < 64 * 16; e += 256) {
      const int row = e / 16, k = e % 16;
      const int v = v0 + row, r = r0 + row, kk = k0 + k;
      sa[k][row] = (v < V1 && kk < K) ? embed[(size_t)v * K + kk] : 0.f;
      sb[k][row] = (r < N && kk < K) ? w[(size_t)r * K + kk] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      float av[4], bv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        av[j] = sa[k][ty * 4 + j];
        bv[j] = sb[k][tx * 4 + j];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int v = v0 + ty * 4 + i;
    if (v > V1) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = r0 + tx * 4 + j;
      if (r < N) out[(size_t)v * N + r] = (v < V1 ? acc[i][j] : 0.f) + b[r];
    }
  }
}

}  // namespace

cudaError_t transducer_gate0_launch(const float* embed, const float* w_ih0, const float* b0, int V1, int H,
                                    float* out, cudaStream_t st) {
  if (V1 < 1 || H < 1) return cudaErrorInvalidValue;
  const int N = 4 * H;
  k_gate0<<<dim3((N + 63) / 64, (V1 + 1 + 63) / 64), 256, 0, st>>>(embed, w_ih0, b0, V1, N, H, out);
  return cudaGetLastError();
}

size_t transducer_smem_bytes(int H, int J, int L, int VP, int grid, int B) {
  return td_layout_for(H, J, L, VP, grid, B).bytes;
}
size_t transducer_smem_limit() { return TD_SMEM_LIMIT; }
int transducer_max_batch(int H, int J, int L, int VP, int grid) {
  const size_t fixed = transducer_smem_bytes(H, J, L, VP, grid, 0);
  return fixed >= TD_SMEM_LIMIT ? 0 : (int)((TD_SMEM_LIMIT - fixed) / (TD_STATE_INTS * sizeof(int)));
}
size_t transducer_key_bytes(int B) { return (size_t)6 * B * sizeof(unsigned long long); }
size_t transducer_partial_bytes(int grid, int B) {
  return transducer_key_bytes(B) + (size_t)2 * grid * B * sizeof(float2);
}

cudaError_t transducer_greedy_launch(const TransducerArgs& a, int grid, cudaStream_t st) {
  if (a.B <= 0) return cudaSuccess;
  const int VP = a.V1 + a.D;
  if (a.H < 4 || a.J < 4 || a.H % 4 || a.J % 4 || a.L < 1 || grid < 1 || a.D < 0 || a.D > TD_MAX_DUR || a.V1 < 2)
    return cudaErrorInvalidValue;
  // bulk copies: 16-byte aligned sources and destinations
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!a.gate0 || !al16(a.w_ih) || !al16(a.w_hh) || !al16(a.w_pred) || !al16(a.w_out) ||
      !al16(a.enc_proj) || a.ld_enc % 4 || !al16(a.h) || !al16(a.pred_proj) || !al16(a.keys))
    return cudaErrorInvalidValue;
  TdLayout lay = td_layout_for(a.H, a.J, a.L, VP, grid, a.B);
  if (const char* e = std::getenv("PKC_DECODE_STREAM"))  // one resident LSTM layer (the streamed path)
    if (std::atoi(e) == 1 && a.L > 1) lay = td_layout(a.H, a.J, a.L, VP, grid, a.B, 1, lay.jres);
  if (const char* e = std::getenv("PKC_DECODE_JOINT_STREAM"))  // joint rows streamed (the large-vocabulary path)
    if (std::atoi(e) == 1) lay = td_layout(a.H, a.J, a.L, VP, grid, a.B, lay.held, 0);
  if (lay.bytes > TD_SMEM_LIMIT) return cudaErrorInvalidValue;
  cudaError_t e =
      cudaFuncSetAttribute(k_transducer_greedy, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lay.bytes);
  if (e != cudaSuccess) return e;
  TransducerArgs ka = a;
  ka.held = lay.held;
  ka.jres = lay.jres;
  void* params[] = {&ka};
  return cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(&k_transducer_greedy), dim3(grid),
                                     dim3(TD_THREADS), params, lay.bytes, st);
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
