// Relative-position multi-head self-attention on the 5th-generation tensor
// cores: tcgen05.mma with f32 accumulators in tensor memory, operands staged
// by TMA (128-byte swizzle), flash-style online softmax (no T x T buffer).
//
// Reference: RelPosAttention::build_graph_batched (src/relpos_attention.cpp:162-306):
//   ac = (q + pos_bias_u) k^T,  bd = (q + pos_bias_v) p^T,
//   bd <- rel_shift(bd)  (pad / reshape / view / cont sequence, :230-238),
//   attn = softmax((ac + bd) / sqrt(dk) + key_mask),  ctx = attn v,
//   padded query rows zeroed.
// rel_shift is an index map: score (i, j) takes bd at positional row
// r = c - 1 - i + j (c = table centre; row r holds relative position c-1-r).
//
// One CTA = one 128-row query tile of one utterance x one head; keys are
// visited in tiles of KN = 64. For query rows q0..q0+127 and key tile t the
// positional rows needed are the window W_t = [rb + 64t, rb + 64t + 191)
// (rb = c - 1 - (q0 + 127)), and score (i, j) reads window column
// 127 - i + j. Consecutive windows overlap by 128 rows, so the positional
// scores are produced as 64-column chunks C_k = Qv * P[rb + 64k, +64)^T:
// tile t reads chunks t, t+1, t+2 and computes exactly one new chunk.
// The positional term therefore costs the same tensor work as Q K^T.
//
// Tensor memory (512 columns x 128 lanes, lane = query row):
//   [0, 128)     O accumulator (DK columns used)
//   [128, 192)   S = Qu K^T of the next key tile
//   [192, 384)   ring of three positional chunks (chunk k in slot k % 3)
//   [384, 448)   Qv = Q + v, f16/bf16 pairs: the A operand of the chunk MMAs
//   [448, 512)   P, two 32-column buffers (key-tile parity): the A operand of P V
// Shared memory: Qu = Q + u (A operand of S, written over the TMA-loaded Q
// tile), an 8-stage ring carrying K tiles, positional chunks and V tiles in
// the order the MMAs consume them, and one 100-word row per query row
// through which the diagonal shift is applied: tensor-memory loads read the
// same columns in every lane, so each row's window is written out and read
// back at the row's own offset.
//
// Warps: 0 = TMA producer, 1 = MMA issuer (one thread), 2..9 = softmax.
// Softmax warp w owns TMEM lanes 32(w%4)..+31 (one query row per lane) and
// keys 32h..32h+31 of every tile, h = (w-2)/4. The softmax is software
// pipelined by one key tile: while the exponentials of tile t run on the
// special-function unit, the same warp moves tile t+1's scores out of tensor
// memory and through the shift rows (load/store unit). S and the positional
// chunks are released as soon as they are in registers, so one S buffer and
// three chunk slots keep the tensor pipe a tile ahead.
// Online softmax with a lazy rescale: the running maximum used for the
// exponentials only moves when a tile maximum exceeds it by more than 8
// (log2 units), so P stays <= 256 and O is rescaled (tcgen05.ld / st by the
// rows' own threads) only on those rare moves. The final O / l is exact.
//
// Frames are packed per utterance (no padding); keys >= T are masked, query
// rows >= T are computed but not stored -- the reference's masking.
#include "common.cuh"
#include "per_device.h"
#include "gemm.h"
#include "kernels.h"

namespace pkc {

namespace {

constexpr int QM = 128;      // query rows per CTA (MMA M, TMEM lanes)
constexpr int KN = 64;       // keys per tile (MMA N of S and of a chunk)
constexpr int SM_WARPS = 8;  // softmax warps
constexpr int THREADS = 64 + 32 * SM_WARPS;
constexpr int RING = 8;      // K / positional / V stages
constexpr int SKEW_LD = 100; // words per query row: 96 + 4 (conflict-free v4 stores and skewed loads)
constexpr float kRescaleLog2 = 8.0f;

enum : int {
  B_QFULL = 0, B_QREADY = 1, B_RFULL = 2, B_REMPTY = B_RFULL + RING,
  B_SFULL = B_REMPTY + RING, B_STFREE = B_SFULL + 1, B_PFULL = B_STFREE + 1, B_PVDONE = B_PFULL + 2,
  B_FINAL = B_PVDONE + 2, B_PSKEW = B_FINAL + 1, B_PMAX = B_PSKEW + 4, N_BARS = B_PMAX + 4
};

template <int DK>
struct TcLayout {
  static constexpr int KB = DK / 64;           // 64-column (128-byte) k-blocks
  static constexpr int Q_BYTES = QM * DK * 2;
  static constexpr int T_BYTES = KN * DK * 2;  // one K, V or positional-chunk tile
  static constexpr int OFF_QU = 0;
  static constexpr int OFF_RING = OFF_QU + Q_BYTES;
  static constexpr int OFF_SKEW = OFF_RING + RING * T_BYTES;
  static constexpr int OFF_RED = OFF_SKEW + QM * SKEW_LD * 4;  // [2 parity][2 half][QM] floats
  static constexpr int OFF_BIAS = OFF_RED + 2 * 2 * QM * 4;  // [u | v] of the head, 2 dk floats
  static constexpr int OFF_BAR = OFF_BIAS + 2 * DK * 4;
  static constexpr int OFF_SLOT = OFF_BAR + N_BARS * 8;
  static constexpr int SMEM = OFF_SLOT + 16 + 1024;  // + alignment slack
};

constexpr uint32_t TM_O = 0, TM_S = 128, TM_BD = 192, TM_QV = 384, TM_P = 448;

struct TcParams {
  const int* tiles;     // [n_tiles][2] (item, q0)
  const int* item_off;
  const int* item_len;
  const float* bias_u;  // [H * dk]
  const float* bias_v;
  void* ctx;            // [M, d]
  int d, centre;
  float scale_log2;
  int* err;
  int qu_folded;        // q columns hold q + bias_u (AttnArgs::qu_folded)
};

// window column wc (0..191) of key tile t -> TMEM column of its chunk slot
__device__ __forceinline__ uint32_t bd_col(int t, int wc) {
  return TM_BD + 64u * (uint32_t)((t + (wc >> 6)) % 3) + (uint32_t)(wc & 63);
}

// Loads in issue (= consumption) order: positional chunks 0, 1, K tile 0,
// chunk 2, then for u = 0 .. nT-2: K tile u+1, chunk u+3, V tile u-1 (u >= 1),
// and finally V tiles nT-2 (if nT >= 2) and nT-1.
//   position of K tile u (u >= 1):  4 + 3(u-1) - (u >= 2)
//   the group of u holds 2 loads for u = 0 and 3 for u >= 1
struct LoadSeq {
  int kind, idx;  // kind 0 = K tile, 1 = positional chunk, 2 = V tile
};
__device__ __forceinline__ int group_start(int u) { return u == 0 ? 4 : 6 + 3 * (u - 1); }
__device__ __forceinline__ LoadSeq load_at(int n, int nT) {
  if (n < 2) return {1, n};
  if (n == 2) return {0, 0};
  if (n == 3) return {1, 2};
  if (nT >= 2) {
    if (n < 6) return n == 4 ? LoadSeq{0, 1} : LoadSeq{1, 3};  // group u = 0
    const int m = n - 6, u = 1 + m / 3, r = m % 3;
    if (u <= nT - 2) return r == 0 ? LoadSeq{0, u + 1} : r == 1 ? LoadSeq{1, u + 3} : LoadSeq{2, u - 1};
    // tail: V(nT-2), V(nT-1)
    const int tail = n - group_start(nT - 1);
    return {2, nT - 2 + tail};
  }
  return {2, 0};  // nT == 1: C0 C1 K0 C2 V0
}
__device__ __forceinline__ int n_loads_for(int nT) { return nT >= 2 ? group_start(nT - 1) + 2 : 5; }
__device__ __forceinline__ int pos_k(int u) { return u == 0 ? 2 : group_start(u - 1); }          // K tile u
__device__ __forceinline__ int pos_c(int c) { return c < 2 ? c : c == 2 ? 3 : group_start(c - 3) + 1; }  // chunk c
__device__ __forceinline__ int pos_v(int u, int nT) {                                          // V tile u
  if (nT == 1) return 4;
  if (u <= nT - 3) return group_start(u + 1) + 2;
  return group_start(nT - 1) + (u - (nT - 2));
}

template <typename H, int DK>
__global__ void __launch_bounds__(THREADS, 1)
    k_relpos_attn_tc(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_pos,
                     TcParams p) {
  using L = TcLayout<DK>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L::OFF_SLOT);
  const uint32_t sbase = smem_u32(sm);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    prefetch_tmap(&tm_qkv);
    prefetch_tmap(&tm_pos);
    for (int i = 0; i < N_BARS; ++i) {
      const bool per_warp = i == B_QREADY || i == B_STFREE || i == B_PFULL || i == B_PFULL + 1;
      mbar_init(bar(i), per_warp ? (uint32_t)SM_WARPS : i >= B_PSKEW ? 2u : 1u);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  // the head's pos_bias_u / pos_bias_v are weights: staged before the
  // dependency wait, so the Q preparation reads them from shared memory
  // ([u | v], or [0 | v - u] when q already carries u)
  {
    float4* sb = reinterpret_cast<float4*>(sm + L::OFF_BIAS);
    const int hd = blockIdx.x;
    for (int j = threadIdx.x; j < DK / 2; j += THREADS) {
      const int jj = j < DK / 4 ? j : j - DK / 4;
      const float4 u = *reinterpret_cast<const float4*>(p.bias_u + hd * DK + 4 * jj);
      if (j < DK / 4) {
        sb[j] = p.qu_folded ? make_float4(0.f, 0.f, 0.f, 0.f) : u;
      } else {
        const float4 v = *reinterpret_cast<const float4*>(p.bias_v + hd * DK + 4 * jj);
        sb[j] = p.qu_folded ? make_float4(v.x - u.x, v.y - u.y, v.z - u.z, v.w - u.w) : v;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  pdl_trigger();

  // heads vary fastest in launch order, so every head of the longest tile
  // (the tile list is sorted longest utterance first) is issued first
  const int head = blockIdx.x, tile = blockIdx.y;
  const int item = p.tiles[2 * tile], q0 = p.tiles[2 * tile + 1];
  const int off = p.item_off[item], T = p.item_len[item];
  const int nT = (T + KN - 1) / KN;
  const int n_loads = n_loads_for(nT);
  const int rb = p.centre - 1 - (q0 + QM - 1);  // first positional row of chunk 0

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    // The whole warp runs the loop (waits are warp-wide); one elected lane
    // arms the barriers and issues the copies.
    const uint32_t leader = elect_one();
    auto wwait = [&](int b, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar(b), parity, p.err, DEV_ERR_TIMEOUT_ATTN)) != 0;
    };
    const int colq = head * DK, colk = p.d + head * DK, colv = 2 * p.d + head * DK;
    mbar_arrive_expect_tx_if(leader, bar(B_QFULL), L::Q_BYTES);
#pragma unroll
    for (int kb = 0; kb < L::KB; ++kb)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        tma_load_2d_if(leader, sbase + L::OFF_QU + kb * QM * 128 + h * 64 * 128, &tm_qkv, bar(B_QFULL),
                       colq + kb * 64, off + q0 + 64 * h);
    int n = 0;
    for (; n < n_loads; ++n) {
      const int s = n % RING;
      if (!wwait(B_REMPTY + s, ((uint32_t)(n / RING) & 1u) ^ 1u)) break;
      const LoadSeq ls = load_at(n, nT);
      const CUtensorMap* map = ls.kind == 1 ? &tm_pos : &tm_qkv;
      const int col = ls.kind == 0 ? colk : ls.kind == 1 ? head * DK : colv;
      const int row = ls.kind == 1 ? rb + KN * ls.idx : off + KN * ls.idx;
      mbar_arrive_expect_tx_if(leader, bar(B_RFULL + s), L::T_BYTES);
#pragma unroll
      for (int kb = 0; kb < L::KB; ++kb)
        tma_load_2d_if(leader, sbase + L::OFF_RING + s * L::T_BYTES + kb * KN * 128, map, bar(B_RFULL + s),
                       col + kb * 64, row);
    }
    if (n < n_loads) {
      // a consumer gave up: let every copy already issued land before the
      // CTA may exit (the last load of each stage; earlier ones on the same
      // stage were consumed, or a later one could not have been issued)
      mbar_wait(bar(B_QFULL), 0, nullptr, 0);
      for (int m = n - RING; m < n; ++m)
        if (m >= 0) mbar_wait(bar(B_RFULL + m % RING), (uint32_t)(m / RING) & 1u, nullptr, 0);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // Whole warp, one elected lane issuing (commits track that lane's MMAs).
    const uint32_t leader = elect_one();
    auto wwait = [&](int b, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar(b), parity, p.err, DEV_ERR_TIMEOUT_ATTN)) != 0;
    };
    constexpr int fmt = is_bf16<H>::value ? 1 : 0;
    constexpr uint32_t id_s = idesc_f16(QM, KN, fmt);
    constexpr uint32_t id_pv = idesc_f16(QM, DK, fmt) | (1u << 16);  // B (V) MN-major
    // q + u in shared memory: the TMA tile itself when q carries u (S(0) can
    // go once it has landed), else after the softmax warps rewrote it
    bool ok = wwait(p.qu_folded ? B_QFULL : B_QREADY, 0);
    tc_fence_after();
    const uint64_t dqu = smem_desc_sw128(sbase + L::OFF_QU);
    // K-step kk (16 elements of dk): k-block kk/4, 32 bytes per step inside it
    auto a_off = [](int kk) { return (uint64_t)(((kk >> 2) * QM * 128 + (kk & 3) * 32) >> 4); };
    auto b_off = [](int kk) { return (uint64_t)(((kk >> 2) * KN * 128 + (kk & 3) * 32) >> 4); };
    auto ring_wait = [&](int n) -> bool {
      if (!wwait(B_RFULL + n % RING, (uint32_t)(n / RING) & 1u)) return false;
      tc_fence_after();
      return true;
    };
    auto ring_addr = [&](int n) { return sbase + L::OFF_RING + (n % RING) * L::T_BYTES; };
    auto s_mma = [&](int u) -> bool {  // S = Qu K(u)^T
      const int n = pos_k(u);
      if (!ring_wait(n)) return false;
      const uint64_t db = smem_desc_sw128(ring_addr(n));
#pragma unroll
      for (int kk = 0; kk < DK / 16; ++kk)
        umma_f16_if(leader, tmem + TM_S, dqu + a_off(kk), db + b_off(kk), id_s, kk > 0 ? 1u : 0u);
      umma_commit_if(leader, bar(B_REMPTY + n % RING));
      return true;
    };
    auto c_mma = [&](int c) -> bool {  // chunk c = Qv (tensor memory) P(c)^T
      const int n = pos_c(c);
      if (!ring_wait(n)) return false;
      const uint64_t db = smem_desc_sw128(ring_addr(n));
      const uint32_t dcol = TM_BD + 64u * (uint32_t)(c % 3);
#pragma unroll
      for (int kk = 0; kk < DK / 16; ++kk)
        umma_f16_ts_if(leader, tmem + dcol, tmem + TM_QV + 8u * kk, db + b_off(kk), id_s, kk > 0 ? 1u : 0u);
      umma_commit_if(leader, bar(B_REMPTY + n % RING));
      return true;
    };
    auto pv = [&](int u) -> bool {  // O += P(u) (tensor memory) V(u)
      if (!wwait(B_PFULL + (u & 1), ((uint32_t)u >> 1) & 1u)) return false;
      const int n = pos_v(u, nT);
      if (!ring_wait(n)) return false;
      const uint64_t dv = smem_desc_sw128_mn(ring_addr(n), KN * 128, 1024);
      const uint32_t pa = tmem + TM_P + 32u * (uint32_t)(u & 1);
#pragma unroll
      for (int kk = 0; kk < KN / 16; ++kk)
        umma_f16_ts_if(leader, tmem + TM_O, pa + 8u * kk, dv + (uint64_t)((kk * 16 * 128) >> 4), id_pv,
                       (u > 0 || kk > 0) ? 1u : 0u);
      umma_commit_if(leader, bar(B_REMPTY + n % RING));
      umma_commit_if(leader, bar(B_PVDONE + (u & 1)));
      return true;
    };
    if (p.qu_folded) {
      // q + v (tensor memory) is ready at QREADY
      ok = ok && s_mma(0) && wwait(B_QREADY, 0);
      tc_fence_after();
      ok = ok && c_mma(0) && c_mma(1) && c_mma(2);
    } else {
      ok = ok && c_mma(0) && c_mma(1) && s_mma(0) && c_mma(2);
    }
    if (ok) umma_commit_if(leader, bar(B_SFULL));
    // S(u+1) and chunk u+3 go to the tensor pipe as soon as the softmax has
    // read tile u, ahead of P(u-1) V(u-1): the softmax waits on S, while
    // P V only has to finish before the P buffer comes round again
    for (int u = 0; u < nT && ok; ++u) {
      if (u + 1 < nT) {
        // S and chunk u are free once the softmax has read tile u
        ok = wwait(B_STFREE, (uint32_t)u & 1u);
        if (!ok) break;
        tc_fence_after();
        ok = s_mma(u + 1) && c_mma(u + 3);
        if (!ok) break;
        umma_commit_if(leader, bar(B_SFULL));
      }
      if (u >= 1) ok = pv(u - 1);
    }
    if (ok) pv(nT - 1);
    // every issued MMA has completed before TMEM can be released
    umma_commit_if(leader, bar(B_FINAL));
    wwait(B_FINAL, 0);
  } else {
    // ---------------------------------------------------------------- softmax warps
    const int q = warp & 3;              // TMEM lane quarter
    const int hh = (warp - 2) >> 2;      // key half of every tile
    const int i = 32 * q + lane;         // query row within the tile = TMEM lane
    const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16);
    bool ok = __all_sync(0xffffffffu, mbar_wait(bar(B_QFULL), 0, p.err, DEV_ERR_TIMEOUT_ATTN)) != 0;
    if (ok) {
      // Row i, dk columns [hh*DK/2, (hh+1)*DK/2): Qu = Q + u back into the
      // swizzled tile (16-byte chunk pc of row r holds logical columns
      // 8 * (pc ^ (r & 7)) of its k-block), Qv = Q + v into tensor memory
      constexpr int CPT = DK / 16;  // 16-byte chunks per thread
      uint32_t qv[DK / 4];
#pragma unroll
      for (int k = 0; k < CPT; ++k) {
        const int lc = hh * CPT + k;          // logical chunk in the row
        const int kb = lc >> 3, c8 = lc & 7;
        const int col = kb * 64 + c8 * 8;
        uint8_t* src = sm + L::OFF_QU + kb * QM * 128 + i * 128 + ((c8 ^ (i & 7)) << 4);
        const uint4 raw = *reinterpret_cast<const uint4*>(src);
        const H* hv = reinterpret_cast<const H*>(&raw);
        const float* sbu = reinterpret_cast<const float*>(sm + L::OFF_BIAS);
        const float4 u0 = *reinterpret_cast<const float4*>(sbu + col);
        const float4 u1 = *reinterpret_cast<const float4*>(sbu + col + 4);
        const float4 v0 = *reinterpret_cast<const float4*>(sbu + DK + col);
        const float4 v1 = *reinterpret_cast<const float4*>(sbu + DK + col + 4);
        const float bu[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
        const float bv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        uint32_t wu[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x0 = from_h(hv[2 * e]), x1 = from_h(hv[2 * e + 1]);
          wu[e] = pack2<H>(x0 + bu[2 * e], x1 + bu[2 * e + 1]);
          qv[4 * k + e] = pack2<H>(x0 + bv[2 * e], x1 + bv[2 * e + 1]);
        }
        if (!p.qu_folded) *reinterpret_cast<uint4*>(src) = make_uint4(wu[0], wu[1], wu[2], wu[3]);
      }
      if constexpr (DK == 128) {
        tmem_st32(trow + TM_QV + 32u * hh, qv);
      } else {
        tmem_st16(trow + TM_QV + 16u * hh, qv);
      }
      tmem_st_wait();
      fence_proxy_async_smem();
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar(B_QREADY));

    // This row's shift buffer: window columns wc0 .. wc0+95 at words 0..95,
    // wc0 = 96 - 32q. Warp hh = 0 writes words [0, 64), warp hh = 1 writes
    // [64, 96) and also reads [32, 64) (after the pair's skew barrier).
    float* skew = reinterpret_cast<float*>(sm + L::OFF_SKEW) + i * SKEW_LD;
    float* red = reinterpret_cast<float*>(sm + L::OFF_RED);
    const float sl2 = p.scale_log2;
    float m_used = -INFINITY, lsum = 0.f, alpha = 1.f;
    bool resc = false;  // O must be scaled by alpha before P V of the current tile

    // warp-wide bounded wait (every lane tests; the vote agrees on the outcome)
    auto wwait = [&](int b, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar(b), parity, p.err, DEV_ERR_TIMEOUT_ATTN)) != 0;
    };
    // Scores of key tile t, in three steps so that the shift-row traffic of
    // tile t+1 can be interleaved with the exponentials of tile t:
    //  fetch:      S(t) and this warp's positional columns into registers, then
    //              S and chunk t are released to the MMA warp
    //  skew_store: the positional columns into this row's shift buffer
    //  skew_read:  (after the pair's skew barrier) the shifted read, plus S,
    //              keys >= T masked -> unscaled scores
    auto fetch = [&](int t, uint32_t (&sv)[32], uint32_t (&b0)[32], uint32_t (&b1)[32]) -> bool {
      if (!wwait(B_SFULL, (uint32_t)t & 1u)) return false;
      tc_fence_after();
      const int wc = 96 - 32 * q + 32 * hh;  // first window column for keys 32hh..
      tmem_ld32(trow + TM_S + 32u * hh, sv);
      if (hh == 0) tmem_ld32(trow + bd_col(t, wc), b0);  // warp hh = 1 does not store these columns
      tmem_ld32(trow + bd_col(t, wc + 32), b1);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_STFREE));
      return true;
    };
    auto skew_store = [&](const uint32_t (&b0)[32], const uint32_t (&b1)[32]) {
      float4* s4 = reinterpret_cast<float4*>(skew + 32 * hh);
      if (hh == 0) {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          s4[k] = make_float4(__uint_as_float(b0[4 * k]), __uint_as_float(b0[4 * k + 1]),
                              __uint_as_float(b0[4 * k + 2]), __uint_as_float(b0[4 * k + 3]));
      }
#pragma unroll
      for (int k = 0; k < 8; ++k)
        s4[8 + k] = make_float4(__uint_as_float(b1[4 * k]), __uint_as_float(b1[4 * k + 1]),
                                __uint_as_float(b1[4 * k + 2]), __uint_as_float(b1[4 * k + 3]));
    };
    auto skew_read = [&](int t, const uint32_t (&sv)[32], float (&x)[32]) {
      // key 32hh + j of row i sits at window column 127 - i + 32hh + j
      //   = wc + (31 - lane) + j, i.e. word 32hh + 31 - lane + j
      const float* src = skew + 32 * hh + (31 - lane);
#pragma unroll
      for (int j = 0; j < 32; ++j) x[j] = __uint_as_float(sv[j]) + src[j];
      if (t == nT - 1) {
        const int kv = T - KN * t - 32 * hh;  // valid keys of this half (may be <= 0)
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j >= kv) x[j] = -INFINITY;
      }
    };
    auto skew_sync = [&](int t) -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_PSKEW + q));
      return hh == 0 || wwait(B_PSKEW + q, (uint32_t)t & 1u);
    };
    auto half_max = [&](const float (&x)[32]) {
      float mx[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx[k] = fmaxf(fmaxf(x[4 * k], x[4 * k + 1]), fmaxf(x[4 * k + 2], x[4 * k + 3]));
      return fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
    };
    // publish this half's value k (max of tile k, or the final row sum at k = nT)
    auto pair_publish = [&](int k, float v) {
      red[(k & 1) * 2 * QM + hh * QM + i] = v;
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_PMAX + q));
    };
    auto pair_fetch = [&](int k, float& v) -> bool {
      if (!wwait(B_PMAX + q, (uint32_t)k & 1u)) return false;
      v = red[(k & 1) * 2 * QM + (hh ^ 1) * QM + i];
      return true;
    };
    // new running maximum for a tile whose row maximum (unscaled) is mrow
    auto update_max = [&](float mrow) {
      const float mt = mrow * sl2;
      resc = mt > m_used + kRescaleLog2;
      alpha = 1.f;
      if (resc) {
        alpha = ex2_approx(m_used - mt);  // 0 on the first tile
        m_used = mt;
        lsum *= alpha;
      }
    };
    // probabilities of keys [16 * part, 16 * part + 16) of a score row
    auto exps = [&](const float (&x)[32], uint32_t (&pk)[16], int part) {
      float rs[2] = {0.f, 0.f};
#pragma unroll
      for (int j = 8 * part; j < 8 * part + 8; ++j) {
        const float p0 = ex2_approx(fmaf(x[2 * j], sl2, -m_used));
        const float p1 = ex2_approx(fmaf(x[2 * j + 1], sl2, -m_used));
        rs[j & 1] += p0 + p1;
        pk[j] = pack2<H>(p0, p1);
      }
      lsum += rs[0] + rs[1];
    };

    // One pipelined step: probabilities of tile t (xc) while tile t+1's
    // scores are moved into xn; then P(t) to tensor memory and the running
    // maximum for tile t+1.
    float mh_next = 0.f;
    auto step = [&](int t, const float (&xc)[32], float (&xn)[32]) -> bool {
      const bool more = t + 1 < nT;
      uint32_t pk[16];
      exps(xc, pk, 0);  // special-function unit; overlaps the wait for S(t+1)
      if (more) {
        uint32_t sv[32], b0[32], b1[32];
        if (!fetch(t + 1, sv, b0, b1)) return false;
        skew_store(b0, b1);  // load/store unit
        exps(xc, pk, 1);     // independent of the stores
        if (!skew_sync(t + 1)) return false;
        skew_read(t + 1, sv, xn);
        mh_next = half_max(xn);
        pair_publish(t + 1, mh_next);
      } else {
        exps(xc, pk, 1);
      }
      // P(t) goes to buffer t&1, which held P(t-2). When there is a next tile
      // its S commit (waited in fetch) arrived after P(t-2) V(t-2) had
      // completed -- commits follow issue order and the MMA warp issues
      // P(t-2) V(t-2) before S(t+1) -- so only the last tile waits here.
      // Rescaling O needs P(t-1) V(t-1) complete: an explicit wait (rare).
      if (t >= 1 && __any_sync(0xffffffffu, resc)) {
        if (!wwait(B_PVDONE + ((t - 1) & 1), ((uint32_t)(t - 1) >> 1) & 1u)) return false;
        tc_fence_after();
#pragma unroll 1
        for (int c = hh * (DK / 64); c < (hh + 1) * (DK / 64); ++c) {
          uint32_t o[32];
          tmem_ld32(trow + TM_O + 32u * c, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(trow + TM_O + 32u * c, o);
        }
      } else if (!more && t >= 2) {
        if (!wwait(B_PVDONE + (t & 1), ((uint32_t)(t - 2) >> 1) & 1u)) return false;
        tc_fence_after();
      }
      tmem_st16(trow + TM_P + 32u * (uint32_t)(t & 1) + 16u * hh, pk);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_PFULL + (t & 1)));
      if (more) {
        float mo;
        if (!pair_fetch(t + 1, mo)) return false;
        update_max(fmaxf(mh_next, mo));
      }
      return true;
    };

    float xa[32], xb[32];
    if (ok) {
      uint32_t sv[32], b0[32], b1[32];
      ok = fetch(0, sv, b0, b1);
      if (ok) {
        skew_store(b0, b1);
        ok = skew_sync(0);
      }
      if (ok) {
        skew_read(0, sv, xa);
        const float mh = half_max(xa);
        pair_publish(0, mh);
        float mo;
        ok = pair_fetch(0, mo);
        if (ok) update_max(fmaxf(mh, mo));
        resc = false;  // nothing accumulated in O yet
      }
    }
    for (int t = 0; t < nT && ok; ++t) {
      ok = step(t, xa, xb);
#pragma unroll
      for (int j = 0; j < 32; ++j) xa[j] = xb[j];
    }
    // row sum over both halves
    if (ok) {
      pair_publish(nT, lsum);
      float lo;
      ok = pair_fetch(nT, lo);
      lsum += lo;
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_PVDONE + ((nT - 1) & 1)), ((uint32_t)(nT - 1) >> 1) & 1u,
                                                  p.err, DEV_ERR_TIMEOUT_ATTN)) != 0;
    // Epilogue: O / l rounded to the operand type, staged through the (now
    // idle) Q tile as [QM rows x DK] with 16-byte chunk c of row r at
    // c ^ (r & 7) (conflict-free both ways), then stored by all 8 softmax
    // warps with the lanes along the rows: each instruction writes whole
    // rows instead of one 16-byte piece of 32 rows.
    constexpr int CH = DK / 8;  // 16-byte chunks per row
    uint8_t* stile = sm + L::OFF_QU;
    if (ok) {
      tc_fence_after();
      const float inv = 1.0f / lsum;
#pragma unroll 1
      for (int c = hh * (DK / 64); c < (hh + 1) * (DK / 64); ++c) {
        uint32_t o[32];
        tmem_ld32(trow + TM_O + 32u * c, o);
        tmem_ld_wait();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int ch = 4 * c + k;  // chunk of this row
          *reinterpret_cast<uint4*>(stile + i * (DK * 2) + ((ch ^ (i & 7)) << 4)) =
              make_uint4(pack2<H>(__uint_as_float(o[8 * k]) * inv, __uint_as_float(o[8 * k + 1]) * inv),
                         pack2<H>(__uint_as_float(o[8 * k + 2]) * inv, __uint_as_float(o[8 * k + 3]) * inv),
                         pack2<H>(__uint_as_float(o[8 * k + 4]) * inv, __uint_as_float(o[8 * k + 5]) * inv),
                         pack2<H>(__uint_as_float(o[8 * k + 6]) * inv, __uint_as_float(o[8 * k + 7]) * inv));
        }
      }
    }
    // every softmax thread arrives here exactly once (no path leaves the
    // branch early); the tile is stored only if all of them had it ready
    uint32_t all_ok;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(all_ok)
        : "r"(ok ? 1u : 0u), "r"(32 * SM_WARPS)
        : "memory");
    if (all_ok) {
      const int t = threadIdx.x - 64;  // 0 .. 32 * SM_WARPS - 1
      H* base = reinterpret_cast<H*>(p.ctx) + (size_t)(off + q0) * p.d + head * DK;
#pragma unroll
      for (int k = 0; k < QM * CH / (32 * SM_WARPS); ++k) {
        const int idx = t + 32 * SM_WARPS * k;
        const int r = idx / CH, c = idx % CH;
        const uint4 v = *reinterpret_cast<const uint4*>(stile + r * (DK * 2) + ((c ^ (r & 7)) << 4));
        if (q0 + r < T) *reinterpret_cast<uint4*>(base + (size_t)r * p.d + 8 * c) = v;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

template <typename H, int DK>
cudaError_t launch_tc(const AttnArgs& a, cudaStream_t st) {
  auto kern = k_relpos_attn_tc<H, DK>;
  constexpr int smem = TcLayout<DK>::SMEM;
  static PerDevice once;
  int unused = 0;
  const cudaError_t ae = per_device(once, &unused, [&](int, int&) {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  });
  if (ae != cudaSuccess) return ae;
  const bool bf = is_bf16<H>::value;
  CUtensorMap tq, tp;
  if (!make_tmap_kmajor(&tq, a.qkv, a.rows, 3 * a.d, 3 * a.d, 64, bf)) return cudaErrorInvalidValue;
  if (!make_tmap_kmajor(&tp, a.ptab, a.ptab_rows, a.d, a.ptab_ld > 0 ? a.ptab_ld : a.d, 64, bf))
    return cudaErrorInvalidValue;
  TcParams p{a.tiles, a.item_off, a.item_len, a.bias_u, a.bias_v, a.ctx, a.d, a.centre,
             1.4426950408889634f / sqrtf((float)DK), a.err, a.qu_folded ? 1 : 0};
  return launch_pdl(kern, dim3(a.n_heads, a.n_tiles), dim3(THREADS), smem, st, tq, tp, p);
}

}  // namespace

int attn_tc_query_tile() { return QM; }

cudaError_t attention_tc_launch(const AttnArgs& a, bool bf16, cudaStream_t st) {
  if (a.n_tiles <= 0) return cudaSuccess;
  if (a.d % a.n_heads != 0 || a.rows <= 0 || (a.d % 8) != 0 ||
      (reinterpret_cast<uintptr_t>(a.qkv) & 15) || (reinterpret_cast<uintptr_t>(a.ptab) & 15) ||
      (reinterpret_cast<uintptr_t>(a.bias_u) & 15) || (reinterpret_cast<uintptr_t>(a.bias_v) & 15))
    return cudaErrorInvalidValue;
  if (a.n_tiles > 65535) return cudaErrorInvalidValue;  // grid y
  const int dk = a.d / a.n_heads;
  if (dk == 128) return bf16 ? launch_tc<__nv_bfloat16, 128>(a, st) : launch_tc<__half, 128>(a, st);
  if (dk == 64) return bf16 ? launch_tc<__nv_bfloat16, 64>(a, st) : launch_tc<__half, 64>(a, st);
  return cudaErrorInvalidValue;
}

}  // namespace pkc
