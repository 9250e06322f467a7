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
// tile t reads chunks t, t+1, t+2 and computes exactly one new chunk (t+2).
// The positional term therefore costs the same tensor work as Q K^T.
//
// Tensor memory (512 columns x 128 lanes, lane = query row):
//   [0, DK)      O accumulator
//   [128, 256)   S = Qu K^T, two 64-column buffers (tile parity)
//   [256, 512)   ring of four positional chunks (chunk k in slot k % 4)
// Shared memory: Qu, Qv (built from the TMA-loaded Q tile plus the biases),
// K / V / positional-chunk rings of 2, the P tile (f16/bf16, the A operand of
// P V), and one private 68-word row per softmax thread used to apply the
// diagonal shift (tensor-memory loads read the same columns in every lane).
//
// Warps: 0 = TMA producer, 1 = MMA issuer (one thread), 2..5 = softmax
// (warp w owns TMEM lanes 32(w%4)..+31, one query row per thread).
// Order of tensor work: S(t) and C(t+2), then P(t-1) V(t-1), so the softmax
// of tile t overlaps P V of tile t-1 and S / C of tile t+1.
// Online softmax with a lazy rescale: the running maximum used for the
// exponentials only moves when the tile maximum exceeds it by more than 8
// (log2 units), so P stays <= 256 and O is rescaled (tcgen05.ld / st by the
// row's own thread) only on those rare moves. The final O / l is exact.
//
// Frames are packed per utterance (no padding); keys >= T are masked, query
// rows >= T are computed but not stored -- the reference's masking.
#include "common.cuh"
#include "gemm.h"
#include "kernels.h"

namespace pkc {

namespace {

constexpr int QM = 128;     // query rows per CTA (MMA M, TMEM lanes)
constexpr int KN = 64;      // keys per tile (MMA N of S and of a chunk)
constexpr int THREADS = 192;
constexpr int SKEW_LD = 68; // words per thread row: 64 + 4 (conflict-free v4 stores / skewed loads)
constexpr float kRescaleLog2 = 8.0f;

enum : int {
  B_QFULL = 0, B_QREADY = 1,
  B_KFULL = 2, B_KEMPTY = 4, B_VFULL = 6, B_VEMPTY = 8, B_PWFULL = 10, B_PWEMPTY = 12,
  B_SFULL = 14, B_STFREE = 16, B_PFULL = 18, B_PVDONE = 19, B_FINAL = 20, N_BARS = 21
};

template <int DK>
struct TcLayout {
  static constexpr int KB = DK / 64;           // 64-column (128-byte) k-blocks
  static constexpr int Q_BYTES = QM * DK * 2;
  static constexpr int T_BYTES = KN * DK * 2;  // one K, V or positional-chunk tile
  static constexpr int P_BYTES = QM * KN * 2;
  static constexpr int OFF_QU = 0;
  static constexpr int OFF_QV = OFF_QU + Q_BYTES;
  static constexpr int OFF_K = OFF_QV + Q_BYTES;
  static constexpr int OFF_V = OFF_K + 2 * T_BYTES;
  static constexpr int OFF_PW = OFF_V + 2 * T_BYTES;
  static constexpr int OFF_P = OFF_PW + 2 * T_BYTES;
  static constexpr int OFF_SKEW = OFF_P + P_BYTES;
  static constexpr int OFF_BAR = OFF_SKEW + QM * SKEW_LD * 4;
  static constexpr int OFF_SLOT = OFF_BAR + N_BARS * 8;
  static constexpr int SMEM = OFF_SLOT + 16 + 1024;  // + alignment slack
};

constexpr uint32_t TM_O = 0, TM_S = 128, TM_BD = 256;

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
};

// window column wc (0..191) of key tile t -> TMEM column of its chunk slot
__device__ __forceinline__ uint32_t bd_col(int t, int wc) {
  return TM_BD + 64u * (uint32_t)((t + (wc >> 6)) & 3) + (uint32_t)(wc & 63);
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
      const bool four = i == B_QREADY || i == B_STFREE || i == B_STFREE + 1 || i == B_PFULL;
      mbar_init(bar(i), four ? 4u : 1u);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  pdl_trigger();

  const int tile = blockIdx.x, head = blockIdx.y;
  const int item = p.tiles[2 * tile], q0 = p.tiles[2 * tile + 1];
  const int off = p.item_off[item], T = p.item_len[item];
  const int nT = (T + KN - 1) / KN;
  const int rb = p.centre - 1 - (q0 + QM - 1);  // first positional row of chunk 0

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- TMA producer
      const int colq = head * DK, colk = p.d + head * DK, colv = 2 * p.d + head * DK;
      mbar_arrive_expect_tx(bar(B_QFULL), L::Q_BYTES);
#pragma unroll
      for (int kb = 0; kb < L::KB; ++kb)
#pragma unroll
        for (int h = 0; h < 2; ++h)
          tma_load_2d(sbase + L::OFF_QU + kb * QM * 128 + h * 64 * 128, &tm_qkv, bar(B_QFULL), colq + kb * 64,
                      off + q0 + 64 * h);
      int issued[3] = {0, 0, 0};  // loads issued per ring: positional chunks, K, V
      auto load_tile = [&](int ring, int fam_full, int fam_empty, int region, const CUtensorMap* map, int col,
                           int row) -> bool {
        const int n = issued[ring], s = n & 1;
        if (!mbar_wait(bar(fam_empty + s), (((uint32_t)n >> 1) & 1u) ^ 1u, p.err, DEV_ERR_TIMEOUT_ATTN)) return false;
        mbar_arrive_expect_tx(bar(fam_full + s), L::T_BYTES);
#pragma unroll
        for (int kb = 0; kb < L::KB; ++kb)
          tma_load_2d(sbase + region + s * L::T_BYTES + kb * KN * 128, map, bar(fam_full + s), col + kb * 64, row);
        ++issued[ring];
        return true;
      };
      bool ok = load_tile(0, B_PWFULL, B_PWEMPTY, L::OFF_PW, &tm_pos, head * DK, rb) &&
                load_tile(0, B_PWFULL, B_PWEMPTY, L::OFF_PW, &tm_pos, head * DK, rb + KN);
      for (int t = 0; t < nT && ok; ++t) {
        ok = load_tile(1, B_KFULL, B_KEMPTY, L::OFF_K, &tm_qkv, colk, off + KN * t) &&
             load_tile(0, B_PWFULL, B_PWEMPTY, L::OFF_PW, &tm_pos, head * DK, rb + KN * (t + 2)) &&
             load_tile(2, B_VFULL, B_VEMPTY, L::OFF_V, &tm_qkv, colv, off + KN * t);
      }
      if (!ok) {
        // a consumer gave up: let every copy already issued land before the
        // CTA may exit (the last load of each stage; earlier ones on the same
        // stage were consumed, or this one could not have been issued)
        mbar_wait(bar(B_QFULL), 0, nullptr, 0);
        const int fam[3] = {B_PWFULL, B_KFULL, B_VFULL};
        for (int r = 0; r < 3; ++r)
          for (int n = issued[r] - 2; n < issued[r]; ++n)
            if (n >= 0) mbar_wait(bar(fam[r] + (n & 1)), ((uint32_t)n >> 1) & 1u, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      constexpr int fmt = is_bf16<H>::value ? 1 : 0;
      constexpr uint32_t id_s = idesc_f16(QM, KN, fmt);
      constexpr uint32_t id_pv = idesc_f16(QM, DK, fmt) | (1u << 16);  // B (V) MN-major
      bool ok = mbar_wait(bar(B_QREADY), 0, p.err, DEV_ERR_TIMEOUT_ATTN);
      tc_fence_after();
      const uint64_t dqu = smem_desc_sw128(sbase + L::OFF_QU);
      const uint64_t dqv = smem_desc_sw128(sbase + L::OFF_QV);
      // K-step kk (16 elements of dk): k-block kk/4, 32 bytes per step inside it
      auto a_off = [](int kk) { return (uint64_t)(((kk >> 2) * QM * 128 + (kk & 3) * 32) >> 4); };
      auto b_off = [](int kk) { return (uint64_t)(((kk >> 2) * KN * 128 + (kk & 3) * 32) >> 4); };
      auto chunk = [&](int c) -> bool {
        const int s = c & 1;
        if (!mbar_wait(bar(B_PWFULL + s), ((uint32_t)c >> 1) & 1u, p.err, DEV_ERR_TIMEOUT_ATTN)) return false;
        tc_fence_after();
        const uint64_t db = smem_desc_sw128(sbase + L::OFF_PW + s * L::T_BYTES);
#pragma unroll
        for (int kk = 0; kk < DK / 16; ++kk)
          umma_f16(tmem + TM_BD + 64u * (uint32_t)(c & 3), dqv + a_off(kk), db + b_off(kk), id_s, kk > 0 ? 1u : 0u);
        umma_commit(bar(B_PWEMPTY + s));
        return true;
      };
      auto pv = [&](int u) -> bool {
        const int s = u & 1;
        if (!mbar_wait(bar(B_PFULL), (uint32_t)u & 1u, p.err, DEV_ERR_TIMEOUT_ATTN)) return false;
        if (!mbar_wait(bar(B_VFULL + s), ((uint32_t)u >> 1) & 1u, p.err, DEV_ERR_TIMEOUT_ATTN)) return false;
        tc_fence_after();
        const uint64_t da = smem_desc_sw128(sbase + L::OFF_P);
        const uint64_t dv = smem_desc_sw128_mn(sbase + L::OFF_V + s * L::T_BYTES, KN * 128, 1024);
#pragma unroll
        for (int kk = 0; kk < KN / 16; ++kk)
          umma_f16(tmem + TM_O, da + (uint64_t)((kk * 32) >> 4), dv + (uint64_t)((kk * 16 * 128) >> 4), id_pv,
                   (u > 0 || kk > 0) ? 1u : 0u);
        umma_commit(bar(B_VEMPTY + s));
        umma_commit(bar(B_PVDONE));
        return true;
      };
      ok = ok && chunk(0) && chunk(1);
      for (int t = 0; t < nT && ok; ++t) {
        if (t >= 2) {
          ok = mbar_wait(bar(B_STFREE + (t & 1)), ((uint32_t)(t - 2) >> 1) & 1u, p.err, DEV_ERR_TIMEOUT_ATTN);
          if (!ok) break;
          tc_fence_after();
        }
        const int s = t & 1;
        ok = mbar_wait(bar(B_KFULL + s), ((uint32_t)t >> 1) & 1u, p.err, DEV_ERR_TIMEOUT_ATTN);
        if (!ok) break;
        tc_fence_after();
        const uint64_t dk = smem_desc_sw128(sbase + L::OFF_K + s * L::T_BYTES);
#pragma unroll
        for (int kk = 0; kk < DK / 16; ++kk)
          umma_f16(tmem + TM_S + 64u * (uint32_t)s, dqu + a_off(kk), dk + b_off(kk), id_s, kk > 0 ? 1u : 0u);
        umma_commit(bar(B_KEMPTY + s));
        ok = chunk(t + 2);
        if (!ok) break;
        umma_commit(bar(B_SFULL + s));
        if (t >= 1) ok = pv(t - 1);
      }
      if (ok) pv(nT - 1);
      // every issued MMA has completed before TMEM can be released
      umma_commit(bar(B_FINAL));
      mbar_wait(bar(B_FINAL), 0, p.err, DEV_ERR_TIMEOUT_ATTN);
    }
  } else {
    // ---------------------------------------------------------------- softmax warps
    const int q = warp & 3;
    const int i = 32 * q + lane;  // query row within the tile = TMEM lane
    const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16);
    const int ts = threadIdx.x - 64;  // 0..127
    bool ok = __all_sync(0xffffffffu, mbar_wait(bar(B_QFULL), 0, p.err, DEV_ERR_TIMEOUT_ATTN)) != 0;
    if (ok) {
      // Qu = Q + u, Qv = Q + v in the swizzled layout TMA wrote: 16-byte chunk
      // pc of row r holds logical columns 8 * (pc ^ (r & 7)) of its k-block
      for (int idx = ts; idx < QM * DK / 8; idx += 128) {
        const int kb = idx / (QM * 8), rem = idx % (QM * 8);
        const int r = rem >> 3, pc = rem & 7;
        const int col = kb * 64 + ((pc ^ (r & 7)) << 3);
        const int ob = kb * QM * 128 + r * 128 + pc * 16;
        const uint4 raw = *reinterpret_cast<const uint4*>(sm + L::OFF_QU + ob);
        const H* hv = reinterpret_cast<const H*>(&raw);
        const float* bu = p.bias_u + head * DK + col;
        const float* bv = p.bias_v + head * DK + col;
        uint32_t wu[4], wv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x0 = from_h(hv[2 * e]), x1 = from_h(hv[2 * e + 1]);
          wu[e] = pack2<H>(x0 + bu[2 * e], x1 + bu[2 * e + 1]);
          wv[e] = pack2<H>(x0 + bv[2 * e], x1 + bv[2 * e + 1]);
        }
        *reinterpret_cast<uint4*>(sm + L::OFF_QU + ob) = make_uint4(wu[0], wu[1], wu[2], wu[3]);
        *reinterpret_cast<uint4*>(sm + L::OFF_QV + ob) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
      }
      fence_proxy_async_smem();
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bar(B_QREADY));

    float* skew = reinterpret_cast<float*>(sm + L::OFF_SKEW) + i * SKEW_LD;
    uint8_t* prow = sm + L::OFF_P + i * 128;
    float m_used = -INFINITY, lsum = 0.f;
    const float sl2 = p.scale_log2;
    for (int t = 0; t < nT && ok; ++t) {
      ok = __all_sync(0xffffffffu, mbar_wait(bar(B_SFULL + (t & 1)), ((uint32_t)t >> 1) & 1u, p.err,
                                             DEV_ERR_TIMEOUT_ATTN)) != 0;
      if (!ok) break;
      tc_fence_after();
      float x[KN];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t sv[32], b0[32], b1[32];
        const int wc = 96 - 32 * q + 32 * h;  // first window column this warp needs for keys 32h..
        tmem_ld32(trow + TM_S + 64u * (uint32_t)(t & 1) + 32u * h, sv);
        tmem_ld32(trow + bd_col(t, wc), b0);
        tmem_ld32(trow + bd_col(t, wc + 32), b1);
        tmem_ld_wait();
        float4* s4 = reinterpret_cast<float4*>(skew);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          s4[k] = make_float4(__uint_as_float(b0[4 * k]), __uint_as_float(b0[4 * k + 1]),
                              __uint_as_float(b0[4 * k + 2]), __uint_as_float(b0[4 * k + 3]));
#pragma unroll
        for (int k = 0; k < 8; ++k)
          s4[8 + k] = make_float4(__uint_as_float(b1[4 * k]), __uint_as_float(b1[4 * k + 1]),
                                  __uint_as_float(b1[4 * k + 2]), __uint_as_float(b1[4 * k + 3]));
        // key 32h + j of row i sits at window column 127 - i + 32h + j = wc + (31 - lane) + j
        const float* src = skew + (31 - lane);
#pragma unroll
        for (int j = 0; j < 32; ++j) x[32 * h + j] = (__uint_as_float(sv[j]) + src[j]) * sl2;
      }
      // S(t) and chunk t are consumed
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_STFREE + (t & 1)));

      if (t == nT - 1) {
        const int kv = T - KN * t;  // valid keys in the last tile (1..64)
#pragma unroll
        for (int j = 0; j < KN; ++j)
          if (j >= kv) x[j] = -INFINITY;
      }
      float mt = x[0];
#pragma unroll
      for (int j = 1; j < KN; ++j) mt = fmaxf(mt, x[j]);
      const bool resc = mt > m_used + kRescaleLog2;
      float alpha = 1.f;
      if (resc) {
        alpha = ex2_approx(m_used - mt);  // 0 on the first tile
        m_used = mt;
        lsum *= alpha;
      }
      uint32_t pk[KN / 2];
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < KN / 2; ++j) {
        const float p0 = ex2_approx(x[2 * j] - m_used), p1 = ex2_approx(x[2 * j + 1] - m_used);
        rs += p0 + p1;
        pk[j] = pack2<H>(p0, p1);
      }
      lsum += rs;
      // the P tile and O are free once P(t-1) V(t-1) has completed
      if (t >= 1) {
        ok = __all_sync(0xffffffffu, mbar_wait(bar(B_PVDONE), (uint32_t)(t - 1) & 1u, p.err,
                                               DEV_ERR_TIMEOUT_ATTN)) != 0;
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, resc)) {
#pragma unroll 1
          for (int c = 0; c < DK / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(trow + TM_O + 32u * c, o);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st32(trow + TM_O + 32u * c, o);
          }
          tmem_st_wait();
        }
      }
      // P row i: 8 chunks of 16 bytes, chunk c at (c ^ (i & 7)) (128-byte swizzle)
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(prow + ((c ^ (i & 7)) << 4)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_PFULL));
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_PVDONE), (uint32_t)(nT - 1) & 1u, p.err,
                                                  DEV_ERR_TIMEOUT_ATTN)) != 0;
    if (ok) {
      tc_fence_after();
      const float inv = 1.0f / lsum;
      const bool store = q0 + i < T;
      H* dst = reinterpret_cast<H*>(p.ctx) + (size_t)(off + q0 + i) * p.d + head * DK;
#pragma unroll 1
      for (int c = 0; c < DK / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(trow + TM_O + 32u * c, o);
        tmem_ld_wait();
        if (store) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + 32 * c);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            d4[k] = make_uint4(pack2<H>(__uint_as_float(o[8 * k]) * inv, __uint_as_float(o[8 * k + 1]) * inv),
                               pack2<H>(__uint_as_float(o[8 * k + 2]) * inv, __uint_as_float(o[8 * k + 3]) * inv),
                               pack2<H>(__uint_as_float(o[8 * k + 4]) * inv, __uint_as_float(o[8 * k + 5]) * inv),
                               pack2<H>(__uint_as_float(o[8 * k + 6]) * inv, __uint_as_float(o[8 * k + 7]) * inv));
        }
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
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set[dev & 63] = true;
  }
  const bool bf = is_bf16<H>::value;
  CUtensorMap tq, tp;
  if (!make_tmap_kmajor(&tq, a.qkv, a.rows, 3 * a.d, 3 * a.d, 64, bf)) return cudaErrorInvalidValue;
  if (!make_tmap_kmajor(&tp, a.ptab, a.ptab_rows, a.d, a.ptab_ld > 0 ? a.ptab_ld : a.d, 64, bf))
    return cudaErrorInvalidValue;
  TcParams p{a.tiles, a.item_off, a.item_len, a.bias_u, a.bias_v, a.ctx, a.d, a.centre,
             1.4426950408889634f / sqrtf((float)DK), a.err};
  return launch_pdl(kern, dim3(a.n_tiles, a.n_heads), dim3(THREADS), smem, st, tq, tp, p);
}

}  // namespace

int attn_tc_query_tile() { return QM; }

cudaError_t attention_tc_launch(const AttnArgs& a, bool bf16, cudaStream_t st) {
  if (a.n_tiles <= 0) return cudaSuccess;
  if (a.d % a.n_heads != 0 || a.rows <= 0 || (a.d % 8) != 0 ||
      (reinterpret_cast<uintptr_t>(a.qkv) & 15) || (reinterpret_cast<uintptr_t>(a.ptab) & 15))
    return cudaErrorInvalidValue;
  const int dk = a.d / a.n_heads;
  if (dk == 128) return bf16 ? launch_tc<__nv_bfloat16, 128>(a, st) : launch_tc<__half, 128>(a, st);
  if (dk == 64) return bf16 ? launch_tc<__nv_bfloat16, 64>(a, st) : launch_tc<__half, 64>(a, st);
  return cudaErrorInvalidValue;
}

}  // namespace pkc
