// Relative-position multi-head self-attention, flash style (no T x T buffer).
//
// Reference: RelPosAttention::build_graph_batched (src/relpos_attention.cpp:162-306):
//   ac = (q + pos_bias_u) k^T,  bd = (q + pos_bias_v) p^T,
//   bd <- rel_shift(bd)  (pad / reshape / view / cont sequence, :230-238),
//   attn = softmax((ac + bd) / sqrt(dk) + key_mask),  ctx = attn v,
//   padded query rows zeroed.
// Here the rel_shift is folded into the score indexing: bd[i][j] uses the
// positional row r = c - (i - j), where row r of the table holds relative
// position (c - r) (c = table centre). For a tile of 64 query rows and 32 keys
// only 95 consecutive rows of p are needed; each warp computes a 16 x 48 skewed
// block Qv * Pwin^T on the tensor cores and reads it back diagonally.
//
// Frames are packed per utterance (no padding): keys beyond an utterance's
// valid length do not exist and are masked by bounds, and query rows beyond
// it are never written, which is exactly the reference's masking.
//
// Layout: qkv [M, 3d] (q | k | v, head h at columns h*dk), ptab [NP, d] (the
// linear_pos output over relative positions centre-1 ... -(centre-1)),
// ctx [M, d]; all f16 or bf16. One CTA = (one 64-row query tile, one head).
#include "common.cuh"
#include "kernels.h"

namespace pkc {

namespace {

constexpr int QT = 64;   // query rows per CTA
constexpr int KT = 32;   // keys per iteration
constexpr int PW = QT + KT - 1;  // positional rows needed per CTA iteration (95)
constexpr int PWR = 96;          // rounded
constexpr int WPWR = 48;         // positional rows per warp: 16 + KT - 1 = 47, rounded to n8
constexpr int NTHREADS = 128;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename H>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4],
                                                 uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4],
                                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename H, int DK>
struct AttnSmem {
  static constexpr int LD = DK + 8;  // padded row (halves): conflict-free ldmatrix
  H qu[QT * LD];
  H qv[QT * LD];
  H k[KT * LD];
  H v[KT * LD];
  H p[PWR * LD];
  float bd[4][16][WPWR + 4];
};

template <typename H, int DK>
__global__ void __launch_bounds__(NTHREADS)
    k_relpos_attn(const H* __restrict__ qkv, const H* __restrict__ ptab, int ptab_rows, int centre,
                  const float* __restrict__ bias_u, const float* __restrict__ bias_v,
                  const int* __restrict__ tiles,     // [n_tiles][2]: item, q0
                  const int* __restrict__ item_off,  // [B] first packed row of each item
                  const int* __restrict__ item_len,  // [B] valid frames
                  H* __restrict__ ctx, int d, float scale_log2) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  using S = AttnSmem<H, DK>;
  constexpr int LD = S::LD;
  S& sm = *reinterpret_cast<S*>(smem_raw);

  const int tile = blockIdx.x;
  const int head = blockIdx.y;
  const int item = tiles[2 * tile];
  const int q0 = tiles[2 * tile + 1];
  const int off = item_off[item];
  const int T = item_len[item];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int ld3 = 3 * d;

  // ---- Q tile -> (q + u), (q + v), rounded to H
  {
    constexpr int CH = DK / 8;
    for (int i = threadIdx.x; i < QT * CH; i += NTHREADS) {
      const int r = i / CH, c = i % CH;
      const int qi = q0 + r;
      float qf[8];
      if (qi < T) {
        uint4 raw = *reinterpret_cast<const uint4*>(qkv + (size_t)(off + qi) * ld3 + head * DK + c * 8);
        const H* hv = reinterpret_cast<const H*>(&raw);
#pragma unroll
        for (int e = 0; e < 8; ++e) qf[e] = from_h(hv[e]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) qf[e] = 0.f;
      }
      H ou[8], ov[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        ou[e] = to_h<H>(qf[e] + bias_u[head * DK + c * 8 + e]);
        ov[e] = to_h<H>(qf[e] + bias_v[head * DK + c * 8 + e]);
      }
      *reinterpret_cast<uint4*>(&sm.qu[r * LD + c * 8]) = *reinterpret_cast<uint4*>(ou);
      *reinterpret_cast<uint4*>(&sm.qv[r * LD + c * 8]) = *reinterpret_cast<uint4*>(ov);
    }
  }

  float o[DK / 8][4];
#pragma unroll
  for (int i = 0; i < DK / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY};
  float lrow[2] = {0.f, 0.f};

  const int iw = q0 + warp * 16;  // first query row of this warp
  const uint32_t qu_base = smem_u32(sm.qu), qv_base = smem_u32(sm.qv);
  const uint32_t k_base = smem_u32(sm.k), v_base = smem_u32(sm.v), p_base = smem_u32(sm.p);

  for (int j0 = 0; j0 < T; j0 += KT) {
    __syncthreads();  // previous iteration's readers are done with k/v/p/bd
    {
      constexpr int CH = DK / 8;
      for (int i = threadIdx.x; i < KT * CH; i += NTHREADS) {
        const int r = i / CH, c = i % CH;
        const int kj = j0 + r;
        uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
        if (kj < T) {
          const H* base = qkv + (size_t)(off + kj) * ld3 + head * DK + c * 8;
          kv = *reinterpret_cast<const uint4*>(base + d);
          vv = *reinterpret_cast<const uint4*>(base + 2 * d);
        }
        *reinterpret_cast<uint4*>(&sm.k[r * LD + c * 8]) = kv;
        *reinterpret_cast<uint4*>(&sm.v[r * LD + c * 8]) = vv;
      }
      // positional window: block rows rb .. rb+PWR-1 with rb = centre-1-(q0+QT-1)+j0
      const int rb = centre - 1 - (q0 + QT - 1) + j0;
      for (int i = threadIdx.x; i < PWR * CH; i += NTHREADS) {
        const int r = i / CH, c = i % CH;
        const int pr = rb + r;
        uint4 pv = make_uint4(0, 0, 0, 0);
        if (r < PW && pr >= 0 && pr < ptab_rows)
          pv = *reinterpret_cast<const uint4*>(ptab + (size_t)pr * d + head * DK + c * 8);
        *reinterpret_cast<uint4*>(&sm.p[r * LD + c * 8]) = pv;
      }
    }
    __syncthreads();

    // ---- skewed positional scores: BD[16][48] = Qv(16 x DK) * Pwin(48 x DK)^T
    // warp window rows start at cw = (QT-16) - 16*warp (see header comment)
    const int cw = (QT - 16) - 16 * warp;
    {
      float bdacc[WPWR / 8][4];
#pragma unroll
      for (int n = 0; n < WPWR / 8; ++n) bdacc[n][0] = bdacc[n][1] = bdacc[n][2] = bdacc[n][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < DK / 16; ++kk) {
        uint32_t a[4];
        {
          const int row = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int col = kk * 16 + (lane >> 4) * 8;
          ldsm_x4(qv_base + (uint32_t)((row * LD + col) * 2), a[0], a[1], a[2], a[3]);
        }
#pragma unroll
        for (int n = 0; n < WPWR / 16; ++n) {
          uint32_t b0, b1, b2, b3;
          const int prow = cw + n * 16 + (lane & 7) + (lane >> 4) * 8;
          const int col = kk * 16 + ((lane >> 3) & 1) * 8;
          ldsm_x4(p_base + (uint32_t)((prow * LD + col) * 2), b0, b1, b2, b3);
          mma16816<H>(bdacc[2 * n], a, b0, b1);
          mma16816<H>(bdacc[2 * n + 1], a, b2, b3);
        }
      }
#pragma unroll
      for (int n = 0; n < WPWR / 8; ++n) {
        sm.bd[warp][g][n * 8 + 2 * t4] = bdacc[n][0];
        sm.bd[warp][g][n * 8 + 2 * t4 + 1] = bdacc[n][1];
        sm.bd[warp][g + 8][n * 8 + 2 * t4] = bdacc[n][2];
        sm.bd[warp][g + 8][n * 8 + 2 * t4 + 1] = bdacc[n][3];
      }
    }
    __syncwarp();

    // ---- content scores: S[16][32] = Qu * K^T, plus the shifted positional term
    float s[KT / 8][4];
#pragma unroll
    for (int n = 0; n < KT / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < DK / 16; ++kk) {
      uint32_t a[4];
      {
        const int row = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = kk * 16 + (lane >> 4) * 8;
        ldsm_x4(qu_base + (uint32_t)((row * LD + col) * 2), a[0], a[1], a[2], a[3]);
      }
#pragma unroll
      for (int n = 0; n < KT / 16; ++n) {
        uint32_t b0, b1, b2, b3;
        const int krow = n * 16 + (lane & 7) + (lane >> 4) * 8;
        const int col = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(k_base + (uint32_t)((krow * LD + col) * 2), b0, b1, b2, b3);
        mma16816<H>(s[2 * n], a, b0, b1);
        mma16816<H>(s[2 * n + 1], a, b2, b3);
      }
    }
    // positional term: local row ri (0..15), local key cj (0..31):
    // P row r = centre-1-(iw+ri)+(j0+cj); warp window starts at
    // r_w = centre-1-(iw+15)+j0, so column = r - r_w = 15 - ri + cj.
    float mnew[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int ri = g + 8 * hr;
      float mx = mrow[hr];
#pragma unroll
      for (int n = 0; n < KT / 8; ++n) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int cj = n * 8 + 2 * t4 + e;
          float val = s[n][2 * hr + e] + sm.bd[warp][ri][15 - ri + cj];
          val = (j0 + cj < T) ? val * scale_log2 : -INFINITY;
          s[n][2 * hr + e] = val;
          mx = fmaxf(mx, val);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      mnew[hr] = mx;
    }
    // online softmax (base-2 exponent; scale_log2 = log2(e)/sqrt(dk))
    float alpha[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      alpha[hr] = exp2f(mrow[hr] - mnew[hr]);
      mrow[hr] = mnew[hr];
      float sum = 0.f;
#pragma unroll
      for (int n = 0; n < KT / 8; ++n) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float pe = exp2f(s[n][2 * hr + e] - mnew[hr]);
          s[n][2 * hr + e] = pe;
          sum += pe;
        }
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      lrow[hr] = lrow[hr] * alpha[hr] + sum;
    }
#pragma unroll
    for (int i = 0; i < DK / 8; ++i) {
      o[i][0] *= alpha[0]; o[i][1] *= alpha[0];
      o[i][2] *= alpha[1]; o[i][3] *= alpha[1];
    }
    // ---- O += P * V
#pragma unroll
    for (int kk = 0; kk < KT / 16; ++kk) {
      uint32_t a[4];
      a[0] = pack2<H>(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack2<H>(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack2<H>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack2<H>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int n = 0; n < DK / 16; ++n) {
        uint32_t b0, b1, b2, b3;
        const int krow = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = n * 16 + (lane >> 4) * 8;
        ldsm_x4_t(v_base + (uint32_t)((krow * LD + col) * 2), b0, b1, b2, b3);
        mma16816<H>(o[2 * n], a, b0, b1);
        mma16816<H>(o[2 * n + 1], a, b2, b3);
      }
    }
  }

  // ---- normalise and store this warp's 16 rows
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int qi = iw + g + 8 * hr;
    if (qi >= T) continue;
    const float inv = 1.0f / lrow[hr];
    H* dst = ctx + (size_t)(off + qi) * d + head * DK;
#pragma unroll
    for (int n = 0; n < DK / 8; ++n) {
      const int c = n * 8 + 2 * t4;
      *reinterpret_cast<uint32_t*>(dst + c) = pack2<H>(o[n][2 * hr] * inv, o[n][2 * hr + 1] * inv);
    }
  }
}

template <typename H, int DK>
cudaError_t launch_attn(const AttnArgs& a, cudaStream_t st) {
  auto kern = k_relpos_attn<H, DK>;
  const int smem = (int)sizeof(AttnSmem<H, DK>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(a.n_tiles, a.n_heads);
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)DK);
  kern<<<grid, NTHREADS, smem, st>>>(reinterpret_cast<const H*>(a.qkv), reinterpret_cast<const H*>(a.ptab),
                                     a.ptab_rows, a.centre, a.bias_u, a.bias_v, a.tiles, a.item_off,
                                     a.item_len, reinterpret_cast<H*>(a.ctx), a.d, scale_log2);
  return cudaGetLastError();
}

}  // namespace

int attn_query_tile() { return QT; }

cudaError_t attention_launch(const AttnArgs& a, bool bf16, cudaStream_t st) {
  if (a.n_tiles <= 0) return cudaSuccess;
  const int dk = a.d / a.n_heads;
  if (a.d % a.n_heads != 0) return cudaErrorInvalidValue;
  if (dk == 128) return bf16 ? launch_attn<__nv_bfloat16, 128>(a, st) : launch_attn<__half, 128>(a, st);
  if (dk == 64) return bf16 ? launch_attn<__nv_bfloat16, 64>(a, st) : launch_attn<__half, 64>(a, st);
  return cudaErrorInvalidValue;
}

}  // namespace pkc
