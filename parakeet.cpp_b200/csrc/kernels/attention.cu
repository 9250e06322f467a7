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
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"

namespace pkc {

namespace {

constexpr int QT = 64;   // query rows per CTA
constexpr int KT = 32;   // keys per iteration
constexpr int PW = QT + KT - 1;  // positional rows needed per CTA iteration (95)
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

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  // zero-fills the 16 bytes when !valid (src-size 0)
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

constexpr int PRING = 128;  // positional rows resident: window (QT+KT-1) + next KT

template <typename H, int DK>
struct AttnSmem {
  static constexpr int LD = DK + 8;  // padded row (halves): conflict-free ldmatrix
  H k[2][KT * LD];
  H v[2][KT * LD];
  H p[PRING * LD];                  // ring over absolute positional rows (row mod PRING)
  float bd[4][16][WPWR + 4];
};

template <typename H, int DK>
__global__ void __launch_bounds__(NTHREADS, 2)
    k_relpos_attn(const H* __restrict__ qkv, const H* __restrict__ ptab, int ptab_rows, int ptab_ld, int centre,
                  const float* __restrict__ bias_u, const float* __restrict__ bias_v,
                  const int* __restrict__ tiles,     // [n_tiles][2]: item, q0
                  const int* __restrict__ item_off,  // [B] first packed row of each item
                  const int* __restrict__ item_len,  // [B] valid frames
                  H* __restrict__ ctx, int d, float scale_log2) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  using S = AttnSmem<H, DK>;
  constexpr int LD = S::LD;
  constexpr int CH = DK / 8;  // 16-byte chunks per row
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
  const int iw = q0 + warp * 16;             // first query row of this warp
  const int rb0 = centre - 1 - (q0 + QT - 1);  // first positional row of key tile 0's window

  auto load_kv = [&](int stage, int j0) {
    for (int i = threadIdx.x; i < KT * CH; i += NTHREADS) {
      const int r = i / CH, c = i % CH;
      const int kj = j0 + r;
      const bool ok = kj < T;
      const H* base = qkv + (size_t)(off + (ok ? kj : 0)) * ld3 + head * DK + c * 8;
      cp_async16(smem_u32(&sm.k[stage][r * LD + c * 8]), base + d, ok);
      cp_async16(smem_u32(&sm.v[stage][r * LD + c * 8]), base + 2 * d, ok);
    }
  };
  auto load_p = [&](int pr0, int nrows) {  // absolute positional rows [pr0, pr0 + nrows)
    for (int i = threadIdx.x; i < nrows * CH; i += NTHREADS) {
      const int r = i / CH, c = i % CH;
      const int pr = pr0 + r;
      const bool ok = pr >= 0 && pr < ptab_rows;
      const int slot = ((pr % PRING) + PRING) % PRING;
      cp_async16(smem_u32(&sm.p[slot * LD + c * 8]), ptab + (size_t)(ok ? pr : 0) * ptab_ld + head * DK + c * 8, ok);
    }
  };

  // ---- prologue: first positional window + first K/V tile in flight
  load_p(rb0, PW);
  load_kv(0, 0);
  cp_async_commit();

  // ---- Q fragments (q + u, q + v) straight from global into registers
  uint32_t qu[DK / 16][4], qv[DK / 16][4];
  {
    const int r0 = iw + g, r1 = iw + g + 8;
    const H* src0 = qkv + (size_t)(off + (r0 < T ? r0 : 0)) * ld3 + head * DK;
    const H* src1 = qkv + (size_t)(off + (r1 < T ? r1 : 0)) * ld3 + head * DK;
#pragma unroll
    for (int kk = 0; kk < DK / 16; ++kk) {
#pragma unroll
      for (int hh = 0; hh < 4; ++hh) {
        // a0: (g, 2t), a1: (g+8, 2t), a2: (g, 2t+8), a3: (g+8, 2t+8)
        const int col = kk * 16 + 2 * t4 + ((hh >> 1) ? 8 : 0);
        const bool hi_row = hh & 1;
        const H* src = hi_row ? src1 : src0;
        const bool ok = (hi_row ? r1 : r0) < T;
        float x0 = 0.f, x1 = 0.f;
        if (ok) {
          x0 = from_h(src[col]);
          x1 = from_h(src[col + 1]);
        }
        const float* bu = bias_u + head * DK + col;
        const float* bv = bias_v + head * DK + col;
        qu[kk][hh] = pack2<H>(x0 + bu[0], x1 + bu[1]);
        qv[kk][hh] = pack2<H>(x0 + bv[0], x1 + bv[1]);
      }
    }
  }

  float o[DK / 8][4];
#pragma unroll
  for (int i = 0; i < DK / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY};
  float lrow[2] = {0.f, 0.f};
  const uint32_t p_base = smem_u32(sm.p);

  int stage = 0;
  for (int j0 = 0; j0 < T; j0 += KT, stage ^= 1) {
    // prefetch the next key tile and the positional rows it adds to the window
    if (j0 + KT < T) {
      load_kv(stage ^ 1, j0 + KT);
      load_p(rb0 + j0 + PW, KT);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    const uint32_t k_base = smem_u32(sm.k[stage]), v_base = smem_u32(sm.v[stage]);
    // ---- skewed positional scores: BD[16][48] = Qv * Pwin^T. The warp's window
    // starts at absolute row rw = rb0 + j0 + (QT-16) - 16*warp.
    const int rw = rb0 + j0 + (QT - 16) - 16 * warp;
    {
      float bdacc[WPWR / 8][4];
#pragma unroll
      for (int n = 0; n < WPWR / 8; ++n) bdacc[n][0] = bdacc[n][1] = bdacc[n][2] = bdacc[n][3] = 0.f;
#pragma unroll
      for (int n = 0; n < WPWR / 16; ++n) {
        const int prow = rw + n * 16 + (lane & 7) + (lane >> 4) * 8;
        const int slot = ((prow % PRING) + PRING) % PRING;
#pragma unroll
        for (int kk = 0; kk < DK / 16; ++kk) {
          uint32_t b0, b1, b2, b3;
          const int col = kk * 16 + ((lane >> 3) & 1) * 8;
          ldsm_x4(p_base + (uint32_t)((slot * LD + col) * 2), b0, b1, b2, b3);
          mma16816<H>(bdacc[2 * n], qv[kk], b0, b1);
          mma16816<H>(bdacc[2 * n + 1], qv[kk], b2, b3);
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

    // ---- content scores S[16][KT] = Qu * K^T plus the shifted positional term
    float s[KT / 8][4];
#pragma unroll
    for (int n = 0; n < KT / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int n = 0; n < KT / 16; ++n) {
      const int krow = n * 16 + (lane & 7) + (lane >> 4) * 8;
#pragma unroll
      for (int kk = 0; kk < DK / 16; ++kk) {
        uint32_t b0, b1, b2, b3;
        const int col = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(k_base + (uint32_t)((krow * LD + col) * 2), b0, b1, b2, b3);
        mma16816<H>(s[2 * n], qu[kk], b0, b1);
        mma16816<H>(s[2 * n + 1], qu[kk], b2, b3);
      }
    }
    // local row ri, local key cj: positional row centre-1-(iw+ri)+(j0+cj), i.e.
    // window column 15 - ri + cj
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
    __syncthreads();  // all warps done with this stage before it is refilled
  }
  cp_async_wait<0>();

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
  return launch_pdl(kern, grid, dim3(NTHREADS), smem, st, reinterpret_cast<const H*>(a.qkv),
                    reinterpret_cast<const H*>(a.ptab), a.ptab_rows, a.ptab_ld > 0 ? a.ptab_ld : a.d, a.centre, a.bias_u, a.bias_v, a.tiles, a.item_off,
                    a.item_len, reinterpret_cast<H*>(a.ctx), a.d, scale_log2);
}

}  // namespace

int attn_mma_query_tile() { return QT; }

cudaError_t attention_mma_launch(const AttnArgs& a, bool bf16, cudaStream_t st) {
  if (a.n_tiles <= 0) return cudaSuccess;
  const int dk = a.d / a.n_heads;
  if (a.d % a.n_heads != 0) return cudaErrorInvalidValue;
  if (dk == 128) return bf16 ? launch_attn<__nv_bfloat16, 128>(a, st) : launch_attn<__half, 128>(a, st);
  if (dk == 64) return bf16 ? launch_attn<__nv_bfloat16, 64>(a, st) : launch_attn<__half, 64>(a, st);
  return cudaErrorInvalidValue;
}

// The tcgen05 kernel (attention_tc.cu) is the product path; PKC_ATTN_MMA_SYNC=1
// selects this warp-level mma.sync kernel instead, for A/B comparisons.
bool attn_use_mma_sync() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("PKC_ATTN_MMA_SYNC");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

int attn_query_tile() { return attn_use_mma_sync() ? attn_mma_query_tile() : attn_tc_query_tile(); }

cudaError_t attention_launch(const AttnArgs& a, bool bf16, cudaStream_t st) {
  return attn_use_mma_sync() ? attention_mma_launch(a, bf16, st) : attention_tc_launch(a, bf16, st);
}

}  // namespace pkc
