// Dense contraction for every projection of the encoder: D = A * B^T with
// A [M, K] activations and B [N, K] weights, both K-major f16 or bf16 in HBM,
// accumulated in f32 in tensor memory by tcgen05.mma (kind::f16), operands
// staged by TMA (128-byte swizzle) through a 4-deep mbarrier pipeline.
//
// Persistent CTAs (one per SM), 6 warps:
//   warp 0 lane 0  TMA producer (runs ahead across tiles through a 4-stage ring)
//   warp 1 lane 0  MMA issuer (single thread, as tcgen05 requires)
//   warps 2..9     epilogue: warp w drains TMEM lanes [32(w%4), 32(w%4)+32),
//                  columns [0,128) for warps 2..5 and [128,256) for warps 6..9
// Two 256-column f32 accumulators in TMEM (all 512 columns): the epilogue of
// tile i runs while the MMAs of tile i+1 fill the other accumulator.
//
#include <cstdlib>

#include "common.cuh"
#include "gemm.h"
#include "per_device.h"

namespace pkc {

namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;  // 64 x 2 bytes = one 128-byte swizzle row
constexpr int STAGES = 4;
constexpr int EPI_WARPS = 8;  // two per TMEM lane quarter, each draining half the columns
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr int A_STAGE_BYTES = BM * BK * 2;
constexpr int B_STAGE_BYTES = BN * BK * 2;
constexpr int SMEM_BYTES = STAGES * (A_STAGE_BYTES + B_STAGE_BYTES) + 8 * 4096 + 256 + 1024;
constexpr uint32_t TMEM_COLS = 512;  // two 128 x 256 f32 accumulators

constexpr int EPI_STAGE_BYTES = 32 * 32 * 4;  // per epilogue warp: 32 rows x 32 f32 columns

// Operand columns of k-block kb: kb * BK for plain operands; in the split
// mode (args.split_k = Ks) pass kb / (Ks / BK) reads (hi, hi), (hi, lo), (lo, hi)
// of the [hi | lo] rows of A and B.
__device__ __forceinline__ void kb_cols(const GemmArgs& a, int kb, int& ca, int& cb) {
  if (!a.split_k) {
    ca = cb = kb * BK;
    return;
  }
  const int kbs = a.split_k / BK;
  const int seg = kb / kbs;
  const int kk = (kb - seg * kbs) * BK;
  ca = kk + (seg == 2 ? a.split_k : 0);
  cb = kk + (seg == 1 ? a.split_k : 0);
}

// Drain this warp's share of one accumulator tile (TMEM lanes row0..row0+31,
// half `half` of the 32-column chunks) through the fused epilogue.
// tcgen05.ld hands each thread one row, but a global access per thread-row
// touches 32 rows (32 cache lines) per instruction. So every chunk is staged
// through a per-warp 32 x 32 f32 tile in shared memory -- 16-byte chunk c of
// row r at (c ^ (r & 7)), conflict-free both ways -- and leaves with lanes
// laid along the rows: each instruction then covers 4 rows x 128 bytes.
// Every lane executes the TMEM loads (.sync.aligned); only rows < M store.
template <typename H, int EPI, int TBN = BN>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& args, uint32_t trow, int row0, int n0,
                                              int half, uint8_t* stage) {
  constexpr bool PAIRED = EPI == EPI_GLU_H || EPI == EPI_POWER_F32;
  // the paired epilogues read value and gate columns of one 256-wide tile
  static_assert(TBN == BN || !PAIRED, "paired epilogues need 256-column tiles");
  const int lane = threadIdx.x & 31;
  const int rr = lane >> 3, cc = lane & 7;  // coalesced layout: rows 4k + rr, 16-byte chunk cc
  const uint32_t sst = smem_u32(stage);
  // output chunk j: columns [32j, 32j + 32) of the output tile (PAIRED: value
  // columns 32j and gate columns BN/2 + 32j of the accumulator)
  const int j0 = PAIRED ? half * (BN / 128) : half * (TBN / 64);
  const int j1 = PAIRED ? j0 + BN / 128 : j0 + TBN / 64;
  const int oc0 = PAIRED ? n0 / 2 : n0;  // output column of chunk 0
  float4 cur[8], nxt[8];
  // EPI_RESID_F32 with stats: lane (rr, cc) merges row 4 * cc + rr's chunk
  // statistics over this half's 128 columns (Chan's update, equal counts)
  float run_mean = 0.f, run_m2 = 0.f;
  auto row_ok = [&](int k) { return row0 + 4 * k + rr < args.M; };
  auto resid = [&](int j, int k) {
    return reinterpret_cast<float4*>(reinterpret_cast<float*>(args.out) + (size_t)(row0 + 4 * k + rr) * args.ldo +
                                     oc0 + 32 * j + 4 * cc);
  };
  // EPI_RESID_F32 without statistics adds alpha (acc + bias) to the residual
  // with a vector reduction in L2 (red.global.add.v4.f32: one update per
  // element, so the sums are those of load + add + store) and loads nothing;
  // with statistics the updated rows are needed here, so they are loaded
  const bool rload = EPI == EPI_RESID_F32 && args.stats != nullptr;
  if constexpr (EPI == EPI_RESID_F32) {
    if (rload) {
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (row_ok(k)) cur[k] = *resid(j0, k);
    }
  }
#pragma unroll 1
  for (int j = j0; j < j1; ++j) {
    uint32_t r[32];
    if constexpr (PAIRED) {
      uint32_t g[32];
      tmem_ld32(trow + 32 * j, r);
      tmem_ld32(trow + BN / 2 + 32 * j, g);
      tmem_ld_wait();
      const float* ba = args.bias ? args.bias + n0 + 32 * j : nullptr;
      const float* bg = args.bias ? args.bias + n0 + BN / 2 + 32 * j : nullptr;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float a = __uint_as_float(r[i]), gg = __uint_as_float(g[i]);
        if constexpr (EPI == EPI_GLU_H) {
          if (ba) {
            a += ba[i];
            gg += bg[i];
          }
          r[i] = __float_as_uint(a * sigmoidf_(gg));
        } else {
          r[i] = __float_as_uint(a * a + gg * gg);
        }
      }
    } else {
      tmem_ld32(trow + 32 * j, r);
      if constexpr (EPI == EPI_RESID_F32) {
        // residual of the next chunk in flight during this one
        if (rload && j + 1 < j1) {
#pragma unroll
          for (int k = 0; k < 8; ++k)
            if (row_ok(k)) nxt[k] = *resid(j + 1, k);
        }
      }
      tmem_ld_wait();
    }
    // row layout -> staging tile
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<uint4*>(stage + lane * 128 + ((c ^ (lane & 7)) << 4)) =
          make_uint4(r[4 * c], r[4 * c + 1], r[4 * c + 2], r[4 * c + 3]);
    __syncwarp();
    // staging tile -> rows (lanes along the row)
    const int oc = oc0 + 32 * j + 4 * cc;
    float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if constexpr (!PAIRED) {
      if (args.bias) b4 = *reinterpret_cast<const float4*>(args.bias + oc);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int rl = 4 * k + rr;
      float4 w;
      asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                   : "=f"(w.x), "=f"(w.y), "=f"(w.z), "=f"(w.w)
                   : "r"(sst + rl * 128 + ((cc ^ (rl & 7)) << 4)));
      const bool okr = row_ok(k);
      const size_t ro = (size_t)(row0 + rl) * args.ldo + oc;
      if constexpr (EPI == EPI_RESID_F32) {
        if (!rload) {
          if (okr) {
            float* dst = reinterpret_cast<float*>(args.out) + ro;
            asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst),
                         "f"(args.alpha * (w.x + b4.x)), "f"(args.alpha * (w.y + b4.y)),
                         "f"(args.alpha * (w.z + b4.z)), "f"(args.alpha * (w.w + b4.w))
                         : "memory");
          }
          continue;
        }
        float4 o = okr ? cur[k] : make_float4(0.f, 0.f, 0.f, 0.f);
        o.x += args.alpha * (w.x + b4.x);
        o.y += args.alpha * (w.y + b4.y);
        o.z += args.alpha * (w.z + b4.z);
        o.w += args.alpha * (w.w + b4.w);
        if (okr) *reinterpret_cast<float4*>(reinterpret_cast<float*>(args.out) + ro) = o;
        if (args.stats) {
          // this chunk's 32 values of the row sit in the 8 lanes with the same rr
          float sum = (o.x + o.y) + (o.z + o.w);
          sum += __shfl_xor_sync(0xffffffffu, sum, 1);
          sum += __shfl_xor_sync(0xffffffffu, sum, 2);
          sum += __shfl_xor_sync(0xffffffffu, sum, 4);
          const float mc = sum * (1.0f / 32.0f);
          const float d0 = o.x - mc, d1 = o.y - mc, d2 = o.z - mc, d3 = o.w - mc;
          float q = (d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3);
          q += __shfl_xor_sync(0xffffffffu, q, 1);
          q += __shfl_xor_sync(0xffffffffu, q, 2);
          q += __shfl_xor_sync(0xffffffffu, q, 4);
          if (cc == k) {
            const int jj = j - j0;
            if (jj == 0) {
              run_mean = mc;
              run_m2 = q;
            } else {
              const float dl = mc - run_mean;
              const float inv = 1.0f / (float)(jj + 1);
              run_mean += dl * inv;
              run_m2 += q + dl * dl * (32.0f * (float)jj * inv);
            }
          }
        }
        continue;
      }
      if (!okr) continue;
      if constexpr (EPI == EPI_STORE_H || EPI == EPI_GLU_H) {
        if (args.ofmt != OUT_H) {
          float x0 = w.x, x1 = w.y, x2 = w.z, x3 = w.w;
          if constexpr (EPI == EPI_STORE_H) {
            x0 += b4.x; x1 += b4.y; x2 += b4.z; x3 += b4.w;
            if (args.act == ACT_SILU) {
              x0 = siluf_(x0); x1 = siluf_(x1); x2 = siluf_(x2); x3 = siluf_(x3);
            } else if (args.act == ACT_RELU) {
              x0 = fmaxf(x0, 0.f); x1 = fmaxf(x1, 0.f); x2 = fmaxf(x2, 0.f); x3 = fmaxf(x3, 0.f);
            }
          }
          if (args.ofmt == OUT_F32) {
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(args.out) + ro) = make_float4(x0, x1, x2, x3);
          } else {
            const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1), h2 = __float2half_rn(x2),
                         h3 = __float2half_rn(x3);
            __half* o = reinterpret_cast<__half*>(args.out) + ro;
            *reinterpret_cast<uint2*>(o) = make_uint2(pack2<__half>(__half2float(h0), __half2float(h1)),
                                                      pack2<__half>(__half2float(h2), __half2float(h3)));
            *reinterpret_cast<uint2*>(o + args.split_ld) =
                make_uint2(pack2<__half>(x0 - __half2float(h0), x1 - __half2float(h1)),
                           pack2<__half>(x2 - __half2float(h2), x3 - __half2float(h3)));
          }
          continue;
        }
      }
      if constexpr (EPI == EPI_STORE_F32) {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(args.out) + ro) =
            make_float4(args.alpha * (w.x + b4.x), args.alpha * (w.y + b4.y), args.alpha * (w.z + b4.z),
                        args.alpha * (w.w + b4.w));
      } else if constexpr (EPI == EPI_POWER_F32) {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(args.out) + ro) = w;
      } else {
        float x0 = w.x, x1 = w.y, x2 = w.z, x3 = w.w;
        if constexpr (EPI == EPI_STORE_H) {
          x0 += b4.x; x1 += b4.y; x2 += b4.z; x3 += b4.w;
          if (args.act == ACT_SILU) {
            x0 = siluf_(x0); x1 = siluf_(x1); x2 = siluf_(x2); x3 = siluf_(x3);
          } else if (args.act == ACT_RELU) {
            x0 = fmaxf(x0, 0.f); x1 = fmaxf(x1, 0.f); x2 = fmaxf(x2, 0.f); x3 = fmaxf(x3, 0.f);
          }
        }
        *reinterpret_cast<uint2*>(reinterpret_cast<H*>(args.out) + ro) = make_uint2(pack2<H>(x0, x1), pack2<H>(x2, x3));
      }
    }
    __syncwarp();  // the staging tile is reused by the next chunk
    if constexpr (EPI == EPI_RESID_F32) {
      if (rload) {
#pragma unroll
        for (int k = 0; k < 8; ++k) cur[k] = nxt[k];
      }
    }
  }
  if constexpr (EPI == EPI_RESID_F32) {
    const int rl = 4 * cc + rr;
    if (args.stats && row0 + rl < args.M)
      *reinterpret_cast<float2*>(args.stats + ((size_t)(row0 + rl) * (args.N / 128) + (oc0 + 32 * j0) / 128) * 2) =
          make_float2(run_mean, run_m2);
  }
}

// Tile index -> row block (tile_mb) and column block (tile_nb). The tiles a
// wave runs at the same time should share the larger operand, so that it
// crosses HBM once while the smaller one stays in L2: column blocks fastest
// when A has more rows than B (the encoder's GEMMs at batch size: the N / 256
// tiles of a row block run together and read its A rows once; row blocks
// fastest would stream all of A once per column block, which for the
// K = 4096 FFN-down at M = 14k frames measured 3.6x its algorithmic bytes),
// row blocks fastest otherwise.
__device__ __forceinline__ int tile_mb(int tile, int tiles_m, int tiles_n, bool nfast) {
  return nfast ? tile / tiles_n : tile % tiles_m;
}
__device__ __forceinline__ int tile_nb(int tile, int tiles_m, int tiles_n, bool nfast) {
  return nfast ? tile % tiles_n : tile / tiles_m;
}

template <typename H, int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE_BYTES;
  uint8_t* sE = sB + STAGES * B_STAGE_BYTES;  // epilogue staging, EPI_STAGE_BYTES per epilogue warp
  uint64_t* bars = reinterpret_cast<uint64_t*>(sE + EPI_WARPS * EPI_STAGE_BYTES);
  // bars: [0,S) full, [S,2S) empty, 2S+{0,1} accumulator full, 2S+{2,3} accumulator empty
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int KB = args.K / BK;
  const int tiles_m = (args.M + BM - 1) / BM;
  const int tiles_n = args.N / BN;
  const int n_tiles = tiles_m * tiles_n;
  const bool nfast = args.M > args.N;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    for (int s = 0; s < 2 * STAGES; ++s) mbar_init(smem_u32(&bars[s]), 1);
    mbar_init(smem_u32(&bars[2 * STAGES + 0]), 1);
    mbar_init(smem_u32(&bars[2 * STAGES + 1]), 1);
    mbar_init(smem_u32(&bars[2 * STAGES + 2]), EPI_WARPS);
    mbar_init(smem_u32(&bars[2 * STAGES + 3]), EPI_WARPS);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // A (and the residual) come from the previous kernel

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
        const int m0 = tile_mb(tile, tiles_m, tiles_n, nfast) * BM;
        const int n0 = tile_nb(tile, tiles_m, tiles_n, nfast) * BN;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(smem_u32(&bars[STAGES + s]), ph ^ 1u, args.err, DEV_ERR_TIMEOUT_EMPTY)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&bars[s]);
          mbar_arrive_expect_tx(fb, A_STAGE_BYTES + B_STAGE_BYTES);
          int ca, cb;
          kb_cols(args, kb, ca, cb);
          tma_load_2d(smem_u32(sA + s * A_STAGE_BYTES), &tmA, fb, ca, m0);
          tma_load_2d(smem_u32(sB + s * B_STAGE_BYTES), &tmB, fb, cb, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer
      constexpr uint32_t idesc = idesc_f16(BM, BN, is_bf16<H>::value ? 1 : 0);
      uint32_t it = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++local) {
        const int buf = local & 1;
        const uint32_t use = (uint32_t)(local >> 1);
        if (!mbar_wait(smem_u32(&bars[2 * STAGES + 2 + buf]), (use & 1u) ^ 1u, args.err,
                       DEV_ERR_TIMEOUT_ACCUM))
          break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(buf * BN);
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(smem_u32(&bars[s]), ph, args.err, DEV_ERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = smem_desc_sw128(smem_u32(sA + s * A_STAGE_BYTES));
          const uint64_t db = smem_desc_sw128(smem_u32(sB + s * B_STAGE_BYTES));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(acc, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc,
                     (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(smem_u32(&bars[STAGES + s]));  // frees the smem stage
        }
        if (ok) umma_commit(smem_u32(&bars[2 * STAGES + buf]));  // accumulator ready
      }
    }
  } else {
    // ---- epilogue warps 2..9
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;
    int local = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++local) {
      const int buf = local & 1;
      const uint32_t use = (uint32_t)(local >> 1);
      const bool have =
          __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars[2 * STAGES + buf]), use & 1u, args.err,
                                            DEV_ERR_TIMEOUT_ACCUM) ? 1 : 0) != 0;
      if (!have) break;
      tc_fence_after();
      const int m0 = tile_mb(tile, tiles_m, tiles_n, nfast) * BM;
      const int n0 = tile_nb(tile, tiles_m, tiles_n, nfast) * BN;
      const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN);
      epilogue_tile<H, EPI>(args, trow, m0 + q * 32, n0, half, sE + (warp - 2) * EPI_STAGE_BYTES);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars[2 * STAGES + 2 + buf]));
    }
  }

  // the next kernel launches once every CTA is here (launched earlier, its
  // CTAs occupied SMs that the other stream's work could use: measured
  // neutral on one stream, slower with two)
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, TMEM_COLS);
}


// ============================================================================
// 2-SM variant: a cluster of two CTAs computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M = 256). Each CTA stages its own 128 rows of A
// and 128 rows (half of N) of B per k-block, so a CTA moves 32 KB per 4 MFLOP
// of its share instead of 48 KB (the 1-SM tile's per-SM load bandwidth and
// shared-memory traffic were the limit), and the ring is 6 stages deep.
//   * both CTAs' producers load into their own smem; the transaction bytes of
//     both complete on the leader's (rank 0) full barrier, which the leader's
//     producer arms for 2 x 32 KB
//   * the leader's single MMA thread issues the M = 256 MMAs and commits with
//     a cluster multicast to both CTAs' empty / accumulator-full barriers
//   * each CTA's 4 epilogue warps drain its own TMEM (its 128 rows x 256
//     columns) and arrive on the leader's accumulator-empty barrier
// TMA loads are plain (no cluster multicast).
constexpr int STAGES2 = 6;
constexpr int HALF_ROWS = 128;
constexpr int A2_BYTES = HALF_ROWS * BK * 2;
constexpr int B2_BYTES = HALF_ROWS * BK * 2;
constexpr int SMEM2_BYTES = STAGES2 * (A2_BYTES + B2_BYTES) + 8 * 4096 + 512 + 1024;

// ---- work schedule of the 2-SM kernel
// Whole tiles: pair p takes tiles p, p + P, p + 2P, ... (P = CTA pairs).
// Stream-K (args.sk_ws set): the W = tiles x KB k-blocks, in tile-major order,
// are cut into P contiguous ranges [p W / P, (p + 1) W / P); a range is a
// sequence of segments (tile, kb0, kb1). A segment with kb0 > 0 is a partial
// sum: its epilogue spills the f32 accumulator to the pair's workspace slot
// and raises a flag. The segment holding a split tile's k-block 0 (the last
// segment of a range) finishes the tile: it adds the partials of the pairs
// that follow, in pair order (so the result does not depend on timing), then
// runs the fused epilogue. Partial segments come first in their ranges, so
// finishers seldom wait. A range holds at most one partial segment, hence one
// workspace slot per pair. Stream-K needs W >= P (no empty range); the kernel
// falls back to whole tiles otherwise.
struct SegIter {
  long long u, b;
  int tile_dp, step, KB, n_tiles;
  bool sk;
  __device__ __forceinline__ SegIter(bool sk_, int pair, int npairs, int KB_, int n_tiles_)
      : tile_dp(pair), step(npairs), KB(KB_), n_tiles(n_tiles_), sk(sk_) {
    const long long W = (long long)n_tiles_ * KB_;
    u = sk_ ? (long long)pair * W / npairs : 0;
    b = sk_ ? (long long)(pair + 1) * W / npairs : 0;
  }
  __device__ __forceinline__ bool next(int& tile, int& kb0, int& kb1) {
    if (sk) {
      if (u >= b) return false;
      tile = (int)(u / KB);
      kb0 = (int)(u - (long long)tile * KB);
      const long long left = b - u;
      kb1 = left < (long long)(KB - kb0) ? kb0 + (int)left : KB;
      u += kb1 - kb0;
      return true;
    }
    if (tile_dp >= n_tiles) return false;
    tile = tile_dp;
    kb0 = 0;
    kb1 = KB;
    tile_dp += step;
    return true;
  }
};

constexpr int SK_SLOT_FLOATS = 32 * 128;  // one epilogue warp: 32 rows x 128 accumulator columns

// Accumulator column of 32-column chunk c (0..3) of the epilogue warp with
// column half `half`: exactly the columns epilogue_tile reads in that warp
// (value and gate chunks for the paired epilogues), so a warp's fix-up never
// depends on another warp.
template <int EPI>
__device__ __forceinline__ int sk_col(int half, int c) {
  constexpr bool PAIRED = EPI == EPI_GLU_H || EPI == EPI_POWER_F32;
  return PAIRED ? (c >> 1) * (BN / 2) + half * (BN / 4) + (c & 1) * 32 : half * (BN / 2) + c * 32;
}

// Partial sum of one epilogue warp (TMEM lanes of `trow`, its 128
// accumulator columns) to its workspace slot, lane-interleaved so each store
// instruction writes 512 contiguous bytes; then the slot's flag.
template <int EPI>
__device__ __forceinline__ void sk_spill(const GemmArgs& args, uint32_t trow, int half, int slot) {
  const int lane = threadIdx.x & 31;
  float* dst = args.sk_ws + (size_t)slot * SK_SLOT_FLOATS;
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t r[32];
    tmem_ld32(trow + (uint32_t)sk_col<EPI>(half, c), r);
    tmem_ld_wait();
#pragma unroll
    for (int e = 0; e < 8; ++e)
      __stcg(reinterpret_cast<float4*>(dst + ((c * 8 + e) * 32 + lane) * 4),
             make_float4(__uint_as_float(r[4 * e]), __uint_as_float(r[4 * e + 1]), __uint_as_float(r[4 * e + 2]),
                         __uint_as_float(r[4 * e + 3])));
  }
  __threadfence();
  __syncwarp();
  if (lane == 0) st_release_gpu(args.sk_flags + slot, 1);
}

// Finisher of split tile `tile` (pair `pair` holds its k-block 0): add the
// partial sums of the pairs after it whose (non-empty) ranges start inside
// the tile, in pair order, into this warp's accumulator columns, back in
// TMEM; clears their flags for the next launch. `slot` = this warp's own
// slot; the same warp of pair q uses slot + (q - pair) * 2 * EPI_WARPS.
template <int EPI>
__device__ __forceinline__ void sk_fixup(const GemmArgs& args, uint32_t trow, int half, int slot, int pair,
                                         int npairs, long long W, long long tile_end) {
  const int lane = threadIdx.x & 31;
  // contributors: pairs pair+1 .. pair+n (W >= npairs: no range is empty)
  int n = 0;
  while (pair + n + 1 < npairs && (long long)(pair + n + 1) * W / npairs < tile_end) ++n;
  bool ok = true;
  if (lane == 0)
    for (int i = 1; i <= n && ok; ++i)
      ok = wait_flag_gpu(args.sk_flags + slot + i * 2 * EPI_WARPS, args.err, DEV_ERR_TIMEOUT_SPLITK);
  __syncwarp();
  // every lane acquires the flags itself before reading the partials
  for (int i = 1; i <= n; ++i) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(args.sk_flags + slot + i * 2 * EPI_WARPS)
                 : "memory");
    (void)v;
  }
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t r[32];
    tmem_ld32(trow + (uint32_t)sk_col<EPI>(half, c), r);
    tmem_ld_wait();
#pragma unroll 1
    for (int i = 1; i <= n; ++i) {
      const float* src = args.sk_ws + (size_t)(slot + i * 2 * EPI_WARPS) * SK_SLOT_FLOATS;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(src + ((c * 8 + e) * 32 + lane) * 4));
        r[4 * e] = __float_as_uint(__uint_as_float(r[4 * e]) + v.x);
        r[4 * e + 1] = __float_as_uint(__uint_as_float(r[4 * e + 1]) + v.y);
        r[4 * e + 2] = __float_as_uint(__uint_as_float(r[4 * e + 2]) + v.z);
        r[4 * e + 3] = __float_as_uint(__uint_as_float(r[4 * e + 3]) + v.w);
      }
    }
    tmem_st32(trow + (uint32_t)sk_col<EPI>(half, c), r);
  }
  tmem_st_wait();
  __syncwarp();
  if (lane == 0)
    for (int i = 1; i <= n; ++i) args.sk_flags[slot + i * 2 * EPI_WARPS] = 0;
}

// TBN = 128: pair tiles of 256 x 128 (each CTA stages 64 rows of B) for
// GEMMs whose 256-wide tiles would fill at most half of the SM pairs (the
// encoder's N = 1024 GEMMs on a few utterances); whole tiles, no row
// statistics, no paired epilogue.
template <typename H, int EPI, bool SK, int TBN = BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    k_gemm_tc2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               GemmArgs args) {
  static_assert(TBN == BN || (TBN == 128 && !SK), "128-column pair tiles are whole tiles only");
  constexpr int TB2 = (TBN / 2) * BK * 2;  // this CTA's B rows per stage
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES2 * A2_BYTES;
  uint8_t* sE = sB + STAGES2 * B2_BYTES;  // epilogue staging, EPI_STAGE_BYTES per epilogue warp
  uint64_t* bars = reinterpret_cast<uint64_t*>(sE + EPI_WARPS * EPI_STAGE_BYTES);
  // bars: [0,S) full, [S,2S) empty, 2S+{0,1} accumulator full, 2S+{2,3} accumulator empty
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES2 + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int KB = args.K / BK;
  const int tiles_m = (args.M + 2 * HALF_ROWS - 1) / (2 * HALF_ROWS);
  const int tiles_n = args.N / TBN;
  const int n_tiles = tiles_m * tiles_n;
  const bool nfast = args.M > args.N;
  // the stream-K instantiation (SK) falls back to whole tiles if W < P
  const bool sk = SK && (long long)n_tiles * KB >= npairs;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    for (int s = 0; s < 2 * STAGES2; ++s) mbar_init(smem_u32(&bars[s]), 1);
    mbar_init(smem_u32(&bars[2 * STAGES2 + 0]), 1);
    mbar_init(smem_u32(&bars[2 * STAGES2 + 1]), 1);
    mbar_init(smem_u32(&bars[2 * STAGES2 + 2]), 2 * EPI_WARPS);
    mbar_init(smem_u32(&bars[2 * STAGES2 + 3]), 2 * EPI_WARPS);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0) {
    tmem_alloc_2sm(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish_2sm();
  }
  tc_fence_before();
  cluster_sync();  // barrier init + TMEM alloc of both CTAs visible cluster-wide
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // A (and the residual) come from the previous kernel

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer (both CTAs)
      uint32_t it = 0;
      bool ok = true;
      SegIter sg(sk, pair, npairs, KB, n_tiles);
      int tile, kb0, kb1;
      while (ok && sg.next(tile, kb0, kb1)) {
        const int m0 = tile_mb(tile, tiles_m, tiles_n, nfast) * 2 * HALF_ROWS + (int)rank * HALF_ROWS;
        const int n0 = tile_nb(tile, tiles_m, tiles_n, nfast) * TBN + (int)rank * (TBN / 2);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES2;
          const uint32_t ph = (it / STAGES2) & 1u;
          if (!mbar_wait(smem_u32(&bars[STAGES2 + s]), ph ^ 1u, args.err, DEV_ERR_TIMEOUT_EMPTY)) {
            ok = false;
            break;
          }
          const uint32_t full_leader = mapa_shared(smem_u32(&bars[s]), 0);
          if (leader) mbar_arrive_expect_tx(smem_u32(&bars[s]), 2 * (A2_BYTES + TB2));
          int ca, cb;
          kb_cols(args, kb, ca, cb);
          tma_load_2d_2sm(smem_u32(sA + s * A2_BYTES), &tmA, full_leader, ca, m0);
          tma_load_2d_2sm(smem_u32(sB + s * B2_BYTES), &tmB, full_leader, cb, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---- MMA issuer (leader CTA only)
      constexpr uint32_t idesc = idesc_f16(2 * HALF_ROWS, TBN, is_bf16<H>::value ? 1 : 0);
      uint32_t it = 0;
      int local = 0;
      bool ok = true;
      SegIter sg(sk, pair, npairs, KB, n_tiles);
      int tile, kb0, kb1;
      for (; ok && sg.next(tile, kb0, kb1); ++local) {
        const int buf = local & 1;
        const uint32_t use = (uint32_t)(local >> 1);
        if (!mbar_wait(smem_u32(&bars[2 * STAGES2 + 2 + buf]), (use & 1u) ^ 1u, args.err,
                       DEV_ERR_TIMEOUT_ACCUM))
          break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(buf * TBN);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES2;
          const uint32_t ph = (it / STAGES2) & 1u;
          if (!mbar_wait(smem_u32(&bars[s]), ph, args.err, DEV_ERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = smem_desc_sw128(smem_u32(sA + s * A2_BYTES));
          const uint64_t db = smem_desc_sw128(smem_u32(sB + s * B2_BYTES));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16_2sm(acc, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc,
                         (kb > kb0 || k > 0) ? 1u : 0u);
          umma_commit_2sm_mc(smem_u32(&bars[STAGES2 + s]), 0x3);  // frees the stage in both CTAs
        }
        if (ok) umma_commit_2sm_mc(smem_u32(&bars[2 * STAGES2 + buf]), 0x3);  // accumulators ready
      }
    }
  } else {
    // ---- epilogue warps 2..9 (both CTAs): this CTA's 128 rows of the tile
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t acce_leader0 = mapa_shared(smem_u32(&bars[2 * STAGES2 + 2]), 0);
    const uint32_t acce_leader1 = mapa_shared(smem_u32(&bars[2 * STAGES2 + 3]), 0);
    int local = 0;
    SegIter sg(sk, pair, npairs, KB, n_tiles);
    int tile, kb0, kb1;
    // this warp's stream-K slot (pair, CTA rank, epilogue warp)
    const int slot = (pair * 2 + (int)rank) * EPI_WARPS + (warp - 2);
    for (; sg.next(tile, kb0, kb1); ++local) {
      const int buf = local & 1;
      const uint32_t use = (uint32_t)(local >> 1);
      const bool have =
          __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars[2 * STAGES2 + buf]), use & 1u, args.err,
                                            DEV_ERR_TIMEOUT_ACCUM) ? 1 : 0) != 0;
      if (!have) break;
      tc_fence_after();
      const int m0 = tile_mb(tile, tiles_m, tiles_n, nfast) * 2 * HALF_ROWS + (int)rank * HALF_ROWS;
      const int n0 = tile_nb(tile, tiles_m, tiles_n, nfast) * TBN;
      const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * TBN);
      if (SK && kb0 > 0) {
        sk_spill<EPI>(args, trow, half, slot);  // partial sum of a split tile
      } else {
        // finisher of a split tile: the pairs after this one whose ranges
        // start inside the tile hold its remaining k-blocks
        if (SK && kb1 < KB)
          sk_fixup<EPI>(args, trow, half, slot, pair, npairs, (long long)n_tiles * KB, (long long)(tile + 1) * KB);
        epilogue_tile<H, EPI, TBN>(args, trow, m0 + q * 32, n0, half, sE + (warp - 2) * EPI_STAGE_BYTES);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote_cta(buf ? acce_leader1 : acce_leader0);
    }
  }

  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 0) tmem_dealloc_2sm(tmem, TMEM_COLS);
}

// ============================================================================
// 2-SM variant with B dequantised inside the kernel (Q8_0 / Q4_K weights).
// Each CTA's producer loads its 128 rows of A (TMA, completing on the pair
// leader's stage barrier, as in k_gemm_tc2) and its 128 rows of the quantised
// B block (TMA into a raw staging ring, completing on a local barrier). Four
// converter warps turn the raw block into the 16-bit, 128-byte-swizzled tile
// the MMA reads -- one B row per converter thread -- then arrive on the
// leader's stage barrier, whose phase therefore completes when A has landed
// in both CTAs and both CTAs' B halves are converted. The dequantisation is
// the load-time one bit for bit: Q8_0 d*q, Q4_K (d*sc)*q - dmin*m, in f32,
// rounded once to f16 / bf16.
// Two rings: QSTAGES stages of {A tile, raw quantised B} loaded by TMA (deep
// enough to cover the load latency), and QBSTAGES stages of converted B (the
// converters run up to that many k-blocks ahead of the MMA).
constexpr int QSTAGES = 5;
constexpr int QBSTAGES = 3;
constexpr int CVT_WARPS = 4;
constexpr int QTHREADS = 64 + 32 * EPI_WARPS + 32 * CVT_WARPS;  // 448

template <int QT>
struct QLayout {
  static constexpr int RAW_Q = QT == QT_Q8_0 ? HALF_ROWS * 64 : HALF_ROWS * 32;  // one k-block of q
  static constexpr int RAW_S = QT == QT_Q8_0 ? 2 * HALF_ROWS * 4 : 2 * 2 * HALF_ROWS * 4;
  static constexpr int RAW = RAW_Q + RAW_S;  // 9216 / 6144: multiples of 1024
  static constexpr int SMEM = QSTAGES * (A2_BYTES + RAW) + QBSTAGES * B2_BYTES + EPI_WARPS * EPI_STAGE_BYTES + 768 + 1024;
};

// Dequantise row r of the CTA's raw B block (one k-block of 64 values) into
// the swizzled 16-bit tile: 16-byte chunk c of row r at (c ^ (r & 7)).
template <typename H, int QT>
__device__ __forceinline__ void dequant_row(const uint8_t* raw, uint8_t* dst, int r) {
  using QL = QLayout<QT>;
  const float* s0 = reinterpret_cast<const float*>(raw + QL::RAW_Q);
  uint32_t w[32];
  if constexpr (QT == QT_Q8_0 && !is_bf16<H>::value) {
    // row r: 64 int8 as four 16-byte chunks, 64-byte TMA swizzle: chunk c at
    // c ^ ((r >> 1) & 3). f16 without conversion instructions: the half with
    // bits 0x64 | (b ^ 0x80) is 1024 + b + 128 exactly, minus 1152 is b
    // exactly, and one f16 multiply by the scale (an f16 value) rounds b * d
    // once -- the same value as the f32 product rounded to f16.
    const __half2 off = __float2half2_rn(1152.f);
    const __half2 dd0 = __float2half2_rn(s0[r]), dd1 = __float2half2_rn(s0[HALF_ROWS + r]);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 v = *reinterpret_cast<const uint4*>(raw + r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
      const uint32_t ws[4] = {v.x, v.y, v.z, v.w};
      const __half2 dd = c < 2 ? dd0 : dd1;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t lo = __byte_perm(ws[i], 0x64646464u, 0x4140) ^ 0x00800080u;
        const uint32_t hi = __byte_perm(ws[i], 0x64646464u, 0x4342) ^ 0x00800080u;
        const __half2 a = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&lo), off), dd);
        const __half2 b = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&hi), off), dd);
        w[8 * c + 2 * i] = *reinterpret_cast<const uint32_t*>(&a);
        w[8 * c + 2 * i + 1] = *reinterpret_cast<const uint32_t*>(&b);
      }
    }
  } else if constexpr (QT == QT_Q8_0) {
    const float d0 = s0[r], d1 = s0[HALF_ROWS + r];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 v = *reinterpret_cast<const uint4*>(raw + r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
      const int8_t* q = reinterpret_cast<const int8_t*>(&v);
      const float d = c < 2 ? d0 : d1;
#pragma unroll
      for (int i = 0; i < 8; ++i) w[8 * c + i] = pack2<H>(d * (float)q[2 * i], d * (float)q[2 * i + 1]);
    }
  } else {
    // row r: 32 bytes of nibbles (byte j = values 2j, 2j+1), 32-byte TMA
    // swizzle: chunk c at c ^ ((r >> 2) & 1); sub-block b = values [32b, 32b+32)
    const float* s1 = s0 + 2 * HALF_ROWS;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const uint4 v = *reinterpret_cast<const uint4*>(raw + r * 32 + ((c ^ ((r >> 2) & 1)) << 4));
      const uint8_t* q = reinterpret_cast<const uint8_t*>(&v);
      const float ds = s0[c * HALF_ROWS + r], dm = s1[c * HALF_ROWS + r];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        // nibble -> f32 without a conversion instruction: the float with
        // bits 0x4B000000 | q is 2^23 + q, minus 2^23 is q exactly
        const float qlo = __uint_as_float(0x4B000000u | (q[i] & 15u)) - 8388608.f;
        const float qhi = __uint_as_float(0x4B000000u | (uint32_t)(q[i] >> 4)) - 8388608.f;
        const float lo = __fsub_rn(__fmul_rn(ds, qlo), dm);
        const float hi = __fsub_rn(__fmul_rn(ds, qhi), dm);
        w[16 * c + i] = pack2<H>(lo, hi);
      }
    }
  }
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<uint4*>(dst + r * 128 + ((c ^ (r & 7)) << 4)) = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}

template <typename H, int EPI, int QT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(512, 1)
    k_gemm_tc2q(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmQ,
                const __grid_constant__ CUtensorMap tmS0, const __grid_constant__ CUtensorMap tmS1,
                GemmArgs args) {
  using QL = QLayout<QT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + QSTAGES * A2_BYTES;          // converted B ring (QBSTAGES)
  uint8_t* sR = sB + QBSTAGES * B2_BYTES;           // raw quantised B ring (QSTAGES)
  uint8_t* sE = sR + QSTAGES * QL::RAW;  // epilogue staging, EPI_STAGE_BYTES per epilogue warp
  uint64_t* bars = reinterpret_cast<uint64_t*>(sE + EPI_WARPS * EPI_STAGE_BYTES);
  // bars: [0,S) full (leader: A bytes of both CTAs + both CTAs' converters),
  //       [S,2S) stage empty (MMA commit + this CTA's converters),
  //       [2S,3S) raw full (local TMA), 3S+{0,1} accumulator full,
  //       3S+{2,3} accumulator empty, 3S+4+[0,SB) converted-B slot empty (MMA commit)
  constexpr int S = QSTAGES;
  constexpr int SB = QBSTAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * S + 4 + SB);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int KB = args.K / BK;
  const int tiles_m = (args.M + 2 * HALF_ROWS - 1) / (2 * HALF_ROWS);
  const int tiles_n = args.N / BN;
  const int n_tiles = tiles_m * tiles_n;
  const bool nfast = args.M > args.N;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmS0);
    if (QT == QT_Q4_K) prefetch_tmap(&tmS1);
    for (int i = 0; i < S; ++i) {
      mbar_init(smem_u32(&bars[i]), 1 + 2 * CVT_WARPS);
      mbar_init(smem_u32(&bars[S + i]), 1 + CVT_WARPS);
      mbar_init(smem_u32(&bars[2 * S + i]), 1);
    }
    mbar_init(smem_u32(&bars[3 * S + 0]), 1);
    mbar_init(smem_u32(&bars[3 * S + 1]), 1);
    mbar_init(smem_u32(&bars[3 * S + 2]), 2 * EPI_WARPS);
    mbar_init(smem_u32(&bars[3 * S + 3]), 2 * EPI_WARPS);
    for (int i = 0; i < SB; ++i) mbar_init(smem_u32(&bars[3 * S + 4 + i]), 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0) {
    tmem_alloc_2sm(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish_2sm();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer (both CTAs): A rows, and the raw quantised B rows
      uint32_t it = 0;
      bool ok = true;
      for (int tile = pair; tile < n_tiles && ok; tile += npairs) {
        const int m0 = tile_mb(tile, tiles_m, tiles_n, nfast) * 2 * HALF_ROWS + (int)rank * HALF_ROWS;
        const int n0 = tile_nb(tile, tiles_m, tiles_n, nfast) * BN + (int)rank * HALF_ROWS;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1u;
          if (!mbar_wait(smem_u32(&bars[S + s]), ph ^ 1u, args.err, DEV_ERR_TIMEOUT_EMPTY)) {
            ok = false;
            break;
          }
          const uint32_t full_leader = mapa_shared(smem_u32(&bars[s]), 0);
          if (leader) mbar_arrive_expect_tx(smem_u32(&bars[s]), 2 * A2_BYTES);
          tma_load_2d_2sm(smem_u32(sA + s * A2_BYTES), &tmA, full_leader, kb * BK, m0);
          const uint32_t rf = smem_u32(&bars[2 * S + s]);
          uint8_t* raw = sR + s * QL::RAW;
          mbar_arrive_expect_tx(rf, QL::RAW);
          tma_load_2d(smem_u32(raw), &tmQ, rf, QT == QT_Q8_0 ? kb * 64 : kb * 32, n0);
          tma_load_2d(smem_u32(raw + QL::RAW_Q), &tmS0, rf, n0, 2 * kb);
          if (QT == QT_Q4_K) tma_load_2d(smem_u32(raw + QL::RAW_Q + 2 * HALF_ROWS * 4), &tmS1, rf, n0, 2 * kb);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---- MMA issuer (leader CTA only)
      constexpr uint32_t idesc = idesc_f16(2 * HALF_ROWS, BN, is_bf16<H>::value ? 1 : 0);
      uint32_t it = 0;
      int local = 0;
      bool ok = true;
      for (int tile = pair; tile < n_tiles && ok; tile += npairs, ++local) {
        const int buf = local & 1;
        const uint32_t use = (uint32_t)(local >> 1);
        if (!mbar_wait(smem_u32(&bars[3 * S + 2 + buf]), (use & 1u) ^ 1u, args.err, DEV_ERR_TIMEOUT_ACCUM))
          break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(buf * BN);
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1u;
          if (!mbar_wait(smem_u32(&bars[s]), ph, args.err, DEV_ERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int sb = it % SB;
          const uint64_t da = smem_desc_sw128(smem_u32(sA + s * A2_BYTES));
          const uint64_t db = smem_desc_sw128(smem_u32(sB + sb * B2_BYTES));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16_2sm(acc, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit_2sm_mc(smem_u32(&bars[S + s]), 0x3);           // A stage (both CTAs)
          umma_commit_2sm_mc(smem_u32(&bars[3 * S + 4 + sb]), 0x3);  // converted B slot (both CTAs)
        }
        if (ok) umma_commit_2sm_mc(smem_u32(&bars[3 * S + buf]), 0x3);
      }
    }
  } else if (warp < 2 + EPI_WARPS) {
    // ---- epilogue warps 2..9 (both CTAs): this CTA's 128 rows of the tile
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t acce_leader0 = mapa_shared(smem_u32(&bars[3 * S + 2]), 0);
    const uint32_t acce_leader1 = mapa_shared(smem_u32(&bars[3 * S + 3]), 0);
    int local = 0;
    for (int tile = pair; tile < n_tiles; tile += npairs, ++local) {
      const int buf = local & 1;
      const uint32_t use = (uint32_t)(local >> 1);
      const bool have = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars[3 * S + buf]), use & 1u, args.err,
                                                          DEV_ERR_TIMEOUT_ACCUM) ? 1 : 0) != 0;
      if (!have) break;
      tc_fence_after();
      const int m0 = tile_mb(tile, tiles_m, tiles_n, nfast) * 2 * HALF_ROWS + (int)rank * HALF_ROWS;
      const int n0 = tile_nb(tile, tiles_m, tiles_n, nfast) * BN;
      const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN);
      epilogue_tile<H, EPI>(args, trow, m0 + q * 32, n0, half, sE + (warp - 2) * EPI_STAGE_BYTES);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote_cta(buf ? acce_leader1 : acce_leader0);
    }
  } else {
    // ---- converter warps (both CTAs): raw quantised B rows -> 16-bit MMA tile
    const int r = (warp - 2 - EPI_WARPS) * 32 + lane;  // B row within this CTA's half
    uint32_t it = 0;
    for (int tile = pair; tile < n_tiles; tile += npairs) {
      bool ok = true;
      for (int kb = 0; kb < KB; ++kb, ++it) {
        const int s = it % S, sb = it % SB;
        const uint32_t ph = (it / S) & 1u, phb = (it / SB) & 1u;
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars[2 * S + s]), ph, args.err,
                                               DEV_ERR_TIMEOUT_FULL) ? 1 : 0) != 0 &&
             __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars[3 * S + 4 + sb]), phb ^ 1u, args.err,
                                               DEV_ERR_TIMEOUT_EMPTY) ? 1 : 0) != 0;
        if (!ok) break;
        dequant_row<H, QT>(sR + s * QL::RAW, sB + sb * B2_BYTES, r);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive_remote_cta(mapa_shared(smem_u32(&bars[s]), 0));  // B half ready (leader's stage)
          mbar_arrive(smem_u32(&bars[S + s]));                      // raw stage consumed (local)
        }
      }
      if (!ok) break;
    }
  }

  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 0) tmem_dealloc_2sm(tmem, TMEM_COLS);
}

// ============================================================================
// 2-SM variant with the LayerNorm fused into the A operand: D = xhat * B^T,
// xhat = (X - mean) * rstd per row. X (the f32 residual stream) is
// TMA-loaded into a raw ring of [128 rows x 32 columns] boxes; four converter
// warps per CTA compute xhat -- mean and rstd of each row merged from the
// per-128-column (mean, M2) partials that the GEMM which produced X wrote
// (EPI_RESID_F32 with stats) -- and write the 16-bit, 128-byte-swizzled A
// tile, one row per converter thread; B comes by TMA as in k_gemm_tc2. The
// LayerNorm's gamma and beta are folded into B and the bias when the weights
// are loaded. No normalised copy of X goes to memory.
// Raw boxes are released by the converters as soon as they are in registers;
// the B stage and the converted A slot of k-block `it` share index
// it % LSTAGES and are released together by the MMA's commit.
// Cost: per CTA and k-block the raw f32 rows add 32 KB of TMA writes, 32 KB of
// converter reads and 16 KB of converter writes to shared memory, on top of
// the 64 KB (TMA in, tensor-core reads) that the plain kernel already moves at
// about the port's rate; measured at M=3277, N=3072, K=1024 it runs one
// k-block per ~1.7k cycles against ~0.55k for k_gemm_tc2, with the MMA waiting
// on the converters. It is therefore opt-in in the encoder.
constexpr int LSTAGES = 4;                        // B stages = converted A slots
constexpr int LRSTAGES = 4;                       // raw X boxes (two per k-block)
constexpr int LRAW = HALF_ROWS * 32 * 4;          // one [128 x 32] f32 box
constexpr int LSMEM = LRSTAGES * LRAW + LSTAGES * (B2_BYTES + A2_BYTES) + EPI_WARPS * EPI_STAGE_BYTES + 768 + 1024;

struct LnParams {
  const float* stats;   // [M][K/128][2]
};

template <typename H, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(512, 1)
    k_gemm_tc2ln(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmB, LnParams lp,
                 GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sR = smem;                                 // raw X boxes
  uint8_t* sB = sR + LRSTAGES * LRAW;                 // B stages
  uint8_t* sA = sB + LSTAGES * B2_BYTES;              // converted A slots
  uint8_t* sE = sA + LSTAGES * A2_BYTES;              // epilogue staging
  uint64_t* bars = reinterpret_cast<uint64_t*>(sE + EPI_WARPS * EPI_STAGE_BYTES);
  // bars: [0,S) full (leader: B bytes of both CTAs + both CTAs' converters),
  //       [S,2S) empty (MMA commit: B stage and A slot), [2S,2S+R) raw full,
  //       [2S+R,2S+2R) raw empty (this CTA's converters),
  //       ACC+{0,1} accumulator full, ACC+{2,3} accumulator empty
  constexpr int S = LSTAGES;
  constexpr int R = LRSTAGES;
  constexpr int ACC = 2 * S + 2 * R;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + ACC + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int KB = args.K / BK;
  const int tiles_m = (args.M + 2 * HALF_ROWS - 1) / (2 * HALF_ROWS);
  const int tiles_n = args.N / BN;
  const int n_tiles = tiles_m * tiles_n;
  const bool nfast = args.M > args.N;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmX);
    prefetch_tmap(&tmB);
    for (int i = 0; i < S; ++i) {
      mbar_init(smem_u32(&bars[i]), 1 + 2 * CVT_WARPS);
      mbar_init(smem_u32(&bars[S + i]), 1);
    }
    for (int i = 0; i < R; ++i) {
      mbar_init(smem_u32(&bars[2 * S + i]), 1);
      mbar_init(smem_u32(&bars[2 * S + R + i]), CVT_WARPS);
    }
    mbar_init(smem_u32(&bars[ACC + 0]), 1);
    mbar_init(smem_u32(&bars[ACC + 1]), 1);
    mbar_init(smem_u32(&bars[ACC + 2]), 2 * EPI_WARPS);
    mbar_init(smem_u32(&bars[ACC + 3]), 2 * EPI_WARPS);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0) {
    tmem_alloc_2sm(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish_2sm();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer (both CTAs): this CTA's B half and raw X rows
      uint32_t it = 0;
      bool ok = true;
      for (int tile = pair; tile < n_tiles && ok; tile += npairs) {
        const int m0 = tile_mb(tile, tiles_m, tiles_n, nfast) * 2 * HALF_ROWS + (int)rank * HALF_ROWS;
        const int n0 = tile_nb(tile, tiles_m, tiles_n, nfast) * BN + (int)rank * HALF_ROWS;
        for (int kb = 0; kb < KB && ok; ++kb, ++it) {
          const int s = it % S;
          if (!mbar_wait(smem_u32(&bars[S + s]), ((it / S) & 1u) ^ 1u, args.err, DEV_ERR_TIMEOUT_EMPTY)) {
            ok = false;
            break;
          }
          const uint32_t full_leader = mapa_shared(smem_u32(&bars[s]), 0);
          if (leader) mbar_arrive_expect_tx(smem_u32(&bars[s]), 2 * B2_BYTES);
          tma_load_2d_2sm(smem_u32(sB + s * B2_BYTES), &tmB, full_leader, kb * BK, n0);
          for (int h = 0; h < 2; ++h) {
            const uint32_t q = 2 * it + (uint32_t)h;
            const int r = q % R;
            if (!mbar_wait(smem_u32(&bars[2 * S + R + r]), ((q / R) & 1u) ^ 1u, args.err, DEV_ERR_TIMEOUT_EMPTY)) {
              ok = false;
              break;
            }
            const uint32_t rf = smem_u32(&bars[2 * S + r]);
            mbar_arrive_expect_tx(rf, LRAW);
            tma_load_2d(smem_u32(sR + r * LRAW), &tmX, rf, kb * BK + 32 * h, m0);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---- MMA issuer (leader CTA only)
      constexpr uint32_t idesc = idesc_f16(2 * HALF_ROWS, BN, is_bf16<H>::value ? 1 : 0);
      uint32_t it = 0;
      int local = 0;
      bool ok = true;
      for (int tile = pair; tile < n_tiles && ok; tile += npairs, ++local) {
        const int buf = local & 1;
        const uint32_t use = (uint32_t)(local >> 1);
        if (!mbar_wait(smem_u32(&bars[ACC + 2 + buf]), (use & 1u) ^ 1u, args.err, DEV_ERR_TIMEOUT_ACCUM))
          break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(buf * BN);
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % S;
          if (!mbar_wait(smem_u32(&bars[s]), (it / S) & 1u, args.err, DEV_ERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = smem_desc_sw128(smem_u32(sA + s * A2_BYTES));
          const uint64_t db = smem_desc_sw128(smem_u32(sB + s * B2_BYTES));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16_2sm(acc, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit_2sm_mc(smem_u32(&bars[S + s]), 0x3);  // B stage + A slot free (both CTAs)
        }
        if (ok) umma_commit_2sm_mc(smem_u32(&bars[ACC + buf]), 0x3);
      }
    }
  } else if (warp < 2 + EPI_WARPS) {
    // ---- epilogue warps 2..9 (both CTAs): this CTA's 128 rows of the tile
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t acce_leader0 = mapa_shared(smem_u32(&bars[ACC + 2]), 0);
    const uint32_t acce_leader1 = mapa_shared(smem_u32(&bars[ACC + 3]), 0);
    int local = 0;
    for (int tile = pair; tile < n_tiles; tile += npairs, ++local) {
      const int buf = local & 1;
      const uint32_t use = (uint32_t)(local >> 1);
      const bool have = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars[ACC + buf]), use & 1u, args.err,
                                                          DEV_ERR_TIMEOUT_ACCUM) ? 1 : 0) != 0;
      if (!have) break;
      tc_fence_after();
      const int m0 = tile_mb(tile, tiles_m, tiles_n, nfast) * 2 * HALF_ROWS + (int)rank * HALF_ROWS;
      const int n0 = tile_nb(tile, tiles_m, tiles_n, nfast) * BN;
      const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN);
      epilogue_tile<H, EPI>(args, trow, m0 + q * 32, n0, half, sE + (warp - 2) * EPI_STAGE_BYTES);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote_cta(buf ? acce_leader1 : acce_leader0);
    }
  } else {
    // ---- converter warps (both CTAs): raw X row -> xhat, 16-bit A row
    const int r = (warp - 2 - EPI_WARPS) * 32 + lane;  // A row within this CTA's 128
    const int nchunk = args.K / 128;
    uint32_t it = 0;
    bool ok = true;
    for (int tile = pair; tile < n_tiles && ok; tile += npairs) {
      // mean / rstd of this row (ggml_norm: population variance, eps 1e-5),
      // merged from its equal-size 128-column partials
      const int grow = tile_mb(tile, tiles_m, tiles_n, nfast) * 2 * HALF_ROWS + (int)rank * HALF_ROWS + r;
      float mean = 0.f, rstd = 0.f;
      if (grow < args.M) {
        const float2* st2 = reinterpret_cast<const float2*>(lp.stats) + (size_t)grow * nchunk;
        float m2 = 0.f;
        for (int c0 = 0; c0 < nchunk; c0 += 8) {
          float2 v[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) v[u] = c0 + u < nchunk ? __ldg(st2 + c0 + u) : make_float2(0.f, 0.f);
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int c = c0 + u;
            if (c == 0) {
              mean = v[u].x;
              m2 = v[u].y;
            } else if (c < nchunk) {
              const float dl = v[u].x - mean;
              const float inv = 1.0f / (float)(c + 1);
              mean += dl * inv;
              m2 += v[u].y + dl * dl * (128.0f * (float)c * inv);
            }
          }
        }
        rstd = 1.0f / sqrtf(m2 / (float)args.K + 1e-5f);
      }
      const float nmr = -mean * rstd;  // xhat = fma(x, rstd, nmr)
      // the next tile's row statistics into L1 while this tile streams
      {
        const int nrow = tile_mb(tile + npairs, tiles_m, tiles_n, nfast) * 2 * HALF_ROWS + (int)rank * HALF_ROWS + r;
        if (tile + npairs < n_tiles && nrow < args.M) {
          const char* p = reinterpret_cast<const char*>(lp.stats + (size_t)nrow * nchunk * 2);
          for (int o = 0; o < nchunk * 8; o += 128) asm volatile("prefetch.global.L1 [%0];" ::"l"(p + o));
        }
      }
      for (int kb = 0; kb < KB; ++kb, ++it) {
        const int s = it % S;
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars[S + s]), ((it / S) & 1u) ^ 1u, args.err,
                                               DEV_ERR_TIMEOUT_EMPTY) ? 1 : 0) != 0;
        if (!ok) break;
        uint8_t* dst = sA + s * A2_BYTES + r * 128;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t qb = 2 * it + (uint32_t)h;
          const int rb = qb % R;
          ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars[2 * S + rb]), (qb / R) & 1u, args.err,
                                                 DEV_ERR_TIMEOUT_FULL) ? 1 : 0) != 0;
          if (!ok) break;
          // row r of the box: 16-byte chunk c (columns 4c..4c+3) at (c ^ (r & 7))
          const uint8_t* raw = sR + rb * LRAW + r * 128;
          float4 x[8];
#pragma unroll
          for (int c = 0; c < 8; ++c) x[c] = *reinterpret_cast<const float4*>(raw + ((c ^ (r & 7)) << 4));
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&bars[2 * S + R + rb]));  // box consumed
#pragma unroll
          for (int c2 = 0; c2 < 4; ++c2) {
            const float4 a = x[2 * c2], b = x[2 * c2 + 1];
            // 16-byte chunk (4h + c2) of the 128-byte A row (8 halves)
            *reinterpret_cast<uint4*>(dst + (((4 * h + c2) ^ (r & 7)) << 4)) =
                make_uint4(pack2<H>(fmaf(a.x, rstd, nmr), fmaf(a.y, rstd, nmr)),
                           pack2<H>(fmaf(a.z, rstd, nmr), fmaf(a.w, rstd, nmr)),
                           pack2<H>(fmaf(b.x, rstd, nmr), fmaf(b.y, rstd, nmr)),
                           pack2<H>(fmaf(b.z, rstd, nmr), fmaf(b.w, rstd, nmr)));
          }
        }
        if (!ok) break;
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote_cta(mapa_shared(smem_u32(&bars[s]), 0));  // A half ready
      }
    }
  }

  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 0) tmem_dealloc_2sm(tmem, TMEM_COLS);
}

}  // namespace

// ------------------------------------------------------------------ host side

static PFN_encodeTiled_t g_encode = nullptr;

static bool get_encode_fn() {
  if (g_encode) return true;
  cudaDriverEntryPointQueryResult q;
  void* fn = nullptr;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !fn)
    return false;
  g_encode = reinterpret_cast<PFN_encodeTiled_t>(fn);
  return true;
}

bool make_tmap_kmajor(CUtensorMap* map, const void* base, int rows, int K, int ld_elems,
                      int box_rows, bool bf16) {
  if (!get_encode_fn()) return false;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld_elems * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = g_encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        2, const_cast<void*>(base), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// CTA pairs of a 2-SM kernel that fit on the device at once (its shared
// memory and thread count; the SM count / 2 if the occupancy query fails).
template <typename K>
static cudaError_t cluster_pairs(K kern, int smem, int threads, int dev, int& n) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute at;
  at.id = cudaLaunchAttributeClusterDimension;
  at.val.clusterDim.x = 2; at.val.clusterDim.y = 1; at.val.clusterDim.z = 1;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    n = sms / 2;
  }
  return cudaSuccess;
}

template <typename H, int EPI>
static cudaError_t launch_t2(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                             cudaStream_t st) {
  auto kern = k_gemm_tc2<H, EPI, false>;
  auto kern_sk = k_gemm_tc2<H, EPI, true>;
  static PerDevice once;
  int mp = 0;
  const cudaError_t ae = per_device(once, &mp, [&](int dev, int& n) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2_BYTES);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kern_sk, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2_BYTES);
    if (e != cudaSuccess) return e;
    return cluster_pairs(kern, SMEM2_BYTES, THREADS, dev, n);
  });
  if (ae != cudaSuccess) return ae;
  const int n_tiles = (a.N / BN) * ((a.M + 2 * HALF_ROWS - 1) / (2 * HALF_ROWS));
  int pairs = n_tiles < mp ? n_tiles : mp;
  if (a.sk_ws && a.sk_flags && mp <= a.sk_pairs && gemm_splitk_enabled()) {
    // stream-K when whole tiles would leave more than 15 % of the last
    // wave's pairs idle, and every pair still gets >= 4 k-blocks
    const int KB = a.K / BK;
    const int waves = (n_tiles + mp - 1) / mp;
    if ((double)n_tiles < 0.85 * (double)waves * mp && (long long)n_tiles * KB >= 4LL * mp)
      return launch_pdl(kern_sk, dim3(2 * mp), dim3(THREADS), SMEM2_BYTES, st, ta, tb, a);
  }
  return launch_pdl(kern, dim3(2 * pairs), dim3(THREADS), SMEM2_BYTES, st, ta, tb, a);
}

// 256 x 128 pair tiles (k_gemm_tc2<.., TBN = 128>); tb's box is 64 rows.
template <typename H, int EPI>
static cudaError_t launch_t2n(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int n_tiles,
                              cudaStream_t st) {
  auto kern = k_gemm_tc2<H, EPI, false, 128>;
  static PerDevice once;
  int unused = 0;
  const cudaError_t ae = per_device(once, &unused, [&](int, int&) {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2_BYTES);
  });
  if (ae != cudaSuccess) return ae;
  return launch_pdl(kern, dim3(2 * n_tiles), dim3(THREADS), SMEM2_BYTES, st, ta, tb, a);
}

// SM pairs of the current device (cached per device)
static int device_sm_pairs() {
  static PerDevice pd;
  int v = 0;
  if (per_device(pd, &v, [](int dev, int& n) {
        int sms = 0;
        const cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        n = sms / 2;
        return e;
      }) != cudaSuccess)
    return 0;
  return v;
}

template <typename H, int EPI>
static cudaError_t launch_t(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                            cudaStream_t st) {
  auto kern = k_gemm_tc<H, EPI>;
  static PerDevice once;
  int n_sm = 0;
  const cudaError_t ae = per_device(once, &n_sm, [&](int dev, int& n) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    return cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  });
  if (ae != cudaSuccess) return ae;
  const int n_tiles = (a.N / BN) * ((a.M + BM - 1) / BM);
  const int grid = n_tiles < n_sm ? n_tiles : n_sm;
  return launch_pdl(kern, dim3(grid), dim3(THREADS), SMEM_BYTES, st, ta, tb, a);
}

// Generic 2-D tensor map (u8 or f32 elements) for the quantised operands.
static bool make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int esize, uint64_t inner,
                         uint64_t outer, uint64_t stride_bytes, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle sw) {
  if (!get_encode_fn()) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  (void)esize;
  return g_encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename H, int EPI, int QT>
static cudaError_t launch_q(const CUtensorMap& ta, const CUtensorMap& tq, const CUtensorMap& t0,
                            const CUtensorMap& t1, const GemmArgs& a, cudaStream_t st) {
  auto kern = k_gemm_tc2q<H, EPI, QT>;
  constexpr int smem = QLayout<QT>::SMEM;
  static PerDevice once;
  int mp = 0;
  const cudaError_t ae = per_device(once, &mp, [&](int dev, int& n) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    return cluster_pairs(kern, smem, QTHREADS, dev, n);
  });
  if (ae != cudaSuccess) return ae;
  const int n_tiles = (a.N / BN) * ((a.M + 2 * HALF_ROWS - 1) / (2 * HALF_ROWS));
  const int pairs = n_tiles < mp ? n_tiles : mp;
  return launch_pdl(kern, dim3(2 * pairs), dim3(QTHREADS), smem, st, ta, tq, t0, t1, a);
}

cudaError_t gemm_launch_q(const void* A, int lda, const QuantB& B, bool bf16, const GemmArgs& args,
                          cudaStream_t st) {
  if (args.M <= 0) return cudaSuccess;
  if (B.type != QT_Q8_0 && B.type != QT_Q4_K) return cudaErrorInvalidValue;
  if (args.split_k || args.ofmt != OUT_H) return cudaErrorInvalidValue;
  if (args.N % BN != 0 || args.K % BK != 0 || args.K <= 0 || (lda % 8) != 0 || !B.q || !B.s0 ||
      (B.type == QT_Q4_K && !B.s1) || (reinterpret_cast<uintptr_t>(A) & 15) ||
      (reinterpret_cast<uintptr_t>(B.q) & 15) || (reinterpret_cast<uintptr_t>(B.s0) & 15) ||
      (reinterpret_cast<uintptr_t>(B.s1) & 15) || (reinterpret_cast<uintptr_t>(args.bias) & 15) ||
      (reinterpret_cast<uintptr_t>(args.out) & 15) || (args.ldo % 8) != 0)
    return cudaErrorInvalidValue;
  CUtensorMap ta, tq, t0, t1;
  if (!make_tmap_kmajor(&ta, A, args.M, args.K, lda, HALF_ROWS, bf16)) return cudaErrorInvalidValue;
  const uint64_t N = (uint64_t)args.N, K = (uint64_t)args.K;
  if (B.type == QT_Q8_0) {
    if (!make_tmap_2d(&tq, B.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, K, 64, HALF_ROWS, CU_TENSOR_MAP_SWIZZLE_64B))
      return cudaErrorInvalidValue;
  } else {
    if (!make_tmap_2d(&tq, B.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K / 2, N, K / 2, 32, HALF_ROWS,
                      CU_TENSOR_MAP_SWIZZLE_32B))
      return cudaErrorInvalidValue;
  }
  if (!make_tmap_2d(&t0, B.s0, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, K / 32, N * 4, HALF_ROWS, 2,
                    CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  t1 = t0;
  if (B.type == QT_Q4_K &&
      !make_tmap_2d(&t1, B.s1, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, K / 32, N * 4, HALF_ROWS, 2,
                    CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  const bool q8 = B.type == QT_Q8_0;
  switch (args.epi) {
#define PKC_GEMMQ_CASE(E)                                                                                     \
  case E:                                                                                                     \
    if (q8) return bf16 ? launch_q<__nv_bfloat16, E, QT_Q8_0>(ta, tq, t0, t1, args, st)                       \
                    : launch_q<__half, E, QT_Q8_0>(ta, tq, t0, t1, args, st);                                 \
    return bf16 ? launch_q<__nv_bfloat16, E, QT_Q4_K>(ta, tq, t0, t1, args, st)                               \
                : launch_q<__half, E, QT_Q4_K>(ta, tq, t0, t1, args, st);
    PKC_GEMMQ_CASE(EPI_STORE_H)
    PKC_GEMMQ_CASE(EPI_RESID_F32)
#undef PKC_GEMMQ_CASE
    default:
      return cudaErrorInvalidValue;
  }
}

template <typename H, int EPI>
static cudaError_t launch_ln(const CUtensorMap& tx, const CUtensorMap& tb, const LnParams& lp, const GemmArgs& a,
                             cudaStream_t st) {
  auto kern = k_gemm_tc2ln<H, EPI>;
  static PerDevice once;
  int mp = 0;
  const cudaError_t ae = per_device(once, &mp, [&](int dev, int& n) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, LSMEM);
    if (e != cudaSuccess) return e;
    return cluster_pairs(kern, LSMEM, QTHREADS, dev, n);
  });
  if (ae != cudaSuccess) return ae;
  const int n_tiles = (a.N / BN) * ((a.M + 2 * HALF_ROWS - 1) / (2 * HALF_ROWS));
  const int pairs = n_tiles < mp ? n_tiles : mp;
  return launch_pdl(kern, dim3(2 * pairs), dim3(QTHREADS), LSMEM, st, tx, tb, lp, a);
}

cudaError_t gemm_launch_ln(const LnA& A, const void* B, int ldb, bool bf16, const GemmArgs& args,
                           cudaStream_t st) {
  if (args.M <= 0) return cudaSuccess;
  if (args.split_k || args.ofmt != OUT_H) return cudaErrorInvalidValue;
  if (args.N % BN != 0 || args.K % 128 != 0 || args.K <= 0 || (A.ldx % 4) != 0 || (ldb % 8) != 0 || !A.x ||
      !A.stats || (reinterpret_cast<uintptr_t>(A.x) & 15) || (reinterpret_cast<uintptr_t>(A.stats) & 7) || (reinterpret_cast<uintptr_t>(B) & 15) ||
      (reinterpret_cast<uintptr_t>(args.bias) & 15) || (reinterpret_cast<uintptr_t>(args.out) & 15) ||
      (args.ldo % 8) != 0)
    return cudaErrorInvalidValue;
  CUtensorMap tx, tb;
  if (!make_tmap_2d(&tx, A.x, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)args.K, (uint64_t)args.M,
                    (uint64_t)A.ldx * 4, 32, HALF_ROWS, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (!make_tmap_kmajor(&tb, B, args.N, args.K, ldb, HALF_ROWS, bf16)) return cudaErrorInvalidValue;
  const LnParams lp{A.stats};
  switch (args.epi) {
#define PKC_GEMMLN_CASE(E)                                                                                   \
  case E:                                                                                                    \
    return bf16 ? launch_ln<__nv_bfloat16, E>(tx, tb, lp, args, st) : launch_ln<__half, E>(tx, tb, lp, args, st);
    PKC_GEMMLN_CASE(EPI_STORE_H)
    PKC_GEMMLN_CASE(EPI_GLU_H)
#undef PKC_GEMMLN_CASE
    default:
      return cudaErrorInvalidValue;
  }
}

size_t gemm_sk_ws_bytes(int pairs) { return (size_t)pairs * 2 * EPI_WARPS * SK_SLOT_FLOATS * sizeof(float); }
int gemm_sk_flag_count(int pairs) { return pairs * 2 * EPI_WARPS; }

// PKC_GEMM_SPLITK=1: let the 2-SM kernel run the stream-K schedule. Off by
// default: at the encoder's shapes the f32 partial sums that every pair
// spills and the finishers read back (~19 MB through L2 at the same moment,
// ~3.5 us each way, measured by per-pair timestamps at M = 3282, N = 1024,
// K = 1024) cost more than the k-blocks the balanced ranges save, and
// whole tiles keep each row's result independent of the batch.
bool gemm_splitk_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("PKC_GEMM_SPLITK");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

// PKC_GEMM_1SM=1 forces the 1-SM kernel (for A/B comparisons)
// PKC_GEMM_NARROW=0: never the 256 x 128 pair tiles
static bool gemm_narrow_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("PKC_GEMM_NARROW");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

bool gemm_2sm_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("PKC_GEMM_1SM");
    v = (e && e[0] == '1') ? 0 : 1;
  }
  return v == 1;
}

int gemm_tile_n() { return BN; }
int gemm_tile_k() { return BK; }
int gemm_tile_m() { return BM; }

// ---------------------------------------------------------------- skinny GEMM
// M <= SKINNY_M rows (the streaming encoder's chunks, a few frames): a
// 128-row tcgen05 tile would leave the tensor cores almost idle and walk K
// through one CTA per 256 columns, so instead every SM streams a slice of the
// weight once: one warp per weight row (per value/gate row pair for GLU),
// 16-byte loads along K, the M rows of A staged in shared memory, f32
// accumulation, a warp reduction and the same epilogues as the tcgen05 GEMM.
constexpr int SKINNY_M = 16;
constexpr int SKINNY_THREADS = 256;
constexpr int SKINNY_WARPS = SKINNY_THREADS / 32;
constexpr int SKINNY_PRE = 8;  // 16-byte weight chunks per lane fetched before the dependency wait (K <= 2048)

template <typename H>
__device__ __forceinline__ void h8_to_f(const uint4& v, float (&f)[8]) {
  const H* h = reinterpret_cast<const H*>(&v);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if constexpr (std::is_same<H, __half>::value) f[i] = __half2float(h[i]);
    else f[i] = __bfloat162float(h[i]);
  }
}

template <typename H, int EPI>
__global__ void __launch_bounds__(SKINNY_THREADS) k_gemm_skinny(const H* __restrict__ A, int lda,
                                                                const H* __restrict__ B, int ldb, GemmArgs args) {
  extern __shared__ uint4 sk_a[];  // A rows [M][K / 8] chunks of 8
  constexpr bool PAIRED = EPI == EPI_GLU_H;
  const int M = args.M, k8 = args.K / 8;
  const int units = PAIRED ? args.N / 2 : args.N;
  // the weight does not depend on the kernel before this one: the warp's first
  // row (first SKINNY_PRE chunks per lane) is fetched before waiting for it
  const int u_first = blockIdx.x * SKINNY_WARPS + (threadIdx.x >> 5);
  uint4 pa[SKINNY_PRE], pg[SKINNY_PRE];
  float pb = 0.f, pbg = 0.f;  // that row's bias (and gate bias)
  if (u_first < units) {
    const int na = PAIRED ? (u_first / (BN / 2)) * BN + u_first % (BN / 2) : u_first;
    const uint4* wa = reinterpret_cast<const uint4*>(B + (size_t)na * ldb);
    const uint4* wg = reinterpret_cast<const uint4*>(B + (size_t)(na + BN / 2) * ldb);
#pragma unroll
    for (int j = 0; j < SKINNY_PRE; ++j) {
      const int c = (threadIdx.x & 31) + 32 * j;
      if (c < k8) {
        pa[j] = __ldg(wa + c);
        if constexpr (PAIRED) pg[j] = __ldg(wg + c);
      }
    }
    if (args.bias) {
      pb = __ldg(args.bias + na);
      if constexpr (PAIRED) pbg = __ldg(args.bias + na + BN / 2);
    }
  }
  // the LayerNorm prologue's gamma / beta (128-byte lines) on their way to L1
  if (args.ln_x)
    for (int i = threadIdx.x; i < args.K / 32; i += SKINNY_THREADS) {
      asm volatile("prefetch.global.L1 [%0];" ::"l"(args.ln_g + 32 * i));
      asm volatile("prefetch.global.L1 [%0];" ::"l"(args.ln_b + 32 * i));
    }
  pdl_wait();
  if (args.ln_x) {
    // LayerNorm of row m by warp m % 8: mean, then the mean square deviation
    // (two passes, as ggml_norm), then the affine, rounded into the staging
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int m = warp; m < M; m += SKINNY_WARPS) {
      const float* xr = args.ln_x + (size_t)m * args.ln_ldx;
      float s = 0.f;
      for (int k = lane * 4; k < args.K; k += 128) {
        const float4 v = *reinterpret_cast<const float4*>(xr + k);
        s += (v.x + v.y) + (v.z + v.w);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      const float mean = s / (float)args.K;
      float q = 0.f;
      for (int k = lane * 4; k < args.K; k += 128) {
        const float4 v = *reinterpret_cast<const float4*>(xr + k);
        const float a0 = v.x - mean, a1 = v.y - mean, a2 = v.z - mean, a3 = v.w - mean;
        q += (a0 * a0 + a1 * a1) + (a2 * a2 + a3 * a3);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
      const float rstd = rsqrtf(q / (float)args.K + 1e-5f);
      for (int c = lane; c < k8; c += 32) {
        const float4 v0 = *reinterpret_cast<const float4*>(xr + 8 * c);
        const float4 v1 = *reinterpret_cast<const float4*>(xr + 8 * c + 4);
        const float4 g0 = *reinterpret_cast<const float4*>(args.ln_g + 8 * c);
        const float4 g1 = *reinterpret_cast<const float4*>(args.ln_g + 8 * c + 4);
        const float4 b0 = *reinterpret_cast<const float4*>(args.ln_b + 8 * c);
        const float4 b1 = *reinterpret_cast<const float4*>(args.ln_b + 8 * c + 4);
        uint4 o;
        o.x = pack2<H>((v0.x - mean) * rstd * g0.x + b0.x, (v0.y - mean) * rstd * g0.y + b0.y);
        o.y = pack2<H>((v0.z - mean) * rstd * g0.z + b0.z, (v0.w - mean) * rstd * g0.w + b0.w);
        o.z = pack2<H>((v1.x - mean) * rstd * g1.x + b1.x, (v1.y - mean) * rstd * g1.y + b1.y);
        o.w = pack2<H>((v1.z - mean) * rstd * g1.z + b1.z, (v1.w - mean) * rstd * g1.w + b1.w);
        sk_a[m * k8 + c] = o;
      }
    }
  } else {
    for (int e = threadIdx.x; e < M * k8; e += SKINNY_THREADS) {
      const int m = e / k8, c = e - m * k8;
      sk_a[e] = __ldg(reinterpret_cast<const uint4*>(A + (size_t)m * lda) + c);
    }
  }
  __syncthreads();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  for (int u = u_first; u < units; u += gridDim.x * SKINNY_WARPS) {
    // GLU: value row blk * BN + c and its gate row BN / 2 later, output column u
    const int na = PAIRED ? (u / (BN / 2)) * BN + u % (BN / 2) : u;
    const int ng = na + BN / 2;
    const uint4* wa = reinterpret_cast<const uint4*>(B + (size_t)na * ldb);
    const uint4* wg = reinterpret_cast<const uint4*>(B + (size_t)(PAIRED ? ng : na) * ldb);
    // the residual this lane updates, in flight during the dot products
    float resid = 0.f;
    if constexpr (EPI == EPI_RESID_F32)
      if (lane < M) resid = reinterpret_cast<const float*>(args.out)[(size_t)lane * args.ldo + u];
    float acc[SKINNY_M], accg[SKINNY_M];
#pragma unroll
    for (int m = 0; m < SKINNY_M; ++m) acc[m] = accg[m] = 0.f;
    auto dot_chunk = [&](const uint4& wav, const uint4& wgv, int c) {
      float fa[8], fg[8];
      h8_to_f<H>(wav, fa);
      if constexpr (PAIRED) h8_to_f<H>(wgv, fg);
#pragma unroll
      for (int m = 0; m < SKINNY_M; ++m) {
        if (m < M) {
          float fx[8];
          h8_to_f<H>(sk_a[m * k8 + c], fx);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            acc[m] = fmaf(fa[i], fx[i], acc[m]);
            if constexpr (PAIRED) accg[m] = fmaf(fg[i], fx[i], accg[m]);
          }
        }
      }
    };
    const bool first = u == u_first;
#pragma unroll
    for (int j = 0; j < SKINNY_PRE; ++j) {
      const int c = lane + 32 * j;
      if (c < k8) {
        const uint4 va = first ? pa[j] : __ldg(wa + c);
        uint4 vg = va;
        if constexpr (PAIRED) vg = first ? pg[j] : __ldg(wg + c);
        dot_chunk(va, vg, c);
      }
    }
#pragma unroll 2
    for (int c = lane + 32 * SKINNY_PRE; c < k8; c += 32) {
      const uint4 va = __ldg(wa + c);
      uint4 vg = va;
      if constexpr (PAIRED) vg = __ldg(wg + c);
      dot_chunk(va, vg, c);
    }
    // row m's sum ends in lane m
    float mine = 0.f, mineg = 0.f;
#pragma unroll
    for (int m = 0; m < SKINNY_M; ++m) {
      if (m < M) {
        float v = acc[m], g = accg[m];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          v += __shfl_xor_sync(0xffffffffu, v, o);
          if constexpr (PAIRED) g += __shfl_xor_sync(0xffffffffu, g, o);
        }
        if (lane == m) {
          mine = v;
          mineg = g;
        }
      }
    }
    if (lane < M) {
      const size_t ro = (size_t)lane * args.ldo + u;
      const float b = args.bias ? (first ? pb : args.bias[na]) : 0.f;
      if constexpr (EPI == EPI_RESID_F32) {
        reinterpret_cast<float*>(args.out)[ro] = resid + args.alpha * (mine + b);
      } else if constexpr (EPI == EPI_STORE_F32) {
        reinterpret_cast<float*>(args.out)[ro] = args.alpha * (mine + b);
      } else if constexpr (EPI == EPI_GLU_H) {
        const float bg = args.bias ? (first ? pbg : args.bias[ng]) : 0.f;
        const float v = (mine + b) * sigmoidf_(mineg + bg);
        reinterpret_cast<H*>(args.out)[ro] = std::is_same<H, __half>::value ? H(__float2half_rn(v)) : H(__float2bfloat16_rn(v));
      } else {
        float v = mine + b;
        if (args.act == ACT_SILU) v = siluf_(v);
        else if (args.act == ACT_RELU) v = fmaxf(v, 0.f);
        reinterpret_cast<H*>(args.out)[ro] = std::is_same<H, __half>::value ? H(__float2half_rn(v)) : H(__float2bfloat16_rn(v));
      }
    }
  }
}

bool gemm_skinny_enabled() {
  static const bool on = [] {
    const char* e = getenv("PKC_GEMM_SKINNY");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <typename H, int EPI>
cudaError_t launch_skinny(const void* A, int lda, const void* B, int ldb, const GemmArgs& args, cudaStream_t st) {
  static PerDevice once;
  int sms = 0;
  const cudaError_t ae = per_device(once, &sms, [](int dev, int& n) {
    return cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  });
  if (ae != cudaSuccess) return ae;
  const size_t smem = (size_t)args.M * args.K * sizeof(H);
  const int units = EPI == EPI_GLU_H ? args.N / 2 : args.N;
  const int grid = std::max(1, std::min((units + SKINNY_WARPS - 1) / SKINNY_WARPS, 2 * sms));
  cudaError_t e = cudaFuncSetAttribute(k_gemm_skinny<H, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(k_gemm_skinny<H, EPI>, dim3(grid), dim3(SKINNY_THREADS), smem, st, static_cast<const H*>(A), lda,
                    static_cast<const H*>(B), ldb, args);
}

cudaError_t gemm_launch(const void* A, int lda, const void* B, int ldb, bool bf16,
                        const GemmArgs& args, cudaStream_t st) {
  if (args.M <= 0) return cudaSuccess;
  auto al16 = [](const void* p) { return !(reinterpret_cast<uintptr_t>(p) & 15); };
  const bool skinny = args.skinny && !args.split_k && args.ofmt == OUT_H && args.M <= SKINNY_M && !args.stats &&
                      args.N % BN == 0 && args.K % 8 == 0 &&
                      args.K <= 4096 && lda % 8 == 0 && ldb % 8 == 0 && (args.ln_x || al16(A)) && al16(B) &&
                      args.epi != EPI_POWER_F32 && gemm_skinny_enabled();
  // the LayerNorm prologue exists on the skinny kernel only
  if (args.ln_x && !(skinny && args.ln_ldx % 4 == 0 && al16(args.ln_x) && al16(args.ln_g) && al16(args.ln_b)))
    return cudaErrorInvalidValue;
  if (skinny) {
    switch (args.epi) {
#define PKC_SKINNY_CASE(E) \
  case E:                  \
    return bf16 ? launch_skinny<__nv_bfloat16, E>(A, lda, B, ldb, args, st) : launch_skinny<__half, E>(A, lda, B, ldb, args, st);
      PKC_SKINNY_CASE(EPI_STORE_H)
      PKC_SKINNY_CASE(EPI_RESID_F32)
      PKC_SKINNY_CASE(EPI_STORE_F32)
      PKC_SKINNY_CASE(EPI_GLU_H)
#undef PKC_SKINNY_CASE
      default:
        break;
    }
  }
  if (args.N % BN != 0 || args.K % BK != 0 || args.K <= 0 || (lda % 8) != 0 || (ldb % 8) != 0 ||
      (reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15) ||
      (reinterpret_cast<uintptr_t>(args.bias) & 15) || (reinterpret_cast<uintptr_t>(args.out) & 15) ||
      (args.ldo % 8) != 0)
    return cudaErrorInvalidValue;
  // split-f16 operands: K = 3 Ks k-steps over [hi | lo] rows of width 2 Ks
  if (args.split_k && (bf16 || args.split_k % BK != 0 || args.K != 3 * args.split_k || lda < 2 * args.split_k ||
                       ldb < 2 * args.split_k))
    return cudaErrorInvalidValue;
  if (args.ofmt == OUT_SPLIT && (bf16 || args.split_ld <= 0 || args.split_ld % 4 != 0)) return cudaErrorInvalidValue;
  const int kmap = args.split_k ? 2 * args.split_k : args.K;
  // 2-SM tiles once there are at least two 128-row blocks of A
  const bool two_sm = args.M > BM && gemm_2sm_enabled();
  const int box = two_sm ? HALF_ROWS : 0;
  // 256 x 128 pair tiles when the 256-wide ones would fill at most half of
  // the SM pairs (twice the tiles at about 0.8 of the per-tile rate: their
  // shared-memory traffic per MMA is higher), for the unpaired epilogues
  // without row statistics. A row's sums run in the same order either way.
  bool narrow = false;
  int n_narrow = 0;
  if (two_sm && gemm_narrow_enabled() && !gemm_splitk_enabled() && !args.stats && !args.split_k &&
      args.N % 128 == 0 && (args.epi == EPI_STORE_H || args.epi == EPI_RESID_F32 || args.epi == EPI_STORE_F32)) {
    const long long rows = (args.M + 2 * HALF_ROWS - 1) / (2 * HALF_ROWS);
    const long long t256 = (long long)(args.N / BN) * rows;
    const int pairs = device_sm_pairs();
    narrow = pairs > 0 && 2 * t256 <= pairs;
    n_narrow = (int)(rows * (args.N / 128));
  }
  CUtensorMap ta, tb;
  if (!make_tmap_kmajor(&ta, A, args.M, kmap, lda, two_sm ? box : BM, bf16)) return cudaErrorInvalidValue;
  if (!make_tmap_kmajor(&tb, B, args.N, kmap, ldb, narrow ? 64 : two_sm ? box : BN, bf16)) return cudaErrorInvalidValue;
  if (narrow) {
    switch (args.epi) {
#define PKC_GEMM_NARROW(E) \
  case E:                  \
    return bf16 ? launch_t2n<__nv_bfloat16, E>(ta, tb, args, n_narrow, st) : launch_t2n<__half, E>(ta, tb, args, n_narrow, st);
      PKC_GEMM_NARROW(EPI_STORE_H)
      PKC_GEMM_NARROW(EPI_RESID_F32)
      PKC_GEMM_NARROW(EPI_STORE_F32)
#undef PKC_GEMM_NARROW
      default:
        return cudaErrorInvalidValue;
    }
  }
  switch (args.epi) {
#define PKC_GEMM_CASE(E)                                                                   \
  case E:                                                                                  \
    if (two_sm)                                                                            \
      return bf16 ? launch_t2<__nv_bfloat16, E>(ta, tb, args, st) : launch_t2<__half, E>(ta, tb, args, st); \
    return bf16 ? launch_t<__nv_bfloat16, E>(ta, tb, args, st) : launch_t<__half, E>(ta, tb, args, st);
    PKC_GEMM_CASE(EPI_STORE_H)
    PKC_GEMM_CASE(EPI_RESID_F32)
    PKC_GEMM_CASE(EPI_STORE_F32)
    PKC_GEMM_CASE(EPI_GLU_H)
    PKC_GEMM_CASE(EPI_POWER_F32)
#undef PKC_GEMM_CASE
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace pkc
