// Host interface of the tcgen05 GEMM (see gemm.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

namespace pkc {

enum EpiKind : int {
  EPI_STORE_H = 0,
  EPI_RESID_F32 = 1,
  EPI_STORE_F32 = 2,
  EPI_GLU_H = 3,
  EPI_POWER_F32 = 4,
};
enum ActKind : int { ACT_NONE = 0, ACT_SILU = 1, ACT_RELU = 2 };
// Output form of EPI_STORE_H / EPI_GLU_H: the operand type (OUT_H), f32, or
// the split-f16 pair of the f32-accurate mode (OUT_SPLIT: hi = f16(v) at the
// column, lo = f16(v - hi) at the column + split_ld; f16 operands only).
enum OutFmt : int { OUT_H = 0, OUT_F32 = 1, OUT_SPLIT = 2 };

struct GemmArgs {
  int M, N, K;
  int epi;            // EpiKind
  int act;            // ActKind, EPI_STORE_H only
  float alpha;        // RESID_F32 / STORE_F32 scale
  const float* bias;  // [N] (GEMM column order) or nullptr
  void* out;          // output base (h or f32 per epilogue)
  int ldo;            // output row stride in elements
  int* err;           // device error word
  // EPI_RESID_F32 only, may be null: per-row statistics of the updated rows,
  // (mean, M2 = sum of squared deviations) of every 128-column chunk, f32
  // [M][N/128][2] -- what a LayerNorm of those rows needs, merged by the
  // consumer (gemm_launch_ln)
  float* stats;
  // Stream-K workspace (may be null: whole tiles only). With it, the 2-SM
  // kernel may split tiles along K across CTA pairs when whole tiles would
  // leave part of the last wave idle: sk_ws >= gemm_sk_ws_bytes(sk_pairs)
  // bytes, sk_flags >= gemm_sk_flag_count(sk_pairs) ints, zero when the
  // launch starts (the kernel leaves them zero). One workspace per stream.
  float* sk_ws;
  int* sk_flags;
  int sk_pairs;       // CTA pairs the workspace has room for
  // nonzero: M <= 16 may run the CUDA-core skinny kernel (16-bit weights, no
  // stats) instead of a 128-row tcgen05 tile. Its f32 sums run in another
  // order, so callers whose output must not depend on the batch composition
  // (the offline encoder) leave it 0.
  int skinny;
  // skinny kernel only: when ln_x is set, A is LayerNorm(ln_x rows) * ln_g +
  // ln_b (ggml_norm, eps 1e-5) rounded to the operand type, computed while
  // the rows are staged (ln_x f32 [M, K], row stride ln_ldx)
  const float* ln_x;
  int ln_ldx;
  const float* ln_g;
  const float* ln_b;
  // f32-accurate mode: split-f16 operands A [M, 2 Ks] = [A_hi | A_lo] and
  // B [N, 2 Ks] = [B_hi | B_lo] (f16, K-major, row strides lda / ldb); the
  // kernel accumulates A_hi B_hi^T + A_hi B_lo^T + A_lo B_hi^T, i.e. K =
  // 3 Ks k-steps whose operand columns are remapped per pass (a product
  // carries ~22 significant bits; A_lo B_lo is below f32 rounding). 0: plain.
  int split_k;
  int ofmt;       // OutFmt (EPI_STORE_H / EPI_GLU_H)
  int split_ld;   // OUT_SPLIT: column offset of the lo half in the output rows
};

// Stream-K workspace sizes for `pairs` CTA pairs (a device's SMs / 2).
size_t gemm_sk_ws_bytes(int pairs);
int gemm_sk_flag_count(int pairs);

typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                      const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                      const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                      CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Encode a 2-D K-major tensor map (inner dim K, outer dim rows) with 128-byte
// swizzle and a [64 x box_rows] box.
bool make_tmap_kmajor(CUtensorMap* map, const void* base, int rows, int K, int ld_elems,
                      int box_rows, bool bf16);

// D[M,N] = A[M,K] * B[N,K]^T with the epilogue in args. A and B hold f16
// (bf16 == false) or bf16 elements with row strides lda / ldb (elements).
// Requires N % 256 == 0, K % 64 == 0, 16-byte aligned bases and strides.
// B and args.bias are weights: the skinny kernel reads them before waiting
// for the previous kernel in the stream (programmatic dependent launch),
// which must not write them; A, the residual and the output wait for it.
cudaError_t gemm_launch(const void* A, int lda, const void* B, int ldb, bool bf16,
                        const GemmArgs& args, cudaStream_t st);

// Weights kept in their GGUF block-quantised form (repacked for TMA) and
// dequantised inside the GEMM, between the TMA stage and the MMA:
//   Q8_0: q int8 [N][K] (row stride K bytes), s0 = block scale d, f32 [K/32][N]
//   Q4_K: q nibbles u8 [N][K/2] (byte j of a row: value 2j in the low nibble,
//         2j+1 in the high one), s0 = d*sc and s1 = dmin*m of each 32-value
//         sub-block, f32 [K/32][N]; value = s0*q - s1
enum QuantType : int { QT_NONE = 0, QT_Q8_0 = 1, QT_Q4_K = 2 };
struct QuantB {
  int type;
  const void* q;
  const float* s0;
  const float* s1;
};
// D[M,N] = A[M,K] * dequant(B)[N,K]^T; K % 64 == 0, N % 256 == 0.
cudaError_t gemm_launch_q(const void* A, int lda, const QuantB& B, bool bf16, const GemmArgs& args,
                          cudaStream_t st);

// D[M,N] = xhat[M,K] * B[N,K]^T with xhat = (X - mean) * rstd per row
// (ggml_norm: population variance, eps 1e-5), computed while A is staged for
// the MMA: X f32 [M, K] (row stride ldx), stats from the EPI_RESID_F32 GEMM
// that produced X. The LayerNorm's gamma / beta are expected folded into B
// (columns scaled by gamma) and the bias (+ B * beta). Dense B only.
struct LnA {
  const float* x;
  int ldx;
  const float* stats;  // [M][K/128][2]
};
cudaError_t gemm_launch_ln(const LnA& A, const void* B, int ldb, bool bf16, const GemmArgs& args,
                           cudaStream_t st);

int gemm_tile_m();
bool gemm_2sm_enabled();
// true when PKC_GEMM_SPLITK=1 (stream-K schedule allowed; whole tiles otherwise)
bool gemm_splitk_enabled();
int gemm_tile_n();
int gemm_tile_k();

}  // namespace pkc
