// Host interface of the non-GEMM kernels (mel front end, subsampling convs,
// LayerNorm, positional table, attention, conv module, output layout).
//
// Data layout in HBM (all packed per utterance, no T_max padding):
//   pcm      f32 [sum S_b]                 utterances concatenated
//   dft_a    f16 [sum Tm_b, 3*n_fft]       [Xhi | Xhi | Xlo] windowed frames
//   power    f32 [sum Tm_b, power_ld]      |X|^2 for bins 0..n_fft/2
//   logmel   f32 [sum Tm_b, F]             time-major log-mel, normalised in place
//   s1       bf16 [sum v1_b, F1, C]        subsampling stage outputs, channel fastest
//   x        f32 [M, d]                    residual stream, M = sum v_b
//   h-type activations (f16 or bf16) [M, *] for every GEMM operand
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

namespace pkc {

// Per-batch item tables (device pointers). Offsets are prefix sums (size B+1).
struct ItemTables {
  int B;
  const int* pcm_off;  // samples
  const int* n_samples;
  const int* mel_off;  // mel frames (Tm_b each)
  const int* mel_T;    // Tm_b
  const int* mel_valid;  // frames the encoder reads (Tm_b - 1)
  const int* v1_off; const int* v1;
  const int* v2_off; const int* v2;
  const int* v_off; const int* v;
};

struct MelArgs {
  const float* pcm;
  const float* window;  // [n_fft], centre-padded
  int n_fft, hop;
  float preemph;
  int total_frames;     // frames row0 .. row0 + total_frames - 1 (of the whole batch)
  __half* dft_a;        // [rows of the batch, 3*n_fft]
  float* power;         // [rows of the batch, power_ld]
  int power_ld;
  int row0;             // first frame (a range of whole utterances; the tables give absolute offsets)
};
cudaError_t mel_frames_launch(const MelArgs& a, const ItemTables& t, cudaStream_t st);

struct FbArgs {
  const float* power; int power_ld;
  const int* fb_start; const int* fb_len; const int* fb_off; const float* fb_w;
  int n_mels;
  float log_guard;
  int total_frames;
  float* logmel;        // [total_frames, n_mels]
};
cudaError_t mel_fb_log_launch(const FbArgs& a, cudaStream_t st);

// Per-feature normalisation in place over each item's first mel_valid frames;
// frames >= mel_valid are zeroed (src/mel_gpu.cpp:137-161).
cudaError_t mel_norm_launch(float* logmel, int n_mels, const ItemTables& t, cudaStream_t st);

// packed [sum Tm_b, F] -> [B][F][T_max] zero padded (the reference MelBatch)
cudaError_t mel_to_batch_launch(const float* logmel, int n_mels, int T_max, float* out,
                                const ItemTables& t, cudaStream_t st);
// [B][F][T_max] -> packed [sum Tm_b, F] (Tm_b = mel_T[b])
cudaError_t batch_to_packed_launch(const float* in, int n_mels, int T_max, float* logmel,
                                   const ItemTables& t, int max_T, cudaStream_t st);

// Subsampling stage 0: Conv2d(1 -> C, 3x3, stride 2, pad 1) + bias + ReLU.
cudaError_t sub_conv0_launch(const float* logmel, int F, const float* w /*[C][9]*/, const float* b,
                             int C, __nv_bfloat16* out, int F1, const ItemTables& t, int total_v1,
                             cudaStream_t st);
// Stage 1 fused (conv.0 + ReLU, then the first depthwise + bias): mel ->
// stage-2 frames [sum v2, F2, C] bf16, no conv.0 map in memory. F1 = 64 or 40.
cudaError_t sub_stage1_launch(const float* logmel, int F, const float* w0, const float* b0, const float* w1,
                              const float* b1, int C, __nv_bfloat16* out, int F1, const ItemTables& t,
                              int max_v2, cudaStream_t st);
// Depthwise Conv2d(C, 3x3, stride 2, pad 1, groups C) + bias.
// stage 1: in = (v1, F_in) -> out = (v2, F_out); stage 2: (v2 -> v)
cudaError_t sub_dw_launch(const __nv_bfloat16* in, int F_in, const int* in_off, const int* in_valid,
                          const float* w /*[9][C]*/, const float* b, int C, __nv_bfloat16* out,
                          int F_out, const int* out_off, const int* out_valid, int B, int max_out,
                          cudaStream_t st);

// LayerNorm over d (ggml_norm, eps 1e-5) * gamma + beta.
// out_h (may be null): normalised result in the compute type.
// If g2 != nullptr: y = LN(x; g, b) is written back to x (f32) and
// out_h = LN(y; g2, b2) (norm_out of one layer fused with the next layer's
// norm_feed_forward1).
// split (f32-accurate path): out_h is f16 [M, 2d], rows [hi | lo].
cudaError_t layernorm_launch(float* x, int M, int d, const float* g, const float* b, void* out_h,
                             bool bf16, const float* g2, const float* b2, bool write_x,
                             cudaStream_t st, bool split = false);

// Sinusoid table over relative positions centre-1 ... -(centre-1): [2*centre-1, d].
cudaError_t pos_table_launch(void* out, int centre, int d, bool bf16, cudaStream_t st);

struct AttnArgs {
  const void* qkv;      // [M, 3d]
  const void* ptab;     // [ptab_rows, ptab_ld] (this layer's d columns)
  int ptab_rows, centre;
  int ptab_ld;          // row stride of ptab in elements (>= d)
  const float* bias_u;  // [H*dk]
  const float* bias_v;
  const int* tiles;     // [n_tiles][2] (item, q0)
  int n_tiles;
  const int* item_off;
  const int* item_len;
  void* ctx;            // [M, d]
  int d, n_heads;
  int rows;             // M: packed frames in qkv / ctx
  int* err;             // device error word (timeouts), may be null
  // nonzero: the q columns of qkv already hold q + bias_u (the QKV GEMM's
  // bias carried it), so the kernel uses them as they are and adds only
  // bias_v - bias_u for the positional term
  int qu_folded = 0;
};
// Dispatcher (the tcgen05 kernel). The tile list in AttnArgs must be built
// with attn_query_tile() rows per tile.
cudaError_t attention_launch(const AttnArgs& a, bool bf16, cudaStream_t st);
int attn_query_tile();
cudaError_t attention_tc_launch(const AttnArgs& a, bool bf16, cudaStream_t st);
int attn_tc_query_tile();

// ---- f32-accurate path (precise.cu): GEMM operands as f16 [hi | lo] rows
// f32 [rows, K] (row stride ldx) -> f16 [rows, 2K] rows [hi | lo] (row stride ldo)
cudaError_t split_rows_launch(const float* x, long long rows, int K, int ldx, __half* out, int ldo,
                              cudaStream_t st);
// sinusoid table [2*centre-1, 2d], rows [hi | lo]
cudaError_t pos_table_split_launch(__half* out, int centre, int d, cudaStream_t st);
// conv.0 + ReLU with f32 output [sum v1, F1, C]
cudaError_t sub_conv0_f32_launch(const float* logmel, int F, const float* w, const float* b, int C, float* out,
                                 int F1, const ItemTables& t, int total_v1, cudaStream_t st);
// subsampling depthwise 3x3 s2 + bias: f32 [frames, F_in, C] -> f16 [frames * F_out, 2C] rows [hi | lo]
cudaError_t sub_dw_f32split_launch(const float* in, int F_in, const int* in_off, const int* in_valid, const float* w,
                                   const float* b, int C, __half* out, int F_out, const int* out_off,
                                   const int* out_valid, int B, int max_out, cudaStream_t st);
// conv module depthwise + BatchNorm + SiLU: f32 [M, d] -> f16 [M, 2d] rows [hi | lo]
cudaError_t dwconv_f32split_launch(const float* in, __half* out, int d, int K, const float* w, const float* bias,
                                   const float* scale, const float* shift, const int* item_off, const int* item_len,
                                   int B, int max_len, cudaStream_t st);
// rel-pos attention in f32: qkv f32 [M, 3d], ptab f32 (ptab_ld), ctx f16 [M, 2d]
// rows [hi | lo]; tiles of attn_f32_query_tile() query rows
cudaError_t attention_f32_launch(const AttnArgs& a, cudaStream_t st);
int attn_f32_query_tile();

// Conv module middle: depthwise Conv1d(K, pad (K-1)/2) over each item's frames
// (zeros outside) + bias -> BatchNorm (folded scale/shift) -> SiLU.
cudaError_t dwconv_bn_silu_launch(const void* in, void* out, int d, int K, const float* w /*[K][d]*/,
                                  const float* bias, const float* scale, const float* shift,
                                  const int* item_off, const int* item_len, int B, int max_len,
                                  bool bf16, cudaStream_t st);

// CTC head (ctc.cu): x f32 [M, d] -> [x_hi | x_hi | x_lo] f16 [M, 3d] (the A
// operand of the ~22-bit split GEMM against [W_hi | W_lo | W_hi])
cudaError_t ctc_split3_launch(const float* x, int M, int d, void* out, cudaStream_t st);
// per frame of logits [M, ld] (V1 real classes): argmax (first maximum),
// maximum log-probability (= -log-sum-exp of the shifted row) and, if
// logprobs != null, the log-probabilities [M, V1]
cudaError_t ctc_rows_launch(const float* logits, int M, int ld, int V1, int* argmax, float* maxlp, float* logprobs,
                            cudaStream_t st);

// Greedy transducer (TDT when D > 0, else RNNT) decode of B utterances in
// lockstep (transducer.cu). Device pointers; state arrays are per utterance
// and must be initialised by the caller (t = sym = 0, cur = 0, have_token = 0,
// pending = 1, done = (item_len == 0), ntok = 0; h = c = 0; bar_count zero and
// the first transducer_key_bytes(B) bytes of partials zero).
// B <= transducer_max_batch(...): every CTA keeps the per-utterance state in
// shared memory, so larger batches are decoded in groups. Weight rows, embed,
// zeros, enc_proj rows, h and pred_proj must be 16-byte aligned (bulk copies).
struct TransducerArgs {
  int B, H, L, J, V1, D, blank, max_symbols, max_iters;
  // weights (f32)
  const float* embed;      // [V1, H]
  const float* w_ih;       // [L][4H, H]
  const float* w_hh;       // [L][4H, H]
  const float* b_lstm;     // [L][4H] (b_ih + b_hh)
  const float* w_pred;     // [J, H]
  const float* b_pred;     // [J]
  const float* w_out;      // [V1 + D, J]
  const float* b_out;      // [V1 + D]
  const int* durations;    // [D]
  const float* zeros;      // [H] zeros
  const float* gate0;      // [V1 + 1, 4H] layer-0 input gates (transducer_gate0_launch)
  // encoder projection, frames of all utterances: [M, ld_enc] (first J columns)
  const float* enc_proj;
  int ld_enc;
  const int* item_off;     // [B] first frame row
  const int* item_len;     // [B] frames
  // state
  float* h;                // [2][L][B][H] (committed buffer cur[b], step output 1 - cur[b])
  float* c;                // [2][L][B][H]
  float* pred_proj;        // [B, J]
  int *t, *sym, *cur, *have_token, *last_token, *pending, *done, *ntok;
  // transducer_partial_bytes(grid, B): argmax keys [2][3][B] u64, then the
  // per-CTA confidence partials [2][grid][B] float2
  unsigned long long* keys;
  // output tokens: utterance b at rows [tok_off[b], tok_off[b] + tok_cap[b]) of
  // int [*, 4] = (id, frame, conf as float bits, span)
  int* tokens;
  const int* tok_off;
  const int* tok_cap;
  unsigned int* bar_count;
  int* err;
  int held;                // set by the launcher (LSTM layers resident in shared memory)
  int jres;                // set by the launcher (joint rows resident, else streamed)
};
// Layer-0 input gates of every token, computed once at load:
// out[v] = W_ih0 embed[v] + b0 for v < V1 and out[V1] = b0 (the SOS step's zero
// input). f32 throughout.
cudaError_t transducer_gate0_launch(const float* embed, const float* w_ih0, const float* b0, int V1, int H,
                                    float* out, cudaStream_t st);
size_t transducer_smem_bytes(int H, int J, int L, int VP, int grid, int B);
size_t transducer_smem_limit();
int transducer_max_batch(int H, int J, int L, int VP, int grid);
size_t transducer_key_bytes(int B);
size_t transducer_partial_bytes(int grid, int B);
int transducer_grid();
cudaError_t transducer_greedy_launch(const TransducerArgs& a, int grid, cudaStream_t st);

// Cache-aware streaming encoder (stream.cu). S streams step together: their
// windows / chunk frames are stacked along the rows, their caches are reached
// through device tables of per-stream pointers.
// Causal subsampling stages: mel windows [S][F][n] f32 -> [S][T1][F1][C] bf16,
// T1 = n/2 + 1, F1 = F/2 + 1; depthwise stage [S][Ti][Fi][C] -> [S][Ti/2 + 1][Fi/2 + 1][C].
cudaError_t causal_conv0_launch(const float* mel, int S, int F, int n, int valid, const float* w, const float* b,
                                int C, int T1, int F1, __nv_bfloat16* out, cudaStream_t st);
cudaError_t causal_dw_launch(const __nv_bfloat16* in, int S, int Ti, int Fi, int valid, const float* w,
                             const float* b, int C, int To, int Fo, __nv_bfloat16* out, cudaStream_t st);
struct StreamAttnArgs {
  const void* qkv;              // [S * Tc, 3d]: the chunks' q | k | v, stream s at rows s * Tc
  const void* const* kv_cache;  // [S]: stream s's k | v cache of every layer, [layers][cache_len][2d]
  size_t kv_layer_off;          // elements from a cache base to this layer's block
  const int* const* filled;     // [S]: stream s's count of valid cache rows (its last ones)
  const void* ptab;             // this layer's projected positions: row r = relative position cache_len + Tc - 1 - r
  int ldp;                      // row stride of ptab (elements)
  const float* bias_u;          // [d]
  const float* bias_v;
  void* ctx;                    // [S * Tc, d]
  int d, n_heads, Tc, cache_len, n_streams;
  int att_left, att_right;
};
cudaError_t stream_attention_launch(const StreamAttnArgs& a, bool bf16, cudaStream_t st);
// Causal depthwise conv over [conv cache (lp = K - 1 rows) | the chunk's GLU
// rows] of every stream, + bias, LayerNorm over d (g, b = gamma, beta) or the
// folded BatchNorm (g, b = scale, shift), SiLU -> out [S * Tc, d]
struct StreamConvArgs {
  const void* const* cv_cache;  // [S]: stream s's conv cache of every layer, [layers][lp][d]
  size_t cv_layer_off;          // elements from a cache base to this layer's block
  const void* glu;              // [S * Tc, d]
  void* out;                    // [S * Tc, d]
  const float* w;               // [K][d]
  const float* bias;            // [d] or null
  const float* g;
  const float* b;
  int d, K, Tc, n_streams, layer_norm;
};
cudaError_t stream_dwconv_launch(const StreamConvArgs& a, bool bf16, cudaStream_t st);
// The next caches of every layer and stream after a chunk (into the other
// buffers): attention k | v = the last cache_len rows of [cache | the chunk's
// k | v], conv = the last lp rows of [conv cache | the chunk's GLU rows]
struct StreamRollArgs {
  void* const* kv_cur;   // [S] -> [layers][cache_len][2d]
  void* const* kv_next;
  void* const* cv_cur;   // [S] -> [layers][lp][d]
  void* const* cv_next;
  const void* qkv;       // [layers][layer_rows][3d]: stream s's chunk rows at s * Tc
  const void* glu;       // [layers][layer_rows][d]
  int layer_rows;
  int layers, d, cache_len, Tc, lp, n_streams;
};
cudaError_t stream_roll_launch(const StreamRollArgs& a, cudaStream_t st);
// *filled[s] = min(cache_len, *filled[s] + Tc) for every stream
cudaError_t stream_advance_launch(int* const* filled, int n_streams, int Tc, int cache_len, cudaStream_t st);

// packed time-major [M, d] -> per item channels-first [d, v_b], items concatenated
cudaError_t to_channels_first_launch(const float* x, float* out, int d, const int* item_off,
                                     const int* item_len, int B, int max_len, cudaStream_t st);

}  // namespace pkc
