// Batch planner and per-device encoder runtime.
#pragma once
#include <cuda_runtime.h>

#include <mutex>
#include <string>
#include <vector>

#include "../../include/pkc.h"
#include "model.hpp"

namespace pkc {

struct ItemTables;  // kernels/kernels.h

// Geometry of one batch on one device: every utterance keeps only its valid
// frames at every stage (the reference pads to T_max and masks).
struct Plan {
  int B = 0;
  std::vector<int> S, pcm_off;        // samples
  std::vector<int> Tm, mel_off;       // mel frames per utterance
  std::vector<int> mval;              // mel frames the encoder reads (Tm - 1)
  std::vector<int> v1, v1_off, v2, v2_off, v, v_off;
  long long total_samples = 0;
  int total_frames = 0, M1 = 0, M2 = 0, M = 0;
  int max_Tm = 0, max_v1 = 0, max_v2 = 0, max_v = 0;
  int centre = 0;                     // positional table centre = max v
  std::vector<int> attn_tiles;        // (item, q0) pairs: part 0's tiles, then part 1's
  // The conformer layers run as two independent parts on two streams when
  // split_b > 0: utterances [0, split_b) (rows [0, v_off[split_b])) and the
  // rest, so one part's kernel tails and latency-bound kernels overlap the
  // other part's work. Every kernel treats rows / utterances independently,
  // so the result is the same bits as one part.
  int split_b = 0;
  int ntiles0 = 0;                    // attention tiles of part 0
};

// n_samples given: PCM path. mel_T given instead (n_samples empty): mel path
// where mel_T[b] = valid mel frames from the caller.
void make_plan(const Config& c, const std::vector<int>& n_samples, const std::vector<int>& mel_T,
               Plan& p);
int mel_frames_for(const Config& c, int n_samples);
int encoder_frames_for(int mel_frames);

struct KernelStatAcc {
  std::string name;
  long long launches = 0;
  double ms = 0, flops = 0, bytes = 0;
};

class DeviceRunner {
 public:
  DeviceRunner(const Config& c, int device) : cfg_(c), device_(device) {}
  ~DeviceRunner();
  // Upload a packed weight image to this runner's device (and create its
  // streams and workspaces).
  std::string init(const PackedWeights& pw);
  // Whether the weights are packed with the pre-norm LayerNorms folded in.
  static bool ln_fused(const Config& c);
  double upload_seconds() const { return upload_s_; }
  int device() const { return device_; }
  cudaStream_t stream() const { return stream_; }
  int last_graph_kernels() const { return last_kernels_; }

  // Runs the front end (if pcm) and the encoder. Inputs either in host memory
  // (copied in) or already on the device. Output: time-major [M, d] f32 in
  // x_out (device, may be the workspace) - see encode_* helpers.
  pkc_status encode_pcm_host(const std::vector<const float*>& pcm, const std::vector<int>& n,
                             int layout, float* host_out, std::string& err);
  // The same with one host destination per clip (the clip's frames copied
  // there by their own device-to-host copy): the multi-device dispatcher's
  // form, which writes each device's clips straight into the caller's buffer.
  pkc_status encode_pcm_host_items(const std::vector<const float*>& pcm, const std::vector<int>& n, int layout,
                                   const std::vector<float*>& item_out, std::string& err);
  pkc_status encode_pcm_device(const float* d_pcm, const std::vector<int>& n, float* d_out,
                               cudaStream_t st, bool sync, std::string& err);
  pkc_status encode_mel_host(const float* mel, int B, int n_mels, int T_max, const int* valid_T,
                             int layout, float* host_out, std::string& err);
  pkc_status mel_host(const std::vector<const float*>& pcm, const std::vector<int>& n, int T_max,
                      float* host_out, std::string& err);

  // CTC head (src/ctc_decoder.cpp:35 + the per-frame part of src/search.cpp:21):
  // encoder, then per frame the argmax class and the maximum log-probability
  // ([sum T'_b] each, clips back to back) and, if logprobs_out != null, the
  // log-probabilities [sum T'_b, V+1]
  pkc_status ctc_pcm_host(const std::vector<const float*>& pcm, const std::vector<int>& n, int* argmax_out,
                          float* maxlp_out, float* logprobs_out, std::string& err);
  int ctc_classes() const { return w_.ctc_v1; }
  // Greedy transducer decode (tdt_greedy, src/tdt.cpp:8; rnnt_greedy,
  // src/rnnt.cpp:110) on the GPU: encoder, encoder projection of the joint,
  // then the lockstep decode kernel. tokens: per clip up to T'_b * max_symbols
  // rows of int [4] (id, frame, conf bits, span) at row offset tok_off[b]
  // (prefix sums of T'_b * max_symbols); n_tok[b] the count.
  pkc_status transducer_pcm_host(const std::vector<const float*>& pcm, const std::vector<int>& n, int* tokens,
                                 int* n_tok, std::string& err);
  // 0: no transducer decoder; 1: RNN-T; 2: TDT
  int transducer_kind() const { return w_.dec_ok ? (cfg_.durations.empty() ? 1 : 2) : 0; }
  int max_symbols() const { return cfg_.max_symbols; }

  void profile_enable(bool on);
  std::vector<KernelStatAcc> profile_read();

  // Cache-aware streaming encoder (StreamingEncoder, src/streaming_encoder.hpp:
  // 33-66): per-stream caches and scratch on this runner's device (stream.cpp).
  struct StreamState;
  StreamState* stream_create(std::string& err);
  static void stream_destroy(StreamState* s);
  pkc_status stream_reset(StreamState& s, std::string& err);
  // One chunk window: mel [n_mels][n_frames] host f32 (feature-major, the
  // pre-encode overlap included); out [valid][d] host f32.
  pkc_status stream_step(StreamState& s, const float* mel, int n_frames, bool is_last, float* out,
                         size_t out_cap_floats, int* n_valid, std::string& err);
  // S streams of this runner stepped together, one window each (all
  // n_frames long; all at their first window or all past it)
  pkc_status stream_step_batch(StreamState* const* ss, int S, const float* const* mels, int n_frames,
                               const int* is_last, float* const* outs, size_t out_cap_floats, int* n_valid,
                               std::string& err);
  static int stream_step_num(const StreamState& s);

 private:
  pkc_status prepare(const Plan& p, cudaStream_t st, std::string& err);
  // device tables of utterances [b0, b1): every table holds absolute offsets,
  // so a range's tables are the batch's shifted to b0
  ItemTables tables_of(int b0, int b1) const;
  // mel front end / subsampling of utterances [b0, b1)
  pkc_status run_frontend(const Plan& p, int b0, int b1, cudaStream_t st, std::string& err);
  pkc_status run_subsampling(const Plan& p, int b0, int b1, cudaStream_t st, std::string& err);
  pkc_status run_pos(const Plan& p, cudaStream_t st, std::string& err);
  // subsampling, positional table and layers of the whole batch (one part, or
  // the layers as two parts on two streams)
  pkc_status run_encoder(const Plan& p, cudaStream_t st, std::string& err);
  // Two-part plans whose front end splits as well: positional table on st,
  // then each half of the utterances runs front end -> subsampling -> layers
  // (-> channels-first output) on its own stream, the front end as two
  // groups. With io_, each group first waits for its ev_in_ and each half
  // records ev_out_[k] when its output is final (external event nodes when
  // captured), so the host's uploads after the first group's, and the first
  // half's download, overlap kernels.
  bool split_front(const Plan& p) const;
  pkc_status run_two_part(const Plan& p, cudaStream_t st, bool transpose, std::string& err);
  // host PCM in, host output out for a two-part plan: each half's uploads on
  // cs_in_, the graph, each half's downloads on cs_out_ after its ev_out_
  // (dst(b) = where utterance b's [v_b, d] block goes)
  template <typename Dst>
  pkc_status encode_host_overlapped(const Plan& p, const std::vector<const float*>& pcm, bool cf, Dst dst,
                                    std::string& err);
  // a contiguous range of utterances / rows the layers are issued for
  struct Part {
    int idx;                  // 0 or 1 (selects the stream-K workspace half)
    int row0, M;              // rows [row0, row0 + M)
    int b0, nb, max_v;        // utterances [b0, b0 + nb)
    const int* tiles;         // attention tiles (item, q0) of these utterances
    int ntiles;
    double attn_flops;
  };
  pkc_status run_layer(const Plan& p, int li, const Part& q, cudaStream_t st, std::string& err);
  // the f32-accurate layer (Config::split): split-f16 GEMM operands, f32 attention
  pkc_status run_layer_split(const Plan& p, int li, const Part& q, cudaStream_t st, std::string& err);
  pkc_status run_subsampling_split(const Plan& p, cudaStream_t st, std::string& err);
  pkc_status finish(cudaStream_t st, std::string& err);
  struct StreamScratch;
  StreamScratch* sscr_ = nullptr;  // scratch, staging and graphs of the streaming chunk step
  void stream_scratch_free();
  pkc_status stream_issue(int S, int n, int Tc, int drop, std::string& err);
  // out = epi(LayerNorm(x rows) * g + b) . B^T on the skinny GEMM (M <= 16, 16-bit weights)
  pkc_status gemm_skinny_ln(const float* x, int ldx, const float* g, const float* b, const void* B, bool bf16, int M,
                            int N, int K, int epi, int act, float alpha, const float* bias, void* out, int ldo,
                            cudaStream_t st, std::string& err);
  bool ensure_ws(size_t bytes);
  void prof_begin(cudaStream_t st);
  void prof_end(cudaStream_t st, const char* name, double flops, double bytes);
  pkc_status gemm(const void* A, int lda, const void* B, int ldb, bool bf16, int M, int N, int K,
                  int epi, int act, float alpha, const float* bias, void* out, int ldo,
                  cudaStream_t st, const char* name, std::string& err, const QWeight* qw = nullptr,
                  float* stats = nullptr);
  // split-f16 GEMM: A [M, 2 Ks] and B [N, 2 Ks] rows [hi | lo] (lda / ldb
  // row strides), output as ofmt (OUT_SPLIT: lo half at column + split_ld)
  pkc_status gemm_split(const void* A, int lda, const void* B, int ldb, int M, int N, int Ks, int epi, int act,
                        float alpha, const float* bias, void* out, int ldo, int ofmt, int split_ld,
                        cudaStream_t st, const char* name, std::string& err);
  // D = xhat * B^T + bias, xhat = (x - mean) * rstd per row computed while
  // the A operand is staged (B and bias carry the LayerNorm's gamma / beta);
  // stats are x's per-128-column (mean, M2) partials
  pkc_status gemm_ln(const float* x, const float* stats, const void* B, bool bf16,
                     int M, int N, int K, int epi, int act, const float* bias, void* out, int ldo, cudaStream_t st,
                     const char* name, std::string& err);

  Config cfg_;
  int device_;
  cudaStream_t stream_ = nullptr;
  DeviceWeights w_;
  void* ws_ = nullptr;
  size_t ws_bytes_ = 0;
  int* err_word_ = nullptr;
  // stream-K workspace of the 2-SM GEMM (flags zero between launches)
  float* sk_ws_ = nullptr;      // two halves, one per layer part
  int* sk_flags_ = nullptr;
  int sk_pairs_ = 0;
  int sk_part_ = 0;             // part whose GEMMs are being issued
  // scratch of the decoder heads (CTC: split operand, logits, per-frame
  // results; transducer: encoder projection, state), grown on demand
  void* ctc_ws_ = nullptr;
  size_t ctc_ws_bytes_ = 0;
  pkc_status ensure_aux(size_t bytes, cudaStream_t st, std::string& err);
  // second stream of the two-part layer schedule, and its fork / join events
  cudaStream_t stream2_ = nullptr;
  cudaEvent_t ev_fork_ = nullptr, ev_join_ = nullptr;
  // host input / output copies of two-part plans, and the events that tie
  // each half's copies to its kernels
  cudaStream_t cs_in_ = nullptr, cs_out_ = nullptr;
  // front-end groups of a two-part plan: each half of the utterances in two
  // groups [gb[g], gb[g + 1]) of about equal audio, group g uploaded before
  // ev_in_[g] is recorded; only the first group's upload is not overlapped
  static constexpr int kFrontGroups = 4;
  void front_groups(const Plan& p, int (&gb)[kFrontGroups + 1]) const;
  cudaEvent_t ev_in_[kFrontGroups] = {}, ev_out_[2] = {nullptr, nullptr};
  cudaEvent_t ev_prior_ = nullptr;  // st's earlier work, before the uploads may overwrite the PCM buffer
  bool io_ = false;  // the launch sequence being issued waits for / records those events
  // The offline encoder's QKV bias with pos_bias_u added to its q columns,
  // [n_layers][3d] f32 (derived at load, not part of the packed weights):
  // the attention then takes q + u as the GEMM wrote it. Null for the
  // f32-accurate and causal models.
  float* qkv_bu_ = nullptr;
  bool sub_unfused_ = false;
  bool ln_unfused_ = false;
  bool skinny_ok_ = false;  // the streaming step issues M <= 16 GEMMs as skinny kernels
  double upload_s_ = 0;
  int* h_tables_ = nullptr;  // pinned staging for the item tables
  size_t h_tables_cap_ = 0;
  // carved workspace pointers for the current plan
  struct Ptrs {
    float* pcm = nullptr; void* dft_a = nullptr; float* power = nullptr; float* logmel = nullptr;
    float* melbatch = nullptr; void* s1 = nullptr; void* s2a = nullptr; void* s2b = nullptr;
    void* s3a = nullptr; void* s3b = nullptr; float* x = nullptr; void* hbuf = nullptr;
    void* ffh = nullptr; void* qkv = nullptr; void* pe = nullptr; void* ptab = nullptr;
    void* ctx = nullptr; float* out = nullptr; int* tables = nullptr; float* stats = nullptr;
  } b_;
  // device table pointers for the current plan
  int *t_pcm_off, *t_S, *t_mel_off, *t_Tm, *t_mval, *t_v1_off, *t_v1, *t_v2_off, *t_v2, *t_v_off,
      *t_v, *t_tiles;
  int power_ld_ = 0;
  // plan cache: the device tables and workspace carve of the last batch
  std::vector<int> last_key_;
  // profiling
  bool prof_on_ = false;
  struct ProfRec { int cls; cudaEvent_t a, b; double flops, bytes; };
  // CUDA graphs of the whole launch sequence, one per (plan, in/out pointers):
  // replaying skips ~380 host launches and tensor-map encodes per batch
  struct GraphEntry {
    std::vector<int> key;
    const void* pcm = nullptr;
    const void* x = nullptr;
    bool transpose = false, prof = false, io = false;
    int kernels = 0;  // kernel nodes of the graph
    cudaGraphExec_t exec = nullptr;
    std::vector<ProfRec> recs;
    std::vector<cudaEvent_t> events;
  };
  std::vector<GraphEntry> graphs_;
  int last_kernels_ = 0;  // kernel nodes of the graph launched last
  std::vector<cudaEvent_t>* capture_events_ = nullptr;
  bool use_graphs_ = true;
  pkc_status run_graphed(const Plan& p, cudaStream_t st, bool transpose, std::string& err);
  pkc_status run_eager(const Plan& p, cudaStream_t st, bool transpose, std::string& err);
  void drop_graphs();
  std::vector<ProfRec> prof_recs_;
  std::vector<cudaEvent_t> ev_pool_;
  size_t ev_next_ = 0;
  std::vector<KernelStatAcc> prof_classes_;
  cudaEvent_t prof_open_ = nullptr;
  bool prof_error_ = false;  // an event call failed while profiling (reported by profile_read)
};

// Error plumbing of the runner's methods (they return pkc_status and fill err).
#define PKC_CK(expr, what)                                                             \
  do {                                                                                 \
    cudaError_t e_ = (expr);                                                           \
    if (e_ != cudaSuccess) {                                                           \
      err = std::string(what) + ": " + cudaGetErrorString(e_);                         \
      return PKC_ERR_CUDA;                                                             \
    }                                                                                  \
  } while (0)
#define PKC_ST(expr)                 \
  do {                               \
    pkc_status s_ = (expr);          \
    if (s_ != PKC_OK) return s_;     \
  } while (0)

}  // namespace pkc
