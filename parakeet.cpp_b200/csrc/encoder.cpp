// Per-device encoder runtime: batch planning, workspace, and the launch
// sequence that replaces the reference's single fused ggml graph
// (Encoder::forward_batch, src/encoder.cpp:97-167; ConformerLayer::
// build_graph_batched, src/conformer.cpp:285-353).
//
// One conformer layer is 15 launches on one stream:
//   LN(ff1) [fused with the previous layer's LN(out)] -> GEMM+SiLU -> GEMM+0.5*res
//   LN(att) -> QKV GEMM -> pos GEMM -> rel-pos flash attention -> out GEMM+res
//   LN(conv) -> pw1 GEMM+GLU -> depthwise+BN+SiLU -> pw2 GEMM+res
//   LN(ff2) -> GEMM+SiLU -> GEMM+0.5*res -> LN(out)
#include "encoder.hpp"

#include <algorithm>
#include <cmath>
#include <chrono>
#include <cstdlib>
#include <cstring>

#include "kernels/gemm.h"
#include "kernels/kernels.h"

namespace pkc {

int mel_frames_for(const Config& c, int S) {
  const int pad = c.n_fft / 2;
  const int padded = S + 2 * pad;
  return padded >= c.n_fft ? 1 + (padded - c.n_fft) / c.hop_length : 0;
}

// Subsampling::valid_out_len with the offline T-1 entry (src/subsampling.cpp:25-46);
// C++ integer division truncates toward zero exactly like the reference's.
static int stage_len(int v) { return (v + 2 - 3) / 2 + 1; }
int encoder_frames_for(int T) { return stage_len(stage_len(stage_len(T - 1))); }

void make_plan(const Config& c, const std::vector<int>& n_samples, const std::vector<int>& mel_T,
               Plan& p) {
  const bool pcm = !n_samples.empty();
  p = Plan();
  p.B = (int)(pcm ? n_samples.size() : mel_T.size());
  const int B = p.B;
  p.S.assign(B, 0); p.pcm_off.assign(B + 1, 0);
  p.Tm.assign(B, 0); p.mel_off.assign(B + 1, 0); p.mval.assign(B, 0);
  p.v1.assign(B, 0); p.v1_off.assign(B + 1, 0);
  p.v2.assign(B, 0); p.v2_off.assign(B + 1, 0);
  p.v.assign(B, 0); p.v_off.assign(B + 1, 0);
  for (int b = 0; b < B; ++b) {
    p.S[b] = pcm ? n_samples[b] : 0;
    p.Tm[b] = pcm ? mel_frames_for(c, n_samples[b]) : mel_T[b];
    p.mval[b] = p.Tm[b] - 1;
    p.v1[b] = stage_len(p.mval[b]);
    p.v2[b] = stage_len(p.v1[b]);
    p.v[b] = stage_len(p.v2[b]);
    p.pcm_off[b + 1] = p.pcm_off[b] + p.S[b];
    p.mel_off[b + 1] = p.mel_off[b] + p.Tm[b];
    p.v1_off[b + 1] = p.v1_off[b] + p.v1[b];
    p.v2_off[b + 1] = p.v2_off[b] + p.v2[b];
    p.v_off[b + 1] = p.v_off[b] + p.v[b];
    p.max_Tm = std::max(p.max_Tm, p.Tm[b]);
    p.max_v1 = std::max(p.max_v1, p.v1[b]);
    p.max_v2 = std::max(p.max_v2, p.v2[b]);
    p.max_v = std::max(p.max_v, p.v[b]);
  }
  p.total_samples = p.pcm_off[B];
  p.total_frames = p.mel_off[B];
  p.M1 = p.v1_off[B];
  p.M2 = p.v2_off[B];
  p.M = p.v_off[B];
  p.centre = p.max_v;
  // attention query tiles, longest utterances first: a tile's cost grows with
  // its utterance's length, so the block scheduler gets the long ones early
  const int qt = c.split ? attn_f32_query_tile() : attn_query_tile();
  std::vector<int> order(B);
  for (int b = 0; b < B; ++b) order[b] = b;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return p.v[a] > p.v[b]; });
  // two-part split: a per-utterance cost of frames x (1 + T / 3.5 d) (the
  // projections per frame, plus attention growing with the length), halves
  // as equal as a contiguous split allows. Only for batches whose halves
  // still fill the GPU: measured at M = 3282 (C2) two parts were 8 % slower
  // (each part's GEMMs fall under one efficient wave), at M ~ 13k (C3) 4 %
  // faster. PKC_STREAMS=1: never split; PKC_STREAMS=2: split any batch of
  // two or more utterances.
  p.split_b = 0;
  const char* sm = getenv("PKC_STREAMS");
  const int mode = sm ? std::atoi(sm) : 0;
  if (B >= 2 && mode != 1 && (mode == 2 || p.M >= 6144)) {
    std::vector<double> cost(B);
    double total = 0.0;
    for (int b = 0; b < B; ++b) {
      cost[b] = p.v[b] * (1.0 + p.v[b] / (3.5 * c.d_model));
      total += cost[b];
    }
    double pre = 0.0, best = 1e300;
    for (int s = 1; s < B; ++s) {
      pre += cost[s - 1];
      const double gap = std::fabs(2.0 * pre - total);
      if (gap < best) {
        best = gap;
        p.split_b = s;
      }
    }
  }
  for (int part = 0; part < 2; ++part) {
    for (int b : order) {
      const bool in1 = p.split_b > 0 && b >= p.split_b;
      if ((part == 1) != in1) continue;
      for (int q0 = 0; q0 < p.v[b]; q0 += qt) {
        p.attn_tiles.push_back(b);
        p.attn_tiles.push_back(q0);
      }
    }
    if (part == 0) p.ntiles0 = (int)p.attn_tiles.size() / 2;
  }
}

namespace {
size_t al(size_t x) { return (x + 255) / 256 * 256; }
}  // namespace

DeviceRunner::~DeviceRunner() {
  cudaSetDevice(device_);
  if (stream_) cudaStreamSynchronize(stream_);
  drop_graphs();
  stream_scratch_free();
  for (cudaEvent_t e : ev_pool_) cudaEventDestroy(e);
  if (ws_) cudaFree(ws_);
  if (err_word_) cudaFree(err_word_);
  if (sk_ws_) cudaFree(sk_ws_);
  if (sk_flags_) cudaFree(sk_flags_);
  if (ctc_ws_) cudaFree(ctc_ws_);
  if (qkv_bu_) cudaFree(qkv_bu_);
  if (stream2_) {
    cudaStreamSynchronize(stream2_);
    cudaStreamDestroy(stream2_);
  }
  if (ev_fork_) cudaEventDestroy(ev_fork_);
  if (ev_join_) cudaEventDestroy(ev_join_);
  for (cudaStream_t s : {cs_in_, cs_out_})
    if (s) {
      cudaStreamSynchronize(s);
      cudaStreamDestroy(s);
    }
  for (cudaEvent_t e : ev_in_)
    if (e) cudaEventDestroy(e);
  for (cudaEvent_t e : {ev_out_[0], ev_out_[1], ev_prior_})
    if (e) cudaEventDestroy(e);
  if (h_tables_) cudaFreeHost(h_tables_);
  free_weights(w_);
  if (stream_) cudaStreamDestroy(stream_);
}

// PKC_LN_FUSED=1: the QKV / pointwise-1 / FFN2-up GEMMs normalise their A
// operand themselves (k_gemm_tc2ln). Off by default: the f32 rows it stages
// through shared memory add ~80 KB of shared-memory traffic per CTA and
// k-block to a mainloop that the plain GEMM already runs at the
// shared-memory port's rate, so it is slower than the separate LayerNorm
// kernel at the encoder's shapes.
bool DeviceRunner::ln_fused(const Config& c) {
  const char* lf = getenv("PKC_LN_FUSED");
  return lf && lf[0] == '1' && c.d_model % 128 == 0 && !c.split;
}

std::string DeviceRunner::init(const PackedWeights& pw) {
  if (cudaSetDevice(device_) != cudaSuccess) return "cannot select CUDA device " + std::to_string(device_);
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device_) != cudaSuccess) return "cudaGetDeviceProperties failed";
  if (prop.major != 10) return std::string("device ") + prop.name + " is not sm_100 (B200); the kernels are sm_100a only";
  if (cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking) != cudaSuccess) return "stream creation failed";
  if (cudaMalloc(&err_word_, sizeof(int)) != cudaSuccess) return "cudaMalloc failed";
  cudaMemset(err_word_, 0, sizeof(int));
  sk_pairs_ = prop.multiProcessorCount / 2;
  if (cudaMalloc(&sk_ws_, 2 * gemm_sk_ws_bytes(sk_pairs_)) != cudaSuccess ||
      cudaMalloc(&sk_flags_, 2 * gemm_sk_flag_count(sk_pairs_) * sizeof(int)) != cudaSuccess)
    return "cudaMalloc of the GEMM stream-K workspace failed";
  cudaMemset(sk_flags_, 0, 2 * gemm_sk_flag_count(sk_pairs_) * sizeof(int));
  if (cudaStreamCreateWithFlags(&stream2_, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&ev_fork_, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&ev_join_, cudaEventDisableTiming) != cudaSuccess)
    return "second stream / event creation failed";
  if (cudaStreamCreateWithFlags(&cs_in_, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&cs_out_, cudaStreamNonBlocking) != cudaSuccess)
    return "copy stream creation failed";
  for (cudaEvent_t& e : ev_in_)
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return "copy event creation failed";
  for (cudaEvent_t* e : {&ev_out_[0], &ev_out_[1], &ev_prior_})
    if (cudaEventCreateWithFlags(e, cudaEventDisableTiming) != cudaSuccess) return "copy event creation failed";
  power_ld_ = cfg_.n_fft / 2 + 8;
  const char* ng = getenv("PKC_NO_GRAPH");
  use_graphs_ = !(ng && ng[0] == '1');
  // PKC_SUB_UNFUSED=1: conv.0 and the first depthwise as two kernels with the
  // conv.0 map in memory (A/B comparisons); the default is the fused kernel
  const char* su = getenv("PKC_SUB_UNFUSED");
  sub_unfused_ = (su && su[0] == '1') || (cfg_.F1 != 64 && cfg_.F1 != 40);
  ln_unfused_ = !ln_fused(cfg_);  // must match the fold the weights were packed with
  const auto t0 = std::chrono::steady_clock::now();
  std::string err = upload_packed(pw, cfg_, w_, stream_);
  upload_s_ = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  if (!err.empty()) return err;
  if (!cfg_.split && !cfg_.causal()) {
    // QKV bias + [pos_bias_u | 0 | 0] per layer, for the offline encoder
    const int d = cfg_.d_model, nl = cfg_.n_layers;
    std::vector<float> hb((size_t)nl * 3 * d, 0.f), hu((size_t)d);
    for (int l = 0; l < nl; ++l) {
      const LayerWeights& lw = w_.layers[l];
      float* row = hb.data() + (size_t)l * 3 * d;
      if (lw.qkv_b && cudaMemcpy(row, lw.qkv_b, (size_t)3 * d * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return "QKV bias download failed";
      if (!lw.pos_u || cudaMemcpy(hu.data(), lw.pos_u, (size_t)d * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return "pos_bias_u download failed";
      for (int k = 0; k < d; ++k) row[k] += hu[k];
    }
    if (cudaMalloc(&qkv_bu_, hb.size() * 4) != cudaSuccess ||
        cudaMemcpy(qkv_bu_, hb.data(), hb.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
      return "QKV + pos_bias_u upload failed";
  }
  return err;
}

bool DeviceRunner::ensure_ws(size_t bytes) {
  if (bytes <= ws_bytes_) return true;
  last_key_.clear();
  cudaStreamSynchronize(stream_);
  drop_graphs();
  if (ws_) cudaFree(ws_);
  ws_ = nullptr;
  ws_bytes_ = 0;
  const size_t want = bytes + bytes / 8;
  if (cudaMalloc(&ws_, want) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  ws_bytes_ = want;
  return true;
}

// ------------------------------------------------------------------ profiling
void DeviceRunner::profile_enable(bool on) {
  cudaSetDevice(device_);
  cudaStreamSynchronize(stream_);
  prof_on_ = on;
  drop_graphs();
  prof_recs_.clear();
  prof_classes_.clear();
  ev_next_ = 0;
}

void DeviceRunner::prof_begin(cudaStream_t st) {
  if (!prof_on_) return;
  if (capture_events_) {
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) { prof_error_ = true; return; }
    capture_events_->push_back(e);
    prof_open_ = e;
    // external: becomes an event-record node that replays re-record
    if (cudaEventRecordWithFlags(prof_open_, st, cudaEventRecordExternal) != cudaSuccess) prof_error_ = true;
    return;
  }
  if (ev_next_ + 2 > ev_pool_.size()) {
    for (int i = 0; i < 256; ++i) {
      cudaEvent_t e;
      cudaEventCreate(&e);
      ev_pool_.push_back(e);
    }
  }
  prof_open_ = ev_pool_[ev_next_++];
  cudaEventRecord(prof_open_, st);
}

void DeviceRunner::prof_end(cudaStream_t st, const char* name, double flops, double bytes) {
  if (!prof_on_) return;
  cudaEvent_t e = nullptr;
  if (capture_events_) {
    if (cudaEventCreate(&e) != cudaSuccess) { prof_error_ = true; return; }
    capture_events_->push_back(e);
  } else {
    e = ev_pool_[ev_next_++];
  }
  const cudaError_t re = capture_events_ ? cudaEventRecordWithFlags(e, st, cudaEventRecordExternal)
                                         : cudaEventRecord(e, st);
  if (re != cudaSuccess) prof_error_ = true;
  int cls = -1;
  for (size_t i = 0; i < prof_classes_.size(); ++i)
    if (prof_classes_[i].name == name) cls = (int)i;
  if (cls < 0) {
    prof_classes_.push_back(KernelStatAcc{name});
    cls = (int)prof_classes_.size() - 1;
  }
  prof_recs_.push_back(ProfRec{cls, prof_open_, e, flops, bytes});
}

std::vector<KernelStatAcc> DeviceRunner::profile_read() {
  cudaSetDevice(device_);
  cudaStreamSynchronize(stream_);
  for (const ProfRec& r : prof_recs_) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, r.a, r.b);
    KernelStatAcc& k = prof_classes_[r.cls];
    k.launches += 1;
    k.ms += ms;
    k.flops += r.flops;
    k.bytes += r.bytes;
  }
  prof_recs_.clear();
  ev_next_ = 0;
  cudaGetLastError();
  std::vector<KernelStatAcc> out = prof_classes_;
  if (prof_error_) out.push_back(KernelStatAcc{"profile_event_error"});
  return out;
}

// ------------------------------------------------------------------ launches
pkc_status DeviceRunner::gemm(const void* A, int lda, const void* B, int ldb, bool bf16, int M,
                              int N, int K, int epi, int act, float alpha, const float* bias,
                              void* out, int ldo, cudaStream_t st, const char* name,
                              std::string& err, const QWeight* qw, float* stats) {
  GemmArgs a{};
  a.M = M; a.N = N; a.K = K; a.epi = epi; a.act = act; a.alpha = alpha; a.bias = bias;
  a.out = out; a.ldo = ldo; a.err = err_word_; a.stats = stats;
  a.skinny = skinny_ok_ ? 1 : 0;
  // the part being issued owns one half of the stream-K workspace
  a.sk_ws = sk_ws_ + (size_t)sk_part_ * (gemm_sk_ws_bytes(sk_pairs_) / sizeof(float));
  a.sk_flags = sk_flags_ + (size_t)sk_part_ * gemm_sk_flag_count(sk_pairs_);
  a.sk_pairs = sk_pairs_;
  prof_begin(st);
  cudaError_t e;
  if (qw && qw->type) {
    // block-quantised weight, dequantised inside the GEMM
    const QuantB qb{qw->type, qw->q, qw->s0, qw->s1};
    e = gemm_launch_q(A, lda, qb, bf16, a, st);
  } else {
    e = gemm_launch(A, lda, B, ldb, bf16, a, st);
  }
  const int osz = (epi == EPI_RESID_F32 || epi == EPI_STORE_F32 || epi == EPI_POWER_F32) ? 4 : 2;
  const int ncols = (epi == EPI_GLU_H || epi == EPI_POWER_F32) ? N / 2 : N;
  prof_end(st, name, 2.0 * M * N * K,
           2.0 * ((double)M * K + (double)N * K) + (double)M * ncols * osz * (epi == EPI_RESID_F32 ? 2 : 1));
  if (e != cudaSuccess) {
    err = std::string("GEMM ") + name + " launch failed: " + cudaGetErrorString(e);
    return PKC_ERR_CUDA;
  }
  return PKC_OK;
}

pkc_status DeviceRunner::gemm_split(const void* A, int lda, const void* B, int ldb, int M, int N, int Ks, int epi,
                                    int act, float alpha, const float* bias, void* out, int ldo, int ofmt,
                                    int split_ld, cudaStream_t st, const char* name, std::string& err) {
  GemmArgs a{};
  a.M = M; a.N = N; a.K = 3 * Ks; a.epi = epi; a.act = act; a.alpha = alpha; a.bias = bias;
  a.out = out; a.ldo = ldo; a.err = err_word_;
  a.split_k = Ks; a.ofmt = ofmt; a.split_ld = split_ld;
  prof_begin(st);
  const cudaError_t e = gemm_launch(A, lda, B, ldb, false, a, st);
  const int ncols = epi == EPI_GLU_H ? N / 2 : N;
  const double osz = (epi == EPI_RESID_F32 || epi == EPI_STORE_F32 || ofmt != OUT_H) ? 4.0 : 2.0;
  // algorithmic work: one f32 contraction (2 M N Ks flops); bytes of the split operands
  prof_end(st, name, 2.0 * M * N * Ks,
           4.0 * ((double)M * Ks + (double)N * Ks) + (double)M * ncols * osz * (epi == EPI_RESID_F32 ? 2 : 1));
  if (e != cudaSuccess) {
    err = std::string("GEMM ") + name + " (split) launch failed: " + cudaGetErrorString(e);
    return PKC_ERR_CUDA;
  }
  return PKC_OK;
}

pkc_status DeviceRunner::gemm_ln(const float* x, const float* stats, const void* B, bool bf16, int M, int N, int K, int epi, int act,
                                 const float* bias, void* out, int ldo, cudaStream_t st, const char* name,
                                 std::string& err) {
  GemmArgs a{};
  a.M = M; a.N = N; a.K = K; a.epi = epi; a.act = act; a.alpha = 1.f; a.bias = bias;
  a.out = out; a.ldo = ldo; a.err = err_word_;
  const LnA la{x, K, stats};
  prof_begin(st);
  const cudaError_t e = gemm_launch_ln(la, B, K, bf16, a, st);
  const int ncols = epi == EPI_GLU_H ? N / 2 : N;
  prof_end(st, name, 2.0 * M * N * K,
           4.0 * M * K + (double)M * (K / 128) * 8 + 2.0 * N * K + 2.0 * M * ncols);
  if (e != cudaSuccess) {
    err = std::string("GEMM ") + name + " (LayerNorm fused) launch failed: " + cudaGetErrorString(e);
    return PKC_ERR_CUDA;
  }
  return PKC_OK;
}

pkc_status DeviceRunner::prepare(const Plan& p, cudaStream_t st, std::string& err) {
  const Config& c = cfg_;
  if (c.causal()) {
    err = "offline encoding of a causal (cache-aware streaming) model is not implemented; use pkc_stream_*";
    return PKC_ERR_UNSUPPORTED;
  }
  const int d = c.d_model, F = c.n_mels, C = c.sub_channels;
  // bytes per logical element of the 16-bit activations: split-f16 [hi | lo]
  // rows (or f32) take 4 in the f32-accurate path
  const size_t hs = c.split ? 4 : 2;
  const int B = p.B;
  // Same geometry as the previous batch on this stream: tables and carve are
  // still valid (lets a device-resident caller launch step after step without
  // a host synchronisation in between).
  std::vector<int> key;
  key.reserve(2 * (size_t)B + 2);
  key.push_back(B);
  for (int b = 0; b < B; ++b) { key.push_back(p.S[b]); key.push_back(p.Tm[b]); }
  if (!last_key_.empty() && key == last_key_) return PKC_OK;
  last_key_.clear();
  const int ntiles = (int)p.attn_tiles.size() / 2;
  const size_t n_tab = (size_t)(B + 1) * 5 + (size_t)B * 6 + (size_t)ntiles * 2 + 8;
  const int np = std::max(1, 2 * p.centre - 1);
  size_t sz = 0;
  auto take = [&](size_t bytes) { const size_t o = sz; sz += al(bytes); return o; };
  const size_t o_tab = take(n_tab * 4);
  const size_t o_pcm = take((size_t)p.total_samples * 4);
  const size_t o_dft = take((size_t)p.total_frames * 3 * c.n_fft * 2);
  const size_t o_pow = take((size_t)p.total_frames * power_ld_ * 4);
  const size_t o_log = take((size_t)p.total_frames * F * 4);
  const size_t o_mb = take((size_t)B * F * p.max_Tm * 4);
  const size_t o_s1 = take((sub_unfused_ || c.split) ? (size_t)p.M1 * c.F1 * C * hs : 0);
  const size_t o_s2a = take((size_t)p.M2 * c.F2 * C * hs);
  const size_t o_s2b = take((size_t)p.M2 * c.F2 * C * hs);
  const size_t o_s3a = take((size_t)p.M * c.F3 * C * hs);
  const size_t o_s3b = take((size_t)p.M * c.F3 * C * hs);
  const size_t o_x = take((size_t)p.M * d * 4);
  const size_t o_h = take((size_t)p.M * d * hs);
  const size_t o_ff = take((size_t)p.M * c.ff_dim * hs);
  const size_t o_qkv = take((size_t)p.M * 3 * d * hs);
  const size_t o_ctx = take((size_t)p.M * d * hs);
  const size_t o_pe = take((size_t)np * d * hs);
  const size_t o_pt = take((size_t)np * d * c.n_layers * hs);
  const size_t o_out = take((size_t)p.M * d * 4);
  const size_t o_st = take(ln_unfused_ ? 0 : (size_t)p.M * (d / 128) * 8);
  if (!ensure_ws(sz)) {
    err = "workspace allocation of " + std::to_string(sz) + " bytes failed";
    return PKC_ERR_OOM;
  }
  uint8_t* base = static_cast<uint8_t*>(ws_);
  b_.tables = reinterpret_cast<int*>(base + o_tab);
  b_.pcm = reinterpret_cast<float*>(base + o_pcm);
  b_.dft_a = base + o_dft;
  b_.power = reinterpret_cast<float*>(base + o_pow);
  b_.logmel = reinterpret_cast<float*>(base + o_log);
  b_.melbatch = reinterpret_cast<float*>(base + o_mb);
  b_.s1 = base + o_s1; b_.s2a = base + o_s2a; b_.s2b = base + o_s2b;
  b_.s3a = base + o_s3a; b_.s3b = base + o_s3b;
  b_.x = reinterpret_cast<float*>(base + o_x);
  b_.hbuf = base + o_h; b_.ffh = base + o_ff; b_.qkv = base + o_qkv; b_.ctx = base + o_ctx;
  b_.pe = base + o_pe; b_.ptab = base + o_pt;
  b_.out = reinterpret_cast<float*>(base + o_out);
  b_.stats = ln_unfused_ ? nullptr : reinterpret_cast<float*>(base + o_st);

  // item tables -> pinned staging -> device (one copy)
  if (h_tables_cap_ < n_tab) {
    cudaStreamSynchronize(st);
    if (h_tables_) cudaFreeHost(h_tables_);
    h_tables_ = nullptr;
    h_tables_cap_ = 0;
    PKC_CK(cudaMallocHost(&h_tables_, n_tab * 2 * 4), "pinned table allocation");
    h_tables_cap_ = n_tab * 2;
  } else {
    cudaStreamSynchronize(st);  // the previous table upload has finished reading
  }
  int* h = h_tables_;
  int* dv = b_.tables;
  size_t pos = 0;
  auto put = [&](const std::vector<int>& v, int*& dst) {
    std::memcpy(h + pos, v.data(), v.size() * 4);
    dst = dv + pos;
    pos += v.size();
  };
  put(p.pcm_off, t_pcm_off); put(p.S, t_S); put(p.mel_off, t_mel_off); put(p.Tm, t_Tm);
  put(p.mval, t_mval); put(p.v1_off, t_v1_off); put(p.v1, t_v1); put(p.v2_off, t_v2_off);
  put(p.v2, t_v2); put(p.v_off, t_v_off); put(p.v, t_v); put(p.attn_tiles, t_tiles);
  PKC_CK(cudaMemcpyAsync(dv, h, pos * 4, cudaMemcpyHostToDevice, st), "table upload");
  last_key_ = std::move(key);
  return PKC_OK;
}

ItemTables DeviceRunner::tables_of(int b0, int b1) const {
  return ItemTables{b1 - b0,         t_pcm_off + b0, t_S + b0,  t_mel_off + b0, t_Tm + b0, t_mval + b0,
                    t_v1_off + b0,   t_v1 + b0,      t_v2_off + b0, t_v2 + b0,  t_v_off + b0, t_v + b0};
}

pkc_status DeviceRunner::run_frontend(const Plan& p, int b0, int b1, cudaStream_t st, std::string& err) {
  const Config& c = cfg_;
  const ItemTables t = tables_of(b0, b1);
  const int f0 = p.mel_off[b0], nf = p.mel_off[b1] - f0;
  const double samples = (double)(p.pcm_off[b1] - p.pcm_off[b0]);
  __half* dft_a = reinterpret_cast<__half*>(b_.dft_a);
  MelArgs ma{b_.pcm, w_.window, c.n_fft, c.hop_length, c.preemph, nf, dft_a, b_.power, power_ld_, f0};
  prof_begin(st);
  PKC_CK(mel_frames_launch(ma, t, st), "mel_frames");
  prof_end(st, "mel_frames", 0.0, samples * 4 * 3.2 + (double)nf * 3 * c.n_fft * 2);
  PKC_ST(gemm(dft_a + (size_t)f0 * 3 * c.n_fft, 3 * c.n_fft, w_.dft_basis, 3 * c.n_fft, false, nf, c.n_fft,
              3 * c.n_fft, EPI_POWER_F32, ACT_NONE, 1.f, nullptr, b_.power + (size_t)f0 * power_ld_, power_ld_, st,
              "gemm_dft", err));
  FbArgs fa{b_.power + (size_t)f0 * power_ld_, power_ld_, w_.fb_start, w_.fb_len, w_.fb_off, w_.fb_w, c.n_mels,
            c.log_zero_guard, nf, b_.logmel + (size_t)f0 * c.n_mels};
  prof_begin(st);
  PKC_CK(mel_fb_log_launch(fa, st), "mel_fb_log");
  prof_end(st, "mel_fb_log", 0.0, (double)nf * (power_ld_ + c.n_mels) * 4);
  prof_begin(st);
  PKC_CK(mel_norm_launch(b_.logmel, c.n_mels, t, st), "mel_norm");
  prof_end(st, "mel_norm", 0.0, (double)nf * c.n_mels * 4 * 3);
  return PKC_OK;
}

pkc_status DeviceRunner::run_subsampling(const Plan& p, int b0, int b1, cudaStream_t st, std::string& err) {
  const Config& c = cfg_;
  const int d = c.d_model, C = c.sub_channels;
  if (c.split) {
    if (b0 != 0 || b1 != p.B) {
      err = "internal: the f32-accurate subsampling runs on whole batches";
      return PKC_ERR_INTERNAL;
    }
    return run_subsampling_split(p, st, err);
  }
  const ItemTables t = tables_of(b0, b1);
  int max_v2 = 0, max_v = 0;
  for (int b = b0; b < b1; ++b) {
    max_v2 = std::max(max_v2, p.v2[b]);
    max_v = std::max(max_v, p.v[b]);
  }
  const int r1 = p.v1_off[b0], M1 = p.v1_off[b1] - r1;
  const int r2 = p.v2_off[b0], M2 = p.v2_off[b1] - r2;
  const int r3 = p.v_off[b0], M = p.v_off[b1] - r3;
  const int nf = p.mel_off[b1] - p.mel_off[b0];
  __nv_bfloat16* s2a = reinterpret_cast<__nv_bfloat16*>(b_.s2a);
  __nv_bfloat16* s2b = reinterpret_cast<__nv_bfloat16*>(b_.s2b);
  __nv_bfloat16* s3a = reinterpret_cast<__nv_bfloat16*>(b_.s3a);
  __nv_bfloat16* s3b = reinterpret_cast<__nv_bfloat16*>(b_.s3b);
  // ---- subsampling (src/subsampling.cpp:48-240)
  if (sub_unfused_) {
    if (b0 != 0 || b1 != p.B) {
      err = "internal: the unfused subsampling runs on whole batches";
      return PKC_ERR_INTERNAL;
    }
    prof_begin(st);
    PKC_CK(sub_conv0_launch(b_.logmel, c.n_mels, w_.c0_w, w_.c0_b, C,
                            reinterpret_cast<__nv_bfloat16*>(b_.s1), c.F1, t, p.M1, st), "conv0");
    prof_end(st, "sub_conv0", 2.0 * p.M1 * c.F1 * C * 9, (double)p.total_frames * c.n_mels * 4 + (double)p.M1 * c.F1 * C * 2);
    prof_begin(st);
    PKC_CK(sub_dw_launch(reinterpret_cast<const __nv_bfloat16*>(b_.s1), c.F1, t_v1_off, t_v1, w_.dw1_w,
                         w_.dw1_b, C, s2a, c.F2, t_v2_off, t_v2, p.B, p.max_v2, st), "dw1");
    prof_end(st, "sub_dw", 2.0 * p.M2 * c.F2 * C * 9, ((double)p.M1 * c.F1 + (double)p.M2 * c.F2) * C * 2);
  } else {
    // conv.0 + ReLU + first depthwise in one kernel; algorithmic bytes: mel
    // read once, stage-2 frames written once
    prof_begin(st);
    PKC_CK(sub_stage1_launch(b_.logmel, c.n_mels, w_.c0_w, w_.c0_b, w_.dw1_w, w_.dw1_b, C, s2a, c.F1, t, max_v2, st),
           "stage1");
    prof_end(st, "sub_stage1", 2.0 * M1 * c.F1 * C * 9 + 2.0 * M2 * c.F2 * C * 9,
             (double)nf * c.n_mels * 4 + (double)M2 * c.F2 * C * 2);
  }
  const size_t o2 = (size_t)r2 * c.F2 * C, o3 = (size_t)r3 * c.F3 * C;
  PKC_ST(gemm(s2a + o2, C, w_.pw1_w, C, true, M2 * c.F2, C, C, EPI_STORE_H, ACT_RELU, 1.f, w_.pw1_b, s2b + o2, C, st,
              "gemm_sub_pw", err));
  prof_begin(st);
  PKC_CK(sub_dw_launch(s2b, c.F2, t_v2_off + b0, t_v2 + b0, w_.dw2_w, w_.dw2_b, C, s3a, c.F3, t_v_off + b0, t_v + b0,
                       b1 - b0, max_v, st), "dw2");
  prof_end(st, "sub_dw", 2.0 * M * c.F3 * C * 9, ((double)M2 * c.F2 + (double)M * c.F3) * C * 2);
  PKC_ST(gemm(s3a + o3, C, w_.pw2_w, C, true, M * c.F3, C, C, EPI_STORE_H, ACT_RELU, 1.f, w_.pw2_b, s3b + o3, C, st,
              "gemm_sub_pw", err));
  const float xs = c.xscaling ? std::sqrt((float)d) : 1.f;
  PKC_ST(gemm(s3b + o3, c.F3 * C, w_.out_w, c.F3 * C, true, M, d, c.F3 * C, EPI_STORE_F32, ACT_NONE, xs, w_.out_b,
              b_.x + (size_t)r3 * d, d, st, "gemm_sub_out", err));
  return PKC_OK;
}

pkc_status DeviceRunner::run_pos(const Plan& p, cudaStream_t st, std::string& err) {
  const Config& c = cfg_;
  const int d = c.d_model;
  const double hs = 2.0;
  // ---- relative positional table (src/pos_enc.cpp:10-34), shared by the batch
  const int np = 2 * p.centre - 1;
  const int Ld = c.n_layers * d;
  if (c.split) {
    prof_begin(st);
    PKC_CK(pos_table_split_launch(reinterpret_cast<__half*>(b_.pe), p.centre, d, st), "pos_table");
    prof_end(st, "pos_table", 0.0, (double)np * d * 4);
    // every layer's linear_pos in one GEMM, f32 out: ptab [np, L*d]
    PKC_ST(gemm_split(b_.pe, 2 * d, w_.pos_all_w, 2 * d, np, Ld, d, EPI_STORE_F32, ACT_NONE, 1.f, nullptr, b_.ptab,
                      Ld, OUT_H, 0, st, "gemm_pos", err));
  } else {
    prof_begin(st);
    PKC_CK(pos_table_launch(b_.pe, p.centre, d, c.bf16, st), "pos_table");
    prof_end(st, "pos_table", 0.0, (double)np * d * hs);
    // every layer's linear_pos (no bias) in one GEMM: ptab [np, L*d], layer l at column l*d
    PKC_ST(gemm(b_.pe, d, w_.pos_all_w, d, c.bf16, np, Ld, d, EPI_STORE_H, ACT_NONE, 1.f, nullptr, b_.ptab, Ld,
                st, "gemm_pos", err, &w_.pos_all_q));
  }
  return PKC_OK;
}

namespace {
double attn_flops_range(const Plan& p, int d, int b0, int b1) {
  double f = 0.0;
  for (int b = b0; b < b1; ++b) {
    const double T = p.v[b];
    f += 2.0 * T * T * d * 2 + 2.0 * T * (2 * T - 1) * d;
  }
  return f;
}
int max_v_range(const Plan& p, int b0, int b1) {
  int m = 0;
  for (int b = b0; b < b1; ++b) m = std::max(m, p.v[b]);
  return m;
}
}  // namespace

pkc_status DeviceRunner::run_encoder(const Plan& p, cudaStream_t st, std::string& err) {
  const Config& c = cfg_;
  const int M = p.M;
  PKC_ST(run_subsampling(p, 0, p.B, st, err));
  PKC_ST(run_pos(p, st, err));

  // ---- conformer layers: one part, or two independent parts on two streams
  const int ntiles = (int)p.attn_tiles.size() / 2;
  const bool two = p.split_b > 0 && !prof_on_;
  auto layer = [&](int li, const Part& q, cudaStream_t s) {
    return c.split ? run_layer_split(p, li, q, s, err) : run_layer(p, li, q, s, err);
  };
  if (!two) {
    const Part all{0, 0, M, 0, p.B, p.max_v, t_tiles, ntiles, attn_flops_range(p, c.d_model, 0, p.B)};
    for (int li = 0; li < c.n_layers; ++li) PKC_ST(layer(li, all, st));
    return PKC_OK;
  }
  const int sb = p.split_b;
  const Part p0{0, 0, p.v_off[sb], 0, sb, max_v_range(p, 0, sb), t_tiles, p.ntiles0,
                attn_flops_range(p, c.d_model, 0, sb)};
  const Part p1{1, p.v_off[sb], M - p.v_off[sb], sb, p.B - sb, max_v_range(p, sb, p.B), t_tiles + 2 * p.ntiles0,
                ntiles - p.ntiles0, attn_flops_range(p, c.d_model, sb, p.B)};
  // fork: the second stream starts after everything issued so far on st
  PKC_CK(cudaEventRecord(ev_fork_, st), "fork event");
  PKC_CK(cudaStreamWaitEvent(stream2_, ev_fork_, 0), "fork wait");
  for (int li = 0; li < c.n_layers; ++li) {
    PKC_ST(layer(li, p0, st));
    PKC_ST(layer(li, p1, stream2_));
  }
  // join: st continues once the second part is done
  PKC_CK(cudaEventRecord(ev_join_, stream2_), "join event");
  PKC_CK(cudaStreamWaitEvent(st, ev_join_, 0), "join wait");
  return PKC_OK;
}

bool DeviceRunner::split_front(const Plan& p) const {
  return p.split_b > 0 && !prof_on_ && !cfg_.split && !sub_unfused_;
}

void DeviceRunner::front_groups(const Plan& p, int (&gb)[kFrontGroups + 1]) const {
  const int bb[3] = {0, p.split_b, p.B};
  for (int k = 0; k < 2; ++k) {
    // the split of [bb[k], bb[k+1]) nearest to half its samples
    const double half = 0.5 * (p.pcm_off[bb[k]] + p.pcm_off[bb[k + 1]]);
    int m = bb[k];
    while (m + 1 < bb[k + 1] && p.pcm_off[m + 1] <= half) ++m;
    if (m == bb[k] && bb[k + 1] - bb[k] > 1) m = bb[k] + 1;
    gb[2 * k] = bb[k];
    gb[2 * k + 1] = m;
  }
  gb[kFrontGroups] = p.B;
}

pkc_status DeviceRunner::run_two_part(const Plan& p, cudaStream_t st, bool transpose, std::string& err) {
  const Config& c = cfg_;
  const int d = c.d_model, M = p.M, sb = p.split_b;
  const int ntiles = (int)p.attn_tiles.size() / 2;
  // the positional table does not depend on the audio: it runs before the fork
  PKC_ST(run_pos(p, st, err));
  PKC_CK(cudaEventRecord(ev_fork_, st), "fork event");
  PKC_CK(cudaStreamWaitEvent(stream2_, ev_fork_, 0), "fork wait");
  cudaStream_t ss[2] = {st, stream2_};
  const int bb[3] = {0, sb, p.B};
  // inside a capture the copy events become external event nodes of the
  // graph; launched eagerly they are plain waits and records
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  PKC_CK(cudaStreamIsCapturing(st, &cap), "capture status");
  const bool ext = cap == cudaStreamCaptureStatusActive;
  const Part parts[2] = {
      {0, 0, p.v_off[sb], 0, sb, max_v_range(p, 0, sb), t_tiles, p.ntiles0, attn_flops_range(p, d, 0, sb)},
      {1, p.v_off[sb], M - p.v_off[sb], sb, p.B - sb, max_v_range(p, sb, p.B), t_tiles + 2 * p.ntiles0,
       ntiles - p.ntiles0, attn_flops_range(p, d, sb, p.B)}};
  int gb[kFrontGroups + 1];
  front_groups(p, gb);
  for (int g = 0; g < kFrontGroups; ++g) {
    cudaStream_t s = ss[g / 2];
    if (io_) PKC_CK(cudaStreamWaitEvent(s, ev_in_[g], ext ? cudaEventWaitExternal : 0), "input wait");
    if (gb[g] == gb[g + 1]) continue;
    PKC_ST(run_frontend(p, gb[g], gb[g + 1], s, err));
    PKC_ST(run_subsampling(p, gb[g], gb[g + 1], s, err));
  }
  for (int li = 0; li < c.n_layers; ++li)
    for (int k = 0; k < 2; ++k) PKC_ST(run_layer(p, li, parts[k], ss[k], err));
  for (int k = 0; k < 2; ++k) {
    if (transpose) {
      prof_begin(ss[k]);
      PKC_CK(to_channels_first_launch(b_.x, b_.out, d, t_v_off + bb[k], t_v + bb[k], bb[k + 1] - bb[k],
                                      parts[k].max_v, ss[k]), "transpose");
      prof_end(ss[k], "to_channels_first", 0.0, (double)parts[k].M * d * 8);
    }
    if (io_)
      PKC_CK(ext ? cudaEventRecordWithFlags(ev_out_[k], ss[k], cudaEventRecordExternal) : cudaEventRecord(ev_out_[k], ss[k]),
             "output event");
  }
  PKC_CK(cudaEventRecord(ev_join_, stream2_), "join event");
  PKC_CK(cudaStreamWaitEvent(st, ev_join_, 0), "join wait");
  return PKC_OK;
}

pkc_status DeviceRunner::run_layer(const Plan& p, int li, const Part& q, cudaStream_t st, std::string& err) {
  const Config& c = cfg_;
  const int d = c.d_model, FF = c.ff_dim, H = c.n_heads, K = c.conv_kernel;
  const bool bf = c.bf16;
  const int M = q.M;
  const double hs = 2.0;
  const int np = 2 * p.centre - 1;
  const int Ld = c.n_layers * d;
  sk_part_ = q.idx;
  // this part's rows of every row-major activation
  const size_t r0 = (size_t)q.row0;
  float* x = b_.x + r0 * d;
  void* hbuf = static_cast<uint8_t*>(b_.hbuf) + r0 * d * 2;
  void* ffh = static_cast<uint8_t*>(b_.ffh) + r0 * FF * 2;
  void* qkv = static_cast<uint8_t*>(b_.qkv) + r0 * 3 * d * 2;
  void* ctx = static_cast<uint8_t*>(b_.ctx) + r0 * d * 2;
  float* stats = b_.stats ? b_.stats + r0 * (d / 128) * 2 : nullptr;
  const int* v_off = t_v_off + q.b0;  // global row offsets of this part's utterances
  const int* v_len = t_v + q.b0;

  const LayerWeights& L = w_.layers[li];
  // FFN1: r = x + 0.5 * FFN(LN(x))
  if (li == 0) {
    prof_begin(st);
    PKC_CK(layernorm_launch(x, M, d, L.ln_ff1_g, L.ln_ff1_b, hbuf, bf, nullptr, nullptr, false, st), "ln");
    prof_end(st, "layernorm", 0.0, (double)M * d * (4 + hs));
  }
  PKC_ST(gemm(hbuf, d, L.ff1_w1, d, bf, M, FF, d, EPI_STORE_H, ACT_SILU, 1.f, L.ff1_b1, ffh, FF, st, "gemm_ffn", err, &L.ff1_q1));
  // LayerNorm inside the consuming GEMM when its weight carries the folded
  // LayerNorm: the GEMM that updates x before it also writes x's
  // per-128-column row statistics
  const bool lnq = L.qkv_ln, lnc = L.pw1_ln, lnf = L.ff2_ln;
  PKC_ST(gemm(ffh, FF, L.ff1_w2, FF, bf, M, d, FF, EPI_RESID_F32, ACT_NONE, 0.5f, L.ff1_b2, x, d, st, "gemm_ffn", err, &L.ff1_q2,
              lnq ? stats : nullptr));
  // MHSA
  // q comes out of the GEMM as q + pos_bias_u when qkv_bu_ carries u
  const float* qkv_bias = qkv_bu_ ? qkv_bu_ + (size_t)li * 3 * d : L.qkv_b;
  if (lnq) {
    PKC_ST(gemm_ln(x, stats, L.qkv_w, bf, M, 3 * d, d, EPI_STORE_H, ACT_NONE, qkv_bias, qkv, 3 * d, st, "gemm_qkv", err));
  } else {
    prof_begin(st);
    PKC_CK(layernorm_launch(x, M, d, L.ln_att_g, L.ln_att_b, hbuf, bf, nullptr, nullptr, false, st), "ln");
    prof_end(st, "layernorm", 0.0, (double)M * d * (4 + hs));
    PKC_ST(gemm(hbuf, d, L.qkv_w, d, bf, M, 3 * d, d, EPI_STORE_H, ACT_NONE, 1.f, qkv_bias, qkv, 3 * d, st, "gemm_qkv", err, &L.qkv_q));
  }
  // attention addresses the whole qkv / ctx buffers by global row offsets
  AttnArgs aa{b_.qkv, static_cast<const uint8_t*>(b_.ptab) + (size_t)li * d * 2, np, p.centre, Ld,
              L.pos_u, L.pos_v, q.tiles, q.ntiles, t_v_off, t_v, b_.ctx, d, H, p.M, err_word_,
              qkv_bu_ ? 1 : 0};
  prof_begin(st);
  PKC_CK(attention_launch(aa, bf, st), "attention");
  prof_end(st, "attention", q.attn_flops, (double)M * (3 * d + d) * hs + (double)np * d * hs);
  PKC_ST(gemm(ctx, d, L.out_w, d, bf, M, d, d, EPI_RESID_F32, ACT_NONE, 1.f, L.out_b, x, d, st, "gemm_out", err, &L.out_q,
              lnc ? stats : nullptr));
  // conv module
  if (lnc) {
    PKC_ST(gemm_ln(x, stats, L.pw1_w, bf, M, 2 * d, d, EPI_GLU_H, ACT_NONE, L.pw1_b, ctx, d, st, "gemm_pw1_glu", err));
  } else {
    prof_begin(st);
    PKC_CK(layernorm_launch(x, M, d, L.ln_conv_g, L.ln_conv_b, hbuf, bf, nullptr, nullptr, false, st), "ln");
    prof_end(st, "layernorm", 0.0, (double)M * d * (4 + hs));
    PKC_ST(gemm(hbuf, d, L.pw1_w, d, bf, M, 2 * d, d, EPI_GLU_H, ACT_NONE, 1.f, L.pw1_b, ctx, d, st, "gemm_pw1_glu", err));
  }
  // the depthwise kernel addresses rows by global offsets too
  prof_begin(st);
  PKC_CK(dwconv_bn_silu_launch(b_.ctx, b_.hbuf, d, K, L.dw_w, L.dw_b, L.bn_scale, L.bn_shift, v_off, v_len, q.nb,
                               q.max_v, bf, st), "dwconv");
  prof_end(st, "dwconv", 2.0 * M * d * K, (double)M * d * hs * 2);
  PKC_ST(gemm(hbuf, d, L.pw2_w, d, bf, M, d, d, EPI_RESID_F32, ACT_NONE, 1.f, L.pw2_b, x, d, st, "gemm_pw2", err, nullptr,
              lnf ? stats : nullptr));
  // FFN2
  if (lnf) {
    PKC_ST(gemm_ln(x, stats, L.ff2_w1, bf, M, FF, d, EPI_STORE_H, ACT_SILU, L.ff2_b1, ffh, FF, st, "gemm_ffn", err));
  } else {
    prof_begin(st);
    PKC_CK(layernorm_launch(x, M, d, L.ln_ff2_g, L.ln_ff2_b, hbuf, bf, nullptr, nullptr, false, st), "ln");
    prof_end(st, "layernorm", 0.0, (double)M * d * (4 + hs));
    PKC_ST(gemm(hbuf, d, L.ff2_w1, d, bf, M, FF, d, EPI_STORE_H, ACT_SILU, 1.f, L.ff2_b1, ffh, FF, st, "gemm_ffn", err, &L.ff2_q1));
  }
  PKC_ST(gemm(ffh, FF, L.ff2_w2, FF, bf, M, d, FF, EPI_RESID_F32, ACT_NONE, 0.5f, L.ff2_b2, x, d, st, "gemm_ffn", err, &L.ff2_q2));
  // norm_out (+ next layer's norm_feed_forward1 in the same pass)
  const bool last = li + 1 == c.n_layers;
  const LayerWeights* N = last ? nullptr : &w_.layers[li + 1];
  prof_begin(st);
  PKC_CK(layernorm_launch(x, M, d, L.ln_out_g, L.ln_out_b, last ? nullptr : hbuf, bf,
                          last ? nullptr : N->ln_ff1_g, last ? nullptr : N->ln_ff1_b, true, st), "ln");
  prof_end(st, "layernorm", 0.0, (double)M * d * (8 + (last ? 0 : hs)));
  return PKC_OK;
}

// Subsampling of the f32-accurate path: conv.0 and the depthwise convs in f32
// on the CUDA cores, the pointwise convs and the output linear as split-f16
// GEMMs (operands written as [hi | lo] rows by the kernel before each).
pkc_status DeviceRunner::run_subsampling_split(const Plan& p, cudaStream_t st, std::string& err) {
  const Config& c = cfg_;
  const int d = c.d_model, C = c.sub_channels, M = p.M, KW = c.F3 * C;
  ItemTables t{p.B, t_pcm_off, t_S, t_mel_off, t_Tm, t_mval, t_v1_off, t_v1, t_v2_off, t_v2, t_v_off, t_v};
  float* s1 = reinterpret_cast<float*>(b_.s1);
  __half* s2a = reinterpret_cast<__half*>(b_.s2a);
  float* s2b = reinterpret_cast<float*>(b_.s2b);
  __half* s3a = reinterpret_cast<__half*>(b_.s3a);
  float* s3b = reinterpret_cast<float*>(b_.s3b);
  prof_begin(st);
  PKC_CK(sub_conv0_f32_launch(b_.logmel, c.n_mels, w_.c0_w, w_.c0_b, C, s1, c.F1, t, p.M1, st), "conv0");
  prof_end(st, "sub_conv0", 2.0 * p.M1 * c.F1 * C * 9, (double)p.total_frames * c.n_mels * 4 + (double)p.M1 * c.F1 * C * 4);
  prof_begin(st);
  PKC_CK(sub_dw_f32split_launch(s1, c.F1, t_v1_off, t_v1, w_.dw1_w, w_.dw1_b, C, s2a, c.F2, t_v2_off, t_v2, p.B,
                                p.max_v2, st), "dw1");
  prof_end(st, "sub_dw", 2.0 * p.M2 * c.F2 * C * 9, ((double)p.M1 * c.F1 + (double)p.M2 * c.F2) * C * 4);
  PKC_ST(gemm_split(s2a, 2 * C, w_.pw1_w, 2 * C, p.M2 * c.F2, C, C, EPI_STORE_H, ACT_RELU, 1.f, w_.pw1_b, s2b, C,
                    OUT_F32, 0, st, "gemm_sub_pw", err));
  prof_begin(st);
  PKC_CK(sub_dw_f32split_launch(s2b, c.F2, t_v2_off, t_v2, w_.dw2_w, w_.dw2_b, C, s3a, c.F3, t_v_off, t_v, p.B,
                                p.max_v, st), "dw2");
  prof_end(st, "sub_dw", 2.0 * M * c.F3 * C * 9, ((double)p.M2 * c.F2 + (double)M * c.F3) * C * 4);
  PKC_ST(gemm_split(s3a, 2 * C, w_.pw2_w, 2 * C, M * c.F3, C, C, EPI_STORE_H, ACT_RELU, 1.f, w_.pw2_b, s3b, C,
                    OUT_F32, 0, st, "gemm_sub_pw", err));
  // [M, F3 * C] f32 -> [hi | lo] rows (s3a is free again)
  prof_begin(st);
  PKC_CK(split_rows_launch(s3b, M, KW, KW, s3a, 2 * KW, st), "split");
  prof_end(st, "split_rows", 0.0, (double)M * KW * 8);
  const float xs = c.xscaling ? std::sqrt((float)d) : 1.f;
  PKC_ST(gemm_split(s3a, 2 * KW, w_.out_w, 2 * KW, M, d, KW, EPI_STORE_F32, ACT_NONE, xs, w_.out_b, b_.x, d, OUT_H,
                    0, st, "gemm_sub_out", err));
  return PKC_OK;
}

// One conformer layer of the f32-accurate path (the same block as run_layer):
// LayerNorms write split-f16 rows, the projections are split-f16 GEMMs with
// f32 (or split) outputs, the attention and the depthwise conv run in f32.
pkc_status DeviceRunner::run_layer_split(const Plan& p, int li, const Part& q, cudaStream_t st, std::string& err) {
  const Config& c = cfg_;
  const int d = c.d_model, FF = c.ff_dim, H = c.n_heads, K = c.conv_kernel;
  const int M = q.M;
  const int np = 2 * p.centre - 1;
  const int Ld = c.n_layers * d;
  const size_t r0 = (size_t)q.row0;
  float* x = b_.x + r0 * d;
  void* hbuf = static_cast<uint8_t*>(b_.hbuf) + r0 * d * 4;   // split [M, 2d]
  void* ffh = static_cast<uint8_t*>(b_.ffh) + r0 * FF * 4;    // split [M, 2 FF]
  void* qkv = static_cast<uint8_t*>(b_.qkv) + r0 * 3 * d * 4; // f32 [M, 3d]
  void* ctx = static_cast<uint8_t*>(b_.ctx) + r0 * d * 4;     // split [M, 2d], or the GLU's f32 [M, d]
  const int* v_off = t_v_off + q.b0;
  const int* v_len = t_v + q.b0;
  const LayerWeights& L = w_.layers[li];
  auto ln = [&](const float* g, const float* b, const float* g2, const float* b2, bool write_x, void* out) {
    prof_begin(st);
    const cudaError_t e = layernorm_launch(x, M, d, g, b, out, false, g2, b2, write_x, st, true);
    prof_end(st, "layernorm", 0.0, (double)M * d * (4 + 4 + (write_x ? 8 : 0)));
    if (e != cudaSuccess) err = std::string("layernorm: ") + cudaGetErrorString(e);
    return e == cudaSuccess ? PKC_OK : PKC_ERR_CUDA;
  };
  // FFN1: x += 0.5 * FFN(LN(x))
  if (li == 0) PKC_ST(ln(L.ln_ff1_g, L.ln_ff1_b, nullptr, nullptr, false, hbuf));
  PKC_ST(gemm_split(hbuf, 2 * d, L.ff1_w1, 2 * d, M, FF, d, EPI_STORE_H, ACT_SILU, 1.f, L.ff1_b1, ffh, 2 * FF,
                    OUT_SPLIT, FF, st, "gemm_ffn", err));
  PKC_ST(gemm_split(ffh, 2 * FF, L.ff1_w2, 2 * FF, M, d, FF, EPI_RESID_F32, ACT_NONE, 0.5f, L.ff1_b2, x, d, OUT_H, 0,
                    st, "gemm_ffn", err));
  // MHSA
  PKC_ST(ln(L.ln_att_g, L.ln_att_b, nullptr, nullptr, false, hbuf));
  PKC_ST(gemm_split(hbuf, 2 * d, L.qkv_w, 2 * d, M, 3 * d, d, EPI_STORE_F32, ACT_NONE, 1.f, L.qkv_b, qkv, 3 * d, OUT_H,
                    0, st, "gemm_qkv", err));
  AttnArgs aa{b_.qkv, reinterpret_cast<const float*>(b_.ptab) + (size_t)li * d, np, p.centre, Ld, L.pos_u, L.pos_v,
              q.tiles, q.ntiles, t_v_off, t_v, b_.ctx, d, H, p.M, err_word_};
  prof_begin(st);
  PKC_CK(attention_f32_launch(aa, st), "attention (f32)");
  prof_end(st, "attention", q.attn_flops, (double)M * (3 * d * 4 + d * 4) + (double)np * d * 4);
  PKC_ST(gemm_split(ctx, 2 * d, L.out_w, 2 * d, M, d, d, EPI_RESID_F32, ACT_NONE, 1.f, L.out_b, x, d, OUT_H, 0, st,
                    "gemm_out", err));
  // conv module
  PKC_ST(ln(L.ln_conv_g, L.ln_conv_b, nullptr, nullptr, false, hbuf));
  PKC_ST(gemm_split(hbuf, 2 * d, L.pw1_w, 2 * d, M, 2 * d, d, EPI_GLU_H, ACT_NONE, 1.f, L.pw1_b, ctx, d, OUT_F32, 0,
                    st, "gemm_pw1_glu", err));
  prof_begin(st);
  PKC_CK(dwconv_f32split_launch(reinterpret_cast<const float*>(b_.ctx), reinterpret_cast<__half*>(b_.hbuf), d, K,
                                L.dw_w, L.dw_b, L.bn_scale, L.bn_shift, v_off, v_len, q.nb, q.max_v, st),
         "dwconv (f32)");
  prof_end(st, "dwconv", 2.0 * M * d * K, (double)M * d * 8);
  PKC_ST(gemm_split(hbuf, 2 * d, L.pw2_w, 2 * d, M, d, d, EPI_RESID_F32, ACT_NONE, 1.f, L.pw2_b, x, d, OUT_H, 0, st,
                    "gemm_pw2", err));
  // FFN2
  PKC_ST(ln(L.ln_ff2_g, L.ln_ff2_b, nullptr, nullptr, false, hbuf));
  PKC_ST(gemm_split(hbuf, 2 * d, L.ff2_w1, 2 * d, M, FF, d, EPI_STORE_H, ACT_SILU, 1.f, L.ff2_b1, ffh, 2 * FF,
                    OUT_SPLIT, FF, st, "gemm_ffn", err));
  PKC_ST(gemm_split(ffh, 2 * FF, L.ff2_w2, 2 * FF, M, d, FF, EPI_RESID_F32, ACT_NONE, 0.5f, L.ff2_b2, x, d, OUT_H, 0,
                    st, "gemm_ffn", err));
  // norm_out (+ next layer's norm_feed_forward1 in the same pass)
  const bool last = li + 1 == c.n_layers;
  const LayerWeights* N = last ? nullptr : &w_.layers[li + 1];
  PKC_ST(ln(L.ln_out_g, L.ln_out_b, last ? nullptr : N->ln_ff1_g, last ? nullptr : N->ln_ff1_b, true,
            last ? nullptr : hbuf));
  return PKC_OK;
}

pkc_status DeviceRunner::finish(cudaStream_t st, std::string& err) {
  int h_err = 0;
  PKC_CK(cudaMemcpyAsync(&h_err, err_word_, sizeof(int), cudaMemcpyDeviceToHost, st), "error word read");
  PKC_CK(cudaStreamSynchronize(st), "stream synchronize");
  if (h_err != 0) {
    cudaMemsetAsync(err_word_, 0, sizeof(int), st);
    // a launch that gave up may have left stream-K flags raised
    if (sk_flags_) cudaMemsetAsync(sk_flags_, 0, 2 * gemm_sk_flag_count(sk_pairs_) * sizeof(int), st);
    cudaStreamSynchronize(st);
    // codes of the device error word (DevErr in kernels/common.cuh)
    const char* what = h_err == 110   ? "bad shape or capacity"
                       : h_err == 111 ? "non-finite decoder logits"
                                      : "bounded wait timed out";
    err = "kernel reported error " + std::to_string(h_err) + " (" + what + ")";
    return PKC_ERR_KERNEL;
  }
  return PKC_OK;
}

void DeviceRunner::drop_graphs() {
  for (GraphEntry& g : graphs_) {
    if (g.exec) cudaGraphExecDestroy(g.exec);
    for (cudaEvent_t e : g.events) cudaEventDestroy(e);
  }
  graphs_.clear();
}

pkc_status DeviceRunner::run_eager(const Plan& p, cudaStream_t st, bool transpose, std::string& err) {
  cudaGetLastError();  // launch checks below must not see an unrelated earlier error
  if (split_front(p)) return run_two_part(p, st, transpose, err);
  PKC_ST(run_frontend(p, 0, p.B, st, err));
  PKC_ST(run_encoder(p, st, err));
  if (transpose) {
    prof_begin(st);
    PKC_CK(to_channels_first_launch(b_.x, b_.out, cfg_.d_model, t_v_off, t_v, p.B, p.max_v, st), "transpose");
    prof_end(st, "to_channels_first", 0.0, (double)p.M * cfg_.d_model * 8);
  }
  return PKC_OK;
}

pkc_status DeviceRunner::run_graphed(const Plan& p, cudaStream_t st, bool transpose, std::string& err) {
  if (!use_graphs_) return run_eager(p, st, transpose, err);
  GraphEntry* hit = nullptr;
  for (GraphEntry& g : graphs_)
    if (g.key == last_key_ && g.pcm == b_.pcm && g.x == b_.x && g.transpose == transpose && g.prof == prof_on_ &&
        g.io == io_)
      hit = &g;
  if (!hit) {
    GraphEntry ge;
    ge.key = last_key_;
    ge.pcm = b_.pcm;
    ge.x = b_.x;
    ge.transpose = transpose;
    ge.prof = prof_on_;
    ge.io = io_;
    std::vector<ProfRec> saved;
    saved.swap(prof_recs_);
    capture_events_ = &ge.events;
    PKC_CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "graph capture begin");
    pkc_status s = run_eager(p, st, transpose, err);
    cudaGraph_t graph = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(st, &graph);
    capture_events_ = nullptr;
    ge.recs.swap(prof_recs_);
    prof_recs_.swap(saved);
    if (s != PKC_OK || ce != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      for (cudaEvent_t e : ge.events) cudaEventDestroy(e);
      cudaGetLastError();
      if (s == PKC_OK) err = std::string("graph capture: ") + cudaGetErrorString(ce);
      return s != PKC_OK ? s : PKC_ERR_CUDA;
    }
    // kernel nodes of the captured sequence (the launch count of one replay)
    size_t n_nodes = 0;
    if (cudaGraphGetNodes(graph, nullptr, &n_nodes) == cudaSuccess && n_nodes > 0) {
      std::vector<cudaGraphNode_t> nodes(n_nodes);
      if (cudaGraphGetNodes(graph, nodes.data(), &n_nodes) == cudaSuccess)
        for (size_t i = 0; i < n_nodes; ++i) {
          cudaGraphNodeType ty;
          if (cudaGraphNodeGetType(nodes[i], &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) ++ge.kernels;
        }
    }
    const cudaError_t ie = cudaGraphInstantiate(&ge.exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) {
      for (cudaEvent_t e : ge.events) cudaEventDestroy(e);
      err = std::string("graph instantiate: ") + cudaGetErrorString(ie);
      return PKC_ERR_CUDA;
    }
    if (graphs_.size() >= 4) {
      cudaStreamSynchronize(st);
      GraphEntry& old = graphs_.front();
      cudaGraphExecDestroy(old.exec);
      for (cudaEvent_t e : old.events) cudaEventDestroy(e);
      graphs_.erase(graphs_.begin());
    }
    graphs_.push_back(std::move(ge));
    hit = &graphs_.back();
  }
  PKC_CK(cudaGraphLaunch(hit->exec, st), "graph launch");
  last_kernels_ = hit->kernels;
  if (hit->prof) {
    // the graph's event nodes are re-recorded on every replay: read them now
    PKC_CK(cudaStreamSynchronize(st), "profile synchronize");
    for (const ProfRec& r : hit->recs) {
      float ms = 0.f;
      PKC_CK(cudaEventElapsedTime(&ms, r.a, r.b), "profile event read");
      KernelStatAcc& k = prof_classes_[r.cls];
      k.launches += 1;
      k.ms += ms;
      k.flops += r.flops;
      k.bytes += r.bytes;
    }
  }
  return PKC_OK;
}

// Copies of the utterances [b0, b1) between host blocks (host(b), n(b) floats)
// and the device rows dev + off(b) (consecutive utterances are consecutive on
// the device), one cudaMemcpyAsync per run of utterances that are also
// consecutive on the host.
template <typename Host, typename Count, typename Off>
static cudaError_t copy_runs(int b0, int b1, Host host, Count n, Off off, float* dev, cudaMemcpyKind kind,
                             cudaStream_t st) {
  int b = b0;
  while (b < b1) {
    if (n(b) <= 0) {
      ++b;
      continue;
    }
    float* h = host(b);
    size_t len = (size_t)n(b);
    int e = b + 1;
    while (e < b1 && (n(e) <= 0 || host(e) == h + len)) len += (size_t)std::max(0, n(e++));
    float* dv = dev + off(b);
    const cudaError_t r = kind == cudaMemcpyHostToDevice ? cudaMemcpyAsync(dv, h, len * 4, kind, st)
                                                         : cudaMemcpyAsync(h, dv, len * 4, kind, st);
    if (r != cudaSuccess) return r;
    b = e;
  }
  return cudaSuccess;
}

template <typename Dst>
pkc_status DeviceRunner::encode_host_overlapped(const Plan& p, const std::vector<const float*>& pcm, bool cf, Dst dst,
                                                std::string& err) {
  const int d = cfg_.d_model;
  const int bb[3] = {0, p.split_b, p.B};
  cudaStream_t st = stream_;
  // the uploads overwrite the PCM buffer: after everything already on st
  PKC_CK(cudaEventRecord(ev_prior_, st), "upload ordering event");
  PKC_CK(cudaStreamWaitEvent(cs_in_, ev_prior_, 0), "upload ordering wait");
  int gb[kFrontGroups + 1];
  front_groups(p, gb);
  for (int g = 0; g < kFrontGroups; ++g) {
    PKC_CK(copy_runs(
               gb[g], gb[g + 1], [&](int b) { return const_cast<float*>(pcm[b]); }, [&](int b) { return p.S[b]; },
               [&](int b) { return (size_t)p.pcm_off[b]; }, b_.pcm, cudaMemcpyHostToDevice, cs_in_),
           "pcm upload");
    PKC_CK(cudaEventRecord(ev_in_[g], cs_in_), "upload event");
  }
  io_ = true;
  const pkc_status s = run_graphed(p, st, cf, err);
  io_ = false;
  if (s != PKC_OK) {
    cudaStreamSynchronize(cs_in_);
    cudaStreamSynchronize(st);
    return s;
  }
  float* src = cf ? b_.out : b_.x;
  cudaError_t ce = cudaSuccess;
  for (int k = 0; k < 2 && ce == cudaSuccess; ++k) {
    ce = cudaStreamWaitEvent(cs_out_, ev_out_[k], 0);
    if (ce == cudaSuccess)
      ce = copy_runs(
          bb[k], bb[k + 1], dst, [&](int b) { return p.v[b] * d; }, [&](int b) { return (size_t)p.v_off[b] * d; },
          src, cudaMemcpyDeviceToHost, cs_out_);
  }
  const pkc_status fs = finish(st, err);
  const cudaError_t se = cudaStreamSynchronize(cs_out_);
  cudaStreamSynchronize(cs_in_);
  if (fs != PKC_OK) return fs;
  if (ce != cudaSuccess || se != cudaSuccess) {
    err = std::string("output download: ") + cudaGetErrorString(ce != cudaSuccess ? ce : se);
    return PKC_ERR_CUDA;
  }
  return PKC_OK;
}

pkc_status DeviceRunner::encode_pcm_host(const std::vector<const float*>& pcm,
                                         const std::vector<int>& n, int layout, float* host_out,
                                         std::string& err) {
  cudaSetDevice(device_);
  Plan p;
  make_plan(cfg_, n, {}, p);
  cudaStream_t st = stream_;
  PKC_ST(prepare(p, st, err));
  const bool cf = layout == PKC_LAYOUT_CHANNELS_FIRST;
  const int d = cfg_.d_model;
  if (split_front(p))
    return encode_host_overlapped(p, pcm, cf, [&](int b) { return host_out + (size_t)p.v_off[b] * d; }, err);
  for (int b = 0; b < p.B; ++b)
    if (n[b] > 0)
      PKC_CK(cudaMemcpyAsync(b_.pcm + p.pcm_off[b], pcm[b], (size_t)n[b] * 4, cudaMemcpyHostToDevice, st), "pcm upload");
  PKC_ST(run_graphed(p, st, cf, err));
  const float* src = cf ? b_.out : b_.x;
  PKC_CK(cudaMemcpyAsync(host_out, src, (size_t)p.M * d * 4, cudaMemcpyDeviceToHost, st), "output download");
  return finish(st, err);
}

pkc_status DeviceRunner::encode_pcm_host_items(const std::vector<const float*>& pcm, const std::vector<int>& n,
                                               int layout, const std::vector<float*>& item_out, std::string& err) {
  cudaSetDevice(device_);
  Plan p;
  make_plan(cfg_, n, {}, p);
  cudaStream_t st = stream_;
  PKC_ST(prepare(p, st, err));
  const bool cf = layout == PKC_LAYOUT_CHANNELS_FIRST;
  if (split_front(p)) return encode_host_overlapped(p, pcm, cf, [&](int b) { return item_out[b]; }, err);
  for (int b = 0; b < p.B; ++b)
    if (n[b] > 0)
      PKC_CK(cudaMemcpyAsync(b_.pcm + p.pcm_off[b], pcm[b], (size_t)n[b] * 4, cudaMemcpyHostToDevice, st), "pcm upload");
  PKC_ST(run_graphed(p, st, cf, err));
  const int d = cfg_.d_model;
  const float* src = cf ? b_.out : b_.x;
  // every clip's block is contiguous in either layout (rows v_off[b] ..)
  for (int b = 0; b < p.B; ++b)
    if (p.v[b] > 0)
      PKC_CK(cudaMemcpyAsync(item_out[b], src + (size_t)p.v_off[b] * d, (size_t)p.v[b] * d * 4, cudaMemcpyDeviceToHost,
                             st), "output download");
  return finish(st, err);
}

pkc_status DeviceRunner::ensure_aux(size_t bytes, cudaStream_t st, std::string& err) {
  if (bytes <= ctc_ws_bytes_) return PKC_OK;
  cudaStreamSynchronize(st);
  if (ctc_ws_) cudaFree(ctc_ws_);
  ctc_ws_ = nullptr;
  ctc_ws_bytes_ = 0;
  PKC_CK(cudaMalloc(&ctc_ws_, bytes + bytes / 8), "decoder scratch allocation");
  ctc_ws_bytes_ = bytes + bytes / 8;
  return PKC_OK;
}

pkc_status DeviceRunner::transducer_pcm_host(const std::vector<const float*>& pcm, const std::vector<int>& n,
                                             int* tokens, int* n_tok, std::string& err) {
  if (!w_.dec_ok) {
    err = "the model has no transducer decoder";
    return PKC_ERR_UNSUPPORTED;
  }
  cudaSetDevice(device_);
  Plan p;
  make_plan(cfg_, n, {}, p);
  cudaStream_t st = stream_;
  PKC_ST(prepare(p, st, err));
  for (int b = 0; b < p.B; ++b)
    if (n[b] > 0)
      PKC_CK(cudaMemcpyAsync(b_.pcm + p.pcm_off[b], pcm[b], (size_t)n[b] * 4, cudaMemcpyHostToDevice, st), "pcm upload");
  PKC_ST(run_graphed(p, st, false, err));  // x: time-major [M, d]
  const Config& c = cfg_;
  const int M = p.M, B = p.B, d = c.d_model, H = c.pred_hidden, L = c.pred_layers, J = c.joint_hidden;
  const int Jp = w_.dec_jpad, MS = std::max(1, c.max_symbols);
  const int grid = transducer_grid();
  // utterances decoded together (every CTA holds their state in shared memory)
  const int V1 = c.vocab_size + 1, VP = V1 + (int)c.durations.size();
  int BG = std::min(B, transducer_max_batch(H, J, L, VP, grid));
  if (const char* e = std::getenv("PKC_DECODE_GROUP")) BG = std::min(BG, std::max(1, std::atoi(e)));
  if (BG < 1) {
    err = "decoder hidden sizes too large for the decode kernel";
    return PKC_ERR_UNSUPPORTED;
  }
  // token rows: utterance b at rows [v_off[b] * MS, v_off[b+1] * MS)
  size_t sz = 0;
  auto take = [&](size_t bytes) { const size_t o = sz; sz += al(bytes); return o; };
  const size_t o_a = take((size_t)M * 3 * d * 2), o_ep = take((size_t)M * Jp * 4);
  const size_t o_h = take((size_t)2 * L * BG * H * 4), o_c = take((size_t)2 * L * BG * H * 4);
  const size_t o_pp = take((size_t)BG * J * 4), o_part = take(transducer_partial_bytes(grid, BG));
  const size_t o_st = take((size_t)B * 12 * 4 + 64), o_tok = take((size_t)M * MS * 16);
  PKC_ST(ensure_aux(sz, st, err));
  uint8_t* ws = static_cast<uint8_t*>(ctc_ws_);
  // per-utterance state (8 ints each), table (off, len, tok_off, tok_cap), barrier word
  std::vector<int> hs((size_t)B * 12 + 16, 0);
  int* s_t = hs.data();
  int* s_pending = s_t + 5 * B;
  int* s_done = s_t + 6 * B;
  int* s_off = s_t + 8 * B;
  int* s_len = s_t + 9 * B;
  int* s_tok_off = s_t + 10 * B;
  int* s_tok_cap = s_t + 11 * B;
  for (int b = 0; b < B; ++b) {
    s_pending[b] = p.v[b] > 0 ? 1 : 0;
    s_done[b] = p.v[b] > 0 ? 0 : 1;
    s_off[b] = p.v_off[b];
    s_len[b] = p.v[b];
    s_tok_off[b] = p.v_off[b] * MS;
    s_tok_cap[b] = p.v[b] * MS;
  }
  int* d_st = reinterpret_cast<int*>(ws + o_st);
  PKC_CK(cudaMemcpyAsync(d_st, hs.data(), hs.size() * 4, cudaMemcpyHostToDevice, st), "decoder state upload");
  sk_part_ = 0;
  // encoder projection of the joint, every frame: [x_hi|x_hi|x_lo] . [W_hi|W_lo|W_hi]^T + b
  PKC_CK(ctc_split3_launch(b_.x, M, d, ws + o_a, st), "decoder split");
  PKC_ST(gemm(ws + o_a, 3 * d, w_.dec_w_enc, 3 * d, false, M, Jp, 3 * d, EPI_STORE_F32, ACT_NONE, 1.f, w_.dec_b_enc,
              ws + o_ep, Jp, st, "gemm_joint_enc", err));
  int* d_ntok = d_st + 7 * B;
  for (int b0 = 0; b0 < B; b0 += BG) {
    const int nb = std::min(BG, B - b0);
    PKC_CK(cudaMemsetAsync(ws + o_h, 0, (size_t)2 * L * nb * H * 4, st), "decoder state reset");
    PKC_CK(cudaMemsetAsync(ws + o_c, 0, (size_t)2 * L * nb * H * 4, st), "decoder state reset");
    PKC_CK(cudaMemsetAsync(ws + o_part, 0, transducer_key_bytes(nb), st), "decoder key reset");
    PKC_CK(cudaMemsetAsync(d_st + 12 * B, 0, 4, st), "decoder barrier reset");
    TransducerArgs a{};
    a.B = nb; a.H = H; a.L = L; a.J = J; a.V1 = V1; a.D = (int)c.durations.size();
    a.blank = c.blank_id; a.max_symbols = MS;
    int maxv = 0;
    for (int b = b0; b < b0 + nb; ++b) maxv = std::max(maxv, p.v[b]);
    a.max_iters = maxv * (MS + 1) + 4;
    a.embed = w_.dec_embed; a.w_ih = w_.dec_w_ih; a.w_hh = w_.dec_w_hh; a.b_lstm = w_.dec_b;
    a.w_pred = w_.dec_w_pred; a.b_pred = w_.dec_b_pred; a.w_out = w_.dec_w_out; a.b_out = w_.dec_b_out;
    a.durations = w_.dec_durations; a.zeros = w_.dec_zeros; a.gate0 = w_.dec_gate0;
    a.enc_proj = reinterpret_cast<const float*>(ws + o_ep); a.ld_enc = Jp;
    a.item_off = d_st + 8 * B + b0; a.item_len = d_st + 9 * B + b0;
    a.h = reinterpret_cast<float*>(ws + o_h); a.c = reinterpret_cast<float*>(ws + o_c);
    a.pred_proj = reinterpret_cast<float*>(ws + o_pp);
    a.t = d_st + b0; a.sym = d_st + B + b0; a.cur = d_st + 2 * B + b0; a.have_token = d_st + 3 * B + b0;
    a.last_token = d_st + 4 * B + b0; a.pending = d_st + 5 * B + b0; a.done = d_st + 6 * B + b0;
    a.ntok = d_ntok + b0;
    a.bar_count = reinterpret_cast<unsigned int*>(d_st + 12 * B);
    a.keys = reinterpret_cast<unsigned long long*>(ws + o_part);
    a.tokens = reinterpret_cast<int*>(ws + o_tok);
    a.tok_off = d_st + 10 * B + b0; a.tok_cap = d_st + 11 * B + b0;
    a.err = err_word_;
    prof_begin(st);
    PKC_CK(transducer_greedy_launch(a, grid, st), "transducer decode launch");
    prof_end(st, "transducer_decode", 0.0, 0.0);
  }
  PKC_CK(cudaMemcpyAsync(n_tok, d_ntok, (size_t)B * 4, cudaMemcpyDeviceToHost, st), "token count download");
  PKC_CK(cudaMemcpyAsync(tokens, ws + o_tok, (size_t)M * MS * 16, cudaMemcpyDeviceToHost, st), "token download");
  return finish(st, err);
}

pkc_status DeviceRunner::ctc_pcm_host(const std::vector<const float*>& pcm, const std::vector<int>& n,
                                      int* argmax_out, float* maxlp_out, float* logprobs_out, std::string& err) {
  if (!w_.ctc_v1) {
    err = "the model has no CTC head";
    return PKC_ERR_UNSUPPORTED;
  }
  cudaSetDevice(device_);
  Plan p;
  make_plan(cfg_, n, {}, p);
  cudaStream_t st = stream_;
  PKC_ST(prepare(p, st, err));
  for (int b = 0; b < p.B; ++b)
    if (n[b] > 0)
      PKC_CK(cudaMemcpyAsync(b_.pcm + p.pcm_off[b], pcm[b], (size_t)n[b] * 4, cudaMemcpyHostToDevice, st), "pcm upload");
  PKC_ST(run_graphed(p, st, false, err));  // x: time-major [M, d]
  const int M = p.M, d = cfg_.d_model, V1 = w_.ctc_v1, Vp = w_.ctc_vpad;
  const size_t o_a = 0, o_l = al((size_t)M * 3 * d * 2), o_am = o_l + al((size_t)M * Vp * 4),
               o_ml = o_am + al((size_t)M * 4), o_lp = o_ml + al((size_t)M * 4);
  const size_t bytes = o_lp + (logprobs_out ? al((size_t)M * V1 * 4) : 0);
  PKC_ST(ensure_aux(bytes, st, err));
  uint8_t* scratch = static_cast<uint8_t*>(ctc_ws_);
  float* logits = reinterpret_cast<float*>(scratch + o_l);
  int* am = reinterpret_cast<int*>(scratch + o_am);
  float* ml = reinterpret_cast<float*>(scratch + o_ml);
  float* lp = logprobs_out ? reinterpret_cast<float*>(scratch + o_lp) : nullptr;
  sk_part_ = 0;
  pkc_status s = PKC_OK;
  do {
    prof_begin(st);
    cudaError_t e = ctc_split3_launch(b_.x, M, d, scratch + o_a, st);
    prof_end(st, "ctc_split", 0.0, (double)M * d * (4 + 6));
    if (e != cudaSuccess) { err = std::string("ctc split: ") + cudaGetErrorString(e); s = PKC_ERR_CUDA; break; }
    // f16 split operands whatever the model's compute type
    s = gemm(scratch + o_a, 3 * d, w_.ctc_w, 3 * d, false, M, Vp, 3 * d, EPI_STORE_F32, ACT_NONE, 1.f, w_.ctc_b,
             logits, Vp, st, "gemm_ctc", err);
    if (s != PKC_OK) break;
    prof_begin(st);
    e = ctc_rows_launch(logits, M, Vp, V1, am, ml, lp, st);
    prof_end(st, "ctc_rows", 0.0, (double)M * V1 * 4 * (lp ? 3 : 2) + (double)M * 8);
    if (e != cudaSuccess) { err = std::string("ctc rows: ") + cudaGetErrorString(e); s = PKC_ERR_CUDA; break; }
    if ((e = cudaMemcpyAsync(argmax_out, am, (size_t)M * 4, cudaMemcpyDeviceToHost, st)) != cudaSuccess ||
        (e = cudaMemcpyAsync(maxlp_out, ml, (size_t)M * 4, cudaMemcpyDeviceToHost, st)) != cudaSuccess ||
        (lp && (e = cudaMemcpyAsync(logprobs_out, lp, (size_t)M * V1 * 4, cudaMemcpyDeviceToHost, st)) != cudaSuccess)) {
      err = std::string("CTC download: ") + cudaGetErrorString(e);
      s = PKC_ERR_CUDA;
      break;
    }
  } while (false);
  if (s != PKC_OK) {
    cudaStreamSynchronize(st);
    return s;
  }
  return finish(st, err);
}

pkc_status DeviceRunner::encode_pcm_device(const float* d_pcm, const std::vector<int>& n, float* d_out,
                                           cudaStream_t st_in, bool sync, std::string& err) {
  cudaSetDevice(device_);
  Plan p;
  make_plan(cfg_, n, {}, p);
  cudaStream_t st = st_in ? st_in : stream_;
  PKC_ST(prepare(p, st, err));
  float* saved_pcm = b_.pcm;
  float* saved_x = b_.x;
  b_.pcm = const_cast<float*>(d_pcm);
  b_.x = d_out;
  pkc_status s = run_graphed(p, st, false, err);
  b_.pcm = saved_pcm;
  b_.x = saved_x;
  if (s != PKC_OK) return s;
  if (sync) return finish(st, err);
  return PKC_OK;
}

pkc_status DeviceRunner::encode_mel_host(const float* mel, int B, int n_mels, int T_max,
                                         const int* valid_T, int layout, float* host_out,
                                         std::string& err) {
  cudaSetDevice(device_);
  std::vector<int> mt(valid_T, valid_T + B);
  Plan p;
  make_plan(cfg_, {}, mt, p);
  cudaStream_t st = stream_;
  PKC_ST(prepare(p, st, err));
  // the planner sized melbatch for max valid_T; the caller's rows are T_max long
  float* staging = nullptr;
  const size_t bytes = (size_t)B * n_mels * T_max * 4;
  float* dst = b_.melbatch;
  if (T_max != p.max_Tm) {
    PKC_CK(cudaMallocAsync(&staging, bytes, st), "mel staging allocation");
    dst = staging;
  }
  PKC_CK(cudaMemcpyAsync(dst, mel, bytes, cudaMemcpyHostToDevice, st), "mel upload");
  ItemTables t{p.B, t_pcm_off, t_S, t_mel_off, t_Tm, t_mval, t_v1_off, t_v1, t_v2_off, t_v2, t_v_off, t_v};
  PKC_CK(batch_to_packed_launch(dst, n_mels, T_max, b_.logmel, t, p.max_Tm, st), "mel repack");
  if (staging) cudaFreeAsync(staging, st);
  PKC_ST(run_encoder(p, st, err));
  const int d = cfg_.d_model;
  const float* src = b_.x;
  if (layout == PKC_LAYOUT_CHANNELS_FIRST) {
    PKC_CK(to_channels_first_launch(b_.x, b_.out, d, t_v_off, t_v, p.B, p.max_v, st), "transpose");
    src = b_.out;
  }
  PKC_CK(cudaMemcpyAsync(host_out, src, (size_t)p.M * d * 4, cudaMemcpyDeviceToHost, st), "output download");
  return finish(st, err);
}

pkc_status DeviceRunner::mel_host(const std::vector<const float*>& pcm, const std::vector<int>& n,
                                  int T_max, float* host_out, std::string& err) {
  cudaSetDevice(device_);
  Plan p;
  make_plan(cfg_, n, {}, p);
  cudaStream_t st = stream_;
  PKC_ST(prepare(p, st, err));
  for (int b = 0; b < p.B; ++b)
    if (n[b] > 0)
      PKC_CK(cudaMemcpyAsync(b_.pcm + p.pcm_off[b], pcm[b], (size_t)n[b] * 4, cudaMemcpyHostToDevice, st), "pcm upload");
  PKC_ST(run_frontend(p, 0, p.B, st, err));
  const ItemTables t = tables_of(0, p.B);
  PKC_CK(mel_to_batch_launch(b_.logmel, cfg_.n_mels, T_max, b_.melbatch, t, st), "mel batch");
  PKC_CK(cudaMemcpyAsync(host_out, b_.melbatch, (size_t)p.B * cfg_.n_mels * T_max * 4,
                         cudaMemcpyDeviceToHost, st), "mel download");
  return finish(st, err);
}

}  // namespace pkc
