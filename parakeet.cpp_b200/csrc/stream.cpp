// Cache-aware streaming encoder on one device (reference: StreamingEncoder,
// src/streaming_encoder.cpp:30-464), for one stream or several stepped
// together.
//
// Per stream, on the device (double-buffered: a chunk reads one buffer and
// writes the next caches into the other):
//   attention cache  per layer [cache_len, 2d]: k | v of the last cache_len
//                    frames. The reference keeps their normalised attention
//                    inputs and projects them again each chunk; the
//                    projection is per row and the same every time, so the
//                    projected rows are kept and the QKV GEMM sees only the
//                    chunk's rows
//   conv cache       per layer [K - 1, d]: the last K - 1 GLU outputs
//   fill count       frames of the attention cache filled so far
//                    (cache_last_channel_len), which the attention mask reads
// A batched step stacks the S streams' windows and chunk frames along the
// rows: the GEMMs see S * Tc rows (each weight read once for all streams) and
// the attention, depthwise and cache kernels reach each stream's caches through
// device tables of per-stream pointers. The chunk's device work is captured as
// a CUDA graph per (streams, window frames, chunk frames); the tables, the
// windows and the outputs go through page-locked staging, so one graph serves
// any set of streams.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "encoder.hpp"
#include "kernels/gemm.h"
#include "kernels/kernels.h"
#include "status.hpp"

namespace pkc {

struct DeviceRunner::StreamState {
  int step = 0;
  int filled = 0;  // valid rows of the attention cache (host copy)
  int cur = 0;     // which cache buffers hold the live caches
  void* kv[2] = {nullptr, nullptr};  // [L][cache_len][2d]
  void* cv[2] = {nullptr, nullptr};  // [L][K - 1][d]
  int* d_filled = nullptr;
};

// Scratch of the chunk step, shared by every stream of this runner.
struct DeviceRunner::StreamScratch {
  void* dev = nullptr;
  size_t bytes = 0;
  int S = -1, n = -1, Tc = -1;  // the shape the carve below was made for
  void** tabs = nullptr;  // device: kv_cur, kv_next, cv_cur, cv_next, filled, each [S]
  float* mel = nullptr;   // right after the tables: one upload carries both
  size_t in_bytes = 0;    // tables + windows
  void *s1 = nullptr, *s2a = nullptr, *s2b = nullptr, *s3a = nullptr, *s3b = nullptr;
  float* x3 = nullptr;  // subsampling output [S * T3, d]
  float* x = nullptr;   // the chunks' frames [S * Tc, d]
  void *hbuf = nullptr, *ffh = nullptr, *ctx = nullptr;
  void* qkv = nullptr;  // [L][S * Tc][3d]
  void* glu = nullptr;  // [L][S * Tc][d]
  void* pe = nullptr;
  void* ptab = nullptr;
  int pos_Tc = -1;        // Tc the positional table was made for
  // page-locked staging: the input mirrors the device's [tables | windows]
  uint8_t* h_in = nullptr;
  float* h_out = nullptr;
  size_t h_in_cap = 0, h_out_cap = 0;
  struct Graph {
    int S, n, Tc;
    cudaGraphExec_t exec;
  };
  std::vector<Graph> graphs;
  void drop_graphs() {
    for (Graph& g : graphs) cudaGraphExecDestroy(g.exec);
    graphs.clear();
  }
};

namespace {
size_t al256(size_t x) { return (x + 255) / 256 * 256; }
int half_up(int n) { return n / 2 + 1; }  // causal k=3, s=2 stage: pads 2 + 1
}  // namespace

pkc_status DeviceRunner::gemm_skinny_ln(const float* x, int ldx, const float* g, const float* b, const void* B,
                                        bool bf16, int M, int N, int K, int epi, int act, float alpha,
                                        const float* bias, void* out, int ldo, cudaStream_t st, std::string& err) {
  GemmArgs a{};
  a.M = M; a.N = N; a.K = K; a.epi = epi; a.act = act; a.alpha = alpha; a.bias = bias;
  a.out = out; a.ldo = ldo; a.err = err_word_; a.skinny = 1;
  a.ln_x = x; a.ln_ldx = ldx; a.ln_g = g; a.ln_b = b;
  PKC_CK(gemm_launch(nullptr, K, B, K, bf16, a, st), "LayerNorm + skinny GEMM");
  return PKC_OK;
}

void DeviceRunner::stream_scratch_free() {
  StreamScratch* x = sscr_;
  if (!x) return;
  cudaSetDevice(device_);
  x->drop_graphs();
  if (x->dev) cudaFree(x->dev);
  if (x->h_in) cudaFreeHost(x->h_in);
  if (x->h_out) cudaFreeHost(x->h_out);
  delete x;
  sscr_ = nullptr;
}

DeviceRunner::StreamState* DeviceRunner::stream_create(std::string& err) {
  const Config& c = cfg_;
  if (!c.stream.present || !c.chunked || !c.causal_downsampling || !c.conv_causal) {
    err = "not a cache-aware streaming model (needs parakeet.streaming.* keys, chunked_limited attention, "
          "causal subsampling and causal conv)";
    return nullptr;
  }
  for (const LayerWeights& L : w_.layers)
    if (L.qkv_ln || L.pw1_ln || L.ff2_ln) {
      err = "streaming needs the unfused LayerNorm weights (PKC_LN_FUSED unset)";
      return nullptr;
    }
  cudaSetDevice(device_);
  auto* s = new StreamState();
  const size_t kb = (size_t)c.n_layers * c.stream.cache_len * 2 * c.d_model * 2;
  const size_t cb = (size_t)c.n_layers * (c.conv_kernel - 1) * c.d_model * 2;
  bool ok = cudaMalloc(&s->d_filled, sizeof(int)) == cudaSuccess;
  for (int i = 0; i < 2 && ok; ++i) {
    if (kb) ok = cudaMalloc(&s->kv[i], kb) == cudaSuccess;
    if (ok && cb) ok = cudaMalloc(&s->cv[i], cb) == cudaSuccess;
  }
  std::string e;
  if (!ok || stream_reset(*s, e) != PKC_OK) {
    err = ok ? e : "cudaMalloc of the stream caches failed";
    stream_destroy(s);
    return nullptr;
  }
  return s;
}

void DeviceRunner::stream_destroy(StreamState* s) {
  if (!s) return;
  for (int i = 0; i < 2; ++i) {
    if (s->kv[i]) cudaFree(s->kv[i]);
    if (s->cv[i]) cudaFree(s->cv[i]);
  }
  if (s->d_filled) cudaFree(s->d_filled);
  delete s;
}

int DeviceRunner::stream_step_num(const StreamState& s) { return s.step; }

pkc_status DeviceRunner::stream_reset(StreamState& s, std::string& err) {
  const Config& c = cfg_;
  cudaSetDevice(device_);
  s.step = 0;
  s.filled = 0;
  s.cur = 0;
  const size_t kb = (size_t)c.n_layers * c.stream.cache_len * 2 * c.d_model * 2;
  const size_t cb = (size_t)c.n_layers * (c.conv_kernel - 1) * c.d_model * 2;
  for (int i = 0; i < 2; ++i) {
    if (s.kv[i]) PKC_CK(cudaMemsetAsync(s.kv[i], 0, kb, stream_), "stream cache reset");
    if (s.cv[i]) PKC_CK(cudaMemsetAsync(s.cv[i], 0, cb, stream_), "stream cache reset");
  }
  PKC_CK(cudaMemsetAsync(s.d_filled, 0, sizeof(int), stream_), "stream counter reset");
  PKC_CK(cudaStreamSynchronize(stream_), "stream reset");
  return PKC_OK;
}

pkc_status DeviceRunner::stream_step(StreamState& s, const float* mel, int n, bool is_last, float* out,
                                     size_t out_cap, int* n_valid, std::string& err) {
  StreamState* ss[1] = {&s};
  const float* mels[1] = {mel};
  const int last[1] = {is_last ? 1 : 0};
  float* outs[1] = {out};
  return stream_step_batch(ss, 1, mels, n, last, outs, out_cap, n_valid, err);
}

pkc_status DeviceRunner::stream_step_batch(StreamState* const* ss, int S, const float* const* mels, int n,
                                           const int* is_last, float* const* outs, size_t out_cap, int* n_valid,
                                           std::string& err) {
  const Config& c = cfg_;
  cudaSetDevice(device_);
  cudaStream_t st = stream_;
  const int F = c.n_mels, C = c.sub_channels, d = c.d_model, FF = c.ff_dim;
  const int Lc = c.n_layers, cache = c.stream.cache_len;
  const bool bf = c.bf16;
  for (int i = 0; i < S; ++i) n_valid[i] = 0;
  if (S <= 0 || n <= 0) {
    err = S <= 0 ? "no streams" : "empty mel window";
    return PKC_ERR_ARG;
  }
  for (int i = 0; i < S; ++i) {
    if (!ss[i] || !mels[i] || !outs[i]) {
      err = "NULL stream, window or output";
      return PKC_ERR_ARG;
    }
    for (int j = 0; j < i; ++j)
      if (ss[j] == ss[i]) {
        err = "a stream appears twice in the batch";
        return PKC_ERR_ARG;
      }
  }
  // the window's leading frames are dropped after a stream's first step, so
  // every stream of a batch must be at its first step or every one past it
  const bool first = ss[0]->step == 0;
  for (int i = 1; i < S; ++i)
    if ((ss[i]->step == 0) != first) {
      err = "the streams of a batch must all be at their first window or all past it";
      return PKC_ERR_ARG;
    }
  // subsampled lengths of the window (src/streaming_encoder.cpp:351-370)
  const int T1 = half_up(n), T2 = half_up(T1), T3 = half_up(T2);
  const int F1 = c.F1, F2 = c.F2, F3 = c.F3;
  const int drop = first ? 0 : c.stream.drop_extra;
  const int Tc = T3 - drop;
  if (Tc <= 0) {  // no output this step (a too-short tail window)
    for (int i = 0; i < S; ++i) ss[i]->step += 1;
    return PKC_OK;
  }
  std::vector<int> valid(S);
  for (int i = 0; i < S; ++i) {
    valid[i] = is_last[i] ? Tc : std::min(c.stream.valid_out_len, Tc);
    if (out_cap < (size_t)valid[i] * d) {
      err = "output buffer holds " + std::to_string(out_cap) + " floats, the chunk needs " +
            std::to_string((size_t)valid[i] * d);
      return PKC_ERR_ARG;
    }
  }
  const int Tk = cache + Tc, P = 2 * Tk - 1, M = S * Tc, Ld = Lc * d;

  // ---- scratch for this shape (the graphs hold its addresses)
  if (!sscr_) sscr_ = new StreamScratch();
  StreamScratch& x = *sscr_;
  {
    size_t sz = 0;
    auto take = [&](size_t b) { const size_t o = sz; sz += al256(b); return o; };
    const size_t tab_b = al256((size_t)5 * S * sizeof(void*)), in_b = tab_b + (size_t)S * F * n * 4;
    const size_t o_in = take(in_b), o_s1 = take((size_t)S * T1 * F1 * C * 2),
                 o_s2a = take((size_t)S * T2 * F2 * C * 2), o_s2b = take((size_t)S * T2 * F2 * C * 2),
                 o_s3a = take((size_t)S * T3 * F3 * C * 2), o_s3b = take((size_t)S * T3 * F3 * C * 2),
                 o_x3 = take((size_t)S * T3 * d * 4), o_x = take((size_t)M * d * 4), o_h = take((size_t)M * d * 2),
                 o_ff = take((size_t)M * FF * 2), o_ctx = take((size_t)M * d * 2),
                 o_qkv = take((size_t)Lc * M * 3 * d * 2), o_glu = take((size_t)Lc * M * d * 2),
                 o_pe = take((size_t)P * d * 2), o_pt = take((size_t)P * Ld * 2);
    if (sz > x.bytes) {
      x.drop_graphs();
      if (x.dev) cudaFree(x.dev);
      x.dev = nullptr;
      x.bytes = 0;
      PKC_CK(cudaMalloc(&x.dev, sz), "cudaMalloc of the streaming scratch");
      x.bytes = sz;
      x.S = -1;
    }
    if (x.S != S || x.n != n || x.Tc != Tc) {  // carve for this shape
      uint8_t* b = static_cast<uint8_t*>(x.dev);
      x.tabs = reinterpret_cast<void**>(b + o_in);
      x.mel = reinterpret_cast<float*>(b + o_in + tab_b);
      x.in_bytes = in_b;
      x.s1 = b + o_s1; x.s2a = b + o_s2a; x.s2b = b + o_s2b; x.s3a = b + o_s3a; x.s3b = b + o_s3b;
      x.x3 = reinterpret_cast<float*>(b + o_x3);
      x.x = reinterpret_cast<float*>(b + o_x);
      x.hbuf = b + o_h; x.ffh = b + o_ff; x.ctx = b + o_ctx; x.qkv = b + o_qkv; x.glu = b + o_glu;
      x.pe = b + o_pe; x.ptab = b + o_pt;
      x.S = S; x.n = n; x.Tc = Tc;
      x.pos_Tc = -1;
    }
  }
  if (x.in_bytes > x.h_in_cap || (size_t)M * d > x.h_out_cap) {
    x.drop_graphs();
    if (x.h_in) cudaFreeHost(x.h_in);
    if (x.h_out) cudaFreeHost(x.h_out);
    x.h_in = nullptr;
    x.h_out = nullptr;
    x.h_in_cap = x.h_out_cap = 0;
    const size_t ic = std::max(x.in_bytes, (size_t)256 + (size_t)F * 64 * 4),
                 oc = std::max((size_t)M * d, (size_t)16 * d);
    PKC_CK(cudaMallocHost(&x.h_in, ic), "page-locked input staging");
    PKC_CK(cudaMallocHost(&x.h_out, oc * 4), "page-locked output staging");
    x.h_in_cap = ic;
    x.h_out_cap = oc;
  }
  sk_part_ = 0;
  cudaGetLastError();

  // positional table over cache + chunk positions and every layer's
  // linear_pos: outside the graphs, only when the chunk length changes
  if (x.pos_Tc != Tc) {
    PKC_CK(pos_table_launch(x.pe, Tk, d, bf, st), "pos_table");
    PKC_ST(gemm(x.pe, d, w_.pos_all_w, d, bf, P, Ld, d, EPI_STORE_H, ACT_NONE, 1.f, nullptr, x.ptab, Ld, st,
                "stream_pos", err, &w_.pos_all_q));
    x.pos_Tc = Tc;
  }
  // staging, laid out as on the device: the per-stream tables (live and
  // next cache buffers, fill counts), then the windows
  void** h_tabs = reinterpret_cast<void**>(x.h_in);
  float* h_mel = reinterpret_cast<float*>(x.h_in + (reinterpret_cast<uint8_t*>(x.mel) -
                                                    reinterpret_cast<uint8_t*>(x.tabs)));
  for (int i = 0; i < S; ++i) {
    const StreamState& s = *ss[i];
    h_tabs[0 * S + i] = s.kv[s.cur];
    h_tabs[1 * S + i] = s.kv[1 - s.cur];
    h_tabs[2 * S + i] = s.cv[s.cur];
    h_tabs[3 * S + i] = s.cv[1 - s.cur];
    h_tabs[4 * S + i] = s.d_filled;
  }
  for (int i = 0; i < S; ++i) std::memcpy(h_mel + (size_t)i * F * n, mels[i], (size_t)F * n * 4);
  StreamScratch::Graph* hit = nullptr;
  for (StreamScratch::Graph& g : x.graphs)
    if (g.S == S && g.n == n && g.Tc == Tc) hit = &g;
  if (use_graphs_ && !hit) {
    cudaGraph_t graph = nullptr;
    PKC_CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "graph capture begin");
    const pkc_status ps = stream_issue(S, n, Tc, drop, err);
    const cudaError_t ce = cudaStreamEndCapture(st, &graph);
    if (ps != PKC_OK || ce != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      cudaGetLastError();
      if (ps == PKC_OK) err = std::string("stream graph capture: ") + cudaGetErrorString(ce);
      return ps != PKC_OK ? ps : PKC_ERR_CUDA;
    }
    cudaGraphExec_t exec = nullptr;
    const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    PKC_CK(ie, "stream graph instantiate");
    if (x.graphs.size() >= 8) {
      cudaStreamSynchronize(st);
      cudaGraphExecDestroy(x.graphs.front().exec);
      x.graphs.erase(x.graphs.begin());
    }
    x.graphs.push_back({S, n, Tc, exec});
    hit = &x.graphs.back();
  }
  if (hit) {
    PKC_CK(cudaGraphLaunch(hit->exec, st), "stream graph launch");
  } else {
    PKC_ST(stream_issue(S, n, Tc, drop, err));
  }
  PKC_ST(finish(st, err));
  for (int i = 0; i < S; ++i) {
    std::memcpy(outs[i], x.h_out + (size_t)i * Tc * d, (size_t)valid[i] * d * 4);
    StreamState& s = *ss[i];
    s.cur = 1 - s.cur;
    s.filled = std::min(cache, s.filled + Tc);
    s.step += 1;
    n_valid[i] = valid[i];
  }
  return PKC_OK;
}

// One chunk step's device work for S streams on the runner's stream, from the
// page-locked windows and tables to the page-locked output (captured into a
// graph per shape).
pkc_status DeviceRunner::stream_issue(int S, int n, int Tc, int drop, std::string& err) {
  // chunk GEMMs have a few rows: the skinny kernel streams each weight once
  // across every SM (the offline encoder keeps tcgen05 tiles for every M)
  struct Skinny {
    bool& f;
    explicit Skinny(bool& v) : f(v) { f = true; }
    ~Skinny() { f = false; }
  } skinny(skinny_ok_);
  const Config& c = cfg_;
  StreamScratch& x = *sscr_;
  cudaStream_t st = stream_;
  const int F = c.n_mels, C = c.sub_channels, d = c.d_model, FF = c.ff_dim, H = c.n_heads, K = c.conv_kernel;
  const int Lc = c.n_layers, LP = K - 1, cache = c.stream.cache_len, Ld = Lc * d;
  const bool bf = c.bf16;
  const int T1 = half_up(n), T2 = half_up(T1), T3 = half_up(T2);
  const int F1 = c.F1, F2 = c.F2, F3 = c.F3;
  const int M = S * Tc;
  void* const* kv_cur = x.tabs;
  void* const* kv_next = x.tabs + S;
  void* const* cv_cur = x.tabs + 2 * S;
  void* const* cv_next = x.tabs + 3 * S;
  int* const* filled = reinterpret_cast<int* const*>(x.tabs + 4 * S);

  PKC_CK(cudaMemcpyAsync(x.tabs, x.h_in, x.in_bytes, cudaMemcpyHostToDevice, st), "stream table and window upload");
  // ---- causal subsampling (each window is all real audio: no time mask bites)
  auto* s1 = static_cast<__nv_bfloat16*>(x.s1);
  PKC_CK(causal_conv0_launch(x.mel, S, F, n, n, w_.c0_w, w_.c0_b, C, T1, F1, s1, st), "causal conv0");
  PKC_CK(causal_dw_launch(s1, S, T1, F1, T1, w_.dw1_w, w_.dw1_b, C, T2, F2, static_cast<__nv_bfloat16*>(x.s2a), st),
         "causal dw1");
  PKC_ST(gemm(x.s2a, C, w_.pw1_w, C, true, S * T2 * F2, C, C, EPI_STORE_H, ACT_RELU, 1.f, w_.pw1_b, x.s2b, C, st,
              "stream_sub_pw", err));
  PKC_CK(causal_dw_launch(static_cast<const __nv_bfloat16*>(x.s2b), S, T2, F2, T2, w_.dw2_w, w_.dw2_b, C, T3, F3,
                          static_cast<__nv_bfloat16*>(x.s3a), st), "causal dw2");
  PKC_ST(gemm(x.s3a, C, w_.pw2_w, C, true, S * T3 * F3, C, C, EPI_STORE_H, ACT_RELU, 1.f, w_.pw2_b, x.s3b, C, st,
              "stream_sub_pw", err));
  const float xs = c.xscaling ? std::sqrt((float)d) : 1.f;
  PKC_ST(gemm(x.s3b, F3 * C, w_.out_w, F3 * C, true, S * T3, d, F3 * C, EPI_STORE_F32, ACT_NONE, xs, w_.out_b, x.x3,
              d, st, "stream_sub_out", err));
  // each stream's chunk frames (after its drop_extra_pre_encoded leading
  // ones), stacked; one stream's, or undropped ones, are stacked already
  float* xa = x.x3 + (size_t)drop * d;
  if (S > 1 && drop > 0) {
    PKC_CK(cudaMemcpy2DAsync(x.x, (size_t)Tc * d * 4, x.x3 + (size_t)drop * d, (size_t)T3 * d * 4,
                             (size_t)Tc * d * 4, S, cudaMemcpyDeviceToDevice, st), "chunk frames");
    xa = x.x;
  }

  // ---- conformer layers with their caches (build_stream_layer, :98-338)
  for (int li = 0; li < Lc; ++li) {
    const LayerWeights& L = w_.layers[li];
    // x -> LayerNorm(g, b) -> GEMM: the norm inside the skinny GEMM's staging
    // when it can run there (few rows, 16-bit weight), else its own kernel
    auto ln_gemm = [&](const float* g, const float* b, const void* W, const QWeight* q, int N, int epi, int act,
                       float alpha, const float* bias, void* out, int ldo, const char* name) -> pkc_status {
      if (M <= 16 && !(q && q->type))
        return gemm_skinny_ln(xa, d, g, b, W, bf, M, N, d, epi, act, alpha, bias, out, ldo, st, err);
      PKC_CK(layernorm_launch(xa, M, d, g, b, x.hbuf, bf, nullptr, nullptr, false, st), "ln");
      return gemm(x.hbuf, d, W, d, bf, M, N, d, epi, act, alpha, bias, out, ldo, st, name, err, q);
    };
    PKC_ST(ln_gemm(L.ln_ff1_g, L.ln_ff1_b, L.ff1_w1, &L.ff1_q1, FF, EPI_STORE_H, ACT_SILU, 1.f, L.ff1_b1, x.ffh, FF,
                   "stream_ffn"));
    PKC_ST(gemm(x.ffh, FF, L.ff1_w2, FF, bf, M, d, FF, EPI_RESID_F32, ACT_NONE, 0.5f, L.ff1_b2, xa, d, st,
                "stream_ffn", err, &L.ff1_q2));
    // q | k | v of the chunks' frames (each layer keeps its rows: the cache
    // roll after the last layer reads them); k | v of the cached frames are
    // in each stream's cache
    uint8_t* qkv = static_cast<uint8_t*>(x.qkv) + (size_t)li * M * 3 * d * 2;
    PKC_ST(ln_gemm(L.ln_att_g, L.ln_att_b, L.qkv_w, &L.qkv_q, 3 * d, EPI_STORE_H, ACT_NONE, 1.f, L.qkv_b, qkv, 3 * d,
                   "stream_qkv"));
    StreamAttnArgs sa{qkv, kv_cur, (size_t)li * cache * 2 * d, filled,
                      static_cast<const uint8_t*>(x.ptab) + (size_t)li * d * 2, Ld, L.pos_u, L.pos_v, x.ctx,
                      d, H, Tc, cache, S, c.att_left, c.att_right};
    PKC_CK(stream_attention_launch(sa, bf, st), "stream attention");
    PKC_ST(gemm(x.ctx, d, L.out_w, d, bf, M, d, d, EPI_RESID_F32, ACT_NONE, 1.f, L.out_b, xa, d, st, "stream_out",
                err, &L.out_q));
    // conv module: causal depthwise over [conv cache | the chunk's GLU rows]
    uint8_t* glu = static_cast<uint8_t*>(x.glu) + (size_t)li * M * d * 2;
    PKC_ST(ln_gemm(L.ln_conv_g, L.ln_conv_b, L.pw1_w, nullptr, 2 * d, EPI_GLU_H, ACT_NONE, 1.f, L.pw1_b, glu, d,
                   "stream_pw1_glu"));
    StreamConvArgs ca{cv_cur, (size_t)li * LP * d, glu, x.hbuf, L.dw_w, L.dw_b, L.bn_scale, L.bn_shift,
                      d, K, Tc, S, c.conv_ln ? 1 : 0};
    PKC_CK(stream_dwconv_launch(ca, bf, st), "stream dwconv");
    PKC_ST(gemm(x.hbuf, d, L.pw2_w, d, bf, M, d, d, EPI_RESID_F32, ACT_NONE, 1.f, L.pw2_b, xa, d, st, "stream_pw2",
                err));
    PKC_ST(ln_gemm(L.ln_ff2_g, L.ln_ff2_b, L.ff2_w1, &L.ff2_q1, FF, EPI_STORE_H, ACT_SILU, 1.f, L.ff2_b1, x.ffh, FF,
                   "stream_ffn"));
    PKC_ST(gemm(x.ffh, FF, L.ff2_w2, FF, bf, M, d, FF, EPI_RESID_F32, ACT_NONE, 0.5f, L.ff2_b2, xa, d, st,
                "stream_ffn", err, &L.ff2_q2));
    PKC_CK(layernorm_launch(xa, M, d, L.ln_out_g, L.ln_out_b, nullptr, bf, nullptr, nullptr, true, st), "ln");
  }
  // every layer's and stream's next caches, in one kernel after the last layer
  StreamRollArgs ra{kv_cur, kv_next, cv_cur, cv_next, x.qkv, x.glu, M, Lc, d, cache, Tc, LP, S};
  PKC_CK(stream_roll_launch(ra, st), "stream cache roll");
  PKC_CK(stream_advance_launch(filled, S, Tc, cache, st), "stream advance");
  PKC_CK(cudaMemcpyAsync(x.h_out, xa, (size_t)M * d * 4, cudaMemcpyDeviceToHost, st), "stream output download");
  return PKC_OK;
}

}  // namespace pkc
