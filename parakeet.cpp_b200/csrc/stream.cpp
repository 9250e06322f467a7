// Cache-aware streaming encoder on one device (reference: StreamingEncoder,
// src/streaming_encoder.cpp:30-464).
//
// Per stream, on the device:
//   attention cache  per layer [cache_len, 2d] compute-type rows: k | v of the
//                    last cache_len frames. The reference keeps their
//                    normalised attention inputs and projects them again each
//                    chunk; the projection is per row and the same every time,
//                    so the projected rows are kept instead and the QKV GEMM
//                    sees only the chunk's rows
//   conv cache       per layer [K - 1 + Tc, d]: the last K - 1 GLU outputs,
//                    then this chunk's (written there by the GLU GEMM)
// Both are double-buffered: the rows that become the next chunk's cache are
// copied into the other buffer (NeMo update_cache / new_x[:, :, -LP:]), and
// the buffers swap after the chunk.
// Host state: the step number and the count of filled attention-cache rows
// (cache_last_channel_len), which the attention mask reads.
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
  int filled = 0;  // valid rows of the attention cache
  int cur = 0;     // which cache buffer holds the live caches
  int Tc_cap = 0, n_cap = 0;
  int pos_Tc = -1;  // Tc the positional table was made for
  void* kv[2] = {nullptr, nullptr};  // [L][cache_len][2d] each
  void* cv[2] = {nullptr, nullptr};
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  // scratch carve
  float* mel = nullptr;
  void *s1 = nullptr, *s2a = nullptr, *s2b = nullptr, *s3a = nullptr, *s3b = nullptr;
  float* x = nullptr;
  void *hbuf = nullptr, *ffh = nullptr, *qkv = nullptr, *ctx = nullptr, *pe = nullptr, *ptab = nullptr;
  int* d_filled = nullptr;  // the attention-cache fill count the kernels read
  // page-locked staging of the window and the chunk's output (graph replays
  // copy from / to fixed addresses)
  float* h_mel = nullptr;
  float* h_out = nullptr;
  size_t h_mel_cap = 0, h_out_cap = 0;
  // captured chunk graphs by (window frames, chunk frames, live cache buffer)
  struct Graph {
    int n, Tc, cur;
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
  auto* s = new StreamState();
  std::string e;
  if (stream_reset(*s, e) != PKC_OK) {
    err = e;
    stream_destroy(s);
    return nullptr;
  }
  return s;
}

void DeviceRunner::stream_destroy(StreamState* s) {
  if (!s) return;
  s->drop_graphs();
  if (s->d_filled) cudaFree(s->d_filled);
  if (s->h_mel) cudaFreeHost(s->h_mel);
  if (s->h_out) cudaFreeHost(s->h_out);
  for (int i = 0; i < 2; ++i) {
    if (s->kv[i]) cudaFree(s->kv[i]);
    if (s->cv[i]) cudaFree(s->cv[i]);
  }
  if (s->scratch) cudaFree(s->scratch);
  delete s;
}

int DeviceRunner::stream_step_num(const StreamState& s) { return s.step; }

pkc_status DeviceRunner::stream_reset(StreamState& s, std::string& err) {
  cudaSetDevice(device_);
  s.step = 0;
  s.filled = 0;
  s.cur = 0;
  if (!s.d_filled) PKC_CK(cudaMalloc(&s.d_filled, sizeof(int)), "cudaMalloc of the stream counter");
  PKC_CK(cudaMemsetAsync(s.d_filled, 0, sizeof(int), stream_), "stream counter reset");
  for (int i = 0; i < 2; ++i) {
    if (!s.kv[i] && cfg_.stream.cache_len > 0)
      PKC_CK(cudaMalloc(&s.kv[i], (size_t)cfg_.n_layers * cfg_.stream.cache_len * 2 * cfg_.d_model * 2),
             "cudaMalloc of the streaming attention cache");
    if (s.kv[i]) PKC_CK(cudaMemsetAsync(s.kv[i], 0, (size_t)cfg_.n_layers * cfg_.stream.cache_len * 2 * cfg_.d_model * 2, stream_), "stream cache reset");
    if (s.cv[i]) PKC_CK(cudaMemsetAsync(s.cv[i], 0, (size_t)cfg_.n_layers * (cfg_.conv_kernel - 1 + s.Tc_cap) * cfg_.d_model * 2, stream_), "stream cache reset");
  }
  PKC_CK(cudaStreamSynchronize(stream_), "stream reset");
  return PKC_OK;
}

pkc_status DeviceRunner::stream_step(StreamState& s, const float* mel, int n, bool is_last, float* out,
                                     size_t out_cap, int* n_valid, std::string& err) {
  const Config& c = cfg_;
  cudaSetDevice(device_);
  cudaStream_t st = stream_;
  const int F = c.n_mels, C = c.sub_channels, d = c.d_model, FF = c.ff_dim, K = c.conv_kernel;
  const int Lc = c.n_layers, LP = K - 1, cache = c.stream.cache_len;
  const bool bf = c.bf16;
  *n_valid = 0;
  if (n <= 0 || !mel) {
    err = "empty mel window";
    return PKC_ERR_ARG;
  }
  // subsampled lengths of the window (src/streaming_encoder.cpp:351-370)
  const int T1 = half_up(n), T2 = half_up(T1), T3 = half_up(T2);
  const int F1 = c.F1, F2 = c.F2, F3 = c.F3;
  const int drop = s.step != 0 ? c.stream.drop_extra : 0;
  const int Tc = T3 - drop;
  if (Tc <= 0) {  // no output this step (a too-short tail window)
    s.step += 1;
    return PKC_OK;
  }
  const int valid = is_last ? Tc : std::min(c.stream.valid_out_len, Tc);
  if (out_cap < (size_t)valid * d) {
    err = "output buffer holds " + std::to_string(out_cap) + " floats, the chunk needs " + std::to_string((size_t)valid * d);
    return PKC_ERR_ARG;
  }
  const int Tk = cache + Tc, P = 2 * Tk - 1;

  // ---- capacity: caches keep their rows when they grow
  if (Tc > s.Tc_cap) {
    const int cap = std::max(Tc, 8);
    for (int i = 0; i < 2; ++i) {  // the conv caches hold the chunk's GLU rows too: they grow with Tc
      void* nc = nullptr;
      const size_t cb = (size_t)Lc * (LP + cap) * d * 2;
      PKC_CK(cudaMalloc(&nc, cb), "cudaMalloc of the streaming conv cache");
      PKC_CK(cudaMemsetAsync(nc, 0, cb, st), "stream cache init");
      if (s.cv[i]) {
        PKC_CK(cudaMemcpy2DAsync(nc, (size_t)(LP + cap) * d * 2, s.cv[i], (size_t)(LP + s.Tc_cap) * d * 2,
                                 (size_t)LP * d * 2, Lc, cudaMemcpyDeviceToDevice, st), "stream cache move");
        PKC_CK(cudaStreamSynchronize(st), "stream cache move");
        cudaFree(s.cv[i]);
      }
      s.cv[i] = nc;
    }
    s.Tc_cap = cap;
    s.drop_graphs();
  }
  const int cap = s.Tc_cap;
  const int Tkc = std::max(cap, Tc) + cache, Pc = 2 * Tkc - 1;
  {
    size_t sz = 0;
    auto take = [&](size_t b) { const size_t o = sz; sz += al256(b); return o; };
    const size_t o_mel = take((size_t)F * n * 4), o_s1 = take((size_t)T1 * F1 * C * 2),
                 o_s2a = take((size_t)T2 * F2 * C * 2), o_s2b = take((size_t)T2 * F2 * C * 2),
                 o_s3a = take((size_t)T3 * F3 * C * 2), o_s3b = take((size_t)T3 * F3 * C * 2),
                 o_x = take((size_t)T3 * d * 4), o_h = take((size_t)cap * d * 2), o_ff = take((size_t)cap * FF * 2),
                 o_qkv = take((size_t)Lc * cap * 3 * d * 2), o_ctx = take((size_t)cap * d * 2), o_pe = take((size_t)Pc * d * 2),
                 o_pt = take((size_t)Pc * Lc * d * 2);
    if (sz > s.scratch_bytes) {
      if (s.scratch) cudaFree(s.scratch);
      s.scratch = nullptr;
      s.scratch_bytes = 0;
      PKC_CK(cudaMalloc(&s.scratch, sz), "cudaMalloc of the streaming scratch");
      s.scratch_bytes = sz;
      s.pos_Tc = -1;
      s.drop_graphs();
    }
    uint8_t* b = static_cast<uint8_t*>(s.scratch);
    s.mel = reinterpret_cast<float*>(b + o_mel);
    s.s1 = b + o_s1; s.s2a = b + o_s2a; s.s2b = b + o_s2b; s.s3a = b + o_s3a; s.s3b = b + o_s3b;
    s.x = reinterpret_cast<float*>(b + o_x);
    s.hbuf = b + o_h; s.ffh = b + o_ff; s.qkv = b + o_qkv; s.ctx = b + o_ctx;
    void* pe = b + o_pe;
    void* pt = b + o_pt;
    if (pe != s.pe || pt != s.ptab || s.mel != reinterpret_cast<float*>(b + o_mel)) {
      s.pos_Tc = -1;
      s.drop_graphs();
    }
    s.pe = pe;
    s.ptab = pt;
  }
  if ((size_t)F * n > s.h_mel_cap || (size_t)T3 * d > s.h_out_cap) {
    s.drop_graphs();
    if (s.h_mel) cudaFreeHost(s.h_mel);
    if (s.h_out) cudaFreeHost(s.h_out);
    s.h_mel = s.h_out = nullptr;
    s.h_mel_cap = s.h_out_cap = 0;
    const size_t mc = std::max((size_t)F * n, (size_t)F * 64), oc = std::max((size_t)T3 * d, (size_t)16 * d);
    PKC_CK(cudaMallocHost(&s.h_mel, mc * 4), "page-locked mel staging");
    PKC_CK(cudaMallocHost(&s.h_out, oc * 4), "page-locked output staging");
    s.h_mel_cap = mc;
    s.h_out_cap = oc;
  }
  sk_part_ = 0;
  cudaGetLastError();

  // positional table over cache + chunk positions and every layer's
  // linear_pos: outside the graphs, only when the chunk length changes
  const int Ld = Lc * d;
  if (s.pos_Tc != Tc) {
    PKC_CK(pos_table_launch(s.pe, Tk, d, bf, st), "pos_table");
    PKC_ST(gemm(s.pe, d, w_.pos_all_w, d, bf, P, Ld, d, EPI_STORE_H, ACT_NONE, 1.f, nullptr, s.ptab, Ld, st,
                "stream_pos", err, &w_.pos_all_q));
    s.pos_Tc = Tc;
  }
  std::memcpy(s.h_mel, mel, (size_t)F * n * 4);
  StreamState::Graph* hit = nullptr;
  for (StreamState::Graph& g : s.graphs)
    if (g.n == n && g.Tc == Tc && g.cur == s.cur) hit = &g;
  if (use_graphs_ && !hit) {
    cudaGraph_t graph = nullptr;
    PKC_CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "graph capture begin");
    const pkc_status ps = stream_issue(s, n, Tc, drop, err);
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
    if (s.graphs.size() >= 8) {
      cudaStreamSynchronize(st);
      cudaGraphExecDestroy(s.graphs.front().exec);
      s.graphs.erase(s.graphs.begin());
    }
    s.graphs.push_back({n, Tc, s.cur, exec});
    hit = &s.graphs.back();
  }
  if (hit) {
    PKC_CK(cudaGraphLaunch(hit->exec, st), "stream graph launch");
  } else {
    PKC_ST(stream_issue(s, n, Tc, drop, err));
  }
  PKC_ST(finish(st, err));
  std::memcpy(out, s.h_out, (size_t)valid * d * 4);
  s.cur = 1 - s.cur;
  s.filled = std::min(cache, s.filled + Tc);
  s.step += 1;
  *n_valid = valid;
  return PKC_OK;
}

// One chunk's device work on the runner's stream, from the page-locked window
// to the page-locked output (captured into a graph per shape).
pkc_status DeviceRunner::stream_issue(StreamState& s, int n, int Tc, int drop, std::string& err) {
  // chunk GEMMs have a few rows: the skinny kernel streams each weight once
  // across every SM (the offline encoder keeps tcgen05 tiles for every M)
  struct Skinny {
    bool& f;
    explicit Skinny(bool& x) : f(x) { f = true; }
    ~Skinny() { f = false; }
  } skinny(skinny_ok_);
  const Config& c = cfg_;
  cudaStream_t st = stream_;
  const int F = c.n_mels, C = c.sub_channels, d = c.d_model, FF = c.ff_dim, H = c.n_heads, K = c.conv_kernel;
  const int Lc = c.n_layers, LP = K - 1, cache = c.stream.cache_len, Ld = Lc * d;
  const bool bf = c.bf16;
  const int T1 = half_up(n), T2 = half_up(T1), T3 = half_up(T2);
  const int F1 = c.F1, F2 = c.F2, F3 = c.F3;
  const int cap = s.Tc_cap;

  // ---- causal subsampling (the window is all real audio: no time mask bites)
  PKC_CK(cudaMemcpyAsync(s.mel, s.h_mel, (size_t)F * n * 4, cudaMemcpyHostToDevice, st), "mel upload");
  auto* s1 = static_cast<__nv_bfloat16*>(s.s1);
  PKC_CK(causal_conv0_launch(s.mel, F, n, n, w_.c0_w, w_.c0_b, C, T1, F1, s1, st), "causal conv0");
  PKC_CK(causal_dw_launch(s1, T1, F1, T1, w_.dw1_w, w_.dw1_b, C, T2, F2, static_cast<__nv_bfloat16*>(s.s2a), st),
         "causal dw1");
  PKC_ST(gemm(s.s2a, C, w_.pw1_w, C, true, T2 * F2, C, C, EPI_STORE_H, ACT_RELU, 1.f, w_.pw1_b, s.s2b, C, st,
              "stream_sub_pw", err));
  PKC_CK(causal_dw_launch(static_cast<const __nv_bfloat16*>(s.s2b), T2, F2, T2, w_.dw2_w, w_.dw2_b, C, T3, F3,
                          static_cast<__nv_bfloat16*>(s.s3a), st), "causal dw2");
  PKC_ST(gemm(s.s3a, C, w_.pw2_w, C, true, T3 * F3, C, C, EPI_STORE_H, ACT_RELU, 1.f, w_.pw2_b, s.s3b, C, st,
              "stream_sub_pw", err));
  const float xs = c.xscaling ? std::sqrt((float)d) : 1.f;
  PKC_ST(gemm(s.s3b, F3 * C, w_.out_w, F3 * C, true, T3, d, F3 * C, EPI_STORE_F32, ACT_NONE, xs, w_.out_b, s.x, d,
              st, "stream_sub_out", err));
  float* x = s.x + (size_t)drop * d;  // drop_extra_pre_encoded leading frames

  // ---- conformer layers with their caches (build_stream_layer, :98-338)
  const size_t kv_rows = (size_t)cache, cv_rows = (size_t)LP + cap;
  for (int li = 0; li < Lc; ++li) {
    const LayerWeights& L = w_.layers[li];
    uint8_t* kvc = cache ? static_cast<uint8_t*>(s.kv[s.cur]) + (size_t)li * kv_rows * 2 * d * 2 : nullptr;
    uint8_t* cvc = static_cast<uint8_t*>(s.cv[s.cur]) + (size_t)li * cv_rows * d * 2;
    // x -> LayerNorm(g, b) -> GEMM: the norm inside the skinny GEMM's staging
    // when it can run there (few rows, 16-bit weight), else its own kernel
    auto ln_gemm = [&](const float* g, const float* b, const void* W, const QWeight* q, int N, int epi, int act,
                       float alpha, const float* bias, void* out, int ldo, const char* name) -> pkc_status {
      if (Tc <= 16 && !(q && q->type)) return gemm_skinny_ln(x, d, g, b, W, bf, Tc, N, d, epi, act, alpha, bias, out, ldo, st, err);
      PKC_CK(layernorm_launch(x, Tc, d, g, b, s.hbuf, bf, nullptr, nullptr, false, st), "ln");
      return gemm(s.hbuf, d, W, d, bf, Tc, N, d, epi, act, alpha, bias, out, ldo, st, name, err, q);
    };
    PKC_ST(ln_gemm(L.ln_ff1_g, L.ln_ff1_b, L.ff1_w1, &L.ff1_q1, FF, EPI_STORE_H, ACT_SILU, 1.f, L.ff1_b1, s.ffh, FF,
                   "stream_ffn"));
    PKC_ST(gemm(s.ffh, FF, L.ff1_w2, FF, bf, Tc, d, FF, EPI_RESID_F32, ACT_NONE, 0.5f, L.ff1_b2, x, d, st,
                "stream_ffn", err, &L.ff1_q2));
    // q | k | v of the chunk's frames; k | v of the cached frames are in kvc
    // (each layer keeps its own qkv rows: the cache roll after the last layer reads them)
    uint8_t* qkv = static_cast<uint8_t*>(s.qkv) + (size_t)li * cap * 3 * d * 2;
    PKC_ST(ln_gemm(L.ln_att_g, L.ln_att_b, L.qkv_w, &L.qkv_q, 3 * d, EPI_STORE_H, ACT_NONE, 1.f, L.qkv_b, qkv, 3 * d,
                   "stream_qkv"));
    StreamAttnArgs sa{qkv, kvc, static_cast<const uint8_t*>(s.ptab) + (size_t)li * d * 2, Ld, L.pos_u, L.pos_v,
                      s.ctx, d, H, Tc, cache, s.d_filled, c.att_left, c.att_right};
    PKC_CK(stream_attention_launch(sa, bf, st), "stream attention");
    PKC_ST(gemm(s.ctx, d, L.out_w, d, bf, Tc, d, d, EPI_RESID_F32, ACT_NONE, 1.f, L.out_b, x, d, st, "stream_out",
                err, &L.out_q));
    // conv module: GLU rows after the conv cache, causal depthwise over both
    PKC_ST(ln_gemm(L.ln_conv_g, L.ln_conv_b, L.pw1_w, nullptr, 2 * d, EPI_GLU_H, ACT_NONE, 1.f, L.pw1_b,
                   cvc + (size_t)LP * d * 2, d, "stream_pw1_glu"));
    PKC_CK(stream_dwconv_launch(cvc, s.hbuf, Tc, d, K, L.dw_w, L.dw_b, L.bn_scale, L.bn_shift, c.conv_ln, bf, st),
           "stream dwconv");
    PKC_ST(gemm(s.hbuf, d, L.pw2_w, d, bf, Tc, d, d, EPI_RESID_F32, ACT_NONE, 1.f, L.pw2_b, x, d, st, "stream_pw2",
                err));
    PKC_ST(ln_gemm(L.ln_ff2_g, L.ln_ff2_b, L.ff2_w1, &L.ff2_q1, FF, EPI_STORE_H, ACT_SILU, 1.f, L.ff2_b1, s.ffh, FF,
                   "stream_ffn"));
    PKC_ST(gemm(s.ffh, FF, L.ff2_w2, FF, bf, Tc, d, FF, EPI_RESID_F32, ACT_NONE, 0.5f, L.ff2_b2, x, d, st,
                "stream_ffn", err, &L.ff2_q2));
    PKC_CK(layernorm_launch(x, Tc, d, L.ln_out_g, L.ln_out_b, nullptr, bf, nullptr, nullptr, true, st), "ln");
  }
  // every layer's next caches, in one kernel after the last layer
  StreamRollArgs ra{s.kv[s.cur], s.kv[1 - s.cur], s.qkv, cap, s.cv[s.cur], s.cv[1 - s.cur], (int)cv_rows, Lc, d, cache,
                    Tc, LP};
  PKC_CK(stream_roll_launch(ra, st), "stream cache roll");
  PKC_CK(stream_advance_launch(s.d_filled, Tc, cache, st), "stream advance");
  PKC_CK(cudaMemcpyAsync(s.h_out, x, (size_t)Tc * d * 4, cudaMemcpyDeviceToHost, st), "stream output download");
  return PKC_OK;
}

}  // namespace pkc
