// GGUF -> device weights. Every tensor is converted once at load into the
// layout its kernel reads (reference counterpart: ModelLoader::realize_weights,
// src/model_loader.cpp:47-98, which uploads ggml tensors unchanged).
//
// Re-packing done here:
//   * linear weights -> the layer compute type (f16, or bf16 for bf16 GGUFs);
//     f32 / q8_0 / q4_k weights are dequantised on the host and rounded once
//   * q, k, v projections concatenated into one [3d, d] weight (one GEMM)
//   * pointwise_conv1 rows paired for the GLU epilogue: within each 256-row
//     tile, rows [0,128) are value channels 128t.. and rows [128,256) the
//     gate channels of the same 128 channels (F.glu: value = first half)
//   * BatchNorm folded to f32 scale/shift exactly as src/conformer.cpp:134-154
//   * depthwise weights transposed to tap-major [K][d] for coalesced reads
//   * subsampling pointwise convs and output linear in bf16 (their activations
//     are bf16: random-init magnitudes there fall below f16's normal range);
//     the output linear's columns permuted from c*F' + f (the reference's
//     channel-major flatten, src/subsampling.cpp:194-202) to f*C + c
//   * the mel DFT basis split into f16 hi/lo parts, [Bhi | Blo | Bhi], with
//     cos/-sin rows of each 128-bin group paired for the POWER epilogue
#include "model.hpp"

#include <algorithm>
#include <chrono>
#include <climits>
#include <cstdio>
#include <type_traits>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <thread>

#include <sys/stat.h>
#include <unistd.h>

#include "half.hpp"
#include "kernels/kernels.h"

namespace pkc {

namespace {

int conv_len(int n) { return (n + 2 - 3) / 2 + 1; }

struct Staging {
  std::vector<uint8_t> buf;
  size_t add(const void* src, size_t n) {
    const size_t off = (buf.size() + 255) / 256 * 256;
    buf.resize(off + n);
    if (src) std::memcpy(buf.data() + off, src, n);
    return off;
  }
};

// Offsets are carried in the pointer fields until the arena exists.
template <typename T>
T* as_off(size_t off) { return reinterpret_cast<T*>(off + 1); }  // +1: 0 means "absent"
template <typename T>
void reloc(T*& p, uint8_t* base) {
  if (p) p = reinterpret_cast<T*>(base + (reinterpret_cast<uintptr_t>(p) - 1));
}

}  // namespace

// Every field of the weight tables that the arena layout defines, in a fixed
// order: the pointer fields (arena offsets + 1 before upload, device addresses
// after) and the sizes and flags beside them. Relocation and the pack cache
// both walk this one list.
template <class F>
void for_each_layer_field(LayerWeights& L, F&& f) {
  f(L.ln_ff1_g); f(L.ln_ff1_b); f(L.ln_att_g); f(L.ln_att_b); f(L.ln_conv_g); f(L.ln_conv_b);
  f(L.ln_ff2_g); f(L.ln_ff2_b); f(L.ln_out_g); f(L.ln_out_b);
  f(L.ff1_w1); f(L.ff1_w2); f(L.ff2_w1); f(L.ff2_w2); f(L.ff1_b1); f(L.ff1_b2); f(L.ff2_b1); f(L.ff2_b2);
  f(L.qkv_w); f(L.qkv_b); f(L.pos_w); f(L.out_w); f(L.out_b); f(L.pos_u); f(L.pos_v);
  f(L.pw1_w); f(L.pw1_b); f(L.dw_w); f(L.dw_b); f(L.bn_scale); f(L.bn_shift); f(L.pw2_w); f(L.pw2_b);
  for (QWeight* q : {&L.ff1_q1, &L.ff1_q2, &L.ff2_q1, &L.ff2_q2, &L.qkv_q, &L.out_q}) {
    f(q->type); f(q->q); f(q->s0); f(q->s1);
  }
  f(L.qkv_ln); f(L.pw1_ln); f(L.ff2_ln);
}

template <class F>
void for_each_top_field(DeviceWeights& w, F&& f) {
  f(w.arena_bytes);
  f(w.window); f(w.dft_basis); f(w.fb_start); f(w.fb_len); f(w.fb_off); f(w.fb_w);
  f(w.c0_w); f(w.c0_b); f(w.dw1_w); f(w.dw1_b); f(w.dw2_w); f(w.dw2_b);
  f(w.pw1_w); f(w.pw2_w); f(w.pw1_b); f(w.pw2_b); f(w.out_w); f(w.out_b);
  f(w.pos_all_w); f(w.pos_all_q.type); f(w.pos_all_q.q); f(w.pos_all_q.s0); f(w.pos_all_q.s1);
  f(w.ctc_w); f(w.ctc_b); f(w.ctc_v1); f(w.ctc_vpad);
  f(w.dec_ok); f(w.dec_embed); f(w.dec_w_ih); f(w.dec_w_hh); f(w.dec_b); f(w.dec_w_pred); f(w.dec_b_pred);
  f(w.dec_w_out); f(w.dec_b_out); f(w.dec_durations); f(w.dec_zeros); f(w.dec_gate0); f(w.dec_w_enc);
  f(w.dec_b_enc); f(w.dec_jpad);
}

template <class F>
void for_each_field(DeviceWeights& w, F&& f) {
  for_each_top_field(w, f);
  for (LayerWeights& L : w.layers) for_each_layer_field(L, f);
}

namespace {

void parallel_rows(int64_t n, const std::function<void(int64_t, int64_t)>& fn) {
  const int nt = (int)std::min<int64_t>(std::max(1u, std::thread::hardware_concurrency()),
                                        std::max<int64_t>(1, n / 64));
  if (nt <= 1) { fn(0, n); return; }
  std::vector<std::thread> th;
  for (int i = 0; i < nt; ++i) {
    const int64_t a = n * i / nt, b = n * (i + 1) / nt;
    th.emplace_back([&fn, a, b] { fn(a, b); });
  }
  for (auto& t : th) t.join();
}

// Read tensor `name` as a row-major f32 [N][K] matrix.
bool read_f32(const GgufFile& g, const std::string& name, int64_t N, int64_t K,
              std::vector<float>& out, std::string& err) {
  const GgufTensor* t = g.tensor(name);
  if (!t) { err = "missing tensor " + name; return false; }
  if (t->nelem() != N * K) {
    err = "tensor " + name + " has " + std::to_string(t->nelem()) + " elements, expected " +
          std::to_string(N * K);
    return false;
  }
  const bool plain = t->type == GT_F32 || t->type == GT_F16 || t->type == GT_BF16;
  if (!plain && t->ne[0] != K) { err = "quantised tensor " + name + " is not K-major"; return false; }
  const size_t rb = ggml_row_bytes(t->type, K);
  if (!rb) { err = "tensor " + name + ": unsupported GGML type " + std::to_string(t->type); return false; }
  out.resize((size_t)(N * K));
  bool ok = true;
  parallel_rows(N, [&](int64_t a, int64_t b) {
    for (int64_t r = a; r < b; ++r)
      if (!ggml_to_f32(t->type, t->data + rb * r, K, out.data() + r * K)) ok = false;
  });
  if (!ok) err = "tensor " + name + ": conversion failed";
  return ok;
}

bool read_vec(const GgufFile& g, const std::string& name, int64_t n, std::vector<float>& out,
              std::string& err) {
  return read_f32(g, name, 1, n, out, err);
}

// Convert f32 rows to 16-bit (f16 or bf16) words.
std::vector<uint16_t> to_h(const std::vector<float>& v, bool bf16) {
  std::vector<uint16_t> h(v.size());
  parallel_rows((int64_t)v.size(), [&](int64_t a, int64_t b) {
    for (int64_t i = a; i < b; ++i) h[i] = bf16 ? f32_to_bf16(v[i]) : f32_to_f16(v[i]);
  });
  return h;
}

// f32 rows [N][K] -> f16 rows [N][2K] = [hi | lo] with hi = f16(w) and
// lo = f16(w - hi): the split-f16 form of the f32-accurate path.
std::vector<uint16_t> to_split(const std::vector<float>& v, int64_t N, int64_t K) {
  std::vector<uint16_t> h((size_t)(N * 2 * K));
  parallel_rows(N, [&](int64_t a, int64_t b) {
    for (int64_t n = a; n < b; ++n)
      for (int64_t k = 0; k < K; ++k) {
        const float x = v[(size_t)(n * K + k)];
        const uint16_t hi = f32_to_f16(x);
        h[(size_t)(n * 2 * K + k)] = hi;
        h[(size_t)(n * 2 * K + K + k)] = f32_to_f16(x - f16_to_f32(hi));
      }
  });
  return h;
}

// Linear weight [N][K] in the target 16-bit type; bytes copied verbatim when
// the GGUF already stores that type.
bool read_h(const GgufFile& g, const std::string& name, int64_t N, int64_t K, bool bf16,
            std::vector<uint16_t>& out, std::string& err) {
  const GgufTensor* t = g.tensor(name);
  if (t && t->nelem() == N * K && ((t->type == GT_F16 && !bf16) || (t->type == GT_BF16 && bf16))) {
    out.resize((size_t)(N * K));
    std::memcpy(out.data(), t->data, out.size() * 2);
    return true;
  }
  std::vector<float> f;
  if (!read_f32(g, name, N, K, f, err)) return false;
  out = to_h(f, bf16);
  return true;
}

// A block-quantised [N][K] weight repacked for the in-kernel dequantising GEMM
// (layout in kernels/gemm.h, QuantB), still on the host.
struct QHost {
  int type = 0;                // QT_Q8_0 = 1, QT_Q4_K = 2
  int64_t N = 0, K = 0;
  std::vector<uint8_t> q;      // Q8_0: int8 [N][K]; Q4_K: nibbles [N][K/2]
  std::vector<float> s0, s1;   // [K/32][N]
};

// Tensor `name` [N][K] as a QHost if the GGUF stores it as Q8_0 or Q4_K in
// K-major rows (type stays 0 otherwise). Per-32-value factors are the ones of
// the reference dequantisation (ggml_to_f32): Q8_0 d; Q4_K d*sc and dmin*m.
bool read_quant(const GgufFile& g, const std::string& name, int64_t N, int64_t K, QHost& out,
                std::string& err) {
  out = QHost{};
  const GgufTensor* t = g.tensor(name);
  if (!t) { err = "missing tensor " + name; return false; }
  if (t->nelem() != N * K || t->ne[0] != K) return true;
  if (t->type != GT_Q8_0 && t->type != GT_Q4_K) return true;
  if (K % 256 || N % 256) return true;
  const size_t rb = ggml_row_bytes(t->type, K);
  out.N = N;
  out.K = K;
  const int64_t nb = K / 32;
  out.s0.assign((size_t)nb * N, 0.f);
  if (t->type == GT_Q8_0) {
    out.type = 1;
    out.q.resize((size_t)N * K);
    parallel_rows(N, [&](int64_t a, int64_t b) {
      for (int64_t r = a; r < b; ++r) {
        const uint8_t* row = t->data + rb * r;
        for (int64_t j = 0; j < nb; ++j) {
          const uint8_t* blk = row + j * 34;
          uint16_t dh;
          std::memcpy(&dh, blk, 2);
          out.s0[(size_t)j * N + r] = f16_to_f32(dh);
          std::memcpy(out.q.data() + (size_t)r * K + j * 32, blk + 2, 32);
        }
      }
    });
  } else {
    out.type = 2;
    out.q.resize((size_t)N * K / 2);
    out.s1.assign((size_t)nb * N, 0.f);
    parallel_rows(N, [&](int64_t a, int64_t b) {
      for (int64_t r = a; r < b; ++r) {
        const uint8_t* row = t->data + rb * r;
        uint8_t* qr = out.q.data() + (size_t)r * (K / 2);
        for (int64_t sb = 0; sb < K / 256; ++sb) {
          const uint8_t* blk = row + sb * 144;
          uint16_t dh, mh;
          std::memcpy(&dh, blk, 2);
          std::memcpy(&mh, blk + 2, 2);
          const float dd = f16_to_f32(dh), dmin = f16_to_f32(mh);
          const uint8_t* sc = blk + 4;
          const uint8_t* qs = blk + 16;
          uint8_t sv[8], mv[8];
          for (int j = 0; j < 4; ++j) {
            sv[j] = sc[j] & 63;
            mv[j] = sc[j + 4] & 63;
            sv[j + 4] = (uint8_t)((sc[j + 8] & 0x0F) | ((sc[j] >> 6) << 4));
            mv[j + 4] = (uint8_t)((sc[j + 8] >> 4) | ((sc[j + 4] >> 6) << 4));
          }
          for (int j = 0; j < 8; ++j) {
            const int64_t blk32 = sb * 8 + j;
            out.s0[(size_t)blk32 * N + r] = dd * sv[j];
            out.s1[(size_t)blk32 * N + r] = dmin * mv[j];
          }
          // value v of the super-block: nibble (v / 32) & 1 of byte 32 * (v / 64) + v % 32
          for (int v = 0; v < 256; v += 2) {
            const int q0 = (qs[32 * (v / 64) + v % 32] >> (4 * ((v / 32) & 1))) & 15;
            const int q1 = (qs[32 * ((v + 1) / 64) + (v + 1) % 32] >> (4 * (((v + 1) / 32) & 1))) & 15;
            qr[sb * 128 + v / 2] = (uint8_t)(q0 | (q1 << 4));
          }
        }
      }
    });
  }
  return true;
}

// Rows of b appended to a (same type and K).
bool q_concat(QHost& a, const QHost& b) {
  if (a.type == 0) { a = b; return true; }
  if (a.type != b.type || a.K != b.K) return false;
  const int64_t nb = a.K / 32, N = a.N + b.N;
  a.q.insert(a.q.end(), b.q.begin(), b.q.end());
  auto merge = [&](std::vector<float>& x, const std::vector<float>& y) {
    if (x.empty()) return;
    std::vector<float> m((size_t)nb * N);
    for (int64_t j = 0; j < nb; ++j) {
      std::memcpy(m.data() + (size_t)j * N, x.data() + (size_t)j * a.N, (size_t)a.N * 4);
      std::memcpy(m.data() + (size_t)j * N + a.N, y.data() + (size_t)j * b.N, (size_t)b.N * 4);
    }
    x.swap(m);
  };
  merge(a.s0, b.s0);
  merge(a.s1, b.s1);
  a.N = N;
  return true;
}

}  // namespace

std::string read_config(const GgufFile& g, Config& c) {
  c.arch = g.str("parakeet.arch");
  c.feat_in = (int)g.u32("parakeet.encoder.feat_in");
  c.d_model = (int)g.u32("parakeet.encoder.d_model");
  c.n_layers = (int)g.u32("parakeet.encoder.n_layers");
  c.n_heads = (int)g.u32("parakeet.encoder.n_heads");
  c.ff_dim = (int)g.u32("parakeet.encoder.ff_dim");
  c.conv_kernel = (int)g.u32("parakeet.encoder.conv_kernel");
  c.conv_norm_type = g.str("parakeet.encoder.conv_norm_type", "batch_norm");
  c.subsampling_factor = (int)g.u32("parakeet.encoder.subsampling_factor");
  c.sub_channels = (int)g.u32("parakeet.encoder.subsampling_conv_channels");
  c.xscaling = g.boolean("parakeet.encoder.xscaling", true);
  c.att_context_style = g.str("parakeet.encoder.att_context_style", "regular");
  c.causal_downsampling = g.boolean("parakeet.encoder.causal_downsampling", false);
  c.conv_causal = g.boolean("parakeet.encoder.conv_causal", false);
  c.sample_rate = (int)g.u32("parakeet.preprocessor.sample_rate", 16000);
  c.n_mels = (int)g.u32("parakeet.preprocessor.n_mels");
  c.n_fft = (int)g.u32("parakeet.preprocessor.n_fft");
  c.win_length = (int)g.u32("parakeet.preprocessor.win_length");
  c.hop_length = (int)g.u32("parakeet.preprocessor.hop_length");
  c.preemph = g.f32("parakeet.preprocessor.preemph", 0.f);
  c.mag_power = g.f32("parakeet.preprocessor.mag_power", 2.f);
  c.normalize = g.str("parakeet.preprocessor.normalize", "per_feature");
  c.log_zero_guard = g.f32("parakeet.preprocessor.log_zero_guard", 0.f);
  c.vocab_size = (int)g.u32("parakeet.vocab_size");
  c.blank_id = (int)g.u32("parakeet.blank_id");
  c.pred_hidden = (int)g.u32("parakeet.decoder.pred_hidden", 0);
  c.pred_layers = (int)g.u32("parakeet.decoder.pred_rnn_layers", 1);
  if (c.pred_layers <= 0) c.pred_layers = 1;  // src/prediction.cpp: default one layer
  c.joint_hidden = (int)g.u32("parakeet.joint.joint_hidden", 0);
  c.max_symbols = (int)g.u32("parakeet.decoding.max_symbols", 10);
  c.durations.clear();
  for (int64_t x : g.int_array("parakeet.tdt.durations")) c.durations.push_back((int)x);
  if (c.d_model <= 0 || c.vocab_size <= 0) return "GGUF lacks parakeet.encoder.d_model / vocab_size";
  if (c.n_layers <= 0 || c.n_heads <= 0 || c.d_model % c.n_heads) return "bad encoder geometry";
  const int dk = c.d_model / c.n_heads;
  if (dk != 64 && dk != 128) return "head size " + std::to_string(dk) + " not supported (64 or 128)";
  if (c.d_model % 256 || c.d_model > 1024) return "d_model must be a multiple of 256, at most 1024";
  if (c.ff_dim % 256) return "ff_dim must be a multiple of 256";
  if (c.sub_channels != 256) return "subsampling_conv_channels must be 256";
  if (c.subsampling_factor != 8) return "only dw_striding 8x subsampling is implemented";
  if (c.conv_norm_type != "batch_norm" && c.conv_norm_type != "layer_norm")
    return "conv_norm_type " + c.conv_norm_type + " not supported (batch_norm, layer_norm)";
  c.conv_ln = c.conv_norm_type == "layer_norm";
  if (c.att_context_style != "regular" && c.att_context_style != "chunked_limited")
    return "att_context_style " + c.att_context_style + " not supported (regular, chunked_limited)";
  c.att_left = g.i32("parakeet.encoder.att_context_left", -1);
  c.att_right = g.i32("parakeet.encoder.att_context_right", -1);
  c.chunked = c.att_context_style == "chunked_limited" && c.att_right >= 0;
  {
    const std::vector<int64_t> cs = g.int_array("parakeet.streaming.chunk_size");
    const std::vector<int64_t> pc = g.int_array("parakeet.streaming.pre_encode_cache_size");
    Config::Streaming& sc = c.stream;
    sc.present = !cs.empty();
    if (cs.size() > 0) sc.chunk_first = (int)cs[0];
    if (cs.size() > 1) sc.chunk_main = (int)cs[1];
    if (pc.size() > 1) sc.pre_cache = (int)pc[1];
    sc.drop_extra = g.i32("parakeet.streaming.drop_extra_pre_encoded", 0);
    sc.cache_len = g.i32("parakeet.streaming.last_channel_cache_size", 0);
    sc.valid_out_len = g.i32("parakeet.streaming.valid_out_len", 0);
    if (sc.present && (sc.chunk_first <= 0 || sc.chunk_main <= 0 || sc.pre_cache < 0 || sc.drop_extra < 0 ||
                       sc.cache_len < 0 || sc.cache_len > 4096 || sc.valid_out_len < 0))
      return "bad parakeet.streaming.* schedule";
  }
  if (c.conv_kernel % 2 == 0 || c.conv_kernel < 3 || c.conv_kernel > 9)
    return "depthwise kernel must be odd, 3..9";
  if (c.n_fft != 512) return "n_fft must be 512";
  if (c.hop_length <= 0 || c.win_length <= 0 || c.win_length > c.n_fft) return "bad STFT geometry";
  if (c.mag_power != 2.f) return "mag_power must be 2";
  if (c.normalize != "per_feature") return "normalize must be per_feature";
  if (c.n_mels <= 0 || c.n_mels > 512) return "bad n_mels";
  // causal subsampling pads 2 before and 1 after (src/subsampling.cpp:25-46)
  auto flen = [&](int n) { return c.causal_downsampling ? n / 2 + 1 : conv_len(n); };
  c.F1 = flen(c.n_mels);
  c.F2 = flen(c.F1);
  c.F3 = flen(c.F2);
  if ((c.F3 * c.sub_channels) % 64) return "subsampling flatten width must be a multiple of 64";
  const GgufTensor* probe = g.tensor("encoder.layers.0.feed_forward1.linear1.weight");
  if (!probe) return "missing encoder.layers.0.feed_forward1.linear1.weight";
  c.weight_type = probe->type;
  c.bf16 = probe->type == GT_BF16;
  // f32 weights run the f32-accurate split-f16 path, as the reference runs an
  // f32 model in f32 (PKC_F32_AS_F16=1: f16 operands instead); the streaming
  // encoder's kernels have no split form
  const char* fa = getenv("PKC_F32_AS_F16");
  c.split = probe->type == GT_F32 && !c.causal() && !(fa && fa[0] == '1');
  return "";
}

// LayerNorm affine folded into the following linear layer:
//   (xhat * gamma + beta) W^T + b = xhat (W diag(gamma))^T + (W beta + b)
// W [N, K] f32 in place; bias [N] (created if the layer had none).
static void fold_layernorm(std::vector<float>& W, int64_t N, int64_t K, const std::vector<float>& gamma,
                           const std::vector<float>& beta, std::vector<float>& bias) {
  if (bias.empty()) bias.assign((size_t)N, 0.f);
  for (int64_t n = 0; n < N; ++n) {
    float* row = W.data() + (size_t)n * K;
    double acc = bias[(size_t)n];
    for (int64_t k = 0; k < K; ++k) {
      acc += (double)row[k] * (double)beta[(size_t)k];
      row[k] *= gamma[(size_t)k];
    }
    bias[(size_t)n] = (float)acc;
  }
}

std::string pack_weights(const GgufFile& g, const Config& c, bool fold_ln, PackedWeights& p) {
  const auto t0 = std::chrono::steady_clock::now();
  std::string err;
  Staging st;
  p = PackedWeights{};
  DeviceWeights& w = p.tmpl;
  const int d = c.d_model, FF = c.ff_dim, C = c.sub_channels, K = c.conv_kernel, H = c.n_heads;
  const bool bf = c.bf16;
  const bool sp = c.split;
  std::vector<float> f, f2, f3, f4;
  std::vector<uint16_t> h;

  auto put_f = [&](const std::vector<float>& v) { return as_off<float>(st.add(v.data(), v.size() * 4)); };
  auto put_h = [&](const std::vector<uint16_t>& v) { return as_off<void>(st.add(v.data(), v.size() * 2)); };
  // PKC_DEQUANT_AT_LOAD=1: dequantise Q8_0 / Q4_K weights on the host (the
  // earlier path, for A/B comparisons); default: keep them block-quantised
  const char* dal = getenv("PKC_DEQUANT_AT_LOAD");
  const bool keep_quant = !(dal && dal[0] == '1');
  auto put_q = [&](const QHost& qh) {
    QWeight qw;
    qw.type = qh.type;
    qw.q = as_off<void>(st.add(qh.q.data(), qh.q.size()));
    qw.s0 = as_off<float>(st.add(qh.s0.data(), qh.s0.size() * 4));
    if (!qh.s1.empty()) qw.s1 = as_off<float>(st.add(qh.s1.data(), qh.s1.size() * 4));
    return qw;
  };
  // a linear weight: block-quantised form when available (qw set, returns
  // null), else the 16-bit form
  auto put_linear = [&](const std::string& name, int64_t N, int64_t Kd, QWeight& qw) -> void* {
    qw = QWeight{};
    if (keep_quant) {
      QHost qh;
      if (!read_quant(g, name, N, Kd, qh, err)) return nullptr;
      if (qh.type) {
        qw = put_q(qh);
        return nullptr;
      }
    }
    if (sp) {
      std::vector<float> wf;
      if (!read_f32(g, name, N, Kd, wf, err)) return nullptr;
      return put_h(to_split(wf, N, Kd));
    }
    if (!read_h(g, name, N, Kd, bf, h, err)) return nullptr;
    return put_h(h);
  };
  auto opt_vec = [&](const std::string& name, int64_t n) -> float* {
    if (!g.tensor(name)) return nullptr;
    std::vector<float> v;
    if (!read_vec(g, name, n, v, err)) return nullptr;
    return put_f(v);
  };

  // ---------------- mel front end
  {
    const int N = c.n_fft, nb = N / 2 + 1;
    std::vector<float> win(N, 0.f);
    if (g.tensor("preprocessor.featurizer.window")) {
      const GgufTensor* t = g.tensor("preprocessor.featurizer.window");
      if (!read_vec(g, "preprocessor.featurizer.window", t->nelem(), f, err)) return err;
      const int wl = (int)f.size(), left = (N - wl) / 2;
      for (int i = 0; i < wl; ++i)
        if (left + i >= 0 && left + i < N) win[left + i] = f[i];
    }
    w.window = put_f(win);
    // DFT basis rows (GEMM columns): tile t of 256 = cos rows of bins 128t..128t+127,
    // then the -sin rows of the same bins; each row [hi | lo | hi] in f16.
    std::vector<uint16_t> basis((size_t)N * 3 * N);
    for (int n = 0; n < N; ++n) {
      const int tile = n / 256, r = n % 256;
      const int bin = tile * 128 + (r % 128);
      const bool is_sin = r >= 128;
      for (int k = 0; k < N; ++k) {
        const double ang = 2.0 * M_PI * (double)bin * (double)k / (double)N;
        const float v = is_sin ? (float)(-std::sin(ang)) : (float)std::cos(ang);
        const uint16_t hi = f32_to_f16(v);
        const uint16_t lo = f32_to_f16(v - f16_to_f32(hi));
        basis[(size_t)n * 3 * N + k] = hi;
        basis[(size_t)n * 3 * N + N + k] = lo;
        basis[(size_t)n * 3 * N + 2 * N + k] = hi;
      }
    }
    w.dft_basis = put_h(basis);
    if (!read_f32(g, "preprocessor.featurizer.fb", c.n_mels, nb, f, err)) return err;
    std::vector<int> fs(c.n_mels), fl(c.n_mels), fo(c.n_mels);
    std::vector<float> fw;
    for (int m = 0; m < c.n_mels; ++m) {
      int a = 0, b = nb;
      while (a < nb && f[(size_t)m * nb + a] == 0.f) ++a;
      while (b > a && f[(size_t)m * nb + b - 1] == 0.f) --b;
      fs[m] = a;
      fl[m] = b - a;
      fo[m] = (int)fw.size();
      for (int k = a; k < b; ++k) fw.push_back(f[(size_t)m * nb + k]);
    }
    if (fw.empty()) fw.push_back(0.f);
    w.fb_start = as_off<int>(st.add(fs.data(), fs.size() * 4));
    w.fb_len = as_off<int>(st.add(fl.data(), fl.size() * 4));
    w.fb_off = as_off<int>(st.add(fo.data(), fo.size() * 4));
    w.fb_w = put_f(fw);
  }

  // ---------------- subsampling
  {
    const std::string p = "encoder.pre_encode.";
    if (!read_f32(g, p + "conv.0.weight", C, 9, f, err)) return err;
    w.c0_w = put_f(f);
    if (!read_vec(g, p + "conv.0.bias", C, f, err)) return err;
    w.c0_b = put_f(f);
    for (int s = 0; s < 2; ++s) {
      const int dwi = s == 0 ? 2 : 5, pwi = dwi + 1;
      if (!read_f32(g, p + "conv." + std::to_string(dwi) + ".weight", C, 9, f, err)) return err;
      std::vector<float> tap(9 * C);
      for (int ch = 0; ch < C; ++ch)
        for (int k = 0; k < 9; ++k) tap[(size_t)k * C + ch] = f[(size_t)ch * 9 + k];
      float* dww = put_f(tap);
      if (!read_vec(g, p + "conv." + std::to_string(dwi) + ".bias", C, f, err)) return err;
      float* dwb = put_f(f);
      if (!read_f32(g, p + "conv." + std::to_string(pwi) + ".weight", C, C, f, err)) return err;
      void* pww = put_h(sp ? to_split(f, C, C) : to_h(f, true));
      if (!read_vec(g, p + "conv." + std::to_string(pwi) + ".bias", C, f, err)) return err;
      float* pwb = put_f(f);
      if (s == 0) { w.dw1_w = dww; w.dw1_b = dwb; w.pw1_w = pww; w.pw1_b = pwb; }
      else { w.dw2_w = dww; w.dw2_b = dwb; w.pw2_w = pww; w.pw2_b = pwb; }
    }
    const int F3 = c.F3, KW = C * F3;
    if (!read_f32(g, p + "out.weight", d, KW, f, err)) return err;
    std::vector<float> perm((size_t)d * KW);
    for (int o = 0; o < d; ++o)
      for (int ch = 0; ch < C; ++ch)
        for (int ff = 0; ff < F3; ++ff)
          perm[(size_t)o * KW + ff * C + ch] = f[(size_t)o * KW + ch * F3 + ff];
    w.out_w = put_h(sp ? to_split(perm, d, KW) : to_h(perm, true));
    if (!read_vec(g, p + "out.bias", d, f, err)) return err;
    w.out_b = put_f(f);
  }

  // ---------------- conformer layers
  w.layers.assign(c.n_layers, LayerWeights{});
  std::vector<uint16_t> pos_all;
  pos_all.reserve((size_t)c.n_layers * d * d);
  QHost pos_q;                // every layer's linear_pos, block-quantised alike
  bool pos_quant = keep_quant;
  for (int li = 0; li < c.n_layers; ++li) {
    LayerWeights& L = w.layers[li];
    const std::string p = "encoder.layers." + std::to_string(li) + ".";
    auto vec = [&](const std::string& n, int64_t len) -> float* {
      std::vector<float> v;
      if (!read_vec(g, p + n, len, v, err)) return nullptr;
      return put_f(v);
    };
    struct { const char* nm; float** gg; float** bb; } lns[] = {
        {"norm_feed_forward1", &L.ln_ff1_g, &L.ln_ff1_b}, {"norm_self_att", &L.ln_att_g, &L.ln_att_b},
        {"norm_conv", &L.ln_conv_g, &L.ln_conv_b}, {"norm_feed_forward2", &L.ln_ff2_g, &L.ln_ff2_b},
        {"norm_out", &L.ln_out_g, &L.ln_out_b}};
    std::vector<float> lng[5], lnb[5];  // host copies (gamma / beta of each norm)
    for (int i = 0; i < 5; ++i) {
      const std::string nm = p + lns[i].nm;
      if (!read_vec(g, nm + ".weight", d, lng[i], err) || !read_vec(g, nm + ".bias", d, lnb[i], err)) return err;
      *lns[i].gg = put_f(lng[i]);
      *lns[i].bb = put_f(lnb[i]);
    }
    struct { const char* nm; void** w1; void** w2; float** b1; float** b2; QWeight* q1; QWeight* q2; } ffs[] = {
        {"feed_forward1", &L.ff1_w1, &L.ff1_w2, &L.ff1_b1, &L.ff1_b2, &L.ff1_q1, &L.ff1_q2},
        {"feed_forward2", &L.ff2_w1, &L.ff2_w2, &L.ff2_b1, &L.ff2_b2, &L.ff2_q1, &L.ff2_q2}};
    for (int fi = 0; fi < 2; ++fi) {
      auto& ff = ffs[fi];
      const std::string n = p + ff.nm;
      *ff.w1 = put_linear(n + ".linear1.weight", FF, d, *ff.q1);
      if (!err.empty()) return err;
      *ff.w2 = put_linear(n + ".linear2.weight", d, FF, *ff.q2);
      if (!err.empty()) return err;
      *ff.b1 = opt_vec(n + ".linear1.bias", FF);
      *ff.b2 = opt_vec(n + ".linear2.bias", d);
      if (!err.empty()) return err;
      if (fi == 1 && fold_ln && !ff.q1->type) {
        // FFN2's linear1 takes norm_feed_forward2 folded in
        std::vector<float> b1;
        if (g.tensor(n + ".linear1.bias") && !read_vec(g, n + ".linear1.bias", FF, b1, err)) return err;
        if (!read_f32(g, n + ".linear1.weight", FF, d, f, err)) return err;
        fold_layernorm(f, FF, d, lng[3], lnb[3], b1);
        *ff.w1 = put_h(to_h(f, bf));
        *ff.b1 = put_f(b1);
        L.ff2_ln = true;
      }
    }
    const std::string a = p + "self_attn.";
    {
      std::vector<uint16_t> qkv((size_t)3 * d * d);
      const char* nms[3] = {"linear_q", "linear_k", "linear_v"};
      std::vector<float> bq((size_t)3 * d, 0.f);
      bool any_b = false;
      // q, k and v block-quantised alike: one quantised [3d, d] weight
      QHost qcat;
      bool all_q = keep_quant;
      for (int i = 0; i < 3 && all_q; ++i) {
        QHost qi;
        if (!read_quant(g, a + nms[i] + ".weight", d, d, qi, err)) return err;
        all_q = qi.type != 0 && q_concat(qcat, qi);
      }
      L.qkv_q = QWeight{};
      if (all_q) L.qkv_q = put_q(qcat);
      for (int i = 0; i < 3; ++i)
        if (g.tensor(a + nms[i] + ".bias")) {
          if (!read_vec(g, a + nms[i] + ".bias", d, f, err)) return err;
          std::memcpy(bq.data() + (size_t)i * d, f.data(), (size_t)d * 4);
          any_b = true;
        }
      if (!all_q && fold_ln) {
        // norm_self_att folded into the [3d, d] weight and its bias
        std::vector<float> wq((size_t)3 * d * d);
        for (int i = 0; i < 3; ++i) {
          if (!read_f32(g, a + nms[i] + ".weight", d, d, f, err)) return err;
          std::memcpy(wq.data() + (size_t)i * d * d, f.data(), (size_t)d * d * 4);
        }
        fold_layernorm(wq, 3 * d, d, lng[1], lnb[1], bq);
        qkv = to_h(wq, bf);
        any_b = true;
        L.qkv_ln = true;
      } else if (sp && !all_q) {
        std::vector<float> wq((size_t)3 * d * d);
        for (int i = 0; i < 3; ++i) {
          if (!read_f32(g, a + nms[i] + ".weight", d, d, f, err)) return err;
          std::memcpy(wq.data() + (size_t)i * d * d, f.data(), (size_t)d * d * 4);
        }
        qkv = to_split(wq, 3 * d, d);
      } else {
        for (int i = 0; i < 3; ++i) {
          if (all_q) break;
          if (!read_h(g, a + nms[i] + ".weight", d, d, bf, h, err)) return err;
          std::memcpy(qkv.data() + (size_t)i * d * d, h.data(), (size_t)d * d * 2);
        }
      }
      L.qkv_w = all_q ? nullptr : put_h(qkv);
      L.qkv_b = any_b ? put_f(bq) : nullptr;
    }
    {
      QHost qp;
      if (pos_quant && !read_quant(g, a + "linear_pos.weight", d, d, qp, err)) return err;
      pos_quant = pos_quant && qp.type != 0 && q_concat(pos_q, qp);
      if (sp) {
        if (!read_f32(g, a + "linear_pos.weight", d, d, f, err)) return err;
        h = to_split(f, d, d);
      } else if (!read_h(g, a + "linear_pos.weight", d, d, bf, h, err)) {
        return err;
      }
      pos_all.insert(pos_all.end(), h.begin(), h.end());
    }
    L.pos_w = nullptr;
    L.out_w = put_linear(a + "linear_out.weight", d, d, L.out_q);
    if (!err.empty()) return err;
    L.out_b = opt_vec(a + "linear_out.bias", d);
    if (!err.empty()) return err;
    L.pos_u = vec("self_attn.pos_bias_u", d);
    L.pos_v = vec("self_attn.pos_bias_v", d);
    if (!L.pos_u || !L.pos_v) return err;
    (void)H;
    // conv module
    {
      if (!read_f32(g, p + "conv.pointwise_conv1.weight", 2 * d, d, f, err)) return err;
      std::vector<float> paired((size_t)2 * d * d);
      std::vector<float> pb((size_t)2 * d, 0.f);
      const bool has_b = g.tensor(p + "conv.pointwise_conv1.bias") != nullptr;
      if (has_b && !read_vec(g, p + "conv.pointwise_conv1.bias", 2 * d, f2, err)) return err;
      for (int n = 0; n < 2 * d; ++n) {
        const int tile = n / 256, r = n % 256;
        const int src = r < 128 ? tile * 128 + r : d + tile * 128 + (r - 128);
        std::memcpy(paired.data() + (size_t)n * d, f.data() + (size_t)src * d, (size_t)d * 4);
        if (has_b) pb[n] = f2[src];
      }
      if (fold_ln) {
        // norm_conv folded into pointwise_conv1 (rows already GLU-paired)
        fold_layernorm(paired, 2 * d, d, lng[2], lnb[2], pb);
        L.pw1_ln = true;
      }
      L.pw1_w = put_h(sp ? to_split(paired, 2 * d, d) : to_h(paired, bf));
      L.pw1_b = (has_b || fold_ln) ? put_f(pb) : nullptr;
      if (!read_f32(g, p + "conv.depthwise_conv.weight", d, K, f, err)) return err;
      std::vector<float> tap((size_t)K * d);
      for (int ch = 0; ch < d; ++ch)
        for (int k = 0; k < K; ++k) tap[(size_t)k * d + ch] = f[(size_t)ch * K + k];
      L.dw_w = put_f(tap);
      L.dw_b = opt_vec(p + "conv.depthwise_conv.bias", d);
      if (!err.empty()) return err;
      if (!read_vec(g, p + "conv.batch_norm.weight", d, f, err) ||
          !read_vec(g, p + "conv.batch_norm.bias", d, f2, err))
        return err;
      if (c.conv_ln) {  // LayerNorm over channels: gamma / beta as they are
        L.bn_scale = put_f(f);
        L.bn_shift = put_f(f2);
      } else {
        if (!read_vec(g, p + "conv.batch_norm.running_mean", d, f3, err) ||
            !read_vec(g, p + "conv.batch_norm.running_var", d, f4, err))
          return err;
        std::vector<float> sc(d), sh(d);
        for (int ch = 0; ch < d; ++ch) {
          sc[ch] = f[ch] / std::sqrt(f4[ch] + 1e-5f);
          sh[ch] = f2[ch] - f3[ch] * sc[ch];
        }
        L.bn_scale = put_f(sc);
        L.bn_shift = put_f(sh);
      }
      if (!read_f32(g, p + "conv.pointwise_conv2.weight", d, d, f, err)) return err;
      L.pw2_w = put_h(sp ? to_split(f, d, d) : to_h(f, bf));
      L.pw2_b = opt_vec(p + "conv.pointwise_conv2.bias", d);
      if (!err.empty()) return err;
    }
  }

  w.pos_all_q = QWeight{};
  if (pos_quant && pos_q.type) {
    w.pos_all_q = put_q(pos_q);
    w.pos_all_w = nullptr;
  } else {
    w.pos_all_w = put_h(pos_all);
  }
  pos_all.clear();
  pos_all.shrink_to_fit();

  // ---------------- CTC head (src/ctc_decoder.cpp:17-28: hybrid name first)
  {
    std::string pre;
    for (const char* cand : {"ctc_decoder.decoder_layers.0.", "decoder.decoder_layers.0."})
      if (g.tensor(std::string(cand) + "weight") && g.tensor(std::string(cand) + "bias")) {
        pre = cand;
        break;
      }
    if (!pre.empty()) {
      const int V1 = c.vocab_size + 1, Vp = (V1 + 255) / 256 * 256;
      if (!read_f32(g, pre + "weight", V1, d, f, err)) return err;
      if (!read_vec(g, pre + "bias", V1, f2, err)) return err;
      std::vector<uint16_t> ws((size_t)Vp * 3 * d, 0);
      for (int v = 0; v < V1; ++v)
        for (int k = 0; k < d; ++k) {
          const float x = f[(size_t)v * d + k];
          const uint16_t hi = f32_to_f16(x);
          const uint16_t lo = f32_to_f16(x - f16_to_f32(hi));
          uint16_t* row = ws.data() + (size_t)v * 3 * d;
          row[k] = hi;
          row[d + k] = lo;
          row[2 * d + k] = hi;
        }
      std::vector<float> bp((size_t)Vp, 0.f);
      std::copy(f2.begin(), f2.end(), bp.begin());
      w.ctc_w = put_h(ws);
      w.ctc_b = put_f(bp);
      w.ctc_v1 = V1;
      w.ctc_vpad = Vp;
    }
  }

  // ---------------- transducer decoder (prediction LSTM + joint), f32
  if (c.pred_hidden > 0 && c.joint_hidden > 0 && g.tensor("decoder.prediction.embed.weight") &&
      g.tensor("joint.joint_net.2.weight")) {
    const int Hp = c.pred_hidden, J = c.joint_hidden, L = c.pred_layers, V1 = c.vocab_size + 1;
    const int D = (int)c.durations.size();
    std::vector<float> emb, wi, wh, bb, t1, t2;
    if (!read_f32(g, "decoder.prediction.embed.weight", V1, Hp, emb, err)) return err;
    for (int l = 0; l < L; ++l) {
      const std::string s = "decoder.prediction.dec_rnn.lstm.";
      const std::string ls = "_l" + std::to_string(l);
      if (!read_f32(g, s + "weight_ih" + ls, 4 * Hp, Hp, t1, err)) return err;
      wi.insert(wi.end(), t1.begin(), t1.end());
      if (!read_f32(g, s + "weight_hh" + ls, 4 * Hp, Hp, t1, err)) return err;
      wh.insert(wh.end(), t1.begin(), t1.end());
      if (!read_vec(g, s + "bias_ih" + ls, 4 * Hp, t1, err) || !read_vec(g, s + "bias_hh" + ls, 4 * Hp, t2, err))
        return err;
      for (int i = 0; i < 4 * Hp; ++i) bb.push_back(t1[i] + t2[i]);
    }
    w.dec_embed = put_f(emb);
    w.dec_w_ih = put_f(wi);
    w.dec_w_hh = put_f(wh);
    w.dec_b = put_f(bb);
    if (!read_f32(g, "joint.pred.weight", J, Hp, t1, err) || !read_vec(g, "joint.pred.bias", J, t2, err)) return err;
    w.dec_w_pred = put_f(t1);
    w.dec_b_pred = put_f(t2);
    if (!read_f32(g, "joint.joint_net.2.weight", V1 + D, J, t1, err) ||
        !read_vec(g, "joint.joint_net.2.bias", V1 + D, t2, err))
      return err;
    w.dec_w_out = put_f(t1);
    w.dec_b_out = put_f(t2);
    std::vector<int> du(c.durations.begin(), c.durations.end());
    if (du.empty()) du.push_back(0);
    w.dec_durations = as_off<int>(st.add(du.data(), du.size() * 4));
    w.dec_zeros = put_f(std::vector<float>((size_t)Hp, 0.f));
    w.dec_gate0 = as_off<float>(st.add(nullptr, (size_t)(V1 + 1) * 4 * Hp * 4));  // filled on the device
    // encoder projection: split f16 rows [W_hi | W_lo | W_hi], padded to 256
    if (!read_f32(g, "joint.enc.weight", J, d, t1, err) || !read_vec(g, "joint.enc.bias", J, t2, err)) return err;
    const int Jp = (J + 255) / 256 * 256;
    std::vector<uint16_t> ws((size_t)Jp * 3 * d, 0);
    for (int j = 0; j < J; ++j)
      for (int k = 0; k < d; ++k) {
        const float x = t1[(size_t)j * d + k];
        const uint16_t hi = f32_to_f16(x), lo = f32_to_f16(x - f16_to_f32(hi));
        uint16_t* row = ws.data() + (size_t)j * 3 * d;
        row[k] = hi;
        row[d + k] = lo;
        row[2 * d + k] = hi;
      }
    std::vector<float> be((size_t)Jp, 0.f);
    std::copy(t2.begin(), t2.end(), be.begin());
    w.dec_w_enc = put_h(ws);
    w.dec_b_enc = put_f(be);
    w.dec_jpad = Jp;
    w.dec_ok = true;
  }

  w.arena_bytes = st.buf.size();
  p.bytes = std::move(st.buf);
  p.pack_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  return "";
}

std::string upload_packed(const PackedWeights& p, const Config& c, DeviceWeights& w, cudaStream_t st) {
  w = p.tmpl;
  int dev_id = 0;
  cudaGetDevice(&dev_id);
  w.device = dev_id;
  void* dev = nullptr;
  if (cudaMalloc(&dev, p.bytes.size()) != cudaSuccess)
    return "cudaMalloc of " + std::to_string(p.bytes.size()) + " weight bytes failed";
  if (cudaMemcpyAsync(dev, p.bytes.data(), p.bytes.size(), cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess) {
    cudaFree(dev);
    return "weight upload failed";
  }
  w.arena = dev;
  uint8_t* base = static_cast<uint8_t*>(dev);
  for_each_field(w, [&](auto& f) {
    using T = std::remove_reference_t<decltype(f)>;
    if constexpr (std::is_pointer_v<T>) reloc(f, base);
  });
  if (w.dec_ok) {
    const int V1 = c.vocab_size + 1, Hp = c.pred_hidden;
    if (transducer_gate0_launch(w.dec_embed, w.dec_w_ih, w.dec_b, V1, Hp, w.dec_gate0, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess) {
      cudaFree(dev);
      w.arena = nullptr;
      return "decoder gate table computation failed";
    }
  }
  return "";
}

std::string upload_weights(const GgufFile& g, const Config& c, DeviceWeights& w, bool fold_ln) {
  PackedWeights p;
  std::string err = pack_weights(g, c, fold_ln, p);
  if (!err.empty()) return err;
  return upload_packed(p, c, w, nullptr);
}

// ---------------------------------------------------------------- pack cache
namespace {

constexpr char kPackMagic[8] = {'P', 'K', 'C', 'P', 'A', 'C', 'K', '1'};
constexpr uint32_t kPackVersion = 1;  // bump when a packed layout or the field list changes

struct PackHeader {
  char magic[8];
  uint32_t version, n_top, n_layer_fields, pad;
  uint64_t key, n_layers, arena_bytes, data_offset;
};

uint64_t fnv1a(uint64_t h, const void* data, size_t n) {
  const uint8_t* b = static_cast<const uint8_t*>(data);
  for (size_t i = 0; i < n; ++i) {
    h ^= b[i];
    h *= 1099511628211ull;
  }
  return h;
}

// Field values of the offset-encoded template as 64-bit words, in visit order.
std::vector<uint64_t> field_words(DeviceWeights& w, size_t& n_top, size_t& n_layer) {
  std::vector<uint64_t> out;
  auto put = [&](auto& f) {
    using T = std::remove_reference_t<decltype(f)>;
    if constexpr (std::is_pointer_v<T>) out.push_back(reinterpret_cast<uintptr_t>(f));
    else out.push_back(static_cast<uint64_t>(f));
  };
  for_each_top_field(w, put);
  n_top = out.size();
  n_layer = 0;
  for (LayerWeights& L : w.layers) {
    const size_t before = out.size();
    for_each_layer_field(L, put);
    n_layer = out.size() - before;
  }
  return out;
}

}  // namespace

uint64_t pack_cache_key(const std::string& gguf_path, const Config& c, bool fold_ln) {
  struct stat sb {};
  char real[PATH_MAX];
  const std::string rp = realpath(gguf_path.c_str(), real) ? std::string(real) : gguf_path;
  uint64_t h = 1469598103934665603ull;
  h = fnv1a(h, kPackMagic, sizeof(kPackMagic));
  h = fnv1a(h, &kPackVersion, sizeof(kPackVersion));
  h = fnv1a(h, rp.data(), rp.size());
  if (stat(rp.c_str(), &sb) == 0) {
    const uint64_t v[4] = {(uint64_t)sb.st_size, (uint64_t)sb.st_mtim.tv_sec, (uint64_t)sb.st_mtim.tv_nsec,
                           (uint64_t)sb.st_ino};
    h = fnv1a(h, v, sizeof(v));
  }
  const char* dal = getenv("PKC_DEQUANT_AT_LOAD");
  const uint32_t opts[5] = {fold_ln ? 1u : 0u, (dal && dal[0] == '1') ? 1u : 0u, (uint32_t)c.n_layers,
                            (uint32_t)sizeof(DeviceWeights), c.split ? 1u : 0u};
  return fnv1a(h, opts, sizeof(opts));
}

std::string pack_cache_path(const std::string& dir, uint64_t key) {
  char name[64];
  snprintf(name, sizeof(name), "pkc_%016llx.pack", (unsigned long long)key);
  return dir + "/" + name;
}

std::string pack_cache_store(const std::string& path, uint64_t key, const PackedWeights& p) {
  DeviceWeights t = p.tmpl;
  size_t n_top = 0, n_layer = 0;
  const std::vector<uint64_t> words = field_words(t, n_top, n_layer);
  PackHeader h{};
  std::memcpy(h.magic, kPackMagic, sizeof(h.magic));
  h.version = kPackVersion;
  h.n_top = (uint32_t)n_top;
  h.n_layer_fields = (uint32_t)n_layer;
  h.key = key;
  h.n_layers = t.layers.size();
  h.arena_bytes = p.bytes.size();
  h.data_offset = (sizeof(h) + words.size() * 8 + 4095) / 4096 * 4096;
  const std::string tmp = path + ".tmp" + std::to_string(getpid());
  FILE* f = fopen(tmp.c_str(), "wb");
  if (!f) return "cannot create " + tmp;
  bool ok = fwrite(&h, sizeof(h), 1, f) == 1 && fwrite(words.data(), 8, words.size(), f) == words.size();
  const std::vector<uint8_t> pad(h.data_offset - sizeof(h) - words.size() * 8, 0);
  ok = ok && (pad.empty() || fwrite(pad.data(), 1, pad.size(), f) == pad.size());
  ok = ok && fwrite(p.bytes.data(), 1, p.bytes.size(), f) == p.bytes.size();
  ok = (fclose(f) == 0) && ok;
  if (!ok || rename(tmp.c_str(), path.c_str()) != 0) {
    unlink(tmp.c_str());
    return "cannot write " + path;
  }
  return "";
}

std::string pack_cache_load(const std::string& path, uint64_t key, const Config& c, PackedWeights& p) {
  const auto t0 = std::chrono::steady_clock::now();
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) return "no cache file " + path;
  std::unique_ptr<FILE, int (*)(FILE*)> guard(f, fclose);
  PackHeader h{};
  if (fread(&h, sizeof(h), 1, f) != 1 || std::memcmp(h.magic, kPackMagic, sizeof(kPackMagic)) != 0 ||
      h.version != kPackVersion)
    return "not a pack cache file: " + path;
  if (h.key != key) return "pack cache key mismatch: " + path;
  DeviceWeights t{};
  t.layers.assign((size_t)c.n_layers, LayerWeights{});
  size_t n_top = 0, n_layer = 0;
  field_words(t, n_top, n_layer);
  if (h.n_layers != t.layers.size() || h.n_top != n_top || h.n_layer_fields != n_layer)
    return "pack cache field layout mismatch: " + path;
  std::vector<uint64_t> words(n_top + n_layer * t.layers.size());
  if (fread(words.data(), 8, words.size(), f) != words.size()) return "truncated pack cache: " + path;
  size_t k = 0;
  auto get = [&](auto& fld) {
    using T = std::remove_reference_t<decltype(fld)>;
    if constexpr (std::is_pointer_v<T>) fld = reinterpret_cast<T>(static_cast<uintptr_t>(words[k++]));
    else fld = static_cast<T>(words[k++]);
  };
  for_each_top_field(t, get);
  for (LayerWeights& L : t.layers) for_each_layer_field(L, get);
  if (t.arena_bytes != h.arena_bytes) return "pack cache size mismatch: " + path;
  // every offset must land inside the arena
  bool inside = true;
  auto check = [&](auto& fld) {
    using T = std::remove_reference_t<decltype(fld)>;
    if constexpr (std::is_pointer_v<T>)
      if (fld && reinterpret_cast<uintptr_t>(fld) - 1 >= h.arena_bytes) inside = false;
  };
  for_each_field(t, check);
  if (!inside) return "pack cache offset out of range: " + path;
  if (fseeko(f, (off_t)h.data_offset, SEEK_SET) != 0) return "truncated pack cache: " + path;
  p = PackedWeights{};
  p.bytes.resize(h.arena_bytes);
  if (fread(p.bytes.data(), 1, p.bytes.size(), f) != p.bytes.size()) return "truncated pack cache: " + path;
  p.tmpl = std::move(t);
  p.from_cache = true;
  p.pack_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  return "";
}

void free_weights(DeviceWeights& w) {
  if (w.arena) cudaFree(w.arena);
  w.arena = nullptr;
}

}  // namespace pkc
