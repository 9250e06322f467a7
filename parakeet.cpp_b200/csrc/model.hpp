// Model configuration (the reference's ParakeetConfig, src/model_loader.hpp:27-52)
// and the per-device weight arena with every tensor re-packed once at load
// into the layout its kernel reads.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "gguf.hpp"

namespace pkc {

struct Config {
  std::string arch;
  int feat_in = 0, d_model = 0, n_layers = 0, n_heads = 0, ff_dim = 0, conv_kernel = 0;
  std::string conv_norm_type = "batch_norm";
  int subsampling_factor = 0, sub_channels = 0;
  bool xscaling = true;
  std::string att_context_style = "regular";
  bool causal_downsampling = false, conv_causal = false;
  // cache-aware streaming (causal) models, src/model_loader.cpp:113-131
  int att_left = -1, att_right = -1;
  bool chunked = false;  // att_context_style chunked_limited with att_right >= 0
  bool conv_ln = false;  // conv_norm_type layer_norm (gamma / beta under conv.batch_norm.*)
  struct Streaming {
    bool present = false;
    int chunk_first = 9, chunk_main = 16;  // mel frames of the first / later chunk windows
    int pre_cache = 9;                     // mel frames of overlap prepended to later windows
    int drop_extra = 0;                    // subsampled frames dropped from later windows
    int cache_len = 0;                     // attention cache (last_channel_cache_size)
    int valid_out_len = 0;                 // frames a mid-stream chunk outputs
  } stream;
  bool causal() const { return causal_downsampling || conv_causal || chunked; }
  int sample_rate = 16000, n_mels = 0, n_fft = 0, win_length = 0, hop_length = 0;
  float preemph = 0.f, mag_power = 2.f, log_zero_guard = 0.f;
  std::string normalize = "per_feature";
  int vocab_size = 0, blank_id = 0;
  // transducer decoder (0 when absent): prediction LSTM, joint, TDT durations
  int pred_hidden = 0, pred_layers = 0, joint_hidden = 0, max_symbols = 0;
  std::vector<int> durations;  // empty: RNN-T
  // derived
  int F1 = 0, F2 = 0, F3 = 0;
  uint32_t weight_type = 0;  // GGUF type of the encoder linear weights
  bool bf16 = false;         // tensor-core operand type of the conformer layers
  // f32-accurate path (f32 GGUF weights, offline encoder): every linear
  // weight and GEMM operand as split-f16 [hi | lo] rows, f32 between GEMMs
  bool split = false;
};

// Read and validate the configuration. Returns an empty string on success,
// else the reason the model cannot run on this library.
std::string read_config(const GgufFile& g, Config& c);

// A linear weight [N][K] kept in its GGUF block format, repacked for TMA
// (layout in kernels/gemm.h, QuantB). type 0 = absent.
struct QWeight {
  int type = 0;
  void* q = nullptr;
  float* s0 = nullptr;
  float* s1 = nullptr;
};

struct LayerWeights {
  float *ln_ff1_g, *ln_ff1_b, *ln_att_g, *ln_att_b, *ln_conv_g, *ln_conv_b;
  float *ln_ff2_g, *ln_ff2_b, *ln_out_g, *ln_out_b;
  void *ff1_w1, *ff1_w2, *ff2_w1, *ff2_w2;           // [FF, d], [d, FF]
  float *ff1_b1, *ff1_b2, *ff2_b1, *ff2_b2;          // optional
  void* qkv_w;                                       // [3d, d]
  float* qkv_b;                                      // [3d] optional
  void* pos_w;                                       // [d, d]
  void* out_w;                                       // [d, d]
  float* out_b;
  float *pos_u, *pos_v;                              // [H * dk]
  void* pw1_w;                                       // [2d, d] GLU-paired rows
  float* pw1_b;                                      // [2d] paired, optional
  float* dw_w;                                       // [K][d]
  float* dw_b;                                       // optional
  float *bn_scale, *bn_shift;                        // [d]
  void* pw2_w;                                       // [d, d]
  float* pw2_b;
  // block-quantised forms (QT_Q8_0 / QT_Q4_K, dequantised inside the GEMM);
  // when set, the matching 16-bit weight above is null
  QWeight ff1_q1, ff1_q2, ff2_q1, ff2_q2, qkv_q, out_q;
  // the preceding LayerNorm's gamma folded into the weight's columns and
  // W * beta into its bias (the GEMM then normalises its A operand itself)
  bool qkv_ln = false, pw1_ln = false, ff2_ln = false;
};

struct DeviceWeights {
  int device = 0;
  void* arena = nullptr;
  size_t arena_bytes = 0;
  // mel front end
  float* window = nullptr;        // [n_fft] centre-padded
  void* dft_basis = nullptr;      // f16 [n_fft, 3*n_fft]
  int* fb_start = nullptr;
  int* fb_len = nullptr;
  int* fb_off = nullptr;
  float* fb_w = nullptr;
  // subsampling
  float *c0_w, *c0_b;             // [C][9], [C]
  float *dw1_w, *dw1_b, *dw2_w, *dw2_b;  // [9][C], [C]
  void *pw1_w, *pw2_w;            // bf16 [C, C]
  float *pw1_b, *pw2_b;
  void* out_w;                    // bf16 [d, F3*C] (columns f*C + c)
  float* out_b;
  void* pos_all_w = nullptr;      // [L*d, d]: every layer's linear_pos, one GEMM per batch
  QWeight pos_all_q;              // its block-quantised form, when every layer's linear_pos is
  std::vector<LayerWeights> layers;
  // CTC head (ctc_decoder.decoder_layers.0 of hybrid models, decoder.* of CTC
  // models), when present: the f32 weight split for the ~22-bit GEMM as f16
  // rows [W_hi | W_lo | W_hi] of length 3d, padded with zero rows to ctc_vpad
  void* ctc_w = nullptr;          // f16 [ctc_vpad, 3d]
  float* ctc_b = nullptr;         // [ctc_vpad]
  int ctc_v1 = 0;                 // vocab + 1 (0: no CTC head)
  int ctc_vpad = 0;               // ctc_v1 rounded up to 256
  // transducer decoder (f32, as in GGUF), when present (dec_ok)
  bool dec_ok = false;
  float* dec_embed = nullptr;     // [V1, H]
  float* dec_w_ih = nullptr;      // [L][4H, H]
  float* dec_w_hh = nullptr;      // [L][4H, H]
  float* dec_b = nullptr;         // [L][4H] (b_ih + b_hh)
  float* dec_w_pred = nullptr;    // [J, H]
  float* dec_b_pred = nullptr;    // [J]
  float* dec_w_out = nullptr;     // [V1 + D, J]
  float* dec_b_out = nullptr;     // [V1 + D]
  int* dec_durations = nullptr;   // [D]
  float* dec_zeros = nullptr;     // [H]
  float* dec_gate0 = nullptr;     // [V1 + 1, 4H] layer-0 input gates W_ih0 embed[v] + b0 (row V1: SOS, b0 only)
  // joint encoder projection as a split-f16 GEMM operand [W_hi | W_lo | W_hi],
  // rows padded to dec_jpad (a multiple of 256), and its bias
  void* dec_w_enc = nullptr;      // f16 [dec_jpad, 3d]
  float* dec_b_enc = nullptr;     // [dec_jpad]
  int dec_jpad = 0;
};

// Host image of one device weight arena: every tensor re-packed into the layout
// its kernel reads, and a DeviceWeights whose pointer fields hold arena offsets
// (+1; 0 = absent) until upload_packed relocates them.
struct PackedWeights {
  std::vector<uint8_t> bytes;
  DeviceWeights tmpl;
  bool from_cache = false;
  double pack_s = 0;  // host seconds to re-pack (or to read the pack cache)
};

// Re-pack every weight of `g` on the host (no CUDA call).
std::string pack_weights(const GgufFile& g, const Config& c, bool fold_ln, PackedWeights& p);
// Copy the image to the current device (p.bytes may be page-locked by the
// caller), relocate the pointers and build the device-side derived tables.
std::string upload_packed(const PackedWeights& p, const Config& c, DeviceWeights& w, cudaStream_t st);

// Pre-pack cache: one file per (GGUF identity, packing options), holding the
// field table and the arena image; a hit skips the re-pack.
uint64_t pack_cache_key(const std::string& gguf_path, const Config& c, bool fold_ln);
std::string pack_cache_path(const std::string& dir, uint64_t key);
std::string pack_cache_store(const std::string& path, uint64_t key, const PackedWeights& p);
std::string pack_cache_load(const std::string& path, uint64_t key, const Config& c, PackedWeights& p);

// Upload every encoder weight of `g` to the current CUDA device.
// Returns an empty string on success, else an error message.
// fold_ln: fold the pre-norm LayerNorms' gamma / beta into the dense QKV,
// pointwise-conv-1 and FFN2-up weights / biases (for the LayerNorm-fused GEMM)
std::string upload_weights(const GgufFile& g, const Config& c, DeviceWeights& w, bool fold_ln);
void free_weights(DeviceWeights& w);

}  // namespace pkc
