// C entry points around parakeet.cpp's own CPU front end, compiled from the
// reference sources in place (see Makefile.ref). TEST INFRASTRUCTURE: the
// parity tests use it to pin the oracle's mel / FFT / positional-encoding
// restatements to the reference's code, and bench.py may time it as the CPU
// baseline of the front end.
//
// The reference's ModelLoader normally reads a GGUF through ggml's gguf API
// (absent here). Its member functions are defined below so that load() takes
// the preprocessor config and the two featurizer tensors from the arguments of
// pkref_mel() instead; MelFrontend and MelKernel are the reference's code.
#include <cstring>
#include <string>
#include <vector>

#include "ggml.h"
#include "backend.hpp"
#include "fft.hpp"
#include "mel.hpp"
#include "model_loader.hpp"
#include "pos_enc.hpp"

namespace {
struct PendingCfg {
  pk::ParakeetConfig cfg;
  ggml_tensor window{}, fb{};
  std::vector<float> window_data, fb_data;
} g_pending;
}  // namespace

namespace pk {
ModelLoader::~ModelLoader() {}
bool ModelLoader::load(const std::string&) {
  cfg_ = g_pending.cfg;
  tensors_.clear();
  tensors_["preprocessor.featurizer.window"] = &g_pending.window;
  tensors_["preprocessor.featurizer.fb"] = &g_pending.fb;
  return true;
}
ggml_tensor* ModelLoader::tensor(const std::string& n) const {
  auto it = tensors_.find(n);
  return it == tensors_.end() ? nullptr : it->second;
}
void weight_to_host_f32(const ModelLoader& ml, const char* name, std::vector<float>& out) {
  ggml_tensor* t = ml.tensor(name);
  size_t n = 1;
  for (int i = 0; i < 4; ++i) n *= (size_t)(t->ne[i] > 0 ? t->ne[i] : 1);
  out.assign((const float*)t->data, (const float*)t->data + n);
}
}  // namespace pk

extern "C" {

// MelFrontend::compute (src/mel.cpp:95-176) on one clip. feats: [n_mels, T]
// row-major, capacity `cap` floats. Returns T, or -1 if cap is too small.
int pkref_mel(const float* samples, int n_samples, int n_mels, int n_fft, int hop, int win_length,
              float preemph, float mag_power, float log_guard, int per_feature,
              const float* window, const float* fb, float* feats, long cap) {
  pk::ParakeetConfig c;
  c.n_mels = n_mels; c.n_fft = n_fft; c.hop_length = hop; c.win_length = win_length;
  c.preemph = preemph; c.mag_power = mag_power; c.log_zero_guard = log_guard;
  c.normalize = per_feature ? "per_feature" : "NA";
  c.d_model = 1; c.vocab_size = 1;
  g_pending.cfg = c;
  const int n_bins = n_fft / 2 + 1;
  g_pending.window_data.assign(window, window + win_length);
  g_pending.fb_data.assign(fb, fb + (size_t)n_mels * n_bins);
  g_pending.window = ggml_tensor{0, {win_length, 1, 1, 1}, g_pending.window_data.data()};
  g_pending.fb = ggml_tensor{0, {n_bins, n_mels, 1, 1}, g_pending.fb_data.data()};
  pk::ModelLoader ml;
  ml.load("");
  pk::MelFrontend mel(ml);
  std::vector<float> s(samples, samples + n_samples), out;
  int nm = 0, T = 0;
  mel.compute(s, out, nm, T);
  if ((long)out.size() > cap) return -1;
  std::memcpy(feats, out.data(), out.size() * sizeof(float));
  return T;
}

// pk::rfft (src/fft.cpp:53-73): n a power of two; re/im receive n/2+1 bins.
void pkref_rfft(const float* x, int n, float* re, float* im) {
  std::vector<float> in(x, x + n), r, i;
  pk::rfft(in, r, i);
  std::memcpy(re, r.data(), r.size() * sizeof(float));
  std::memcpy(im, i.data(), i.size() * sizeof(float));
}

// pk::rel_pos_encoding (src/pos_enc.cpp:10-34): out [2T-1, d].
void pkref_rel_pos_encoding(int T, int d, float* out) {
  std::vector<float> v;
  pk::rel_pos_encoding(T, d, v);
  std::memcpy(out, v.data(), v.size() * sizeof(float));
}

}  // extern "C"
