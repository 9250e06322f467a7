// The model-level C ABI (include/pkc.h): open/close, mel front end, encoder,
// multi-GPU sharding and profiling. No exception crosses this boundary.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <cmath>
#include <memory>
#include <mutex>
#include <numeric>
#include <thread>

#include "../../include/pkc.h"
#include "encoder.hpp"
#include "gguf.hpp"
#include "model.hpp"
#include "status.hpp"

struct pkc_model {
  pkc::Config cfg;
  std::vector<std::unique_ptr<pkc::DeviceRunner>> runners;
  std::mutex mu;
  std::string last_error;
  double pack_s = 0, upload_s = 0;  // load: re-pack (or pack-cache read), slowest device's upload
  int from_cache = 0;
};

struct pkc_stream {
  pkc_model* m;
  pkc::DeviceRunner* r;
  pkc::DeviceRunner::StreamState* st;
};

namespace pkc {
const char* model_error(const pkc_model* m) { return m->last_error.c_str(); }
}  // namespace pkc

namespace {

pkc_status fail(pkc_model* m, pkc_status st, const std::string& msg) {
  m->last_error = msg;
  return st;
}

// Encoder frames (T') of a clip, and the sharding cost T'(1 + T'/8192):
// linear work per frame plus the attention's quadratic term.
double clip_cost(int v) { return (double)v * (1.0 + (double)v / 8192.0); }

// Host-side failure injection for the failure-detection tests: when the
// environment variable PKC_FAULT_DEVICE_SLOT names device slot k, the
// multi-device dispatcher's worker for slot k throws before it touches its
// device (a failed worker, made on the host: no GPU is faulted). Read on
// every call so a test can switch it on and off.
bool fault_injected(int slot) {
  const char* e = std::getenv("PKC_FAULT_DEVICE_SLOT");
  return e && e[0] && std::atoi(e) == slot;
}

void lpt_assign(const std::vector<double>& cost, int n_dev, std::vector<int>& assign) {
  const int B = (int)cost.size();
  std::vector<int> order(B);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return cost[a] > cost[b]; });
  std::vector<double> load(n_dev, 0.0);
  assign.assign(B, 0);
  for (int b : order) {
    int best = 0;
    for (int k = 1; k < n_dev; ++k)
      if (load[k] < load[best]) best = k;
    assign[b] = best;
    load[best] += cost[b];
  }
}

}  // namespace

extern "C" {

pkc_status pkc_model_open(const char* gguf_path, const int* devices, int n_devices, pkc_model** out) {
  if (!out) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_model_open: out is NULL");
  *out = nullptr;
  if (!gguf_path) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_model_open: path is NULL");
  try {
    auto g = std::make_unique<pkc::GgufFile>();
    std::string err;
    if (!g->open(gguf_path, err))
      return pkc::set_thread_error(err.rfind("cannot open", 0) == 0 ? PKC_ERR_IO : PKC_ERR_FORMAT, err);
    auto m = std::make_unique<pkc_model>();
    err = pkc::read_config(*g, m->cfg);
    if (!err.empty()) return pkc::set_thread_error(PKC_ERR_UNSUPPORTED, err);
    std::vector<int> devs;
    if (!devices || n_devices <= 0) devs.push_back(0);
    else devs.assign(devices, devices + n_devices);
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0)
      return pkc::set_thread_error(PKC_ERR_CUDA, "no CUDA device available");
    for (int dv : devs)
      if (dv < 0 || dv >= count)
        return pkc::set_thread_error(PKC_ERR_ARG, "device index " + std::to_string(dv) + " out of range");
    // one host image for every device: from the pre-pack cache when it holds
    // this GGUF (PKC_PACK_CACHE=<dir>), else re-packed here (and stored there)
    const bool fold = pkc::DeviceRunner::ln_fused(m->cfg);
    pkc::PackedWeights pw;
    const char* cache_dir = getenv("PKC_PACK_CACHE");
    std::string cache_path;
    uint64_t key = 0;
    if (cache_dir && cache_dir[0]) {
      key = pkc::pack_cache_key(gguf_path, m->cfg, fold);
      cache_path = pkc::pack_cache_path(cache_dir, key);
      if (!pkc::pack_cache_load(cache_path, key, m->cfg, pw).empty()) pw = pkc::PackedWeights{};
    }
    if (!pw.from_cache) {
      err = pkc::pack_weights(*g, m->cfg, fold, pw);
      if (!err.empty())
        return pkc::set_thread_error(err.find("tensor") != std::string::npos ? PKC_ERR_FORMAT : PKC_ERR_UNSUPPORTED, err);
    }
    const bool store = !pw.from_cache && !cache_path.empty();
    m->pack_s = pw.pack_s;
    m->from_cache = pw.from_cache ? 1 : 0;
    // page-locked source: every device's copy runs at DMA rate, concurrently
    const bool pinned = cudaHostRegister(pw.bytes.data(), pw.bytes.size(), cudaHostRegisterPortable) == cudaSuccess;
    if (!pinned) cudaGetLastError();
    std::vector<std::unique_ptr<pkc::DeviceRunner>> rs(devs.size());
    std::vector<std::string> errs(devs.size());
    {
      std::vector<std::thread> th;
      for (size_t k = 0; k < devs.size(); ++k)
        th.emplace_back([&, k] {
          try {
            rs[k] = std::make_unique<pkc::DeviceRunner>(m->cfg, devs[k]);
            errs[k] = rs[k]->init(pw);
          } catch (const std::exception& e) {
            errs[k] = std::string("device init: ") + e.what();
          }
        });
      if (store) pkc::pack_cache_store(cache_path, key, pw);  // best effort, while the devices upload
      for (auto& t : th) t.join();
    }
    if (pinned) cudaHostUnregister(pw.bytes.data());
    for (size_t k = 0; k < devs.size(); ++k) {
      if (!errs[k].empty()) {
        const bool oom = errs[k].find("cudaMalloc") != std::string::npos;
        return pkc::set_thread_error(oom ? PKC_ERR_OOM : PKC_ERR_CUDA, "device " + std::to_string(devs[k]) + ": " + errs[k]);
      }
      m->upload_s = std::max(m->upload_s, rs[k]->upload_seconds());
    }
    m->runners = std::move(rs);
    *out = m.release();
    return PKC_OK;
  } catch (const std::bad_alloc&) {
    return pkc::set_thread_error(PKC_ERR_OOM, "host allocation failed");
  } catch (const std::exception& e) {
    return pkc::set_thread_error(PKC_ERR_INTERNAL, e.what());
  }
}

pkc_status pkc_stream_schedule_get(const pkc_model* m, pkc_stream_schedule* o) {
  if (!m || !o) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_stream_schedule_get: NULL argument");
  const pkc::Config& c = m->cfg;
  if (!c.stream.present) return pkc::set_thread_error(PKC_ERR_UNSUPPORTED, "not a cache-aware streaming model");
  o->chunk_size_first = c.stream.chunk_first;
  o->chunk_size = c.stream.chunk_main;
  o->pre_encode_cache_size = c.stream.pre_cache;
  o->valid_out_len = c.stream.valid_out_len;
  o->drop_extra_pre_encoded = c.stream.drop_extra;
  o->attention_cache_size = c.stream.cache_len;
  return PKC_OK;
}

pkc_status pkc_stream_begin(pkc_model* m, int device_slot, pkc_stream** out) {
  if (!m || !out) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_stream_begin: NULL argument");
  *out = nullptr;
  if (device_slot < 0 || device_slot >= (int)m->runners.size())
    return fail(m, PKC_ERR_ARG, "pkc_stream_begin: device slot " + std::to_string(device_slot) + " out of range");
  try {
    std::lock_guard<std::mutex> lk(m->mu);
    std::string err;
    pkc::DeviceRunner* r = m->runners[device_slot].get();
    pkc::DeviceRunner::StreamState* st = r->stream_create(err);
    if (!st) return fail(m, err.find("cudaMalloc") != std::string::npos ? PKC_ERR_OOM : PKC_ERR_UNSUPPORTED, err);
    *out = new pkc_stream{m, r, st};
    return PKC_OK;
  } catch (const std::bad_alloc&) {
    return fail(m, PKC_ERR_OOM, "host allocation failed");
  }
}

pkc_status pkc_stream_reset(pkc_stream* s) {
  if (!s) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_stream_reset: NULL stream");
  std::lock_guard<std::mutex> lk(s->m->mu);
  std::string err;
  const pkc_status st = s->r->stream_reset(*s->st, err);
  return st == PKC_OK ? PKC_OK : fail(s->m, st, err);
}

pkc_status pkc_stream_step(pkc_stream* s, const float* mel, int n_frames, int is_last, float* out,
                           size_t out_cap_floats, int* n_valid_out) {
  if (!s || !mel || !out || !n_valid_out) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_stream_step: NULL argument");
  *n_valid_out = 0;
  if (n_frames <= 0) return fail(s->m, PKC_ERR_ARG, "pkc_stream_step: n_frames must be positive");
  try {
    std::lock_guard<std::mutex> lk(s->m->mu);
    std::string err;
    const pkc_status st = s->r->stream_step(*s->st, mel, n_frames, is_last != 0, out, out_cap_floats, n_valid_out, err);
    return st == PKC_OK ? PKC_OK : fail(s->m, st, "pkc_stream_step: " + err);
  } catch (const std::bad_alloc&) {
    return fail(s->m, PKC_ERR_OOM, "host allocation failed");
  }
}

pkc_status pkc_stream_step_batch(pkc_stream* const* streams, int n_streams, const float* const* mels, int n_frames,
                                 const int* is_last, float* const* outs, size_t out_cap_floats, int* n_valid_out) {
  if (!streams || n_streams <= 0 || !mels || !is_last || !outs || !n_valid_out)
    return pkc::set_thread_error(PKC_ERR_ARG, "pkc_stream_step_batch: NULL argument or no streams");
  pkc_model* m = streams[0] ? streams[0]->m : nullptr;
  if (!m) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_stream_step_batch: NULL stream");
  std::vector<pkc::DeviceRunner::StreamState*> ss((size_t)n_streams);
  for (int i = 0; i < n_streams; ++i) {
    if (!streams[i]) return fail(m, PKC_ERR_ARG, "pkc_stream_step_batch: NULL stream " + std::to_string(i));
    if (streams[i]->m != m || streams[i]->r != streams[0]->r)
      return fail(m, PKC_ERR_ARG, "pkc_stream_step_batch: the streams must belong to one model and device");
    ss[(size_t)i] = streams[i]->st;
  }
  try {
    std::lock_guard<std::mutex> lk(m->mu);
    std::string err;
    const pkc_status st = streams[0]->r->stream_step_batch(ss.data(), n_streams, mels, n_frames, is_last, outs,
                                                           out_cap_floats, n_valid_out, err);
    return st == PKC_OK ? PKC_OK : fail(m, st, "pkc_stream_step_batch: " + err);
  } catch (const std::bad_alloc&) {
    return fail(m, PKC_ERR_OOM, "host allocation failed");
  }
}

int pkc_stream_step_num(const pkc_stream* s) { return s ? pkc::DeviceRunner::stream_step_num(*s->st) : -1; }

void pkc_stream_free(pkc_stream* s) {
  if (!s) return;
  {
    std::lock_guard<std::mutex> lk(s->m->mu);
    cudaSetDevice(s->r->device());
    cudaStreamSynchronize(s->r->stream());
    pkc::DeviceRunner::stream_destroy(s->st);
  }
  delete s;
}

pkc_status pkc_model_load_stats(const pkc_model* m, double* pack_seconds, double* upload_seconds, int* from_cache) {
  if (!m) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_model_load_stats: model is NULL");
  if (pack_seconds) *pack_seconds = m->pack_s;
  if (upload_seconds) *upload_seconds = m->upload_s;
  if (from_cache) *from_cache = m->from_cache;
  return PKC_OK;
}

pkc_status pkc_pack_cache_build(const char* gguf_path, const char* cache_dir, char* path_out, int path_cap) {
  if (!gguf_path || !cache_dir) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_pack_cache_build: NULL argument");
  try {
    pkc::GgufFile g;
    std::string err;
    if (!g.open(gguf_path, err))
      return pkc::set_thread_error(err.rfind("cannot open", 0) == 0 ? PKC_ERR_IO : PKC_ERR_FORMAT, err);
    pkc::Config cfg;
    err = pkc::read_config(g, cfg);
    if (!err.empty()) return pkc::set_thread_error(PKC_ERR_UNSUPPORTED, err);
    const bool fold = pkc::DeviceRunner::ln_fused(cfg);
    const uint64_t key = pkc::pack_cache_key(gguf_path, cfg, fold);
    const std::string path = pkc::pack_cache_path(cache_dir, key);
    pkc::PackedWeights pw;
    if (!pkc::pack_cache_load(path, key, cfg, pw).empty()) {
      err = pkc::pack_weights(g, cfg, fold, pw);
      if (!err.empty()) return pkc::set_thread_error(PKC_ERR_FORMAT, err);
      err = pkc::pack_cache_store(path, key, pw);
      if (!err.empty()) return pkc::set_thread_error(PKC_ERR_IO, err);
    }
    if (path_out && path_cap > 0) {
      if ((int)path.size() >= path_cap) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_pack_cache_build: path_cap too small");
      std::memcpy(path_out, path.c_str(), path.size() + 1);
    }
    return PKC_OK;
  } catch (const std::bad_alloc&) {
    return pkc::set_thread_error(PKC_ERR_OOM, "host allocation failed");
  } catch (const std::exception& e) {
    return pkc::set_thread_error(PKC_ERR_INTERNAL, e.what());
  }
}

void pkc_model_close(pkc_model* m) {
  if (!m) return;
  try {
    delete m;
  } catch (...) {
  }
}

pkc_status pkc_model_info_get(const pkc_model* m, pkc_model_info* o) {
  if (!m || !o) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_model_info_get: NULL argument");
  const pkc::Config& c = m->cfg;
  std::memset(o, 0, sizeof(*o));
  o->d_model = c.d_model; o->n_layers = c.n_layers; o->n_heads = c.n_heads; o->ff_dim = c.ff_dim;
  o->conv_kernel = c.conv_kernel; o->n_mels = c.n_mels; o->n_fft = c.n_fft;
  o->win_length = c.win_length; o->hop_length = c.hop_length; o->sample_rate = c.sample_rate;
  o->subsampling_factor = c.subsampling_factor; o->subsampling_conv_channels = c.sub_channels;
  o->xscaling = c.xscaling ? 1 : 0; o->weight_type = (int)c.weight_type;
  o->compute_bf16 = c.bf16 ? 1 : 0; o->n_devices = (int)m->runners.size();
  o->vocab_size = c.vocab_size; o->blank_id = c.blank_id;
  std::strncpy(o->arch, c.arch.c_str(), sizeof(o->arch) - 1);
  return PKC_OK;
}

int pkc_mel_frames(const pkc_model* m, int n_samples) {
  if (!m || n_samples < 0) return 0;
  return pkc::mel_frames_for(m->cfg, n_samples);
}

int pkc_encoder_frames(const pkc_model* m, int mel_frames) {
  if (!m || mel_frames <= 0) return 0;
  return pkc::encoder_frames_for(mel_frames);
}

int pkc_ctc_classes(const pkc_model* m) {
  if (!m || m->runners.empty()) return 0;
  return m->runners[0]->ctc_classes();
}

// The greedy fold of ctc_greedy (src/search.cpp:21-90): the state it keeps
// (previous class, previous token's emit frame, the run's minimum confidence)
// and its start-offset rule are the reference's, so the tokens, frames and
// confidences match it exactly; only the per-frame argmax moved to the GPU.
int pkc_ctc_fold(const int32_t* argmax, const float* max_logprob, int T, int n_classes, int blank_id,
                 pkc_token* out, int cap) {
  if (T < 0 || n_classes <= 1 || (T > 0 && (!argmax || !max_logprob)) || (cap > 0 && !out)) return -1;
  // NeMo's rescaled max_prob confidence of one frame: (N p_max - 1) / (N - 1)
  const float N = (float)n_classes;
  auto conf = [&](float lp) { return (N * std::exp(lp) - 1.0f) / (N - 1.0f); };
  // fold_consecutive: emit p when it differs from the previous frame's class
  // (or that was blank) and is not blank; a token's frame is the previous
  // token's emit frame (the first token's: its own minus one, floored at 0);
  // its confidence the minimum over its argmax run
  int n = 0;
  int32_t previous = blank_id;
  int prev_peak = 0;
  bool have_prev = false;
  float run_min = 1.0f;
  for (int t = 0; t < T; ++t) {
    const int32_t p = argmax[t];
    const bool emit = (p != previous || previous == blank_id) && p != blank_id;
    if (emit) {
      if (n >= cap) return -1;
      if (n > 0) out[n - 1].conf = run_min;
      out[n] = pkc_token{p, have_prev ? (int32_t)prev_peak : (int32_t)(t > 0 ? t - 1 : 0), 0.0f, 1};
      ++n;
      run_min = conf(max_logprob[t]);
      prev_peak = t;
      have_prev = true;
    } else if (p == previous && p != blank_id) {
      run_min = std::min(run_min, conf(max_logprob[t]));
    }
    previous = p;
  }
  if (n > 0) out[n - 1].conf = run_min;
  return n;
}

pkc_status pkc_ctc_greedy_pcm_batch(pkc_model* m, const float* const* pcm, const int* n_samples, int B,
                                    pkc_token* tokens_out, size_t tokens_cap, int* n_tokens,
                                    float* logprobs_out, size_t logprobs_cap) {
  if (!m) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_ctc_greedy_pcm_batch: model is NULL");
  std::lock_guard<std::mutex> lk(m->mu);
  if (!pcm || !n_samples || B <= 0 || !n_tokens || (tokens_cap > 0 && !tokens_out))
    return fail(m, PKC_ERR_ARG, "pkc_ctc_greedy_pcm_batch: bad arguments");
  const int V1 = m->runners[0]->ctc_classes();
  if (!V1) return fail(m, PKC_ERR_UNSUPPORTED, "pkc_ctc_greedy_pcm_batch: the model has no CTC head");
  try {
    std::vector<size_t> off(B + 1, 0);  // frame offsets
    for (int b = 0; b < B; ++b) {
      if (n_samples[b] <= 0 || !pcm[b]) return fail(m, PKC_ERR_ARG, "pkc_ctc_greedy_pcm_batch: empty clip " + std::to_string(b));
      off[b + 1] = off[b] + (size_t)pkc::encoder_frames_for(pkc::mel_frames_for(m->cfg, n_samples[b]));
    }
    const size_t M = off[B];
    if (logprobs_out && logprobs_cap < M * (size_t)V1)
      return fail(m, PKC_ERR_ARG, "pkc_ctc_greedy_pcm_batch: logprobs_out too small");
    std::vector<int32_t> am(M);
    std::vector<float> ml(M);
    const int nd = (int)m->runners.size();
    std::vector<double> cost(B);
    for (int b = 0; b < B; ++b) cost[b] = clip_cost((int)(off[b + 1] - off[b]));
    std::vector<int> assign(B, 0);
    if (nd > 1) lpt_assign(cost, nd, assign);
    std::vector<std::vector<int>> items(nd);
    for (int b = 0; b < B; ++b) items[assign[b]].push_back(b);
    std::vector<pkc_status> st(nd, PKC_OK);
    std::vector<std::string> errs(nd);
    auto run = [&](int k) {
      try {
        std::vector<const float*> p;
        std::vector<int> n;
        size_t tot = 0;
        for (int b : items[k]) { p.push_back(pcm[b]); n.push_back(n_samples[b]); tot += off[b + 1] - off[b]; }
        std::vector<int32_t> a(tot);
        std::vector<float> l(tot), lp(logprobs_out ? tot * V1 : 0);
        st[k] = m->runners[k]->ctc_pcm_host(p, n, a.data(), l.data(), logprobs_out ? lp.data() : nullptr, errs[k]);
        if (st[k] != PKC_OK) return;
        size_t pos = 0;  // scatter this device's clips back into batch order
        for (int b : items[k]) {
          const size_t t = off[b + 1] - off[b];
          std::memcpy(am.data() + off[b], a.data() + pos, t * 4);
          std::memcpy(ml.data() + off[b], l.data() + pos, t * 4);
          if (logprobs_out) std::memcpy(logprobs_out + off[b] * V1, lp.data() + pos * V1, t * V1 * 4);
          pos += t;
        }
      } catch (const std::exception& e) {
        st[k] = PKC_ERR_INTERNAL;
        errs[k] = e.what();
      }
    };
    std::vector<std::thread> th;
    for (int k = 0; k < nd; ++k)
      if (!items[k].empty()) th.emplace_back(run, k);
    for (auto& t : th) t.join();
    for (int k = 0; k < nd; ++k)
      if (st[k] != PKC_OK) return fail(m, st[k], "device " + std::to_string(m->runners[k]->device()) + ": " + errs[k]);
    size_t used = 0;
    for (int b = 0; b < B; ++b) {
      const int T = (int)(off[b + 1] - off[b]);
      const int cap = (int)std::min<size_t>(tokens_cap - used, (size_t)0x7fffffff);
      const int n = pkc_ctc_fold(am.data() + off[b], ml.data() + off[b], T, V1, m->cfg.blank_id,
                                 tokens_out ? tokens_out + used : nullptr, cap);
      if (n < 0) return fail(m, PKC_ERR_ARG, "pkc_ctc_greedy_pcm_batch: tokens_out too small");
      n_tokens[b] = n;
      used += (size_t)n;
    }
    return PKC_OK;
  } catch (const std::exception& e) {
    return fail(m, PKC_ERR_INTERNAL, e.what());
  }
}

int pkc_transducer_kind(const pkc_model* m) {
  if (!m || m->runners.empty()) return 0;
  return m->runners[0]->transducer_kind();
}

pkc_status pkc_transducer_greedy_pcm_batch(pkc_model* m, const float* const* pcm, const int* n_samples, int B,
                                           pkc_token* tokens_out, size_t tokens_cap, int* n_tokens) {
  if (!m) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_transducer_greedy_pcm_batch: model is NULL");
  std::lock_guard<std::mutex> lk(m->mu);
  if (!pcm || !n_samples || B <= 0 || !n_tokens || (tokens_cap > 0 && !tokens_out))
    return fail(m, PKC_ERR_ARG, "pkc_transducer_greedy_pcm_batch: bad arguments");
  if (!m->runners[0]->transducer_kind())
    return fail(m, PKC_ERR_UNSUPPORTED, "pkc_transducer_greedy_pcm_batch: the model has no transducer decoder");
  try {
    const int MS = std::max(1, m->runners[0]->max_symbols());
    std::vector<int> T(B);
    for (int b = 0; b < B; ++b) {
      if (n_samples[b] <= 0 || !pcm[b])
        return fail(m, PKC_ERR_ARG, "pkc_transducer_greedy_pcm_batch: empty clip " + std::to_string(b));
      T[b] = pkc::encoder_frames_for(pkc::mel_frames_for(m->cfg, n_samples[b]));
    }
    const int nd = (int)m->runners.size();
    std::vector<double> cost(B);
    for (int b = 0; b < B; ++b) cost[b] = clip_cost(T[b]);
    std::vector<int> assign(B, 0);
    if (nd > 1) lpt_assign(cost, nd, assign);
    std::vector<std::vector<int>> items(nd);
    for (int b = 0; b < B; ++b) items[assign[b]].push_back(b);
    // per clip: its token rows as the device wrote them
    std::vector<std::vector<int>> rows(B);
    std::vector<int> cnt(B, 0);
    std::vector<pkc_status> st(nd, PKC_OK);
    std::vector<std::string> errs(nd);
    auto run = [&](int k) {
      try {
        std::vector<const float*> p;
        std::vector<int> n;
        size_t frames = 0;
        for (int b : items[k]) { p.push_back(pcm[b]); n.push_back(n_samples[b]); frames += (size_t)T[b]; }
        std::vector<int> tok(frames * MS * 4), nt(items[k].size());
        st[k] = m->runners[k]->transducer_pcm_host(p, n, tok.data(), nt.data(), errs[k]);
        if (st[k] != PKC_OK) return;
        size_t pos = 0;  // token rows of this device's clips, in its order
        for (size_t i = 0; i < items[k].size(); ++i) {
          const int b = items[k][i];
          cnt[b] = nt[i];
          rows[b].assign(tok.begin() + pos * 4, tok.begin() + (pos + (size_t)nt[i]) * 4);
          pos += (size_t)T[b] * MS;
        }
      } catch (const std::exception& e) {
        st[k] = PKC_ERR_INTERNAL;
        errs[k] = e.what();
      }
    };
    std::vector<std::thread> th;
    for (int k = 0; k < nd; ++k)
      if (!items[k].empty()) th.emplace_back(run, k);
    for (auto& t : th) t.join();
    for (int k = 0; k < nd; ++k)
      if (st[k] != PKC_OK) return fail(m, st[k], "device " + std::to_string(m->runners[k]->device()) + ": " + errs[k]);
    size_t used = 0;
    for (int b = 0; b < B; ++b) {
      if (used + (size_t)cnt[b] > tokens_cap)
        return fail(m, PKC_ERR_ARG, "pkc_transducer_greedy_pcm_batch: tokens_out too small");
      if (cnt[b]) std::memcpy(tokens_out + used, rows[b].data(), (size_t)cnt[b] * sizeof(pkc_token));
      n_tokens[b] = cnt[b];
      used += (size_t)cnt[b];
    }
    return PKC_OK;
  } catch (const std::exception& e) {
    return fail(m, PKC_ERR_INTERNAL, e.what());
  }
}

size_t pkc_encode_out_floats(const pkc_model* m, const int* n_samples, int B) {
  if (!m || !n_samples || B <= 0) return 0;
  size_t n = 0;
  for (int b = 0; b < B; ++b)
    n += (size_t)pkc::encoder_frames_for(pkc::mel_frames_for(m->cfg, n_samples[b])) * m->cfg.d_model;
  return n;
}

pkc_status pkc_shard_plan(const int* n_samples, int B, int n_dev, int hop, int* assign) {
  if (!n_samples || !assign || B < 0 || n_dev <= 0 || hop <= 0)
    return pkc::set_thread_error(PKC_ERR_ARG, "pkc_shard_plan: bad arguments");
  std::vector<double> cost(B);
  for (int b = 0; b < B; ++b) {
    if (n_samples[b] <= 0) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_shard_plan: empty clip");
    cost[b] = clip_cost(pkc::encoder_frames_for(1 + n_samples[b] / hop));
  }
  std::vector<int> a;
  lpt_assign(cost, n_dev, a);
  std::copy(a.begin(), a.end(), assign);
  return PKC_OK;
}

pkc_status pkc_mel_batch(pkc_model* m, const float* const* pcm, const int* n_samples, int B,
                         float* feats_out, size_t feats_cap, int* T_out) {
  if (!m) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_mel_batch: model is NULL");
  std::lock_guard<std::mutex> lk(m->mu);
  if (!pcm || !n_samples || B <= 0 || !feats_out || !T_out) return fail(m, PKC_ERR_ARG, "pkc_mel_batch: bad arguments");
  try {
    std::vector<const float*> p(pcm, pcm + B);
    std::vector<int> n(n_samples, n_samples + B);
    int Tmax = 0;
    for (int b = 0; b < B; ++b) {
      if (n[b] <= 0 || !p[b]) return fail(m, PKC_ERR_ARG, "pkc_mel_batch: empty clip " + std::to_string(b));
      T_out[b] = pkc::mel_frames_for(m->cfg, n[b]);
      Tmax = std::max(Tmax, T_out[b]);
    }
    if ((size_t)B * m->cfg.n_mels * Tmax > feats_cap) return fail(m, PKC_ERR_ARG, "pkc_mel_batch: feats_out too small");
    std::string err;
    const pkc_status s = m->runners[0]->mel_host(p, n, Tmax, feats_out, err);
    return s == PKC_OK ? s : fail(m, s, err);
  } catch (const std::exception& e) {
    return fail(m, PKC_ERR_INTERNAL, e.what());
  }
}

pkc_status pkc_encode_batch(pkc_model* m, const float* mel, int B, int n_mels, int T_max,
                            const int* valid_T, int layout, float* out, size_t out_cap,
                            int* valid_Tout, int* d_model_out) {
  if (!m) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_encode_batch: model is NULL");
  std::lock_guard<std::mutex> lk(m->mu);
  if (!mel || B <= 0 || T_max <= 0 || !valid_T || !out || !valid_Tout)
    return fail(m, PKC_ERR_ARG, "pkc_encode_batch: bad arguments");
  if (n_mels != m->cfg.n_mels) return fail(m, PKC_ERR_ARG, "pkc_encode_batch: n_mels does not match the model");
  if (layout != PKC_LAYOUT_CHANNELS_FIRST && layout != PKC_LAYOUT_TIME_MAJOR)
    return fail(m, PKC_ERR_ARG, "pkc_encode_batch: unknown layout");
  try {
    size_t need = 0;
    for (int b = 0; b < B; ++b) {
      if (valid_T[b] < 1 || valid_T[b] > T_max) return fail(m, PKC_ERR_ARG, "pkc_encode_batch: valid_T out of range");
      valid_Tout[b] = pkc::encoder_frames_for(valid_T[b]);
      need += (size_t)valid_Tout[b] * m->cfg.d_model;
    }
    if (need > out_cap) return fail(m, PKC_ERR_ARG, "pkc_encode_batch: out too small");
    if (d_model_out) *d_model_out = m->cfg.d_model;
    std::string err;
    const pkc_status s = m->runners[0]->encode_mel_host(mel, B, n_mels, T_max, valid_T, layout, out, err);
    return s == PKC_OK ? s : fail(m, s, err);
  } catch (const std::exception& e) {
    return fail(m, PKC_ERR_INTERNAL, e.what());
  }
}

pkc_status pkc_encode_pcm_batch(pkc_model* m, const float* const* pcm, const int* n_samples, int B,
                                int layout, float* out, size_t out_cap, int* valid_Tout) {
  if (!m) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_encode_pcm_batch: model is NULL");
  std::lock_guard<std::mutex> lk(m->mu);
  if (!pcm || !n_samples || B <= 0 || !out || !valid_Tout)
    return fail(m, PKC_ERR_ARG, "pkc_encode_pcm_batch: bad arguments");
  if (layout != PKC_LAYOUT_CHANNELS_FIRST && layout != PKC_LAYOUT_TIME_MAJOR)
    return fail(m, PKC_ERR_ARG, "pkc_encode_pcm_batch: unknown layout");
  try {
    const int d = m->cfg.d_model;
    std::vector<size_t> off(B + 1, 0);
    for (int b = 0; b < B; ++b) {
      if (n_samples[b] <= 0 || !pcm[b]) return fail(m, PKC_ERR_ARG, "pkc_encode_pcm_batch: empty clip " + std::to_string(b));
      valid_Tout[b] = pkc::encoder_frames_for(pkc::mel_frames_for(m->cfg, n_samples[b]));
      off[b + 1] = off[b] + (size_t)valid_Tout[b] * d;
    }
    if (off[B] > out_cap) return fail(m, PKC_ERR_ARG, "pkc_encode_pcm_batch: out too small");
    const int nd = (int)m->runners.size();
    if (nd == 1) {
      std::string err;
      std::vector<const float*> p(pcm, pcm + B);
      std::vector<int> n(n_samples, n_samples + B);
      const pkc_status s = m->runners[0]->encode_pcm_host(p, n, layout, out, err);
      return s == PKC_OK ? s : fail(m, s, err);
    }
    // shard whole utterances across devices (no collective: each device runs
    // its own clips end to end), then scatter the outputs back in order
    std::vector<double> cost(B);
    for (int b = 0; b < B; ++b) cost[b] = clip_cost(valid_Tout[b]);
    std::vector<int> assign;
    lpt_assign(cost, nd, assign);
    std::vector<std::vector<int>> items(nd);
    for (int b = 0; b < B; ++b) items[assign[b]].push_back(b);
    // each device copies its clips' outputs straight to their places in
    // `out` (one device-to-host copy per clip, no intermediate host buffer)
    std::vector<pkc_status> st(nd, PKC_OK);
    std::vector<std::string> errs(nd);
    std::vector<std::thread> th;
    for (int k = 0; k < nd; ++k) {
      if (items[k].empty()) continue;
      th.emplace_back([&, k] {
        try {
          if (fault_injected(k)) throw std::runtime_error("injected host fault (PKC_FAULT_DEVICE_SLOT)");
          std::vector<const float*> p;
          std::vector<int> n;
          std::vector<float*> dst;
          for (int b : items[k]) {
            p.push_back(pcm[b]);
            n.push_back(n_samples[b]);
            dst.push_back(out + off[b]);
          }
          st[k] = m->runners[k]->encode_pcm_host_items(p, n, layout, dst, errs[k]);
        } catch (const std::exception& e) {
          st[k] = PKC_ERR_INTERNAL;
          errs[k] = e.what();
        }
      });
    }
    for (auto& t : th) t.join();
    for (int k = 0; k < nd; ++k)
      if (st[k] != PKC_OK) return fail(m, st[k], "device " + std::to_string(m->runners[k]->device()) + ": " + errs[k]);
    return PKC_OK;
  } catch (const std::exception& e) {
    return fail(m, PKC_ERR_INTERNAL, e.what());
  }
}

pkc_status pkc_encode_pcm_device(pkc_model* m, int device_slot, const float* d_pcm,
                                 const int* n_samples, int B, float* d_out, void* stream, int sync) {
  if (!m) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_encode_pcm_device: model is NULL");
  std::lock_guard<std::mutex> lk(m->mu);
  if (!d_pcm || !n_samples || B <= 0 || !d_out) return fail(m, PKC_ERR_ARG, "pkc_encode_pcm_device: bad arguments");
  if (device_slot < 0 || device_slot >= (int)m->runners.size())
    return fail(m, PKC_ERR_ARG, "pkc_encode_pcm_device: bad device slot");
  try {
    std::vector<int> n(n_samples, n_samples + B);
    for (int b = 0; b < B; ++b)
      if (n[b] <= 0) return fail(m, PKC_ERR_ARG, "pkc_encode_pcm_device: empty clip");
    std::string err;
    const pkc_status s = m->runners[device_slot]->encode_pcm_device(
        d_pcm, n, d_out, reinterpret_cast<cudaStream_t>(stream), sync != 0, err);
    return s == PKC_OK ? s : fail(m, s, err);
  } catch (const std::exception& e) {
    return fail(m, PKC_ERR_INTERNAL, e.what());
  }
}

void* pkc_model_stream(const pkc_model* m, int device_slot) {
  if (!m || device_slot < 0 || device_slot >= (int)m->runners.size()) return nullptr;
  return reinterpret_cast<void*>(m->runners[device_slot]->stream());
}

int pkc_last_graph_kernels(const pkc_model* m, int device_slot) {
  if (!m || device_slot < 0 || device_slot >= (int)m->runners.size()) return 0;
  return m->runners[device_slot]->last_graph_kernels();
}

pkc_status pkc_profile_enable(pkc_model* m, int enable) {
  if (!m) return pkc::set_thread_error(PKC_ERR_ARG, "pkc_profile_enable: model is NULL");
  std::lock_guard<std::mutex> lk(m->mu);
  for (auto& r : m->runners) r->profile_enable(enable != 0);
  return PKC_OK;
}

int pkc_profile_read(pkc_model* m, pkc_kernel_stat* out, int cap) {
  if (!m || !out || cap <= 0) return 0;
  std::lock_guard<std::mutex> lk(m->mu);
  std::vector<pkc::KernelStatAcc> all;
  for (auto& r : m->runners)
    for (const auto& k : r->profile_read()) {
      auto it = std::find_if(all.begin(), all.end(), [&](const pkc::KernelStatAcc& a) { return a.name == k.name; });
      if (it == all.end()) all.push_back(k);
      else { it->launches += k.launches; it->ms += k.ms; it->flops += k.flops; it->bytes += k.bytes; }
    }
  const int n = std::min<int>(cap, (int)all.size());
  for (int i = 0; i < n; ++i) {
    std::memset(&out[i], 0, sizeof(out[i]));
    std::strncpy(out[i].name, all[i].name.c_str(), sizeof(out[i].name) - 1);
    out[i].launches = all[i].launches;
    out[i].total_ms = all[i].ms;
    out[i].flops = all[i].flops;
    out[i].bytes = all[i].bytes;
  }
  return n;
}

}  // extern "C"
