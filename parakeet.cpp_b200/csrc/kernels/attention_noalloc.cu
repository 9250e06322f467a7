// Rel-pos attention entry point that allocates no device memory.
//
// Who needs it: host programs that own all of the GPU's memory through their
// own allocator. Examples are a serving runtime that reserves HBM up front
// and forbids raw cudaMalloc, or an embedding host whose memory accounting
// must see every byte. For them a cudaMalloc is either refused or, worse,
// synchronises the whole device in the middle of a request.
// pkc_relpos_attention allocates its small per-call tables (tile list,
// per-utterance offsets and lengths). This variant keeps them in one
// file-scope __device__ array of fixed size instead. The caller passes every
// input and output buffer.
//
// Properties of the shared table array:
//   * It is allocated when the library is loaded, on every GPU that loads it,
//     and stays until the process exits (kNoAllocTableInts * 4 bytes = 80 KiB).
//   * Every call rewrites the part of it that the call uses, so no stale
//     contents are read. Calls that overlap on the GPU (different streams or
//     host threads at the same time) race on it and must be serialised by
//     the caller.
//   * Its device address is looked up with cudaGetSymbolAddress once per
//     device, with that device current, on the first call on that device.
//     Host code never passes the symbol itself (in host code the name is
//     only a host-side stand-in).
#include <cuda_runtime.h>

#include <mutex>
#include <string>
#include <vector>

#include "../../../include/pkc.h"
#include "../status.hpp"
#include "kernels.h"

namespace pkc {

// tiles (2 ints each) + offsets (B+1) + lengths (B)
constexpr int kNoAllocTableInts = 20480;
constexpr int kNoAllocMaxItems = 1024;

static __device__ __align__(256) int g_noalloc_tables[kNoAllocTableInts];

namespace {

int* noalloc_table_ptr(int dev, std::string& err) {
  static std::mutex mu;
  static int* ptrs[64] = {};
  static bool done[64] = {};
  if (dev < 0 || dev >= 64) {
    err = "device index out of range";
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (!done[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_tables);
    if (e != cudaSuccess || !p) {
      err = std::string("cudaGetSymbolAddress failed: ") + cudaGetErrorString(e);
      return nullptr;
    }
    ptrs[dev] = static_cast<int*>(p);
    done[dev] = true;
  }
  return ptrs[dev];
}

}  // namespace
}  // namespace pkc

extern "C" pkc_status pkc_relpos_attention_noalloc(const void* qkv, const void* ptab, int centre,
                                                   const float* bias_u, const float* bias_v,
                                                   const int* lens, int B, int d, int n_heads,
                                                   int dtype, void* ctx, void* stream) {
  using namespace pkc;
  if (!qkv || !ptab || !bias_u || !bias_v || !lens || B <= 0 || !ctx || n_heads <= 0 ||
      (dtype != 0 && dtype != 1))
    return set_thread_error(PKC_ERR_ARG, "pkc_relpos_attention_noalloc: bad arguments");
  if (B > kNoAllocMaxItems)
    return set_thread_error(PKC_ERR_ARG, "pkc_relpos_attention_noalloc: at most " +
                                             std::to_string(kNoAllocMaxItems) + " utterances per call");
  std::vector<int> host;
  host.reserve((size_t)2 * B + 1 + 64);
  host.push_back(0);
  for (int b = 0; b < B; ++b) {
    if (lens[b] <= 0 || lens[b] > centre)
      return set_thread_error(PKC_ERR_ARG, "pkc_relpos_attention_noalloc: lens must be in [1, centre]");
    host.push_back(host.back() + lens[b]);
  }
  host.insert(host.end(), lens, lens + B);
  const int qt = attn_query_tile();
  long long n_tiles = 0;
  for (int b = 0; b < B; ++b) n_tiles += (lens[b] + qt - 1) / qt;
  if ((long long)host.size() + 2 * n_tiles + 1 > kNoAllocTableInts)
    return set_thread_error(PKC_ERR_ARG,
                            "pkc_relpos_attention_noalloc: " + std::to_string(n_tiles) +
                                " query tiles exceed the fixed table (" +
                                std::to_string((kNoAllocTableInts - 1 - (int)host.size()) / 2) + " max)");
  const size_t tiles_at = host.size();
  for (int b = 0; b < B; ++b)
    for (int q0 = 0; q0 < lens[b]; q0 += qt) {
      host.push_back(b);
      host.push_back(q0);
    }
  host.push_back(0);  // device error word
  int dev = 0;
  cudaGetDevice(&dev);
  std::string err;
  int* tab = noalloc_table_ptr(dev, err);
  if (!tab) return set_thread_error(PKC_ERR_CUDA, "pkc_relpos_attention_noalloc: " + err);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(tab, host.data(), host.size() * sizeof(int), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) {
    AttnArgs a{qkv, ptab, 2 * centre - 1, centre, d, bias_u, bias_v, tab + tiles_at, (int)n_tiles,
               tab, tab + B + 1, ctx, d, n_heads, host[B], tab + host.size() - 1};
    e = attention_launch(a, dtype == 1, st);
  }
  // the host table vector must outlive the copy
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  int h_err = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&h_err, tab + host.size() - 1, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess)
    return set_thread_error(PKC_ERR_CUDA, std::string("pkc_relpos_attention_noalloc: ") + cudaGetErrorString(e));
  if (h_err != 0)
    return set_thread_error(PKC_ERR_KERNEL, "pkc_relpos_attention_noalloc: kernel error word " + std::to_string(h_err));
  return PKC_OK;
}
