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
//   * Every call rewrites the part of it that the call uses (the device error
//     word included, which starts each call at zero), so no stale contents
//     are read. Calls that overlapped on the GPU would race on it, so the
//     entry point holds one process-wide lock from its table upload until its
//     stream has finished the call's work.
//   * Its device address is looked up with cudaGetSymbolAddress once per
//     device, with that device current, on the first call on that device;
//     make that first call before any stream capture begins. The address is
//     kept for the life of the process, so the entry point must not be used
//     on a device after cudaDeviceReset (or after the primary context was
//     destroyed and re-created). Host code never passes the symbol itself (in
//     host code the name is only a host-side stand-in).
//   * The tables are built in a fixed file-scope host array of the same size
//     (under the same lock), so a call allocates nothing on the host either.
//   * Size limit: at most kNoAllocMaxItems utterances, and at most
//     (kNoAllocTableInts - 2 - 2B) / 2 query tiles of attn_query_tile() frames
//     (128), where B is the number of utterances of the call.
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <string>

#include "../../../include/pkc.h"
#include "../status.hpp"
#include "kernels.h"

namespace pkc {

// tiles (2 ints each) + offsets (B+1) + lengths (B)
constexpr int kNoAllocTableInts = 20480;
constexpr int kNoAllocMaxItems = 1024;

static __device__ __align__(256) int g_noalloc_tables[kNoAllocTableInts];

namespace {

std::mutex g_noalloc_call_mu;             // one call at a time, until its GPU work is done
int g_noalloc_host[kNoAllocTableInts];    // host image of the tables of the current call

int* noalloc_table_ptr(int dev, std::string& err) {
  static std::mutex mu;
  static std::map<int, int*> ptrs;
  std::lock_guard<std::mutex> lk(mu);
  auto it = ptrs.find(dev);
  if (it != ptrs.end()) return it->second;
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_tables);
  if (e != cudaSuccess || !p) {
    err = std::string("cudaGetSymbolAddress failed: ") + cudaGetErrorString(e);
    return nullptr;
  }
  ptrs[dev] = static_cast<int*>(p);
  return static_cast<int*>(p);
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
  for (int b = 0; b < B; ++b)
    if (lens[b] <= 0 || lens[b] > centre)
      return set_thread_error(PKC_ERR_ARG, "pkc_relpos_attention_noalloc: lens must be in [1, centre]");
  const int qt = attn_query_tile();
  long long n_tiles = 0;
  for (int b = 0; b < B; ++b) n_tiles += (lens[b] + qt - 1) / qt;
  const int n_head = 2 * B + 1;  // offsets (B + 1), then lengths (B)
  if (n_head + 2 * n_tiles + 1 > kNoAllocTableInts)
    return set_thread_error(PKC_ERR_ARG,
                            "pkc_relpos_attention_noalloc: " + std::to_string(n_tiles) + " query tiles of " +
                                std::to_string(qt) + " frames exceed the fixed table (" +
                                std::to_string((kNoAllocTableInts - 1 - n_head) / 2) + " max for " +
                                std::to_string(B) + " utterances)");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // the call waits for its stream and reads its error word back before it
  // returns, which a stream in capture mode cannot do
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cap) != cudaSuccess) {
    cudaGetLastError();
    return set_thread_error(PKC_ERR_ARG, "pkc_relpos_attention_noalloc: invalid stream");
  }
  if (cap != cudaStreamCaptureStatusNone)
    return set_thread_error(PKC_ERR_ARG,
                            "pkc_relpos_attention_noalloc: stream is capturing; this entry point synchronises "
                            "its stream and reads its error word back before returning");
  // the table address is the current device's: the stream must belong to it
  int dev = 0;
  cudaGetDevice(&dev);
  if (st) {
    int sdev = -1;
    if (cudaStreamGetDevice(st, &sdev) != cudaSuccess) {
      cudaGetLastError();
      return set_thread_error(PKC_ERR_ARG, "pkc_relpos_attention_noalloc: invalid stream");
    }
    if (sdev != dev)
      return set_thread_error(PKC_ERR_ARG, "pkc_relpos_attention_noalloc: stream belongs to device " +
                                               std::to_string(sdev) + " but device " + std::to_string(dev) +
                                               " is current; make the stream's device current");
  }
  std::lock_guard<std::mutex> call_lock(g_noalloc_call_mu);
  int* host = g_noalloc_host;
  int n = 0;
  host[n++] = 0;
  for (int b = 0; b < B; ++b, ++n) host[n] = host[n - 1] + lens[b];
  for (int b = 0; b < B; ++b) host[n++] = lens[b];
  const int tiles_at = n;
  for (int b = 0; b < B; ++b)
    for (int q0 = 0; q0 < lens[b]; q0 += qt) {
      host[n++] = b;
      host[n++] = q0;
    }
  host[n++] = 0;  // device error word
  std::string err;
  int* tab = noalloc_table_ptr(dev, err);
  if (!tab) return set_thread_error(PKC_ERR_CUDA, "pkc_relpos_attention_noalloc: " + err);
  cudaError_t e = cudaMemcpyAsync(tab, host, (size_t)n * sizeof(int), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) {
    AttnArgs a{qkv, ptab, 2 * centre - 1, centre, d, bias_u, bias_v, tab + tiles_at, (int)n_tiles,
               tab, tab + B + 1, ctx, d, n_heads, host[B], tab + n - 1};
    e = attention_launch(a, dtype == 1, st);
  }
  // the host tables are reused by the next call: finish this one's copy and kernel first
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  int h_err = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&h_err, tab + n - 1, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess)
    return set_thread_error(PKC_ERR_CUDA, std::string("pkc_relpos_attention_noalloc: ") + cudaGetErrorString(e));
  if (h_err != 0)
    return set_thread_error(PKC_ERR_KERNEL, "pkc_relpos_attention_noalloc: kernel error word " + std::to_string(h_err));
  return PKC_OK;
}
