/*
 * pkc.h — C ABI of the B200 FastConformer encoder library (libpkc.so).
 *
 * This is the seam parakeet.cpp's host code calls instead of building ggml
 * graphs for the encoder hot path. Every entry point is plain C: opaque
 * handles, raw pointers and sizes, integer status codes, no exceptions and no
 * torch or CUDA types in the signatures (CUDA streams travel as void*).
 *
 * Reference interfaces replaced (paths inside parakeet.cpp):
 *   pkc_model_open        ModelLoader::load + realize_weights + Backend init
 *                         (src/model_loader.cpp:99-166, :47-98; src/backend.cpp:61-113)
 *   pkc_mel_batch         GpuMel::compute per clip + build_mel_batch
 *                         (src/mel_gpu.cpp:34-162; src/model.cpp:119-144)
 *   pkc_encode_batch      Encoder::forward_batch (src/encoder.hpp:43-46, src/encoder.cpp:97-167)
 *   pkc_encode_pcm_batch  steps 1-2 of Model::transcribe_16k_batch (src/model.cpp:164-181)
 *   pkc_last_error        parakeet_capi_last_error (include/parakeet_capi.h:136)
 *
 * Threading: one call per pkc_model at a time (the reference serialises every
 * graph on one global mutex, src/ggml_graph.cpp:84). Different models may be
 * used from different threads.
 *
 * Ownership: the caller owns every buffer passed in; the model owns its device
 * weights and workspaces. Nothing returned needs freeing except the model.
 */
#ifndef PKC_H
#define PKC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PKC_ABI_VERSION 1

typedef struct pkc_model pkc_model;

typedef enum pkc_status {
  PKC_OK = 0,
  PKC_ERR_ARG = 1,          /* invalid argument (NULL pointer, bad size, ...) */
  PKC_ERR_IO = 2,           /* file could not be opened or read */
  PKC_ERR_FORMAT = 3,       /* malformed GGUF or missing tensor / key */
  PKC_ERR_UNSUPPORTED = 4,  /* configuration outside what the kernels implement */
  PKC_ERR_CUDA = 5,         /* CUDA runtime error (launch, copy, allocation) */
  PKC_ERR_OOM = 6,          /* device or host allocation failed */
  PKC_ERR_KERNEL = 7,       /* a kernel reported an error through its error word */
  PKC_ERR_INTERNAL = 8
} pkc_status;

/* Output layouts of the encoder entry points. */
typedef enum pkc_layout {
  /* per item channels-first [d_model, valid_Tout[b]] (enc[c*T + t]), items
     concatenated; this is what Encoder::forward_batch returns per item */
  PKC_LAYOUT_CHANNELS_FIRST = 0,
  /* per item time-major [valid_Tout[b], d_model] (enc[t*d + c]), items
     concatenated; what the transducer decoders consume (src/model.cpp:148-162) */
  PKC_LAYOUT_TIME_MAJOR = 1
} pkc_layout;

typedef struct pkc_model_info {
  int d_model, n_layers, n_heads, ff_dim, conv_kernel;
  int n_mels, n_fft, win_length, hop_length, sample_rate;
  int subsampling_factor, subsampling_conv_channels;
  int xscaling;
  int weight_type;  /* GGUF type id of the encoder linear weights (0 f32, 1 f16, 8 q8_0, 12 q4_k, 30 bf16) */
  int compute_bf16; /* 1: bf16 tensor-core operands, 0: f16 */
  int n_devices;
  int vocab_size, blank_id;
  char arch[32];
} pkc_model_info;

/* ABI version of this header/implementation (PKC_ABI_VERSION). */
int pkc_abi_version(void);

/* Human-readable description of the last error on `m`, or of the last failed
   pkc_model_open on this thread when m is NULL. Never NULL. */
const char* pkc_last_error(const pkc_model* m);

/* Load a parakeet GGUF and upload the encoder weights to each listed CUDA
   device (devices == NULL or n_devices == 0: device 0). Weights are re-packed
   once on the host into the kernels' layouts, page-locked, and copied to all
   listed devices concurrently (one host thread per device).
   Pre-pack cache: when the environment variable PKC_PACK_CACHE names a
   directory, the packed image is read from there if a file for this GGUF
   (path, size, modification time) and these packing options exists, else it
   is written there after packing; a damaged or stale file is ignored. */
pkc_status pkc_model_open(const char* gguf_path, const int* devices, int n_devices,
                          pkc_model** out);

/* ---- Cache-aware streaming encoder (StreamingEncoder, src/streaming_encoder.hpp:33-66).
   For models with a parakeet.streaming.* schedule, chunked-limited attention,
   causal subsampling and causal depthwise conv (e.g. the 120M EOU model). The
   caller computes the log-mel of the audio and feeds it window by window: the
   first window is chunk_size_first frames, later ones chunk_size new frames
   preceded by pre_encode_cache_size frames of overlap. Each step returns the
   chunk's valid encoder frames; the concatenation equals the offline
   encoder's output except the final chunk's valid_out_len tail. */
typedef struct pkc_stream pkc_stream;

typedef struct pkc_stream_schedule {
  int chunk_size_first;       /* mel frames of the first window */
  int chunk_size;             /* new mel frames per later window (also the shift) */
  int pre_encode_cache_size;  /* overlap frames prepended to later windows */
  int valid_out_len;          /* encoder frames a mid-stream step returns */
  int drop_extra_pre_encoded; /* subsampled frames dropped from later windows */
  int attention_cache_size;   /* frames of left attention context kept per layer */
} pkc_stream_schedule;

/* chunk_size_first() / chunk_size() / pre_encode_cache_size() / valid_out_len()
   of the reference; PKC_ERR_UNSUPPORTED for a model without a streaming schedule. */
pkc_status pkc_stream_schedule_get(const pkc_model* m, pkc_stream_schedule* out);

/* StreamingEncoder(ml) + reset(): a stream with zero caches on the model's
   device_slot-th device (index into the devices passed to pkc_model_open).
   PKC_ERR_UNSUPPORTED unless the model is a cache-aware streaming model. The
   model must outlive the stream. Steps of different streams on one model run
   one at a time. */
pkc_status pkc_stream_begin(pkc_model* m, int device_slot, pkc_stream** out);

/* reset(): zero the caches, step counter to 0 (a fresh stream). */
pkc_status pkc_stream_reset(pkc_stream* s);

/* step(mel_chunk_frames, n_mel_frames, is_last, n_valid_out): mel is
   [n_mels][n_frames] f32 host memory, feature-major (mel[m * n_frames + t]),
   the whole window including the overlap. out receives [n_valid_out][d_model]
   time-major f32 (out_cap_floats >= valid frames * d_model, at most
   (n_frames / 8 + 2) * d_model); mid-stream steps return valid_out_len
   frames, the last (is_last != 0) all of the chunk's frames. A window too
   short to produce a frame returns 0 frames and still advances the step. */
pkc_status pkc_stream_step(pkc_stream* s, const float* mel, int n_frames, int is_last, float* out,
                           size_t out_cap_floats, int* n_valid_out);

/* Several streams of one model stepped together, one window each: their
   frames are stacked so every weight is read once for all of them (the
   serving form of step()). All streams belong to the same model and device
   slot, every window is n_frames long, and the streams are all at their first
   window or all past it. outs[i] receives stream i's valid frames
   (n_valid_out[i] of them, out_cap_floats >= that * d_model); is_last[i] as in
   pkc_stream_step. Up to 16 stacked frames the result equals stepping each
   stream alone bit for bit. */
pkc_status pkc_stream_step_batch(pkc_stream* const* streams, int n_streams, const float* const* mels, int n_frames,
                                 const int* is_last, float* const* outs, size_t out_cap_floats, int* n_valid_out);

/* step_num(): steps taken since begin / reset; -1 for NULL. */
int pkc_stream_step_num(const pkc_stream* s);

/* Release the stream's device caches. Safe on NULL. */
void pkc_stream_free(pkc_stream* s);

/* Timing of the last pkc_model_open of m: host seconds spent re-packing (or
   reading the pre-pack cache), seconds of the slowest device's upload, and
   whether the image came from the cache (1) or was packed (0). */
pkc_status pkc_model_load_stats(const pkc_model* m, double* pack_seconds, double* upload_seconds,
                                int* from_cache);

/* Host only (no CUDA call): make sure the pre-pack cache directory holds the
   packed image of gguf_path for the current packing options, packing it if
   needed. Writes the cache file's path to path_out (path_cap bytes) if given. */
pkc_status pkc_pack_cache_build(const char* gguf_path, const char* cache_dir, char* path_out, int path_cap);

/* Release the model and all device memory it holds. Safe on NULL. */
void pkc_model_close(pkc_model* m);

pkc_status pkc_model_info_get(const pkc_model* m, pkc_model_info* out);

/* Number of mel frames the front end produces for a clip of n samples
   (1 + n / hop, the reference's n_frames for n_fft == 2*pad). */
int pkc_mel_frames(const pkc_model* m, int n_samples);

/* Number of encoder output frames for a clip whose mel has T frames (the
   reference's Subsampling::valid_out_len with the offline T-1 convention). */
int pkc_encoder_frames(const pkc_model* m, int mel_frames);

/* Batched log-mel front end (16 kHz mono f32 PCM, one pointer per clip).
   feats_out: [B][n_mels][T_max] f32, zero padded (the reference's MelBatch),
   where T_max = max_b mel_frames(n_samples[b]); T_out[b] receives each clip's
   frame count. feats_cap is the capacity of feats_out in floats. */
pkc_status pkc_mel_batch(pkc_model* m, const float* const* pcm, const int* n_samples, int B,
                         float* feats_out, size_t feats_cap, int* T_out);

/* Batched encoder on a host MelBatch ([B][n_mels][T_max] f32, valid_T[b] true
   mel frames). Writes every item's encoder output into `out` (layout as
   requested, items concatenated), valid_Tout[b] its frame count. out_cap is
   the capacity of out in floats; d_model_out may be NULL. */
pkc_status pkc_encode_batch(pkc_model* m, const float* mel, int B, int n_mels, int T_max,
                            const int* valid_T, int layout, float* out, size_t out_cap,
                            int* valid_Tout, int* d_model_out);

/* PCM -> encoder output in one call (mel front end + encoder), host buffers.
   With several devices the clips are sharded across them by length (one host
   thread per device, each copying its clips' outputs straight into `out`); a
   device's failure returns that device's status and message. Failure
   injection for tests: the environment variable PKC_FAULT_DEVICE_SLOT=k makes
   the worker of device slot k fail on the host before it touches its device
   (PKC_ERR_INTERNAL). */
pkc_status pkc_encode_pcm_batch(pkc_model* m, const float* const* pcm, const int* n_samples,
                                int B, int layout, float* out, size_t out_cap, int* valid_Tout);

/* One decoded token, laid out as the reference's TokenInfo
   (src/decode_types.hpp:27-32): vocabulary id, frame (the token's
   start_offset in encoder frames), confidence (NeMo's max_prob, min over the
   token's argmax run) and span (1, as ctc_greedy emits it). */
typedef struct pkc_token {
  int32_t id;
  int32_t frame;
  float conf;
  int32_t span;
} pkc_token;

/* Classes of the model's CTC head (vocab + 1, the blank included), 0 if the
   GGUF has no CTC head (ctc_decoder.decoder_layers.0.* of hybrid models or
   decoder.decoder_layers.0.* of CTC models, src/ctc_decoder.cpp:17-28). */
int pkc_ctc_classes(const pkc_model* m);

/* CTC transcription of B clips of PCM: mel front end + encoder + CTC head on
   the GPU (the linear d -> V+1 and log_softmax of CTCDecoder::forward,
   src/ctc_decoder.cpp:35-116, with the per-frame argmax and maximum
   log-probability), then the greedy fold of ctc_greedy (src/search.cpp:21-90)
   on the host. tokens_out receives the clips' tokens back to back,
   n_tokens[b] clip b's count (a clip yields at most its encoder frame count,
   so tokens_cap = the sum of those always suffices). logprobs_out may be NULL;
   else it receives the log-probabilities [sum T'_b, V+1] time-major, clips
   back to back (logprobs_cap floats). */
pkc_status pkc_ctc_greedy_pcm_batch(pkc_model* m, const float* const* pcm, const int* n_samples, int B,
                                    pkc_token* tokens_out, size_t tokens_cap, int* n_tokens,
                                    float* logprobs_out, size_t logprobs_cap);

/* The greedy fold alone (host arithmetic, no device): T frames of per-frame
   argmax class and maximum log-probability -> tokens, following ctc_greedy
   (src/search.cpp:21-90) over n_classes classes with the given blank id.
   Returns the token count, or -1 if it exceeds cap (cap >= T always
   suffices) or the arguments are invalid. */
int pkc_ctc_fold(const int32_t* argmax, const float* max_logprob, int T, int n_classes, int blank_id,
                 pkc_token* out, int cap);

/* Kind of the model's transducer decoder: 0 none, 1 RNN-T, 2 TDT (durations
   in parakeet.tdt.durations). */
int pkc_transducer_kind(const pkc_model* m);

/* Greedy transducer transcription of B clips of PCM, all on the GPU: mel front
   end + encoder, the joint's encoder projection, then the greedy loop of
   tdt_greedy (src/tdt.cpp:8-126) or rnnt_greedy (src/rnnt.cpp:110-122) --
   prediction LSTM, joint, argmax, max_symbols -- for all clips in lockstep.
   Tokens as the reference's TokenInfo: frame = encoder frame of the emission,
   conf = max_prob over the token classes, span = the TDT duration (1 for
   RNN-T). tokens_out receives the clips' tokens back to back, n_tokens[b]
   clip b's count (at most T'_b * max_symbols). */
pkc_status pkc_transducer_greedy_pcm_batch(pkc_model* m, const float* const* pcm, const int* n_samples, int B,
                                           pkc_token* tokens_out, size_t tokens_cap, int* n_tokens);

/* Floats needed by pkc_encode_pcm_batch's `out` for these clip lengths. */
size_t pkc_encode_out_floats(const pkc_model* m, const int* n_samples, int B);

/* Device-resident variant on one device of the model: d_pcm holds the clips
   concatenated (f32, already in that device's memory), d_out receives the
   outputs (time-major, items concatenated). `stream` is a cudaStream_t or
   NULL for the model's own stream. Asynchronous with respect to the host
   unless sync != 0. */
pkc_status pkc_encode_pcm_device(pkc_model* m, int device_slot, const float* d_pcm,
                                 const int* n_samples, int B, float* d_out, void* stream,
                                 int sync);

/* The CUDA stream (a cudaStream_t, as void*) that the host-buffer entry points
   of device slot `device_slot` run on; lets a caller bracket a call with its
   own events. NULL for a bad slot. */
void* pkc_model_stream(const pkc_model* m, int device_slot);

/* Kernel launches of the CUDA graph that device slot `device_slot` launched
   most recently (its kernel nodes, counted once when the graph was
   instantiated); 0 before any graph launch, with PKC_NO_GRAPH=1, or for a bad
   slot. A diagnostic with no counterpart in the reference. */
int pkc_last_graph_kernels(const pkc_model* m, int device_slot);

/* Per-kernel-class timing (CUDA events around every launch on the model's
   stream). enable != 0 turns it on and clears the accumulators. */
pkc_status pkc_profile_enable(pkc_model* m, int enable);
/* Copy up to cap entries of {name, launches, total_ms, flops, bytes}. Returns
   the number of kernel classes recorded. */
typedef struct pkc_kernel_stat {
  char name[32];
  long long launches;
  double total_ms;
  double flops;  /* algorithmic FLOPs summed over launches */
  double bytes;  /* algorithmic HBM bytes summed over launches */
} pkc_kernel_stat;
int pkc_profile_read(pkc_model* m, pkc_kernel_stat* out, int cap);

/* Assign B clips to n_dev devices (longest-processing-time greedy on the
   cost T'(c1 + c2 T') of each clip's encoder length). assign[b] receives the
   device slot of clip b. Pure host arithmetic. */
pkc_status pkc_shard_plan(const int* n_samples, int B, int n_dev, int hop, int* assign);

/* ---- kernel-level entry points (used by the parity tests; device pointers) */

/* D[M,N] = A[M,K] * B[N,K]^T with a fused epilogue on the tcgen05 GEMM.
   dtype 0 = f16, 1 = bf16 operands; epi/act as in the kernel header. M <= 16
   (K <= 4096, epi 0-3) runs the skinny CUDA-core kernel the streaming encoder
   uses (PKC_GEMM_SKINNY=0: the tcgen05 tile for every M). Bw and bias are
   treated as weights: the kernel may start reading them before the kernel
   launched before it on `stream` has finished (programmatic dependent
   launch), so that kernel must not write them; A and out wait for it. */
pkc_status pkc_gemm(const void* A, int lda, const void* Bw, int ldb, int M, int N, int K,
                    int dtype, int epi, int act, float alpha, const float* bias, void* out,
                    int ldo, void* stream);

/* x[M,N] += alpha * (A[M,K] * B[N,K]^T + bias) in f32 (the residual update of
   the encoder's FFN-down, attention-out and pointwise-conv-2 GEMMs), and, if
   stats is not null, the per-row statistics of the updated x in 128-column
   chunks: stats[(m * (N/128) + c) * 2 + {0,1}] = (mean, sum of squared
   deviations) of x[m, 128c .. 128c+127]. No counterpart in the reference (its
   graph keeps ggml_add and ggml_norm as separate nodes, src/encoder.cpp). */
pkc_status pkc_gemm_resid_stats(const void* A, int lda, const void* Bw, int ldb, int M, int N, int K,
                                int dtype, float alpha, const float* bias, float* x, int ldx,
                                float* stats, void* stream);

/* out = xhat * Bw[N,K]^T + bias with a fused epilogue, xhat = (x - mean) *
   rstd per row (ggml_norm: population variance over K, eps 1e-5) computed
   while the A operand is staged. With Bw = W diag(gamma) and bias = W beta + b
   this is LayerNorm(x; gamma, beta) * W^T + b, the pre-norm + linear of the
   reference's MHSA / conv / FFN blocks (src/encoder.cpp: ggml_norm ->
   ggml_mul -> ggml_add -> ggml_mul_mat); the encoder folds gamma / beta that
   way when it loads the weights. x f32 [M, ldx]; stats as written by
   pkc_gemm_resid_stats for the same x (N there = K here); K a multiple of
   128. epi 0 (store) or 3 (GLU); act as in pkc_gemm. */
pkc_status pkc_gemm_ln(const float* x, int ldx, const float* stats, const void* Bw, int ldb, int M,
                       int N, int K, int dtype, int epi, int act, const float* bias, void* out, int ldo,
                       void* stream);

/* The split-f16 GEMM of the f32-accurate path (f32 GGUF weights): A is
   [M, 2Ks] f16 rows [A_hi | A_lo] and Bw [N, 2Ks] rows [B_hi | B_lo] with
   hi = f16(v), lo = f16(v - hi) (row strides lda / ldb elements); the kernel
   accumulates A_hi B_hi^T + A_hi B_lo^T + A_lo B_hi^T in f32 (~22 significant
   bits per product) and applies epilogue epi / act as pkc_gemm. ofmt (epi 0
   and 3 only): 0 f16, 1 f32, 2 split-f16 rows with the lo half at column +
   split_ld. Replaces the F32 mul_mat of the reference's graphs
   (src/conformer.cpp:319-324, src/relpos_attention.cpp:191-194,305). */
pkc_status pkc_gemm_split(const void* A, int lda, const void* Bw, int ldb, int M, int N, int Ks, int epi, int act,
                          float alpha, const float* bias, void* out, int ldo, int ofmt, int split_ld, void* stream);

/* Relative-position attention of one layer for B utterances packed along
   rows (item b owns rows [off_b, off_b + len[b])). qkv [M, 3d] and ptab
   [2*centre-1, d] in the compute type (dtype 0 f16, 1 bf16), bias_u/v [d] f32,
   ctx [M, d] out. centre >= max len. Device pointers; lens on the host. */
pkc_status pkc_relpos_attention(const void* qkv, const void* ptab, int centre,
                                const float* bias_u, const float* bias_v, const int* lens, int B,
                                int d, int n_heads, int dtype, void* ctx, void* stream);

/* The conv module's depthwise stage for B utterances packed along rows (item
   b owns rows [off_b, off_b + lens[b]), lens on the host, zero allowed):
   out = SiLU((depthwise Conv1d(in; w, pad (K-1)/2, zeros outside the item) +
   bias) * scale + shift), i.e. the BatchNorm folded to scale / shift. in /
   out [sum lens, d] in the compute type (dtype 0 f16, 1 bf16), w [K][d],
   bias (may be null), scale, shift [d] f32; K in {3, 5, 7, 9}, d % 8 == 0.
   Device pointers. Replaces the depthwise conv + batch_norm + silu nodes of
   src/conformer.cpp:112-154. */
pkc_status pkc_conv_depthwise(const void* in, const int* lens, int B, int d, int K, const float* w,
                              const float* bias, const float* scale, const float* shift, int dtype,
                              void* out, void* stream);

/* Failure detection check: runs this library's bounded-wait helpers (every
   mbarrier wait and cross-CTA flag wait of its kernels uses them) on a
   condition that never comes true -- kind 0: an mbarrier no thread arrives
   on, kind 1: a global flag no thread sets -- with a limit of limit_ms
   (0 < limit_ms <= 2000; the kernels' own limit is 2000 ms). The wait runs
   out, records its code in the device error word (*error_code, 108) and the
   kernel returns: PKC_ERR_KERNEL, with the CUDA context still usable. No
   counterpart in the reference (its failures are host status codes only,
   src/parakeet_capi.cpp:207-294). */
pkc_status pkc_bounded_wait_check(int kind, double limit_ms, int* error_code);

/* The attention of the f32-accurate path: qkv f32 [M, 3d], ptab f32
   [2*centre-1, d], everything in f32 (softmax with expf); ctx receives f16
   rows [hi | lo] of width 2d (hi = f16(v), lo = f16(v - hi)), the split
   operand of the output projection. Other arguments as pkc_relpos_attention
   (src/relpos_attention.cpp:162-306). */
pkc_status pkc_relpos_attention_f32(const float* qkv, const float* ptab, int centre, const float* bias_u,
                                    const float* bias_v, const int* lens, int B, int d, int n_heads, void* ctx,
                                    void* stream);

/* The same attention as pkc_relpos_attention, for callers that may not
   allocate device memory: hosts whose own allocator owns all of HBM (a serving
   runtime that reserves memory up front, or one whose accounting must see
   every byte), where a cudaMalloc is refused or stalls the whole device. No
   counterpart in the reference. Its small tables live in one fixed 80 KiB
   device array that the library holds on each GPU until exit. Limits: at most
   1024 utterances, and at most (20478 - 2B) / 2 query tiles of 128 frames
   (about 10,000 tiles; B = utterances of the call); larger calls fail with
   PKC_ERR_ARG. `stream` must belong to the current device (else PKC_ERR_ARG),
   and a stream in capture mode is rejected with PKC_ERR_ARG. The first call
   on a device looks up the array's address; make it before any stream
   capture begins, and do not use this entry point on a device after
   cudaDeviceReset. Calls that overlapped on the GPU would race on the shared
   array, so the library runs one call at a time per process and returns only
   after the call's work on `stream` has finished. */
pkc_status pkc_relpos_attention_noalloc(const void* qkv, const void* ptab, int centre,
                                        const float* bias_u, const float* bias_v, const int* lens,
                                        int B, int d, int n_heads, int dtype, void* ctx,
                                        void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PKC_H */
