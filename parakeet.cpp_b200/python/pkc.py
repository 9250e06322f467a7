"""ctypes binding of libpkc.so (include/pkc.h).

This is the Python face of the C ABI used by the tests, bench.py and
__graft_entry__.py. It mirrors the reference's operator interface for the
encoder path: Encoder::forward_batch (src/encoder.hpp:43), GpuMel::compute +
build_mel_batch (src/mel_gpu.hpp:20, src/model.cpp:119) and the C-API error
convention (status code + last_error string, include/parakeet_capi.h:136).

There is no fallback: if libpkc.so is missing or a call fails, an exception is
raised.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char, c_char_p, c_double, c_float, c_int, c_longlong, c_size_t, c_void_p

import numpy as np

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "libpkc.so")

PKC_OK = 0
STATUS_NAMES = {
    0: "PKC_OK", 1: "PKC_ERR_ARG", 2: "PKC_ERR_IO", 3: "PKC_ERR_FORMAT",
    4: "PKC_ERR_UNSUPPORTED", 5: "PKC_ERR_CUDA", 6: "PKC_ERR_OOM", 7: "PKC_ERR_KERNEL",
    8: "PKC_ERR_INTERNAL",
}
(PKC_ERR_ARG, PKC_ERR_IO, PKC_ERR_FORMAT, PKC_ERR_UNSUPPORTED, PKC_ERR_CUDA, PKC_ERR_OOM, PKC_ERR_KERNEL,
 PKC_ERR_INTERNAL) = range(1, 9)
LAYOUT_CHANNELS_FIRST = 0
LAYOUT_TIME_MAJOR = 1

EPI_STORE_H, EPI_RESID_F32, EPI_STORE_F32, EPI_GLU_H, EPI_POWER_F32 = range(5)
ACT_NONE, ACT_SILU, ACT_RELU = range(3)


class PkcError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


class ModelInfo(ctypes.Structure):
    _fields_ = [
        ("d_model", c_int), ("n_layers", c_int), ("n_heads", c_int), ("ff_dim", c_int),
        ("conv_kernel", c_int), ("n_mels", c_int), ("n_fft", c_int), ("win_length", c_int),
        ("hop_length", c_int), ("sample_rate", c_int), ("subsampling_factor", c_int),
        ("subsampling_conv_channels", c_int), ("xscaling", c_int), ("weight_type", c_int),
        ("compute_bf16", c_int), ("n_devices", c_int), ("vocab_size", c_int),
        ("blank_id", c_int), ("arch", c_char * 32),
    ]


class StreamSchedule(ctypes.Structure):
    _fields_ = [(n, c_int) for n in ("chunk_size_first", "chunk_size", "pre_encode_cache_size", "valid_out_len",
                                     "drop_extra_pre_encoded", "attention_cache_size")]


class Token(ctypes.Structure):
    """pkc_token: the reference's TokenInfo (src/decode_types.hpp:27)."""
    _fields_ = [("id", ctypes.c_int32), ("frame", ctypes.c_int32), ("conf", c_float), ("span", ctypes.c_int32)]


class KernelStat(ctypes.Structure):
    _fields_ = [("name", c_char * 32), ("launches", c_longlong), ("total_ms", c_double),
                ("flops", c_double), ("bytes", c_double)]


_lib = None


def lib():
    """Load libpkc.so once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(f"{LIB_PATH} not built; run __graft_entry__.build()")
        L = ctypes.CDLL(LIB_PATH)
        _declare(L)
        _lib = L
    return _lib


def _declare(L):
    def fn(name, res, *args):
        f = getattr(L, name)
        f.restype = res
        f.argtypes = list(args)
    fn("pkc_abi_version", c_int)
    fn("pkc_last_error", c_char_p, c_void_p)
    fn("pkc_gemm", c_int, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
       c_int, c_float, c_void_p, c_void_p, c_int, c_void_p)
    optional = [
        ("pkc_model_open", c_int, c_char_p, POINTER(c_int), c_int, POINTER(c_void_p)),
        ("pkc_model_close", None, c_void_p),
        ("pkc_model_load_stats", c_int, c_void_p, POINTER(ctypes.c_double), POINTER(ctypes.c_double), POINTER(c_int)),
        ("pkc_stream_schedule_get", c_int, c_void_p, POINTER(StreamSchedule)),
        ("pkc_stream_begin", c_int, c_void_p, c_int, POINTER(c_void_p)),
        ("pkc_stream_reset", c_int, c_void_p),
        ("pkc_stream_step", c_int, c_void_p, c_void_p, c_int, c_int, c_void_p, c_size_t, POINTER(c_int)),
        ("pkc_stream_step_num", c_int, c_void_p),
        ("pkc_stream_step_batch", c_int, POINTER(c_void_p), c_int, POINTER(c_void_p), c_int, POINTER(c_int),
         POINTER(c_void_p), c_size_t, POINTER(c_int)),
        ("pkc_stream_free", None, c_void_p),
        ("pkc_pack_cache_build", c_int, c_char_p, c_char_p, ctypes.c_char_p, c_int),
        ("pkc_model_info_get", c_int, c_void_p, POINTER(ModelInfo)),
        ("pkc_mel_frames", c_int, c_void_p, c_int),
        ("pkc_encoder_frames", c_int, c_void_p, c_int),
        ("pkc_mel_batch", c_int, c_void_p, POINTER(c_void_p), POINTER(c_int), c_int, c_void_p,
         c_size_t, POINTER(c_int)),
        ("pkc_encode_batch", c_int, c_void_p, c_void_p, c_int, c_int, c_int, POINTER(c_int), c_int,
         c_void_p, c_size_t, POINTER(c_int), POINTER(c_int)),
        ("pkc_encode_pcm_batch", c_int, c_void_p, POINTER(c_void_p), POINTER(c_int), c_int, c_int,
         c_void_p, c_size_t, POINTER(c_int)),
        ("pkc_encode_out_floats", c_size_t, c_void_p, POINTER(c_int), c_int),
        ("pkc_encode_pcm_device", c_int, c_void_p, c_int, c_void_p, POINTER(c_int), c_int,
         c_void_p, c_void_p, c_int),
        ("pkc_profile_enable", c_int, c_void_p, c_int),
        ("pkc_model_stream", c_void_p, c_void_p, c_int),
        ("pkc_last_graph_kernels", c_int, c_void_p, c_int),
        ("pkc_profile_read", c_int, c_void_p, POINTER(KernelStat), c_int),
        ("pkc_shard_plan", c_int, POINTER(c_int), c_int, c_int, c_int, POINTER(c_int)),
        ("pkc_ctc_classes", c_int, c_void_p),
        ("pkc_transducer_kind", c_int, c_void_p),
        ("pkc_transducer_greedy_pcm_batch", c_int, c_void_p, POINTER(c_void_p), POINTER(c_int), c_int,
         POINTER(Token), c_size_t, POINTER(c_int)),
        ("pkc_ctc_greedy_pcm_batch", c_int, c_void_p, POINTER(c_void_p), POINTER(c_int), c_int, POINTER(Token),
         c_size_t, POINTER(c_int), c_void_p, c_size_t),
        ("pkc_ctc_fold", c_int, c_void_p, c_void_p, c_int, c_int, c_int, POINTER(Token), c_int),
        ("pkc_gemm_resid_stats", c_int, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int,
         c_float, c_void_p, c_void_p, c_int, c_void_p, c_void_p),
        ("pkc_gemm_ln", c_int, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
         c_int, c_int, c_void_p, c_void_p, c_int, c_void_p),
        ("pkc_relpos_attention", c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p, POINTER(c_int),
         c_int, c_int, c_int, c_int, c_void_p, c_void_p),
        ("pkc_relpos_attention_noalloc", c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p,
         POINTER(c_int), c_int, c_int, c_int, c_int, c_void_p, c_void_p),
        ("pkc_gemm_split", c_int, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
         c_float, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p),
        ("pkc_relpos_attention_f32", c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p, POINTER(c_int),
         c_int, c_int, c_int, c_void_p, c_void_p),
        ("pkc_bounded_wait_check", c_int, c_int, ctypes.c_double, POINTER(c_int)),
        ("pkc_conv_depthwise", c_int, c_void_p, POINTER(c_int), c_int, c_int, c_int, c_void_p, c_void_p,
         c_void_p, c_void_p, c_int, c_void_p, c_void_p),
    ]
    for name, res, *args in optional:
        if hasattr(L, name):
            fn(name, res, *args)


def _check(status: int, model=None):
    if status != PKC_OK:
        msg = lib().pkc_last_error(model)
        raise PkcError(status, msg.decode() if msg else "")


def _ints(xs):
    arr = (c_int * len(xs))(*[int(x) for x in xs])
    return arr


def gemm(A, B, M, N, K, *, bf16, epi, act=ACT_NONE, alpha=1.0, bias=None, out, ldo,
         lda=None, ldb=None, stream=0):
    """D = A[M,K] * B[N,K]^T with a fused epilogue (device pointers as ints)."""
    _check(lib().pkc_gemm(c_void_p(A), lda or K, c_void_p(B), ldb or K, M, N, K, 1 if bf16 else 0,
                          epi, act, alpha, c_void_p(bias) if bias else None, c_void_p(out), ldo,
                          c_void_p(stream) if stream else None))


OUT_H, OUT_F32, OUT_SPLIT = 0, 1, 2


def gemm_split(A, B, M, N, Ks, *, epi, act=ACT_NONE, alpha=1.0, bias=None, out, ldo, ofmt=OUT_H, split_ld=0,
               lda=None, ldb=None, stream=0):
    """Split-f16 GEMM of the f32-accurate path: A [M, 2Ks] and B [N, 2Ks] f16
    rows [hi | lo] (device pointers as ints)."""
    _check(lib().pkc_gemm_split(c_void_p(A), lda or 2 * Ks, c_void_p(B), ldb or 2 * Ks, M, N, Ks, epi, act, alpha,
                                c_void_p(bias) if bias else None, c_void_p(out), ldo, ofmt, split_ld,
                                c_void_p(stream) if stream else None))


def relpos_attention_f32(qkv, ptab, centre, bias_u, bias_v, lens, d, n_heads, *, ctx, stream=0):
    """f32 rel-pos attention (f32 qkv / ptab in, split-f16 [M, 2d] ctx out)."""
    _check(lib().pkc_relpos_attention_f32(c_void_p(qkv), c_void_p(ptab), centre, c_void_p(bias_u), c_void_p(bias_v),
                                          _ints(lens), len(lens), d, n_heads, c_void_p(ctx),
                                          c_void_p(stream) if stream else None))


def bounded_wait_check(kind, limit_ms):
    """pkc_bounded_wait_check: (status, device error code) of a bounded wait
    on a condition that never comes true (kind 0 mbarrier, 1 global flag)."""
    code = c_int(0)
    st = lib().pkc_bounded_wait_check(kind, float(limit_ms), ctypes.byref(code))
    return st, code.value


def ctc_fold(argmax, max_logprob, n_classes, blank_id):
    """The greedy CTC fold (host arithmetic): per-frame argmax classes and
    maximum log-probabilities -> list of (id, frame, conf, span)."""
    a = np.ascontiguousarray(argmax, dtype=np.int32)
    lp = np.ascontiguousarray(max_logprob, dtype=np.float32)
    T = len(a)
    out = (Token * max(T, 1))()
    n = lib().pkc_ctc_fold(a.ctypes.data, lp.ctypes.data, T, n_classes, blank_id, out, max(T, 1))
    if n < 0:
        raise PkcError(1, "pkc_ctc_fold: bad arguments")
    return [(t.id, t.frame, t.conf, t.span) for t in out[:n]]


def gemm_resid_stats(A, B, M, N, K, *, bf16, alpha=1.0, bias=None, x, ldx=None, stats=None,
                     lda=None, ldb=None, stream=0):
    """x[M,N] += alpha * (A * B^T + bias) in f32, plus x's per-128-column row
    statistics (mean, M2) into stats [M, N/128, 2] when given (device pointers)."""
    _check(lib().pkc_gemm_resid_stats(c_void_p(A), lda or K, c_void_p(B), ldb or K, M, N, K,
                                      1 if bf16 else 0, alpha, c_void_p(bias) if bias else None,
                                      c_void_p(x), ldx or N, c_void_p(stats) if stats else None,
                                      c_void_p(stream) if stream else None))


def gemm_ln(x, stats, B, M, N, K, *, bf16, epi=EPI_STORE_H, act=ACT_NONE, bias=None, out, ldo, ldx=None,
            ldb=None, stream=0):
    """out = xhat * B^T + bias, xhat = (x - mean) * rstd per row computed
    while the GEMM stages its A operand; a LayerNorm's gamma / beta go into B
    (B = W diag(gamma)) and the bias (W beta + b). Device pointers as ints."""
    _check(lib().pkc_gemm_ln(c_void_p(x), ldx or K, c_void_p(stats), c_void_p(B), ldb or K, M, N, K,
                             1 if bf16 else 0, epi, act, c_void_p(bias) if bias else None, c_void_p(out), ldo,
                             c_void_p(stream) if stream else None))


def relpos_attention(qkv, ptab, centre, bias_u, bias_v, lens, d, n_heads, *, bf16, ctx, stream=0):
    """Rel-pos attention kernel on packed rows (device pointers as ints)."""
    _check(lib().pkc_relpos_attention(c_void_p(qkv), c_void_p(ptab), centre, c_void_p(bias_u),
                                      c_void_p(bias_v), _ints(lens), len(lens), d, n_heads,
                                      1 if bf16 else 0, c_void_p(ctx), c_void_p(stream) if stream else None))


def conv_depthwise(x, lens, d, K, w, bias, scale, shift, *, bf16, out, stream=0):
    """Conv module depthwise stage (depthwise Conv1d + bias, folded BatchNorm,
    SiLU) on packed rows; device pointers as ints, bias may be 0."""
    _check(lib().pkc_conv_depthwise(c_void_p(x), _ints(lens), len(lens), d, K, c_void_p(w),
                                    c_void_p(bias) if bias else None, c_void_p(scale), c_void_p(shift),
                                    1 if bf16 else 0, c_void_p(out), c_void_p(stream) if stream else None))


def relpos_attention_noalloc(qkv, ptab, centre, bias_u, bias_v, lens, d, n_heads, *, bf16, ctx,
                             stream=0):
    """The attention entry point that allocates no device memory (fixed
    tables inside the library); same arguments as relpos_attention."""
    _check(lib().pkc_relpos_attention_noalloc(c_void_p(qkv), c_void_p(ptab), centre, c_void_p(bias_u),
                                              c_void_p(bias_v), _ints(lens), len(lens), d, n_heads,
                                              1 if bf16 else 0, c_void_p(ctx),
                                              c_void_p(stream) if stream else None))


def pack_cache_build(gguf_path: str, cache_dir: str) -> str:
    """pkc_pack_cache_build: the packed weight image of gguf_path in cache_dir
    (made there if absent, host only); returns the cache file's path."""
    buf = ctypes.create_string_buffer(4096)
    _check(lib().pkc_pack_cache_build(gguf_path.encode(), cache_dir.encode(), buf, len(buf)))
    return buf.value.decode()


def shard_plan(n_samples, n_dev, hop=160):
    out = (c_int * len(n_samples))()
    _check(lib().pkc_shard_plan(_ints(n_samples), len(n_samples), n_dev, hop, out))
    return list(out)


class Model:
    """An open GGUF model on one or more CUDA devices (pkc_model)."""

    def __init__(self, gguf_path: str, devices=(0,)):
        L = lib()
        h = c_void_p()
        devs = _ints(devices)
        st = L.pkc_model_open(gguf_path.encode(), devs, len(devices), ctypes.byref(h))
        _check(st, None)
        self._h = h
        info = ModelInfo()
        _check(L.pkc_model_info_get(h, ctypes.byref(info)), h)
        self.info = info

    def stream_schedule(self):
        """pkc_stream_schedule_get as a dict."""
        o = StreamSchedule()
        _check(lib().pkc_stream_schedule_get(self._h, ctypes.byref(o)), self._h)
        return {n: getattr(o, n) for n, _ in StreamSchedule._fields_}

    def load_stats(self):
        """pkc_model_load_stats: {"pack_s", "upload_s", "from_cache"} of this open."""
        a, b, c = ctypes.c_double(), ctypes.c_double(), c_int()
        _check(lib().pkc_model_load_stats(self._h, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c)), self._h)
        return {"pack_s": a.value, "upload_s": b.value, "from_cache": bool(c.value)}

    def close(self):
        if getattr(self, "_h", None):
            lib().pkc_model_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def mel_frames(self, n):
        return lib().pkc_mel_frames(self._h, int(n))

    def encoder_frames(self, mel_frames):
        return lib().pkc_encoder_frames(self._h, int(mel_frames))

    def mel_batch(self, pcms):
        """GpuMel::compute per clip stacked as MelBatch: ([B, n_mels, T_max], T[B])."""
        B = len(pcms)
        pcms = [np.ascontiguousarray(p, dtype=np.float32) for p in pcms]
        ptrs = (c_void_p * B)(*[p.ctypes.data for p in pcms])
        ns = _ints([len(p) for p in pcms])
        T = [self.mel_frames(len(p)) for p in pcms]
        Tmax = max(T) if T else 0
        out = np.zeros((B, self.info.n_mels, Tmax), dtype=np.float32)
        T_out = (c_int * B)()
        _check(lib().pkc_mel_batch(self._h, ptrs, ns, B, out.ctypes.data, out.size, T_out), self._h)
        return out, list(T_out)

    def encode_batch(self, mel, valid_T, layout=LAYOUT_CHANNELS_FIRST):
        """Encoder::forward_batch: list of per-item outputs ([d, T_b] or [T_b, d])."""
        mel = np.ascontiguousarray(mel, dtype=np.float32)
        B, F, Tmax = mel.shape
        vout = [self.encoder_frames(int(t)) for t in valid_T]
        d = self.info.d_model
        out = np.zeros(sum(vout) * d, dtype=np.float32)
        vt = (c_int * B)()
        dm = c_int()
        _check(lib().pkc_encode_batch(self._h, mel.ctypes.data, B, F, Tmax, _ints(valid_T), layout,
                                      out.ctypes.data, out.size, vt, ctypes.byref(dm)), self._h)
        return _split(out, list(vt), d, layout)

    def encode_pcm_batch(self, pcms, layout=LAYOUT_CHANNELS_FIRST, out=None):
        """Encode B clips of 16 kHz mono PCM (host arrays). Returns one array
        per clip ([d, T'] channels-first or [T', d] time-major). `out`: an
        optional contiguous float32 host array of at least
        out_floats(lengths) elements to write into (the returned arrays are
        views of it); pass page-locked memory (e.g. a pinned torch tensor's
        .numpy()) and the download runs at full copy speed with no allocation
        per call."""
        B = len(pcms)
        pcms = [np.ascontiguousarray(p, dtype=np.float32) for p in pcms]
        ptrs = (c_void_p * B)(*[p.ctypes.data for p in pcms])
        ns = _ints([len(p) for p in pcms])
        n = lib().pkc_encode_out_floats(self._h, ns, B)
        if out is None:
            out = np.empty(n, dtype=np.float32)
        else:
            if out.dtype != np.float32 or not out.flags["C_CONTIGUOUS"] or out.size < n:
                raise ValueError(f"out must be a contiguous float32 array of at least {n} elements")
            out = out.reshape(-1)[:n]
        vt = (c_int * B)()
        _check(lib().pkc_encode_pcm_batch(self._h, ptrs, ns, B, layout, out.ctypes.data, out.size,
                                          vt), self._h)
        return _split(out, list(vt), self.info.d_model, layout)

    def ctc_classes(self):
        """Classes of the CTC head (vocab + 1), 0 without one."""
        return int(lib().pkc_ctc_classes(self._h))

    def ctc_greedy_pcm_batch(self, pcms, logprobs=False):
        """CTC transcription: per clip a list of (id, frame, conf, span); with
        logprobs=True also per clip the [T', V+1] log-probabilities."""
        B = len(pcms)
        pcms = [np.ascontiguousarray(p, dtype=np.float32) for p in pcms]
        ptrs = (c_void_p * B)(*[p.ctypes.data for p in pcms])
        ns = _ints([len(p) for p in pcms])
        frames = [self.encoder_frames(self.mel_frames(len(p))) for p in pcms]
        cap = max(1, sum(frames))
        toks = (Token * cap)()
        nt = (c_int * B)()
        V1 = self.ctc_classes()
        lp = np.empty((sum(frames), V1), dtype=np.float32) if logprobs else None
        _check(lib().pkc_ctc_greedy_pcm_batch(self._h, ptrs, ns, B, toks, cap, nt,
                                              lp.ctypes.data if logprobs else None,
                                              lp.size if logprobs else 0), self._h)
        out, pos = [], 0
        for b in range(B):
            out.append([(t.id, t.frame, t.conf, t.span) for t in toks[pos:pos + nt[b]]])
            pos += nt[b]
        if not logprobs:
            return out
        lps, f0 = [], 0
        for T in frames:
            lps.append(lp[f0:f0 + T])
            f0 += T
        return out, lps

    def transducer_kind(self):
        """0: no transducer decoder, 1: RNN-T, 2: TDT."""
        return int(lib().pkc_transducer_kind(self._h))

    def transducer_greedy_pcm_batch(self, pcms, max_symbols=10):
        """Greedy RNN-T / TDT transcription on the GPU: per clip a list of
        (id, frame, conf, span)."""
        B = len(pcms)
        pcms = [np.ascontiguousarray(p, dtype=np.float32) for p in pcms]
        ptrs = (c_void_p * B)(*[p.ctypes.data for p in pcms])
        ns = _ints([len(p) for p in pcms])
        frames = [self.encoder_frames(self.mel_frames(len(p))) for p in pcms]
        cap = max(1, sum(frames) * max_symbols)
        toks = (Token * cap)()
        nt = (c_int * B)()
        _check(lib().pkc_transducer_greedy_pcm_batch(self._h, ptrs, ns, B, toks, cap, nt), self._h)
        out, pos = [], 0
        for b in range(B):
            out.append([(t.id, t.frame, t.conf, t.span) for t in toks[pos:pos + nt[b]]])
            pos += nt[b]
        return out

    def out_floats(self, n_samples):
        """Floats the encoder output of clips with these sample counts takes."""
        return int(lib().pkc_encode_out_floats(self._h, _ints(n_samples), len(n_samples)))

    def encode_pcm_device(self, d_pcm, n_samples, d_out, stream=0, slot=0, sync=False):
        _check(lib().pkc_encode_pcm_device(self._h, slot, c_void_p(d_pcm), _ints(n_samples),
                                           len(n_samples), c_void_p(d_out),
                                           c_void_p(stream) if stream else None, 1 if sync else 0),
               self._h)

    def last_graph_kernels(self, slot=0):
        """Kernel launches of the CUDA graph this device slot launched last."""
        return int(lib().pkc_last_graph_kernels(self._h, slot))

    def stream(self, slot=0):
        """cudaStream_t (as int) that the host-buffer entry points use."""
        return lib().pkc_model_stream(self._h, slot) or 0

    def profile_enable(self, on=True):
        _check(lib().pkc_profile_enable(self._h, 1 if on else 0), self._h)

    def profile_read(self):
        cap = 64
        arr = (KernelStat * cap)()
        n = lib().pkc_profile_read(self._h, arr, cap)
        return [dict(name=a.name.decode(), launches=a.launches, total_ms=a.total_ms,
                     flops=a.flops, bytes=a.bytes) for a in arr[:n]]


def _split(flat, vt, d, layout):
    outs, off = [], 0
    for t in vt:
        blk = flat[off:off + t * d]
        outs.append(blk.reshape(d, t) if layout == LAYOUT_CHANNELS_FIRST else blk.reshape(t, d))
        off += t * d
    return outs


class Stream:
    """A cache-aware streaming encoder session (pkc_stream_*, the reference's
    StreamingEncoder)."""

    def __init__(self, model: "Model", device_slot: int = 0):
        self.model = model
        h = c_void_p()
        _check(lib().pkc_stream_begin(model.handle, device_slot, ctypes.byref(h)), model.handle)
        self._h = h
        self.d = model.info.d_model

    def step(self, mel_window, is_last: bool = False) -> np.ndarray:
        """One window [n_mels, n] (feature-major, overlap included) -> the
        chunk's valid frames [valid, d_model]."""
        mel = np.ascontiguousarray(mel_window, dtype=np.float32)
        n = mel.shape[1]
        cap = (n // 8 + 2) * self.d
        out = np.empty(cap, dtype=np.float32)
        nv = c_int()
        _check(lib().pkc_stream_step(self._h, mel.ctypes.data, n, 1 if is_last else 0, out.ctypes.data, cap,
                                     ctypes.byref(nv)), self.model.handle)
        return out[: nv.value * self.d].reshape(nv.value, self.d).copy()

    def reset(self):
        _check(lib().pkc_stream_reset(self._h), self.model.handle)

    @property
    def step_num(self) -> int:
        return lib().pkc_stream_step_num(self._h)

    def close(self):
        if getattr(self, "_h", None):
            lib().pkc_stream_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def stream_step_batch(streams, mel_windows, is_last):
    """pkc_stream_step_batch: one window [n_mels, n] per stream (all the same
    n) -> list of [valid_i, d_model] arrays."""
    S = len(streams)
    mels = [np.ascontiguousarray(m, dtype=np.float32) for m in mel_windows]
    n = mels[0].shape[1]
    d = streams[0].d
    cap = (n // 8 + 2) * d
    outs = [np.empty(cap, dtype=np.float32) for _ in range(S)]
    hs = (c_void_p * S)(*[s._h.value for s in streams])
    mp = (c_void_p * S)(*[m.ctypes.data for m in mels])
    op = (c_void_p * S)(*[o.ctypes.data for o in outs])
    last = (c_int * S)(*[1 if x else 0 for x in is_last])
    nv = (c_int * S)()
    _check(lib().pkc_stream_step_batch(hs, S, mp, n, last, op, cap, nv), streams[0].model.handle)
    return [o[: nv[i] * d].reshape(nv[i], d).copy() for i, o in enumerate(outs)]
