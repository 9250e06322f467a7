"""ORACLE — CPU restatement of parakeet.cpp's encoder hot path.

TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline legs may import this module, and only as the checker (or as the
timed CPU baseline); the product path (libpkc.so) never calls it.

What it restates (paths inside parakeet.cpp, the reference):
  * MelFrontend::compute + MelKernel::frame_logmel   src/mel.cpp:63-176
  * GpuMel::compute (DFT-as-matmul front end)        src/mel_gpu.cpp:15-162
  * rel_pos_encoding                                 src/pos_enc.cpp:10-34
  * Subsampling::build_graph_batched, valid_out_len  src/subsampling.cpp:25-240
  * RelPosAttention::build_graph_batched             src/relpos_attention.cpp:162-306
  * build_conv_module (batched)                      src/conformer.cpp:38-164
  * ConformerLayer::build_graph_batched              src/conformer.cpp:285-353
  * Encoder::forward_batch                           src/encoder.cpp:97-167
  * CTCDecoder::forward (CTC head)                   src/ctc_decoder.cpp:35-116
  * ctc_greedy (greedy fold, token frame / conf)     src/search.cpp:8-90
  * PredictionNet::step, Joint::step_logits          src/prediction.cpp, src/joint.hpp
  * tdt_greedy, rnnt_decode_frames / rnnt_greedy     src/tdt.cpp:8-126, src/rnnt.cpp:17-122
  * causal models offline (B = 1): causal subsampling, chunked-limited
    attention mask, causal depthwise conv, layer_norm conv norm
      src/subsampling.cpp:25-46,260-388, src/relpos_attention.cpp:30-37,113-131,
      src/conformer.cpp:38-164
  * StreamingEncoder::step (cache-aware streaming)   src/streaming_encoder.cpp:98-460
The batched graph is restated literally: every item is zero-padded to the
batch's T_max and every mask the reference builds (per-stage subsampling time
masks, output-frame mask, attention key mask and padded-query zeroing, conv
pre-depthwise mask) is applied, so padding effects are modelled, not assumed.

Arithmetic is float64 throughout (the reference computes in f32 with ggml);
the op semantics follow ggml: ggml_norm = (x-mean)/sqrt(var+eps) with the
population variance; soft_max_ext(a, mask, scale) = softmax(a*scale + mask);
silu(x) = x*sigmoid(x); GLU = first half * sigmoid(second half); BatchNorm
folded into f32 scale/shift on the host exactly as conformer.cpp:134-154 does.

Pinning: ggml itself (the library that executes these graphs) is absent from
the reference checkout, so the graph arithmetic cannot be run here. The oracle
is pinned against (a) the reference's own CPU mel front end and positional
encoding compiled from its sources (oracle/_ref, see Makefile.ref), (b) the
reference's known-answer test (tests/test_fft.cpp: a cosine at bin 8 peaks at
bin 8) and its GpuMel-vs-MelFrontend tolerance (tests/test_mel_gpu.cpp: < 0.05),
(c) a literal pad/reshape/view restatement of rel_shift, and (d) the
reference's batched == standalone padding-invariance property
(tests/test_encoder_batch.cpp). The encoder graph beyond those anchors is
"parity unpinned" against ggml's own kernels. The streaming restatement is
pinned to the offline causal restatement by the reference's cache-aware
equivalence (tests/test_streaming_encoder.cpp: the concatenated chunk outputs
equal the offline encoder output except the final chunk's valid_out_len tail).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

LN_EPS = 1e-5
BN_EPS = 1e-5

# Arithmetic type of the encoder restatement: float64 for every parity use.
# compute_dtype(np.float32) runs the same graph in float32 (weights are stored
# float32, so every op then stays float32): only the timed CPU baseline of
# bench.py uses it, to time the reference's f32 CPU path fairly.
_DT = np.float64


class compute_dtype:
    """Context manager: run the encoder restatement in the given numpy type."""

    def __init__(self, dt):
        self.dt = dt

    def __enter__(self):
        global _DT
        self.prev, _DT = _DT, self.dt
        return self

    def __exit__(self, *exc):
        global _DT
        _DT = self.prev
NORM_EPS = 1e-5       # per-feature mel normalisation (src/mel.cpp:13)
INF_VAL = 10000.0     # sinusoid base (src/pos_enc.cpp:8)


def cdiv_trunc(a: int, b: int) -> int:
    """C integer division (truncates toward zero), as the reference's int math."""
    q = abs(a) // abs(b)
    return q if (a >= 0) == (b >= 0) else -q


def valid_out_len(T: int, in_valid: int = -1) -> int:
    """Subsampling::valid_out_len (src/subsampling.cpp:25-46), offline path."""
    valid = in_valid if in_valid >= 0 else T - 1
    for _ in range(3):
        valid = cdiv_trunc(valid + 2 - 3, 2) + 1
    return valid


def conv_out_len(n: int) -> int:
    """Spatial output of a k=3, s=2, p=1 convolution."""
    return (n + 2 - 3) // 2 + 1


# =========================================================== weights

class Weights:
    """GGUF tensors as float32 arrays in torch/numpy shape (dequantised with
    gguf-py: exactly the values ggml's mul_mat sees for f16/q8_0/q4_k weights);
    every op promotes them to float64."""

    def __init__(self, gguf_path: str):
        import gguf
        r = gguf.GGUFReader(gguf_path)
        self.kv = {}
        for f in r.fields.values():
            try:
                self.kv[f.name] = f.contents()
            except Exception:
                pass
        self.t = {}
        self.types = {}
        for t in r.tensors:
            ne = [int(x) for x in t.shape]
            shape = tuple(reversed(ne))
            qt = t.tensor_type
            self.types[t.name] = int(qt)
            if qt in (gguf.GGMLQuantizationType.F32, gguf.GGMLQuantizationType.F16):
                arr = np.asarray(t.data).astype(np.float32).reshape(shape)
            else:
                arr = gguf.quants.dequantize(np.asarray(t.data), qt).astype(np.float32).reshape(shape)
            self.t[t.name] = arr
        kv = self.kv
        self.d = int(kv["parakeet.encoder.d_model"])
        self.L = int(kv["parakeet.encoder.n_layers"])
        self.H = int(kv["parakeet.encoder.n_heads"])
        self.K = int(kv["parakeet.encoder.conv_kernel"])
        self.C = int(kv["parakeet.encoder.subsampling_conv_channels"])
        self.xscaling = bool(kv.get("parakeet.encoder.xscaling", True))
        self.n_mels = int(kv["parakeet.preprocessor.n_mels"])
        self.n_fft = int(kv["parakeet.preprocessor.n_fft"])
        self.hop = int(kv["parakeet.preprocessor.hop_length"])
        self.preemph = float(kv.get("parakeet.preprocessor.preemph", 0.0))
        self.mag_power = float(kv.get("parakeet.preprocessor.mag_power", 2.0))
        self.log_guard = float(kv.get("parakeet.preprocessor.log_zero_guard", 0.0))
        self.per_feature = kv.get("parakeet.preprocessor.normalize", "per_feature") == "per_feature"

    def get(self, name):
        return self.t.get(name)

    def window(self) -> np.ndarray:
        """Hann window centre-padded to n_fft (src/mel.cpp:29-44), f32."""
        w = np.zeros(self.n_fft, dtype=np.float32)
        src = self.t.get("preprocessor.featurizer.window")
        if src is not None:
            src = src.astype(np.float32).reshape(-1)
            left = (self.n_fft - len(src)) // 2
            w[left:left + len(src)] = src
        return w

    def fb(self) -> np.ndarray:
        nb = self.n_fft // 2 + 1
        return self.t["preprocessor.featurizer.fb"].astype(np.float32).reshape(self.n_mels, nb)


# =========================================================== mel front end

def _preemph_pad(samples: np.ndarray, n_fft: int, hop: int, preemph: float):
    S = len(samples)
    s = samples.astype(np.float64)
    x = s.copy()
    if preemph > 0 and S > 0:
        x[1:] = s[1:] - float(np.float32(preemph)) * s[:-1]
    pad = n_fft // 2
    padded = np.zeros(S + 2 * pad, dtype=np.float64)
    padded[pad:pad + S] = x
    T = 1 + (S + 2 * pad - n_fft) // hop if S + 2 * pad >= n_fft else 0
    idx = np.arange(T)[:, None] * hop + np.arange(n_fft)[None, :]
    return padded[idx], T, (S // hop if S > 0 else 0)


def _normalize(feats: np.ndarray, seq_len: int) -> np.ndarray:
    """Per-feature normalisation (src/mel.cpp:150-174), double precision."""
    F, T = feats.shape
    valid = min(seq_len, T)
    out = np.zeros_like(feats)
    for m in range(F):
        row = feats[m].astype(np.float64)
        mean = row[:valid].sum() / valid if valid > 0 else 0.0
        var = ((row[:valid] - mean) ** 2).sum() / (valid - 1) if valid > 1 else 0.0
        sd = math.sqrt(var) + NORM_EPS
        out[m, :valid] = ((row[:valid] - mean) / sd).astype(np.float32)
    return out


def mel_frontend(w: Weights, samples: np.ndarray) -> np.ndarray:
    """MelFrontend::compute: FFT front end, feats [n_mels, T] f32."""
    if len(samples) == 0:
        return np.zeros((w.n_mels, 0), dtype=np.float32)
    frames, T, seq_len = _preemph_pad(samples, w.n_fft, w.hop, w.preemph)
    win = w.window().astype(np.float64)
    fr = (frames * win[None, :]).astype(np.float32)
    spec = np.fft.rfft(fr.astype(np.float64), axis=1)
    re = spec.real.astype(np.float32).astype(np.float64)
    im = spec.imag.astype(np.float32).astype(np.float64)
    mag = np.sqrt(re * re + im * im)
    power = mag if w.mag_power == 1.0 else mag ** w.mag_power
    mel = power @ w.fb().astype(np.float64).T                     # [T, F]
    feats = np.log(mel + float(np.float32(w.log_guard))).astype(np.float32).T
    return _normalize(feats, seq_len) if w.per_feature else feats


def mel_gpu_graph(w: Weights, samples: np.ndarray) -> np.ndarray:
    """GpuMel::compute: DFT as f32 matmuls, power, filterbank, log (f32)."""
    if len(samples) == 0:
        return np.zeros((w.n_mels, 0), dtype=np.float32)
    frames, T, seq_len = _preemph_pad(samples, w.n_fft, w.hop, w.preemph)
    win = w.window().astype(np.float64)
    xw = (frames * win[None, :]).astype(np.float32).astype(np.float64)
    N = w.n_fft
    nb = N // 2 + 1
    ang = 2.0 * np.pi * np.outer(np.arange(nb), np.arange(N)) / N
    cosb = np.cos(ang).astype(np.float32).astype(np.float64)
    sinb = (-np.sin(ang)).astype(np.float32).astype(np.float64)
    re = (xw @ cosb.T).astype(np.float32)
    im = (xw @ sinb.T).astype(np.float32)
    power = (re * re + im * im).astype(np.float32).astype(np.float64)
    mel = (power @ w.fb().astype(np.float64).T).astype(np.float32)
    lm = np.log(mel + np.float32(w.log_guard)).astype(np.float32).T
    return _normalize(lm, seq_len) if w.per_feature else lm


def mel_batch(w: Weights, pcms, gpu_graph: bool = True):
    """build_mel_batch (src/model.cpp:119-144): [B, F, T_max] zero padded + T[b]."""
    feats = [(mel_gpu_graph if gpu_graph else mel_frontend)(w, p) for p in pcms]
    Ts = [f.shape[1] for f in feats]
    Tmax = max(Ts) if Ts else 0
    out = np.zeros((len(pcms), w.n_mels, Tmax), dtype=np.float32)
    for b, f in enumerate(feats):
        out[b, :, :f.shape[1]] = f
    return out, Ts


# =========================================================== positional encoding

def rel_pos_encoding(T: int, d: int) -> np.ndarray:
    """rel_pos_encoding (src/pos_enc.cpp:10-34): [2T-1, d] f32, positions
    T-1 ... -(T-1), sin on even dims, cos on odd dims."""
    half = d // 2
    factor = -(math.log(INF_VAL) / d)
    div = np.exp(np.arange(half, dtype=np.float64) * 2 * factor)
    pos = (T - 1) - np.arange(2 * T - 1, dtype=np.float64)
    arg = pos[:, None] * div[None, :]
    pe = np.zeros((2 * T - 1, d), dtype=np.float32)
    pe[:, 0::2] = np.sin(arg)
    pe[:, 1::2] = np.cos(arg)
    return pe


# =========================================================== subsampling

def _conv3x3_s2(x: np.ndarray, wk: np.ndarray) -> np.ndarray:
    """x [..., H, W] zero-padded by 1; wk [..., 3, 3] broadcast against x's
    leading dims; returns sum_{kh,kw} wk*x at stride 2 -> [..., H', W']."""
    H, W = x.shape[-2:]
    Ho, Wo = conv_out_len(H), conv_out_len(W)
    xp = np.zeros(x.shape[:-2] + (H + 2, W + 2), dtype=_DT)
    xp[..., 1:H + 1, 1:W + 1] = x
    out = 0
    for kh in range(3):
        for kw in range(3):
            sl = xp[..., kh:kh + 2 * Ho - 1:2, kw:kw + 2 * Wo - 1:2]
            out = out + wk[..., kh, kw][..., None, None] * sl
    return out


def subsampling_batched(w: Weights, mel: np.ndarray, valid_in: list[int]):
    """Subsampling::build_graph_batched (src/subsampling.cpp:48-240).
    mel [B, F, T] -> (x [B, Tp, d], out_valid [B])."""
    B, F, T = mel.shape
    C = w.C
    x = mel.astype(_DT).transpose(0, 2, 1)                    # [B, T, F] (H=T, W=F)
    vt0 = [v if v >= 0 else T - 1 for v in valid_in]
    vt1 = [cdiv_trunc(v - 1, 2) + 1 for v in vt0]
    vt2 = [cdiv_trunc(v - 1, 2) + 1 for v in vt1]

    def mask_time(t, vt):                                    # t [B, C?, H, W]
        H = t.shape[-2]
        m = (np.arange(H)[None, :] < np.array(vt)[:, None]).astype(_DT)
        return t * m.reshape((t.shape[0],) + (1,) * (t.ndim - 3) + (H, 1))

    g = lambda n: w.get("encoder.pre_encode." + n)
    x = mask_time(x, vt0)                                      # [B, T, F]
    w0 = g("conv.0.weight")[:, 0]                              # [C, 3, 3]
    y = _conv3x3_s2(x[:, None], w0[None])                      # [B, C, T1, F1]
    y = np.maximum(y + g("conv.0.bias")[None, :, None, None], 0.0)
    for dw_i, pw_i, vt in ((2, 3, vt1), (5, 6, vt2)):
        y = mask_time(y, vt)
        y = _conv3x3_s2(y, g(f"conv.{dw_i}.weight")[:, 0][None]) + g(f"conv.{dw_i}.bias")[None, :, None, None]
        pw = g(f"conv.{pw_i}.weight")[:, :, 0, 0]               # [C_out, C_in]
        y = np.einsum("oc,bchw->bohw", pw, y) + g(f"conv.{pw_i}.bias")[None, :, None, None]
        y = np.maximum(y, 0.0)
    _, _, Tp, Fp = y.shape
    flat = y.transpose(0, 2, 1, 3).reshape(B, Tp, C * Fp)      # idx c*F' + f
    out_valid = [min(valid_out_len(T, v), Tp) for v in valid_in]
    m = (np.arange(Tp)[None, :] < np.array(out_valid)[:, None]).astype(_DT)
    flat = flat * m[:, :, None]
    out = flat @ g("out.weight").T + g("out.bias")
    return out, out_valid


# =========================================================== conformer layer

def layer_norm(x, g, b):
    mean = x.mean(axis=-1, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=-1, keepdims=True)
    return (x - mean) / np.sqrt(var + LN_EPS) * g + b


def silu(x):
    return x / (1.0 + np.exp(-x))


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def linear(x, W, b=None):
    y = x @ W.T
    return y + b if b is not None else y


def rel_shift_index(bd_raw: np.ndarray) -> np.ndarray:
    """bd[..., i, j] = bd_raw[..., i, j - i + T - 1] (bd_raw [..., T, 2T-1])."""
    T = bd_raw.shape[-2]
    i = np.arange(T)[:, None]
    j = np.arange(T)[None, :]
    return np.take_along_axis(bd_raw, np.broadcast_to(j - i + T - 1, bd_raw.shape[:-2] + (T, T)), axis=-1)


def rel_shift_literal(bd_raw: np.ndarray) -> np.ndarray:
    """The reference's rel_shift op sequence (src/relpos_attention.cpp:230-238)
    replayed on a C-ordered buffer, for one [T_q, 2T-1] slab. ggml ne0 is the
    fastest axis, so a ggml tensor [ne0, ne1] is a numpy array [ne1, ne0]."""
    T = bd_raw.shape[0]
    P = 2 * T - 1
    padded = np.concatenate([np.zeros((T, 1)), bd_raw], axis=1)       # pad_ext lp0=1 -> [2T, T]
    flat = padded.reshape(-1)                                          # contiguous
    as_T_2T = flat.reshape(2 * T, T)                                   # reshape_4d(T, 2T)
    view = as_T_2T[1:]                                                 # view: 2T-1 rows, offset nb[1]
    cont = np.ascontiguousarray(view).reshape(-1)                      # cont
    as_P_T = cont.reshape(T, P)                                        # reshape_4d(2T-1, T)
    return np.ascontiguousarray(as_P_T[:, :T])                         # view [T, T] offset 0 + cont


def chunked_visible(gq, gk, att_left: int, att_right: int):
    """Chunked-limited attention (att_context_style "chunked_limited",
    src/relpos_attention.cpp:113-131, src/streaming_encoder.cpp:231-260): with
    chunk = att_right + 1, a key is visible iff 0 <= gq/chunk - gk/chunk <=
    att_left/chunk (global query / key frame indices)."""
    chunk = att_right + 1
    left_chunks = att_left // chunk if chunk > 0 else 0
    diff = np.asarray(gq)[:, None] // chunk - np.asarray(gk)[None, :] // chunk
    return (diff >= 0) & (diff <= left_chunks)


def relpos_attention(w: Weights, li: int, x: np.ndarray, pe: np.ndarray, valid: int,
                     literal_shift: bool = False, chunked=None) -> np.ndarray:
    """RelPosAttention::build_graph_batched for one item (src/relpos_attention.cpp:162-306).
    x [T, d] (the normalised attention input), pe [2T-1, d]; chunked = (att_left,
    att_right) for chunked-limited models."""
    T, d = x.shape
    H = w.H
    dk = d // H
    pre = f"encoder.layers.{li}.self_attn."
    g = lambda n: w.get(pre + n)
    q = linear(x, g("linear_q.weight"), g("linear_q.bias")).reshape(T, H, dk).transpose(1, 0, 2)
    k = linear(x, g("linear_k.weight"), g("linear_k.bias")).reshape(T, H, dk).transpose(1, 0, 2)
    v = linear(x, g("linear_v.weight"), g("linear_v.bias")).reshape(T, H, dk).transpose(1, 0, 2)
    p = linear(pe.astype(_DT), g("linear_pos.weight")).reshape(2 * T - 1, H, dk).transpose(1, 0, 2)
    qu = q + g("pos_bias_u")[:, None, :]
    qv = q + g("pos_bias_v")[:, None, :]
    ac = qu @ k.transpose(0, 2, 1)                              # [H, Tq, Tk]
    bd_raw = qv @ p.transpose(0, 2, 1)                          # [H, Tq, 2T-1]
    if literal_shift:
        bd = np.stack([rel_shift_literal(bd_raw[h]) for h in range(H)])
    else:
        bd = rel_shift_index(bd_raw)
    scale = 1.0 / math.sqrt(dk)
    vis = np.broadcast_to(np.arange(T)[None, :] < valid, (T, T))
    if chunked is not None:
        vis = vis & chunked_visible(np.arange(T), np.arange(T), *chunked)
    mask = np.where(vis, 0.0, -np.inf).astype(_DT)[None]
    s = (ac + bd) * scale + mask
    s = s - s.max(axis=-1, keepdims=True)
    e = np.exp(s)
    attn = e / e.sum(axis=-1, keepdims=True)
    ctx = (attn @ v).transpose(1, 0, 2).reshape(T, d)
    ctx[valid:] = 0.0
    return linear(ctx, g("linear_out.weight"), g("linear_out.bias"))


def bn_fold(w: Weights, pre: str):
    """Host BatchNorm fold in f32 (src/conformer.cpp:134-154)."""
    gmm = w.get(pre + "conv.batch_norm.weight").astype(np.float32)
    bb = w.get(pre + "conv.batch_norm.bias").astype(np.float32)
    m = w.get(pre + "conv.batch_norm.running_mean").astype(np.float32)
    var = w.get(pre + "conv.batch_norm.running_var").astype(np.float32)
    sc = (gmm / np.sqrt(var + np.float32(BN_EPS))).astype(np.float32)
    sh = (bb - m * sc).astype(np.float32)
    return sc.astype(_DT), sh.astype(_DT)


def conv_norm(w: Weights, pre: str, dw: np.ndarray, norm: str) -> np.ndarray:
    """The norm between the depthwise conv and SiLU (src/conformer.cpp:128-154):
    LayerNorm over channels (gamma / beta stored as conv.batch_norm.weight /
    bias) or the host-folded BatchNorm."""
    if norm == "layer_norm":
        return layer_norm(dw, w.get(pre + "conv.batch_norm.weight"), w.get(pre + "conv.batch_norm.bias"))
    sc, sh = bn_fold(w, pre)
    return dw * sc + sh


def conv_module(w: Weights, li: int, c: np.ndarray, valid: int, causal: bool = False,
                norm: str = "batch_norm") -> np.ndarray:
    """build_conv_module for one item (src/conformer.cpp:38-164); causal: the
    depthwise input is padded K-1 on the left only (:102-108)."""
    T, d = c.shape
    pre = f"encoder.layers.{li}."
    g = lambda n: w.get(pre + n)
    y = linear(c, g("conv.pointwise_conv1.weight")[:, :, 0], g("conv.pointwise_conv1.bias"))
    glu = y[:, :d] * sigmoid(y[:, d:])
    glu[valid:] = 0.0
    K = w.K
    left = K - 1 if causal else (K - 1) // 2
    dww = g("conv.depthwise_conv.weight")[:, 0, :]             # [d, K]
    gp = np.zeros((T + K - 1, d), dtype=_DT)
    gp[left:left + T] = glu
    dw = np.zeros((T, d), dtype=_DT)
    for k in range(K):
        dw += gp[k:k + T] * dww[:, k][None, :]
    if g("conv.depthwise_conv.bias") is not None:
        dw += g("conv.depthwise_conv.bias")
    nrm = silu(conv_norm(w, pre, dw, norm))
    return linear(nrm, g("conv.pointwise_conv2.weight")[:, :, 0], g("conv.pointwise_conv2.bias"))


def conformer_layer(w: Weights, li: int, x: np.ndarray, pe: np.ndarray, valid: int, sc=None) -> np.ndarray:
    """ConformerLayer::build_graph_batched for one item (src/conformer.cpp:285-353);
    sc (StreamCfg) switches on a causal model's attention mask, conv and conv norm."""
    pre = f"encoder.layers.{li}."
    g = lambda n: w.get(pre + n)
    ln = lambda t, nm: layer_norm(t, g(nm + ".weight"), g(nm + ".bias"))

    def ff(t, nm):
        h = silu(linear(t, g(nm + ".linear1.weight"), g(nm + ".linear1.bias")))
        return linear(h, g(nm + ".linear2.weight"), g(nm + ".linear2.bias"))

    r = x + 0.5 * ff(ln(x, "norm_feed_forward1"), "feed_forward1")
    chunked = (sc.att_left, sc.att_right) if sc is not None and sc.chunked else None
    r = r + relpos_attention(w, li, ln(r, "norm_self_att"), pe, valid, chunked=chunked)
    r = r + conv_module(w, li, ln(r, "norm_conv"), valid, causal=bool(sc and sc.conv_causal),
                        norm=sc.conv_norm if sc is not None else "batch_norm")
    r = r + 0.5 * ff(ln(r, "norm_feed_forward2"), "feed_forward2")
    return ln(r, "norm_out")


@dataclass
class EncodeResult:
    outs: list            # per item [valid_b, d] (time-major) float64
    valid: list
    Tp: int
    sub_out: np.ndarray   # subsampling output [B, Tp, d]


def encoder_forward_batch(w: Weights, mel: np.ndarray, valid_T: list[int], n_layers: int | None = None,
                          capture: dict | None = None) -> EncodeResult:
    """Encoder::forward_batch (src/encoder.cpp:97-167). mel [B, F, T_max]."""
    B = mel.shape[0]
    vin = [v - 1 for v in valid_T]
    x, vout = subsampling_batched(w, mel, vin)
    sub_out = x.copy()
    if w.xscaling:
        x = x * math.sqrt(w.d)
    Tp = x.shape[1]
    pe = rel_pos_encoding(Tp, w.d)
    L = w.L if n_layers is None else n_layers
    outs = []
    for b in range(B):
        xb = x[b]
        for li in range(L):
            xb = conformer_layer(w, li, xb, pe, vout[b])
            if capture is not None:
                capture.setdefault(li, []).append(xb[:vout[b]].copy())
        outs.append(xb[:vout[b]])
    return EncodeResult(outs, vout, Tp, sub_out)


def encode_pcm_batch(w: Weights, pcms, n_layers: int | None = None, gpu_graph_mel: bool = True):
    """Model::transcribe_16k_batch steps 1-2 (src/model.cpp:164-181)."""
    mel, Ts = mel_batch(w, pcms, gpu_graph=gpu_graph_mel)
    return encoder_forward_batch(w, mel, Ts, n_layers=n_layers)


# ------------------------------------------------------------------ CTC head

# =========================================================== causal / cache-aware streaming models

class StreamCfg:
    """The causal-model and streaming-schedule keys of a GGUF
    (src/model_loader.cpp:113-131, src/streaming_encoder.cpp:30-60)."""

    def __init__(self, w: Weights):
        kv = w.kv
        self.style = str(kv.get("parakeet.encoder.att_context_style", "regular"))
        self.att_left = int(kv.get("parakeet.encoder.att_context_left", -1))
        self.att_right = int(kv.get("parakeet.encoder.att_context_right", -1))
        self.chunked = self.style == "chunked_limited" and self.att_right >= 0
        self.causal_sub = bool(kv.get("parakeet.encoder.causal_downsampling", False))
        self.conv_causal = bool(kv.get("parakeet.encoder.conv_causal", False))
        self.conv_norm = str(kv.get("parakeet.encoder.conv_norm_type", "batch_norm"))
        arr = lambda k: [int(v) for v in kv.get(k, [])]
        cs, pc = arr("parakeet.streaming.chunk_size"), arr("parakeet.streaming.pre_encode_cache_size")
        self.chunk_first = cs[0] if len(cs) > 0 else 9
        self.chunk_main = cs[1] if len(cs) > 1 else 16
        self.pre_cache = pc[1] if len(pc) > 1 else 9
        self.drop_extra = int(kv.get("parakeet.streaming.drop_extra_pre_encoded", 0))
        self.cache_len = int(kv.get("parakeet.streaming.last_channel_cache_size", 0))
        self.valid_out_len = int(kv.get("parakeet.streaming.valid_out_len", 0))
        self.present = "parakeet.streaming.chunk_size" in kv


def causal_valid_out_len(T: int, in_valid: int = -1) -> int:
    """Subsampling::valid_out_len with causal paddings (all_paddings = 3)."""
    v = in_valid if in_valid >= 0 else T - 1
    for _ in range(3):
        v = v // 2 + 1
    return v


def _conv3x3_s2_causal(x: np.ndarray, wk: np.ndarray) -> np.ndarray:
    """NeMo CausalConv2D as the reference builds it (src/subsampling.cpp:283-295):
    both spatial axes padded 2 before and 1 after, k=3, stride 2, no other pad."""
    H, W = x.shape[-2:]
    Ho, Wo = H // 2 + 1, W // 2 + 1
    xp = np.zeros(x.shape[:-2] + (H + 3, W + 3), dtype=np.float64)
    xp[..., 2:H + 2, 2:W + 2] = x
    out = 0
    for kh in range(3):
        for kw in range(3):
            sl = xp[..., kh:kh + 2 * Ho - 1:2, kw:kw + 2 * Wo - 1:2]
            out = out + wk[..., kh, kw][..., None, None] * sl
    return out


def subsampling_causal(w: Weights, mel_tf: np.ndarray, in_valid: int = -1):
    """Subsampling::build_graph, causal branch, one item (src/subsampling.cpp:260-388):
    every stage's input time frames >= its valid length are zeroed before the
    causal pad. mel_tf [T, F] -> (x [Tp, d], out_valid)."""
    T, F = mel_tf.shape
    v0 = in_valid if in_valid >= 0 else T - 1
    v1 = v0 // 2 + 1
    v2 = v1 // 2 + 1
    mask_time = lambda t, v: t * (np.arange(t.shape[-2]) < v).astype(np.float64)[:, None]
    g = lambda n: w.get("encoder.pre_encode." + n)
    x = mask_time(mel_tf.astype(np.float64), v0)
    y = _conv3x3_s2_causal(x[None], g("conv.0.weight")[:, 0])             # [C, T1, F1]
    y = np.maximum(y + g("conv.0.bias")[:, None, None], 0.0)
    for dw_i, pw_i, v in ((2, 3, v1), (5, 6, v2)):
        y = mask_time(y, v)
        y = _conv3x3_s2_causal(y, g(f"conv.{dw_i}.weight")[:, 0]) + g(f"conv.{dw_i}.bias")[:, None, None]
        y = np.einsum("oc,chw->ohw", g(f"conv.{pw_i}.weight")[:, :, 0, 0], y) + g(f"conv.{pw_i}.bias")[:, None, None]
        y = np.maximum(y, 0.0)
    C, Tp, Fp = y.shape
    flat = y.transpose(1, 0, 2).reshape(Tp, C * Fp)                       # idx c*F' + f
    out_valid = min(causal_valid_out_len(T, in_valid), Tp)
    flat[out_valid:] = 0.0
    return flat @ g("out.weight").T + g("out.bias"), out_valid


def encode_causal_offline(w: Weights, mel_ft: np.ndarray, n_layers: int | None = None) -> np.ndarray:
    """The offline encoder on a causal (streaming-trained) model, one clip:
    causal subsampling, chunked-limited attention, causal depthwise conv and its
    conv norm (src/encoder.cpp + the causal branches above). mel [F, T] ->
    [valid, d]."""
    sc = StreamCfg(w)
    x, vout = subsampling_causal(w, mel_ft.T, -1)
    if w.xscaling:
        x = x * math.sqrt(w.d)
    pe = rel_pos_encoding(x.shape[0], w.d)
    for li in range(w.L if n_layers is None else n_layers):
        x = conformer_layer(w, li, x, pe, vout, sc)
    return x[:vout]


class StreamingEncoder:
    """StreamingEncoder (src/streaming_encoder.cpp): per-layer attention cache
    (the last cache_len normalised attention inputs), depthwise-conv cache (the
    last K-1 GLU outputs) and the count of filled attention-cache frames."""

    def __init__(self, w: Weights, n_layers: int | None = None):
        self.w = w
        self.sc = StreamCfg(w)
        self.nl = w.L if n_layers is None else n_layers
        self.reset()

    def reset(self):
        d, K = self.w.d, self.w.K
        self.step_num = 0
        self.clc = 0
        self.ch = [np.zeros((self.sc.cache_len, d)) for _ in range(self.nl)]
        self.tm = [np.zeros((K - 1, d)) for _ in range(self.nl)]

    def _attention(self, li, attn_in, kv, pe, Tc):
        w, sc = self.w, self.sc
        d, H = w.d, w.H
        dk = d // H
        cache_len = sc.cache_len
        Tk = cache_len + Tc
        pre = f"encoder.layers.{li}.self_attn."
        g = lambda n: w.get(pre + n)
        q = linear(attn_in, g("linear_q.weight"), g("linear_q.bias")).reshape(Tc, H, dk).transpose(1, 0, 2)
        k = linear(kv, g("linear_k.weight"), g("linear_k.bias")).reshape(Tk, H, dk).transpose(1, 0, 2)
        v = linear(kv, g("linear_v.weight"), g("linear_v.bias")).reshape(Tk, H, dk).transpose(1, 0, 2)
        P = 2 * Tk - 1
        p = linear(pe.astype(np.float64), g("linear_pos.weight")).reshape(P, H, dk).transpose(1, 0, 2)
        qu = q + g("pos_bias_u")[:, None, :]
        qv = q + g("pos_bias_v")[:, None, :]
        ac = qu @ k.transpose(0, 2, 1)                                     # [H, Tc, Tk]
        bd_raw = qv @ p.transpose(0, 2, 1)                                 # [H, Tc, P]
        i = np.arange(Tc)[:, None]
        j = np.arange(Tk)[None, :]
        bd = np.take_along_axis(bd_raw, np.broadcast_to(j + Tc - 1 - i, (H, Tc, Tk)), axis=-1)
        gq = cache_len + np.arange(Tc)
        vis = chunked_visible(gq, np.arange(Tk), sc.att_left, sc.att_right)
        vis &= (np.arange(Tk) >= cache_len - self.clc)[None, :]           # empty-cache mask
        s = (ac + bd) / math.sqrt(dk) + np.where(vis, 0.0, -np.inf)[None]
        s = s - s.max(axis=-1, keepdims=True)
        e = np.exp(s)
        ctx = ((e / e.sum(axis=-1, keepdims=True)) @ v).transpose(1, 0, 2).reshape(Tc, d)
        return linear(ctx, g("linear_out.weight"), g("linear_out.bias"))

    def _layer(self, li, x, pe, Tc):
        """build_stream_layer (src/streaming_encoder.cpp:98-338)."""
        w, sc = self.w, self.sc
        d, K = w.d, w.K
        pre = f"encoder.layers.{li}."
        g = lambda n: w.get(pre + n)
        ln = lambda t, nm: layer_norm(t, g(nm + ".weight"), g(nm + ".bias"))

        def ff(t, nm):
            h = silu(linear(t, g(nm + ".linear1.weight"), g(nm + ".linear1.bias")))
            return linear(h, g(nm + ".linear2.weight"), g(nm + ".linear2.bias"))

        r = x + 0.5 * ff(ln(x, "norm_feed_forward1"), "feed_forward1")
        attn_in = ln(r, "norm_self_att")
        kv = np.concatenate([self.ch[li], attn_in], axis=0)
        r = r + self._attention(li, attn_in, kv, pe, Tc)
        next_ch = kv[-sc.cache_len:].copy() if sc.cache_len > 0 else kv[:0].copy()
        c = ln(r, "norm_conv")
        y = linear(c, g("conv.pointwise_conv1.weight")[:, :, 0], g("conv.pointwise_conv1.bias"))
        glu = y[:, :d] * sigmoid(y[:, d:])
        dw_in = np.concatenate([self.tm[li], glu], axis=0)               # [K-1+Tc, d]
        next_tm = dw_in[-(K - 1):].copy()
        dww = g("conv.depthwise_conv.weight")[:, 0, :]
        dw = np.zeros((Tc, d))
        for kk in range(K):
            dw += dw_in[kk:kk + Tc] * dww[:, kk][None, :]
        if g("conv.depthwise_conv.bias") is not None:
            dw += g("conv.depthwise_conv.bias")
        nrm = silu(conv_norm(w, pre, dw, sc.conv_norm))
        r = r + linear(nrm, g("conv.pointwise_conv2.weight")[:, :, 0], g("conv.pointwise_conv2.bias"))
        r = r + 0.5 * ff(ln(r, "norm_feed_forward2"), "feed_forward2")
        return ln(r, "norm_out"), next_ch, next_tm

    def step(self, mel_window_ft: np.ndarray, is_last: bool) -> np.ndarray:
        """StreamingEncoder::step (src/streaming_encoder.cpp:340-460): mel
        window [F, n] (already holding the pre-encode overlap) -> the chunk's
        valid frames [valid, d]."""
        w, sc = self.w, self.sc
        n = mel_window_ft.shape[1]
        x, _ = subsampling_causal(w, mel_window_ft.T, in_valid=n)
        drop = sc.drop_extra if self.step_num != 0 else 0
        Tc = x.shape[0] - drop
        if Tc <= 0:
            self.step_num += 1
            return np.zeros((0, w.d))
        x = x[drop:]
        if w.xscaling:
            x = x * math.sqrt(w.d)
        pe = rel_pos_encoding(sc.cache_len + Tc, w.d)
        nch, ntm = [], []
        for li in range(self.nl):
            x, a, b = self._layer(li, x, pe, Tc)
            nch.append(a)
            ntm.append(b)
        self.ch, self.tm = nch, ntm
        self.clc = min(sc.cache_len, self.clc + Tc)
        self.step_num += 1
        valid = Tc if is_last else min(sc.valid_out_len, Tc)
        return x[:valid]


def stream_schedule(sc: StreamCfg, T: int):
    """The chunk windows (lo, hi, is_last) of a T-frame mel under the model's
    schedule (CacheAwareStreamingAudioBuffer, tests/test_streaming_encoder.cpp:70-100)."""
    out, idx, first = [], 0, True
    while idx < T:
        size = sc.chunk_first if first else sc.chunk_main
        hi = min(idx + size, T)
        if hi - idx <= 0:
            break
        lo = idx if first else max(0, idx - sc.pre_cache)
        out.append((lo, hi, hi >= T))
        idx += size
        first = False
    return out


def ctc_head_weights(w: Weights):
    """The CTC head's weight [V+1, d] and bias [V+1] (hybrid name first, then
    the standalone CTC model's, as src/ctc_decoder.cpp:17-28), or None."""
    for pre in ("ctc_decoder.decoder_layers.0.", "decoder.decoder_layers.0."):
        if pre + "weight" in w.t and pre + "bias" in w.t:
            W = w.t[pre + "weight"].astype(np.float64)
            return W.reshape(W.shape[0], -1), w.t[pre + "bias"].astype(np.float64)
    return None


def ctc_log_probs(w: Weights, x: np.ndarray) -> np.ndarray:
    """CTCDecoder::forward (src/ctc_decoder.cpp:35-116): log_softmax(x W^T + b)
    over the V+1 classes. x [T, d] time-major -> [T, V+1], float64."""
    W, b = ctc_head_weights(w)
    y = x.astype(np.float64) @ W.T + b
    m = y.max(axis=1, keepdims=True)
    return y - m - np.log(np.exp(y - m).sum(axis=1, keepdims=True))


def ctc_greedy(logp: np.ndarray, blank_id: int):
    """ctc_greedy (src/search.cpp:21-90): per-frame argmax (first maximum),
    fold_consecutive emission, token frame = previous token's emit frame (the
    first token's: max(0, t-1)), confidence = min over the token's argmax run of
    (N exp(max logp) - 1) / (N - 1), span 1. Returns [(id, frame, conf, span)]."""
    T, N = logp.shape
    out = []
    previous, prev_peak, have_prev, run_min = blank_id, 0, False, 1.0
    for t in range(T):
        p = int(np.argmax(logp[t]))
        c = (N * math.exp(float(logp[t, p])) - 1.0) / (N - 1.0)
        emit = (p != previous or previous == blank_id) and p != blank_id
        if emit:
            if out:
                out[-1][2] = run_min
            out.append([p, prev_peak if have_prev else max(0, t - 1), 0.0, 1])
            run_min, prev_peak, have_prev = c, t, True
        elif p == previous and p != blank_id:
            run_min = min(run_min, c)
        previous = p
    if out:
        out[-1][2] = run_min
    return [tuple(o) for o in out]


# ------------------------------------------------------------ transducer decode

class Transducer:
    """Prediction network + joint of a transducer model, float64."""

    def __init__(self, w: Weights):
        kv = w.kv
        self.H = int(kv["parakeet.decoder.pred_hidden"])
        self.L = max(1, int(kv.get("parakeet.decoder.pred_rnn_layers", 1)))
        self.J = int(kv["parakeet.joint.joint_hidden"])
        self.V1 = int(kv["parakeet.vocab_size"]) + 1
        self.blank = int(kv["parakeet.blank_id"])
        self.max_symbols = int(kv.get("parakeet.decoding.max_symbols", 10))
        du = kv.get("parakeet.tdt.durations")
        self.durations = [int(x) for x in du] if du is not None else []
        f = lambda n: w.t[n].astype(np.float64)
        self.embed = f("decoder.prediction.embed.weight").reshape(self.V1, self.H)
        p = "decoder.prediction.dec_rnn.lstm."
        self.lstm = [(f(p + f"weight_ih_l{l}").reshape(4 * self.H, self.H), f(p + f"weight_hh_l{l}").reshape(4 * self.H, self.H),
                      f(p + f"bias_ih_l{l}"), f(p + f"bias_hh_l{l}")) for l in range(self.L)]
        self.w_enc, self.b_enc = f("joint.enc.weight").reshape(self.J, -1), f("joint.enc.bias")
        self.w_pred, self.b_pred = f("joint.pred.weight").reshape(self.J, self.H), f("joint.pred.bias")
        self.w_out, self.b_out = f("joint.joint_net.2.weight").reshape(-1, self.J), f("joint.joint_net.2.bias")

    def zero_state(self):
        return [np.zeros(self.H) for _ in range(self.L)], [np.zeros(self.H) for _ in range(self.L)]

    def step(self, token, is_sos, state):
        """PredictionNet::step: embedding (zero SOS input), stacked LSTM, gate
        order i f g o; returns (g = top h', new state)."""
        hs, cs = state
        x = np.zeros(self.H) if is_sos else self.embed[token]
        nh, nc = [], []
        for l, (wi, wh, bi, bh) in enumerate(self.lstm):
            z = wi @ x + bi + wh @ hs[l] + bh
            H = self.H
            i, fg, g, o = sigmoid(z[:H]), sigmoid(z[H:2 * H]), np.tanh(z[2 * H:3 * H]), sigmoid(z[3 * H:])
            c = fg * cs[l] + i * g
            h = o * np.tanh(c)
            nh.append(h)
            nc.append(c)
            x = h
        return x, (nh, nc)

    def logits(self, enc_proj_t, g):
        """Joint::step_logits: W_out ReLU(enc_proj[t] + W_pred g + b_pred) + b_out."""
        f = np.maximum(enc_proj_t + self.w_pred @ g + self.b_pred, 0.0)
        return self.w_out @ f + self.b_out


def _argmax_gap(v):
    """first argmax and the gap to the runner-up (inf for one element)"""
    k = int(np.argmax(v))
    if len(v) < 2:
        return k, math.inf
    s = np.sort(v)
    return k, float(s[-1] - s[-2])


def _max_prob_conf(a, k):
    """decode_max_prob_conf (src/decode_common.hpp): (N p_k - 1) / (N - 1)"""
    m = a.max()
    p = math.exp(a[k] - m) / float(np.exp(a - m).sum())
    N = float(len(a))
    return (N * p - 1.0) / (N - 1.0)


def transducer_greedy(tr: Transducer, enc: np.ndarray, trace=None):
    """tdt_greedy (durations present) or rnnt_greedy on one utterance's
    encoder output enc [T, d]. Returns ([(id, frame, conf, span)], the smallest
    top-two gap over every argmax taken). If trace is a list, every joint
    decision appends (tokens emitted before it, its top-two gap (TDT: the
    smaller of the token and duration gaps), frame t, prediction output g)."""
    enc_proj = enc.astype(np.float64) @ tr.w_enc.T + tr.b_enc
    T = enc.shape[0]
    out, gap = [], math.inf
    state = tr.zero_state()
    last, have = -1, False
    g = nstate = None
    g_valid = False
    t = 0
    if tr.durations:
        ND = len(tr.durations)
        while t < T:
            sym, need, skip = 0, True, 0
            while need and sym < tr.max_symbols:
                if not g_valid:
                    g, nstate = tr.step(last if have else tr.blank, not have, state)
                    g_valid = True
                lg = tr.logits(enc_proj[t], g)
                k, g1 = _argmax_gap(lg[:tr.V1])
                dk, g2 = _argmax_gap(lg[tr.V1:tr.V1 + ND])
                gap = min(gap, g1, g2)
                if trace is not None:
                    trace.append((len(out), min(g1, g2), t, g))
                skip = tr.durations[dk]
                if k != tr.blank:
                    out.append((k, t, _max_prob_conf(lg[:tr.V1], k), skip))
                    last, have, state, g_valid = k, True, nstate, False
                sym += 1
                t += skip
                need = skip == 0
            if sym == tr.max_symbols:
                t += 1
    else:
        while t < T:
            emitted = 0
            while emitted < tr.max_symbols:
                if not g_valid:
                    g, nstate = tr.step(last if have else tr.blank, not have, state)
                    g_valid = True
                lg = tr.logits(enc_proj[t], g)
                k, g1 = _argmax_gap(lg)
                gap = min(gap, g1)
                if trace is not None:
                    trace.append((len(out), g1, t, g))
                if k == tr.blank:
                    break
                out.append((k, t, _max_prob_conf(lg, k), 1))
                last, have, state, g_valid = k, True, nstate, False
                emitted += 1
            t += 1
    return out, gap
