"""Seeded synthetic models and audio for the benchmark configurations.

There is no network here, so no NeMo checkpoint and no LibriSpeech: models are
random-init FastConformers written to GGUF with the reference converter's key
schema and tensor names (scripts/convert_parakeet_to_gguf.py:152-300 of
parakeet.cpp; docs/conversion.md), and audio is a seeded mix of sines plus
noise with the lengths the benchmark configurations name.

Weight init (identical for every config): linear/conv weights and biases,
pos_bias_u/v ~ N(0, 0.02); LayerNorm gamma 1, beta 0; BatchNorm running mean 0,
var 1, gamma 1, beta 0. Biases of the conformer linears/convs exist only for the
110M class (the 0.6B/1.1B checkpoints use bias=False there). The filterbank is
the Slaney-normalised mel matrix and the window a symmetric Hann of win_length.

Weight dtypes follow the converter's quantisation allowlist (FFN linears,
q/k/v/out/pos, pre_encode.out, joint.enc/pred); everything else stays f32.
"""
from __future__ import annotations

import hashlib
import os
import re
from dataclasses import dataclass, field, asdict

import numpy as np

SR = 16000


@dataclass
class ModelCfg:
    name: str
    arch: str
    d_model: int
    n_layers: int
    n_heads: int
    ff_dim: int
    conv_kernel: int
    n_mels: int
    sub_channels: int = 256
    vocab: int = 1024
    pred_hidden: int = 640
    joint_hidden: int = 640
    pred_layers: int = 1
    streaming: bool = False     # cache-aware streaming (causal) FastConformer
    durations: tuple = ()
    dtype: str = "f32"          # f32 | f16 | bf16 | q8_0 | q4_k
    biases: bool = False
    xscaling: bool = False
    # LayerNorm affines of the conformer layers: gamma 1 + N(0, 0.1), beta
    # N(0, 0.05) instead of the BASELINE init's (1, 0), so that the parity
    # tests see a non-trivial LayerNorm scale and shift
    ln_affine: bool = False
    n_fft: int = 512
    win_length: int = 400
    hop_length: int = 160
    seed: int = 1234

    def key(self) -> str:
        items = asdict(self)
        if items["pred_layers"] == 1:  # keeps the names of files made before the field existed
            del items["pred_layers"]
        if not items["streaming"]:
            del items["streaming"]
        if not items["ln_affine"]:
            del items["ln_affine"]
        h = hashlib.sha1(repr(sorted(items.items())).encode()).hexdigest()[:12]
        return f"{self.name}_{self.dtype}_{h}"


# The five BASELINE.json configurations (model part).
CONFIGS = {
    "c1_110m": ModelCfg("c1_110m", "hybrid_tdt_ctc", 512, 17, 8, 2048, 9, 80,
                        durations=(0, 1, 2, 3, 4), dtype="f32", biases=True),
    "c2_0.6b_f16": ModelCfg("c2_0.6b_f16", "tdt", 1024, 24, 8, 4096, 9, 128,
                            durations=(0, 1, 2, 3, 4), dtype="f16"),
    "c3_0.6b_q8": ModelCfg("c3_0.6b_q8", "rnnt", 1024, 24, 8, 4096, 9, 128, dtype="q8_0"),
    "c4_1.1b_q4k": ModelCfg("c4_1.1b_q4k", "hybrid_tdt_ctc", 1024, 42, 8, 4096, 9, 128,
                            durations=(0, 1, 2, 3, 4), dtype="q4_k"),
    "c5_0.6b_bf16_long": ModelCfg("c5_0.6b_bf16_long", "tdt", 1024, 24, 8, 4096, 9, 128,
                                  vocab=8192, durations=(0, 1, 2, 3, 4), dtype="bf16"),
}

# The cache-aware streaming model class of the reference (parakeet_realtime_eou_120m:
# 17 layers, d 512, causal subsampling, chunked-limited attention, layer_norm conv norm).
STREAM_CONFIGS = {
    "eou_120m_stream": ModelCfg("eou_120m_stream", "rnnt", 512, 17, 8, 2048, 9, 128, vocab=1026,
                                dtype="f16", biases=True, streaming=True),
}

# Batch part of each configuration: (batch, min_s, max_s) with lengths U(min,max).
BATCHES = {
    "c1_110m": (1, 10.0, 10.0),
    "c2_0.6b_f16": (16, 2.0, 35.0),
    "c3_0.6b_q8": (64, 2.0, 35.0),
    "c4_1.1b_q4k": (128, 2.0, 35.0),
    "c5_0.6b_bf16_long": (8, 120.0, 120.0),
}

QUANT_PATTERNS = [re.compile(p) for p in (
    r"^encoder\.layers\.\d+\.feed_forward[12]\.linear[12]\.weight$",
    r"^encoder\.layers\.\d+\.self_attn\.linear_(q|k|v|out|pos)\.weight$",
    r"^encoder\.pre_encode\.out\.weight$",
    r"^joint\.enc\.weight$",
    r"^joint\.pred\.weight$",
)]


def quantizable(name: str) -> bool:
    return any(p.match(name) for p in QUANT_PATTERNS)


# ----------------------------------------------------------------- front end

def slaney_mel_fb(sr: int, n_fft: int, n_mels: int, fmin: float = 0.0, fmax: float | None = None):
    """Slaney-style mel filterbank [n_mels, n_fft//2+1] (librosa's published
    formula: linear below 1 kHz, log above, area-normalised triangles)."""
    fmax = sr / 2 if fmax is None else fmax
    f_sp = 200.0 / 3
    min_log_hz = 1000.0
    min_log_mel = min_log_hz / f_sp
    logstep = np.log(6.4) / 27.0

    def hz_to_mel(f):
        f = np.asarray(f, dtype=np.float64)
        m = f / f_sp
        return np.where(f >= min_log_hz, min_log_mel + np.log(np.maximum(f, 1e-10) / min_log_hz) / logstep, m)

    def mel_to_hz(m):
        m = np.asarray(m, dtype=np.float64)
        f = f_sp * m
        return np.where(m >= min_log_mel, min_log_hz * np.exp(logstep * (m - min_log_mel)), f)

    fftfreqs = np.linspace(0, sr / 2, 1 + n_fft // 2)
    mel_f = mel_to_hz(np.linspace(hz_to_mel(fmin), hz_to_mel(fmax), n_mels + 2))
    fdiff = np.diff(mel_f)
    ramps = mel_f[:, None] - fftfreqs[None, :]
    w = np.zeros((n_mels, len(fftfreqs)))
    for i in range(n_mels):
        lower = -ramps[i] / fdiff[i]
        upper = ramps[i + 2] / fdiff[i + 1]
        w[i] = np.maximum(0, np.minimum(lower, upper))
    enorm = 2.0 / (mel_f[2:n_mels + 2] - mel_f[:n_mels])
    w *= enorm[:, None]
    return w.astype(np.float32)


def hann_symmetric(n: int):
    k = np.arange(n, dtype=np.float64)
    return (0.5 - 0.5 * np.cos(2 * np.pi * k / (n - 1))).astype(np.float32)


# ----------------------------------------------------------------- q4_k

def quantize_q4_k(x: np.ndarray) -> np.ndarray:
    """Quantise rows of x (last dim a multiple of 256) to the q4_k super-block
    layout gguf-py dequantises (gguf/quants.py Q4_K): per 256 values
    f16 d, f16 dmin, 12 bytes of 6-bit sub-block scales/mins, 128 bytes of
    nibbles; value = d*sc_j*q - dmin*m_j for sub-block j of 32 values."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows = x.reshape(-1, 256)
    nb = rows.shape[0]
    sub = rows.reshape(nb, 8, 32)
    mn = np.minimum(sub.min(axis=2), 0.0)            # <= 0
    mx = sub.max(axis=2)
    scale = (mx - mn) / 15.0                          # >= 0
    d = scale.max(axis=1) / 63.0
    dmin = (-mn).max(axis=1) / 63.0
    d16 = d.astype(np.float16)
    dmin16 = dmin.astype(np.float16)
    df = d16.astype(np.float32)
    dminf = dmin16.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(df[:, None] > 0, np.rint(scale / df[:, None]), 0).clip(0, 63).astype(np.uint8)
        mq = np.where(dminf[:, None] > 0, np.rint(-mn / dminf[:, None]), 0).clip(0, 63).astype(np.uint8)
        eff_s = df[:, None] * sc.astype(np.float32)
        eff_m = dminf[:, None] * mq.astype(np.float32)
        q = np.where(eff_s[:, :, None] > 0, np.rint((sub + eff_m[:, :, None]) / eff_s[:, :, None]), 0)
    q = q.clip(0, 15).astype(np.uint8)                 # [nb, 8, 32]
    scales = np.zeros((nb, 12), dtype=np.uint8)
    scales[:, 0:4] = (sc[:, 0:4] & 0x3F) | ((sc[:, 4:8] >> 4) << 6)
    scales[:, 4:8] = (mq[:, 0:4] & 0x3F) | ((mq[:, 4:8] >> 4) << 6)
    scales[:, 8:12] = (sc[:, 4:8] & 0x0F) | ((mq[:, 4:8] & 0x0F) << 4)
    qs = np.zeros((nb, 4, 32), dtype=np.uint8)
    qs[:] = q[:, 0::2, :] | (q[:, 1::2, :] << 4)
    out = np.concatenate([d16.view(np.uint8).reshape(nb, 2), dmin16.view(np.uint8).reshape(nb, 2),
                          scales, qs.reshape(nb, 128)], axis=1)
    return out.reshape(*x.shape[:-1], x.shape[-1] // 256 * 144)


# ----------------------------------------------------------------- model

def model_tensors(cfg: ModelCfg):
    """Yield (name, float32 array in torch/numpy shape) for every tensor."""
    rng = np.random.default_rng(cfg.seed)

    def nrm(*shape):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02))

    d, C, H = cfg.d_model, cfg.sub_channels, cfg.n_heads
    dk = d // H
    F3 = cfg.n_mels
    for _ in range(3):  # causal subsampling pads 2 + 1, offline 1 + 1
        F3 = F3 // 2 + 1 if cfg.streaming else (F3 - 1) // 2 + 1
    nb = cfg.n_fft // 2 + 1
    yield "preprocessor.featurizer.fb", slaney_mel_fb(SR, cfg.n_fft, cfg.n_mels)[None]
    yield "preprocessor.featurizer.window", hann_symmetric(cfg.win_length)
    pre = "encoder.pre_encode."
    yield pre + "conv.0.weight", nrm(C, 1, 3, 3)
    yield pre + "conv.0.bias", nrm(C)
    for i in (2, 5):
        yield pre + f"conv.{i}.weight", nrm(C, 1, 3, 3)
        yield pre + f"conv.{i}.bias", nrm(C)
        yield pre + f"conv.{i + 1}.weight", nrm(C, C, 1, 1)
        yield pre + f"conv.{i + 1}.bias", nrm(C)
    yield pre + "out.weight", nrm(d, C * F3)
    yield pre + "out.bias", nrm(d)
    ones = lambda n: np.ones(n, dtype=np.float32)
    zeros = lambda n: np.zeros(n, dtype=np.float32)
    for li in range(cfg.n_layers):
        p = f"encoder.layers.{li}."
        for ln in ("norm_feed_forward1", "norm_self_att", "norm_conv", "norm_feed_forward2", "norm_out"):
            if cfg.ln_affine:
                yield p + ln + ".weight", ones(d) + nrm(d) * np.float32(5.0)
                yield p + ln + ".bias", nrm(d) * np.float32(2.5)
            else:
                yield p + ln + ".weight", ones(d)
                yield p + ln + ".bias", zeros(d)
        for ff in ("feed_forward1", "feed_forward2"):
            yield p + ff + ".linear1.weight", nrm(cfg.ff_dim, d)
            if cfg.biases:
                yield p + ff + ".linear1.bias", nrm(cfg.ff_dim)
            yield p + ff + ".linear2.weight", nrm(d, cfg.ff_dim)
            if cfg.biases:
                yield p + ff + ".linear2.bias", nrm(d)
        for nm in ("linear_q", "linear_k", "linear_v", "linear_out"):
            yield p + "self_attn." + nm + ".weight", nrm(d, d)
            if cfg.biases:
                yield p + "self_attn." + nm + ".bias", nrm(d)
        yield p + "self_attn.linear_pos.weight", nrm(d, d)
        yield p + "self_attn.pos_bias_u", nrm(H, dk)
        yield p + "self_attn.pos_bias_v", nrm(H, dk)
        yield p + "conv.pointwise_conv1.weight", nrm(2 * d, d, 1)
        if cfg.biases:
            yield p + "conv.pointwise_conv1.bias", nrm(2 * d)
        yield p + "conv.depthwise_conv.weight", nrm(d, 1, cfg.conv_kernel)
        if cfg.biases:
            yield p + "conv.depthwise_conv.bias", nrm(d)
        if cfg.streaming:  # conv_norm_type layer_norm: gamma / beta under the batch_norm names
            yield p + "conv.batch_norm.weight", ones(d) + nrm(d) * np.float32(10.0)
            yield p + "conv.batch_norm.bias", nrm(d) * np.float32(10.0)
        else:
            yield p + "conv.batch_norm.weight", ones(d)
            yield p + "conv.batch_norm.bias", zeros(d)
            yield p + "conv.batch_norm.running_mean", zeros(d)
            yield p + "conv.batch_norm.running_var", ones(d)
        yield p + "conv.pointwise_conv2.weight", nrm(d, d, 1)
        if cfg.biases:
            yield p + "conv.pointwise_conv2.bias", nrm(d)
    V1 = cfg.vocab + 1
    if cfg.arch in ("ctc", "hybrid_tdt_ctc", "hybrid_rnnt_ctc"):
        head = "decoder" if cfg.arch == "ctc" else "ctc_decoder"
        yield head + ".decoder_layers.0.weight", nrm(V1, d, 1)
        yield head + ".decoder_layers.0.bias", nrm(V1)
    if cfg.arch != "ctc":
        Hp = cfg.pred_hidden
        yield "decoder.prediction.embed.weight", nrm(V1, Hp)
        for l in range(cfg.pred_layers):
            yield f"decoder.prediction.dec_rnn.lstm.weight_ih_l{l}", nrm(4 * Hp, Hp)
            yield f"decoder.prediction.dec_rnn.lstm.weight_hh_l{l}", nrm(4 * Hp, Hp)
            yield f"decoder.prediction.dec_rnn.lstm.bias_ih_l{l}", nrm(4 * Hp)
            yield f"decoder.prediction.dec_rnn.lstm.bias_hh_l{l}", nrm(4 * Hp)
        J = cfg.joint_hidden
        yield "joint.enc.weight", nrm(J, d)
        yield "joint.enc.bias", nrm(J)
        yield "joint.pred.weight", nrm(J, Hp)
        yield "joint.pred.bias", nrm(J)
        yield "joint.joint_net.2.weight", nrm(V1 + len(cfg.durations), J)
        yield "joint.joint_net.2.bias", nrm(V1 + len(cfg.durations))


def write_gguf(cfg: ModelCfg, path: str) -> str:
    import gguf
    w = gguf.GGUFWriter(path, "parakeet")
    w.add_string("general.name", cfg.name)
    w.add_string("parakeet.arch", cfg.arch)
    w.add_uint32("parakeet.encoder.feat_in", cfg.n_mels)
    w.add_uint32("parakeet.encoder.d_model", cfg.d_model)
    w.add_uint32("parakeet.encoder.n_layers", cfg.n_layers)
    w.add_uint32("parakeet.encoder.n_heads", cfg.n_heads)
    w.add_uint32("parakeet.encoder.ff_dim", cfg.ff_dim)
    w.add_uint32("parakeet.encoder.conv_kernel", cfg.conv_kernel)
    w.add_string("parakeet.encoder.conv_norm_type", "layer_norm" if cfg.streaming else "batch_norm")
    if cfg.streaming:
        # the cache-aware schedule of the 120M EOU streaming model (att_context_size [70, 1])
        w.add_string("parakeet.encoder.att_context_style", "chunked_limited")
        w.add_int32("parakeet.encoder.att_context_left", 70)
        w.add_int32("parakeet.encoder.att_context_right", 1)
        w.add_bool("parakeet.encoder.causal_downsampling", True)
        w.add_bool("parakeet.encoder.conv_causal", True)
        w.add_array("parakeet.streaming.chunk_size", [9, 16])
        w.add_array("parakeet.streaming.shift_size", [9, 16])
        w.add_array("parakeet.streaming.pre_encode_cache_size", [0, 9])
        w.add_int32("parakeet.streaming.cache_drop_size", 0)
        w.add_int32("parakeet.streaming.last_channel_cache_size", 70)
        w.add_int32("parakeet.streaming.valid_out_len", 2)
        w.add_int32("parakeet.streaming.drop_extra_pre_encoded", 2)
    w.add_uint32("parakeet.encoder.subsampling_factor", 8)
    w.add_uint32("parakeet.encoder.subsampling_conv_channels", cfg.sub_channels)
    w.add_bool("parakeet.encoder.xscaling", cfg.xscaling)
    w.add_uint32("parakeet.encoder.pos_emb_max_len", 5000)
    w.add_uint32("parakeet.preprocessor.sample_rate", SR)
    w.add_uint32("parakeet.preprocessor.n_mels", cfg.n_mels)
    w.add_uint32("parakeet.preprocessor.n_fft", cfg.n_fft)
    w.add_uint32("parakeet.preprocessor.win_length", cfg.win_length)
    w.add_uint32("parakeet.preprocessor.hop_length", cfg.hop_length)
    w.add_float32("parakeet.preprocessor.preemph", 0.97)
    w.add_float32("parakeet.preprocessor.mag_power", 2.0)
    w.add_string("parakeet.preprocessor.normalize", "per_feature")
    w.add_float32("parakeet.preprocessor.log_zero_guard", 2.0 ** -24)
    w.add_uint32("parakeet.vocab_size", cfg.vocab)
    w.add_uint32("parakeet.blank_id", cfg.vocab)
    w.add_array("parakeet.tokenizer.pieces", [f"▁t{i}" for i in range(cfg.vocab)])
    if cfg.arch != "ctc":
        w.add_uint32("parakeet.decoder.pred_hidden", cfg.pred_hidden)
        w.add_uint32("parakeet.decoder.pred_rnn_layers", cfg.pred_layers)
        w.add_uint32("parakeet.joint.joint_hidden", cfg.joint_hidden)
        w.add_string("parakeet.joint.activation", "relu")
        w.add_uint32("parakeet.decoding.max_symbols", 10)
    if cfg.durations:
        w.add_array("parakeet.tdt.durations", [int(x) for x in cfg.durations])
    qt = gguf.GGMLQuantizationType
    for name, arr in model_tensors(cfg):
        arr = np.ascontiguousarray(arr, dtype=np.float32)
        ne0 = arr.shape[-1]
        if cfg.dtype == "f32" or not quantizable(name) or arr.ndim < 2 or min(arr.shape[-1], arr.shape[0]) < 32:
            w.add_tensor(name, arr)
        elif cfg.dtype == "f16":
            w.add_tensor(name, arr.astype(np.float16))
        elif cfg.dtype == "bf16":
            raw = gguf.quants.quantize(arr, qt.BF16)
            w.add_tensor(name, raw, raw_shape=raw.shape, raw_dtype=qt.BF16)
        elif cfg.dtype == "q8_0" and ne0 % 32 == 0:
            raw = gguf.quants.quantize(arr, qt.Q8_0)
            w.add_tensor(name, raw, raw_shape=raw.shape, raw_dtype=qt.Q8_0)
        elif cfg.dtype == "q4_k" and ne0 % 256 == 0:
            raw = quantize_q4_k(arr)
            w.add_tensor(name, raw, raw_shape=raw.shape, raw_dtype=qt.Q4_K)
        else:
            w.add_tensor(name, arr)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path


def ensure_gguf(cfg: ModelCfg, cache_dir: str | None = None) -> str:
    """Write cfg's GGUF once into cache_dir (default: $PKC_CACHE or /tmp/pkc_models)."""
    cache_dir = cache_dir or os.environ.get("PKC_CACHE", "/tmp/pkc_models")
    os.makedirs(cache_dir, exist_ok=True)
    path = os.path.join(cache_dir, cfg.key() + ".gguf")
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        write_gguf(cfg, tmp)
        os.replace(tmp, path)
    return path


def small_cfg(base: str = "c2_0.6b_f16", **over) -> ModelCfg:
    """A reduced copy of a configuration for fast parity runs."""
    c = CONFIGS[base] if base in CONFIGS else STREAM_CONFIGS[base]
    d = asdict(c)
    d.update(over)
    d["name"] = d.get("name", c.name) + "_small"
    return ModelCfg(**d)


# ----------------------------------------------------------------- audio

def synth_audio(n_samples: int, seed: int) -> np.ndarray:
    """3 sines (f ~ U(100, 4000) Hz, amplitude ~ U(0.1, 0.5), phase ~ U(0, 2pi))
    plus N(0, 0.05) noise, clipped to [-1, 1], 16 kHz f32."""
    rng = np.random.default_rng(seed)
    t = np.arange(n_samples, dtype=np.float64) / SR
    f = rng.uniform(100.0, 4000.0, 3)
    a = rng.uniform(0.1, 0.5, 3)
    ph = rng.uniform(0.0, 2 * np.pi, 3)
    x = (a[:, None] * np.sin(2 * np.pi * f[:, None] * t[None, :] + ph[:, None])).sum(0)
    x = x + rng.standard_normal(n_samples) * 0.05
    return np.clip(x, -1.0, 1.0).astype(np.float32)


def batch_lengths(batch: int, min_s: float, max_s: float, seed: int) -> list[int]:
    """Clip lengths in samples, U(min_s, max_s) seconds from their own stream."""
    if min_s == max_s:
        return [int(round(min_s * SR))] * batch
    rng = np.random.default_rng(seed + 7919)
    return [int(round(s * SR)) for s in rng.uniform(min_s, max_s, batch)]


def synth_batch(config: str, seed: int = 0, batch: int | None = None):
    """PCM clips for configuration `config` (batch size overridable)."""
    b, lo, hi = BATCHES[config]
    b = batch if batch is not None else b
    lens = batch_lengths(b, lo, hi, seed)
    return [synth_audio(n, seed * 100003 + i) for i, n in enumerate(lens)]
