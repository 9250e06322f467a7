"""CPU: pin the oracle against parakeet.cpp's own code, its known-answer tests
and its self-consistency properties (no GPU needed).

Anchors:
  * tests/golden/ref_frontend.npz — outputs of the reference's compiled
    MelFrontend::compute, pk::rfft and pk::rel_pos_encoding (made by
    tests/golden/make_golden.py from oracle/_ref)
  * the reference's test_fft known answer (tests/test_fft.cpp:5-18)
  * the reference's GpuMel-vs-MelFrontend bound (tests/test_mel_gpu.cpp:65, 0.05)
  * rel_shift's literal pad/reshape/view sequence (src/relpos_attention.cpp:230-238)
  * batched == standalone (tests/test_encoder_batch.cpp)
"""
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden", "ref_frontend.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="module")
def tiny_model(tmp_path_factory):
    import synth
    cfg = synth.small_cfg("c1_110m", n_layers=2, d_model=256, n_heads=4, ff_dim=512, vocab=32,
                          pred_hidden=32, joint_hidden=32)
    return synth.ensure_gguf(cfg, str(tmp_path_factory.mktemp("m")))


class _W:
    """Stand-in for oracle.Weights carrying only the front-end fields."""

    def __init__(self, n_mels, fb, window):
        self.n_mels, self.n_fft, self.hop = n_mels, 512, 160
        self.preemph, self.mag_power, self.log_guard, self.per_feature = 0.97, 2.0, 2.0 ** -24, True
        self._fb, self._win = fb, window

    def window(self):
        w = np.zeros(512, dtype=np.float32)
        w[56:456] = self._win
        return w

    def fb(self):
        return self._fb


def test_fft_known_answer(golden):
    """tests/test_fft.cpp: a cosine at bin 8 peaks at bin 8."""
    re, im = golden["rfft_cos8_re"], golden["rfft_cos8_im"]
    assert int(np.argmax(re * re + im * im)) == 8
    x = np.cos(2 * np.pi * 8 * np.arange(512) / 512)
    spec = np.fft.rfft(x)
    assert int(np.argmax(np.abs(spec))) == 8
    np.testing.assert_allclose(spec.real.astype(np.float32), re, atol=1e-4)
    np.testing.assert_allclose(spec.imag.astype(np.float32), im, atol=1e-4)


@pytest.mark.parametrize("n_mels", [80, 128])
def test_mel_frontend_matches_reference(golden, n_mels):
    import oracle
    from golden.make_golden import golden_clips
    w = _W(n_mels, golden[f"fb{n_mels}"], golden["window"])
    for name, clip in golden_clips().items():
        ref = golden[f"mel{n_mels}_{name}"]
        got = oracle.mel_frontend(w, clip)
        assert got.shape == ref.shape
        assert np.abs(got - ref).max() <= 1e-5, (name, np.abs(got - ref).max())


def test_gpumel_graph_within_reference_bound(golden):
    """The DFT-as-matmul front end (GpuMel) against MelFrontend: the reference
    asserts max |diff| < 0.05 on its seeded 4 s signal."""
    import oracle
    from golden.make_golden import golden_clips
    w = _W(80, golden["fb80"], golden["window"])
    clip = golden_clips()["refsig"]
    d = np.abs(oracle.mel_gpu_graph(w, clip) - golden["mel80_refsig"]).max()
    assert d < 0.05
    assert d < 1e-3  # the f64 restatement is far inside the reference's bound


def test_pos_enc_matches_reference(golden):
    import oracle
    for T, d in ((7, 64), (31, 128)):
        np.testing.assert_array_equal(oracle.rel_pos_encoding(T, d), golden[f"pe_{T}_{d}"])


@pytest.mark.parametrize("T", [1, 2, 3, 7, 16, 33])
def test_rel_shift_literal_equals_index(T):
    import oracle
    rng = np.random.default_rng(T)
    bd = rng.standard_normal((T, 2 * T - 1))
    np.testing.assert_array_equal(oracle.rel_shift_literal(bd), oracle.rel_shift_index(bd[None])[0])


def test_valid_out_len_known_values():
    """Frame counts the benchmark configurations quote: 10 s -> 125,
    35 s -> 438, 120 s -> 1500 encoder frames (mel T = 1 + S/160)."""
    import oracle
    for sec, want in ((10, 125), (35, 438), (120, 1500)):
        T = 1 + sec * 16000 // 160
        assert oracle.valid_out_len(T) == want
    # zero valid mel frames still yield one frame (C integer division)
    assert oracle.valid_out_len(1) == 1
    assert oracle.cdiv_trunc(-1, 2) == 0


def test_batched_equals_standalone(tiny_model):
    """tests/test_encoder_batch.cpp: a short utterance padded into a batch
    equals its standalone run (the per-stage masks make padding invisible)."""
    import oracle
    import synth
    w = oracle.Weights(tiny_model)
    pcm = [synth.synth_audio(16000 * 2 + 77, 1), synth.synth_audio(16000 + 160 * 3, 2), synth.synth_audio(900, 3)]
    both = oracle.encode_pcm_batch(w, pcm)
    for i, p in enumerate(pcm):
        alone = oracle.encode_pcm_batch(w, [p])
        np.testing.assert_allclose(both.outs[i], alone.outs[0], atol=1e-12, rtol=0)


def test_literal_rel_shift_in_attention(tiny_model):
    """The full attention block with the literal view sequence equals the
    index form."""
    import oracle
    w = oracle.Weights(tiny_model)
    rng = np.random.default_rng(0)
    T = 9
    x = rng.standard_normal((T, w.d))
    pe = oracle.rel_pos_encoding(T, w.d)
    a = oracle.relpos_attention(w, 0, x, pe, valid=7, literal_shift=True)
    b = oracle.relpos_attention(w, 0, x, pe, valid=7, literal_shift=False)
    np.testing.assert_allclose(a, b, atol=1e-12, rtol=0)


def test_q4_k_quantiser_matches_gguf_dequant():
    """Our q4_k writer against gguf-py's reference dequantiser (the layout the
    reference's ggml reads): round trip error bounded by the 4-bit step."""
    import gguf
    import synth
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((8, 512)) * 0.02).astype(np.float32)
    raw = synth.quantize_q4_k(x)
    assert raw.shape == (8, 512 // 256 * 144)
    back = gguf.quants.dequantize(raw, gguf.GGMLQuantizationType.Q4_K).reshape(x.shape)
    step = (x.reshape(-1, 32).max(1) - np.minimum(x.reshape(-1, 32).min(1), 0)) / 15
    err = np.abs(back - x).reshape(-1, 32).max(1)
    assert np.all(err <= step * 0.75 + 1e-4)


@pytest.mark.parametrize("T", [150, 1201])
def test_streaming_oracle_equals_offline_causal(tmp_path, T):
    """Cache-aware equivalence (tests/test_streaming_encoder.cpp of the
    reference): the streaming restatement fed the model's chunk schedule gives
    the offline causal encoder's output on every frame but the final chunk's
    valid_out_len tail. 1201 mel frames (151 output frames) run the 70-frame
    attention cache past full, so its roll and the chunked-limited left
    context are exercised."""
    import synth
    import oracle
    cfg = synth.small_cfg("eou_120m_stream", n_layers=2, d_model=128, n_heads=4, ff_dim=256, n_mels=64,
                          sub_channels=32, vocab=16, pred_hidden=16, joint_hidden=16)
    w = oracle.Weights(synth.ensure_gguf(cfg, str(tmp_path)))
    sc = oracle.StreamCfg(w)
    assert sc.chunked and sc.causal_sub and sc.conv_causal and sc.conv_norm == "layer_norm"
    mel = np.random.default_rng(T).standard_normal((64, T))
    off = oracle.encode_causal_offline(w, mel)
    enc = oracle.StreamingEncoder(w)
    st = np.concatenate([enc.step(mel[:, lo:hi], last) for lo, hi, last in oracle.stream_schedule(sc, T)])
    assert st.shape == off.shape
    m = len(st) - sc.valid_out_len
    assert np.abs(st[:m] - off[:m]).max() <= 1e-12 * np.abs(off[:m]).max()
    assert np.abs(st[m:] - off[m:]).max() > 1e-6   # the tail differs by design
