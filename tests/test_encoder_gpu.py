"""GPU parity: libpkc.so (through the C ABI) against the CPU oracle, which
restates parakeet.cpp's batched encoder graph in float64.

Tolerances (stated per the north star), per element with the reference's
comparator form |gpu - oracle| <= atol + rtol |oracle| (tests/parity.py:
atol = rtol * rms of the output): rtol 1e-3 for f32 weights (the
f32-accurate split-f16 path), 2e-2 for the f16 / bf16 compute path; the
log-mel front end within 2e-3 absolute on normalised features (the
reference's own GPU-vs-CPU mel test allows 0.05). Quantised weights (q8_0 /
q4_k) are dequantised to the compute type exactly as the oracle dequantises
them, so they carry the f16 path's bound.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SR = 16000


def rel_err(got, ref):
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


# per-element bound of each model kind (f32 weights: the f32-accurate path)
RTOL = {"f32_bias": 1e-3, "f32_xs": 1e-3, "f32_ln": 1e-3}


@pytest.fixture(scope="session")
def models(tmp_path_factory):
    import synth
    d = str(tmp_path_factory.mktemp("models"))
    small = dict(n_layers=3, d_model=256, n_heads=4, ff_dim=1024, vocab=64, pred_hidden=64,
                 joint_hidden=64)
    cfgs = {
        "f16": synth.small_cfg("c2_0.6b_f16", n_mels=80, **small),
        "f32_bias": synth.small_cfg("c1_110m", **small),
        # the reference scales the subsampling output by sqrt(d_model) when
        # parakeet.encoder.xscaling is set (src/encoder.cpp:59-61,123)
        "f32_xs": synth.small_cfg("c1_110m", xscaling=True, **small),
        "bf16": synth.small_cfg("c5_0.6b_bf16_long", n_mels=128, **small),
        # non-trivial LayerNorm gamma / beta (the BASELINE init has 1 / 0)
        "f16_ln": synth.small_cfg("c2_0.6b_f16", n_mels=80, ln_affine=True, **small),
        "bf16_ln": synth.small_cfg("c5_0.6b_bf16_long", n_mels=128, ln_affine=True, **small),
        "q8_ln": synth.small_cfg("c3_0.6b_q8", n_mels=80, ln_affine=True, **small),
        "q4_ln": synth.small_cfg("c4_1.1b_q4k", n_mels=128, ln_affine=True, **small),
        "f32_ln": synth.small_cfg("c1_110m", ln_affine=True, **small),
        "q8_0": synth.small_cfg("c3_0.6b_q8", n_mels=80, **small),
        "q4_k": synth.small_cfg("c4_1.1b_q4k", n_mels=128, **small),
        "dk128": synth.small_cfg("c2_0.6b_f16", n_layers=2, d_model=512, n_heads=4, ff_dim=1024,
                                 vocab=64, pred_hidden=64, joint_hidden=64),
        "tdt2": synth.small_cfg("c2_0.6b_f16", n_layers=2, d_model=256, n_heads=4, ff_dim=1024, n_mels=80,
                                vocab=64, pred_hidden=128, joint_hidden=96, pred_layers=2),
        # C5's decoder geometry (8192 tokens, pred / joint 640) on a small encoder
        "tdt_bigv": synth.small_cfg("c5_0.6b_bf16_long", n_layers=2, d_model=256, n_heads=4, ff_dim=1024,
                                    n_mels=128),
    }
    return {k: synth.ensure_gguf(c, d) for k, c in cfgs.items()}


@pytest.fixture(scope="session")
def opened(models):
    import pkc
    cache = {}

    def get(kind):
        if kind not in cache:
            cache[kind] = pkc.Model(models[kind])
        return cache[kind]
    yield get
    for m in cache.values():
        m.close()


@pytest.fixture(scope="session")
def oracles(models):
    import oracle
    cache = {}

    def get(kind):
        if kind not in cache:
            cache[kind] = oracle.Weights(models[kind])
        return cache[kind]
    return get


def clips(lengths, seed=0):
    import synth
    return [synth.synth_audio(n, seed * 1000 + i) for i, n in enumerate(lengths)]


def test_mel_front_end_matches_oracle(opened, oracles):
    import oracle
    m, w = opened("f16"), oracles("f16")
    pcm = clips([SR * 2 + 77, SR, 5000, 161, 1600])
    got, T = m.mel_batch(pcm)
    ref, Tr = oracle.mel_batch(w, pcm, gpu_graph=True)
    assert T == Tr
    assert np.abs(got - ref).max() < 2e-3, np.abs(got - ref).max()
    ref_fft, _ = oracle.mel_batch(w, pcm, gpu_graph=False)
    assert np.abs(got - ref_fft).max() < 2e-3


@pytest.mark.parametrize("kind", ["f16", "f32_bias", "f32_xs", "bf16", "q8_0", "q4_k", "dk128", "f16_ln", "bf16_ln",
                                  "q8_ln", "q4_ln", "f32_ln"])
def test_encoder_matches_oracle(opened, oracles, kind):
    import oracle
    from parity import max_rel_err
    m, w = opened(kind), oracles(kind)
    pcm = clips([SR * 3 + 500, SR * 1 + 1234, SR * 2], seed=1)
    outs = m.encode_pcm_batch(pcm)
    ref = oracle.encode_pcm_batch(w, pcm)
    assert [o.shape[1] for o in outs] == ref.valid
    errs = [max_rel_err(got, r.T) for got, r in zip(outs, ref.outs)]
    print(f"encoder {kind}: per-element max rel err {[f'{e:.2e}' for e in errs]}")
    assert max(errs) <= RTOL.get(kind, 2e-2), (kind, errs)


def test_batched_equals_standalone(opened):
    """A clip's output does not depend on its batch mates, bit for bit (every
    kernel computes a row the same way whatever the batch), and the same
    batch twice gives the same bits."""
    m = opened("f16")
    pcm = clips([SR * 4 + 17, SR * 2 + 999, 3000], seed=2)
    together = m.encode_pcm_batch(pcm)
    again = m.encode_pcm_batch(pcm)
    for a, b in zip(together, again):
        np.testing.assert_array_equal(a, b)
    for i, p in enumerate(pcm):
        alone = m.encode_pcm_batch([p])[0]
        np.testing.assert_array_equal(together[i], alone)


def test_mel_entry_matches_pcm_entry(opened):
    import pkc
    m = opened("f16")
    pcm = clips([SR * 2 + 5, SR + 160 * 7], seed=3)
    mel, T = m.mel_batch(pcm)
    a = m.encode_batch(mel, T)
    b = m.encode_pcm_batch(pcm)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)
    tm = m.encode_pcm_batch(pcm, layout=pkc.LAYOUT_TIME_MAJOR)
    for x, y in zip(tm, b):
        np.testing.assert_array_equal(x.T, y)


def test_tiny_and_boundary_clips(opened, oracles):
    """Edge lengths: one hop, just under one hop (0 valid mel frames: the
    reference's integer recurrence still yields one output frame), and lengths
    that make every stage's frame count odd/even."""
    import oracle
    m, w = opened("f16"), oracles("f16")
    lengths = [100, 160, 161, 1280, 1281, 1440, 2560 + 160]
    pcm = clips(lengths, seed=4)
    outs = m.encode_pcm_batch(pcm)
    ref = oracle.encode_pcm_batch(w, pcm)
    for got, r in zip(outs, ref.outs):
        assert got.shape == r.T.shape
        assert rel_err(got, r.T) < 2e-2


def test_bad_arguments(opened):
    import pkc
    m = opened("f16")
    with pytest.raises(pkc.PkcError) as e:
        m.encode_pcm_batch([np.zeros(0, dtype=np.float32)])
    assert e.value.status == 1
    mel = np.zeros((1, 81, 50), dtype=np.float32)
    with pytest.raises(pkc.PkcError) as e:
        m.encode_batch(mel, [50])
    assert e.value.status == 1


@pytest.mark.parametrize("kind", ["q8_0", "q4_k"])
def test_in_kernel_dequant_equals_load_time_dequant(models, kind, monkeypatch):
    """Q8_0 / Q4_K weights dequantised inside the GEMM (the default) give the
    same encoder output, bit for bit, as weights dequantised once on the host
    at load (PKC_DEQUANT_AT_LOAD=1): same per-value arithmetic (d*q, or
    (d*sc)*q - dmin*m in f32 rounded once) and the same MMA order."""
    import pkc
    pcm = clips([SR * 3 + 11, SR + 400, 5000], seed=7)
    m = pkc.Model(models[kind])
    try:
        inkernel = m.encode_pcm_batch(pcm)
    finally:
        m.close()
    monkeypatch.setenv("PKC_DEQUANT_AT_LOAD", "1")
    m = pkc.Model(models[kind])
    try:
        atload = m.encode_pcm_batch(pcm)
    finally:
        m.close()
    for a, b in zip(inkernel, atload):
        np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("kind", ["f16", "bf16", "q8_0"])
def test_fused_layernorm_matches_separate_layernorm(models, oracles, kind, monkeypatch):
    """The pre-norm LayerNorms applied inside the QKV / pointwise-1 / FFN2-up
    GEMMs (PKC_LN_FUSED=1: gamma / beta folded into the weights at load, row
    statistics from the residual GEMM's epilogue) and as separate kernels (the
    default) both stay within the oracle bound and agree well inside it. With
    q8_0 weights only pointwise-1 (dense) takes the fused form."""
    import pkc
    pcm = clips([SR * 2 + 123, 7000, SR + 1], seed=21)
    m = pkc.Model(models[kind])
    try:
        sep = m.encode_pcm_batch(pcm)
    finally:
        m.close()
    monkeypatch.setenv("PKC_LN_FUSED", "1")
    m = pkc.Model(models[kind])
    try:
        fused = m.encode_pcm_batch(pcm)
    finally:
        m.close()
    import oracle
    ref = oracle.encode_pcm_batch(oracles(kind), pcm)
    for a, b, r in zip(fused, sep, ref.outs):
        assert rel_err(a, r.T) < 2e-2
        assert rel_err(b, r.T) < 2e-2
        assert rel_err(a, b) < 1e-2


@pytest.mark.parametrize("kind", ["f16", "q8_0"])
def test_two_part_layer_schedule_is_bitwise_single_stream(models, oracles, kind, monkeypatch):
    """Large batches run their conformer layers as two utterance-contiguous
    parts on two streams inside the CUDA graph (forced here with
    PKC_STREAMS=2); every kernel computes a row / utterance the same way in
    either schedule, so the output equals the one-stream schedule
    (PKC_STREAMS=1) bit for bit, and stays within the oracle bound."""
    import oracle
    import pkc
    pcm = clips([SR * 15 + 1000 * i for i in range(8)], seed=31)
    monkeypatch.setenv("PKC_STREAMS", "2")
    m = pkc.Model(models[kind])
    try:
        two = m.encode_pcm_batch(pcm)
    finally:
        m.close()
    monkeypatch.setenv("PKC_STREAMS", "1")
    m = pkc.Model(models[kind])
    try:
        one = m.encode_pcm_batch(pcm)
    finally:
        m.close()
    for a, b in zip(two, one):
        np.testing.assert_array_equal(a, b)
    ref = oracle.encode_pcm_batch(oracles(kind), pcm[:2])
    for a, r in zip(two[:2], ref.outs):
        assert rel_err(a, r.T) < 2e-2


@pytest.mark.parametrize("kind", ["f16", "q8_0"])
def test_two_part_host_copies_pair_with_their_half(models, kind, monkeypatch):
    """Two-part plans split the mel front end and subsampling by utterance
    half as well, and the host entry points overlap their copies with the
    other half's kernels: each half's uploads go on a copy stream whose event
    its first kernel waits for (an external event node of the CUDA graph), and
    each half's downloads wait for an event its last kernel records. Checked
    bit for bit against the one-stream schedule: two calls of one geometry
    with different audio (the graph replays, and every call's copies must pair
    with its own kernels), both output layouts, the device-resident entry (the
    split front end without copies), eager launches (PKC_NO_GRAPH=1) and two
    runners on one device (the per-clip output path of the multi-device
    dispatcher)."""
    import pkc
    import torch
    lens = [SR * 15 + 1000 * i for i in range(8)]
    a, b = clips(lens, seed=41), clips(lens, seed=42)

    def run(streams, devices=(0,), eager=False):
        monkeypatch.setenv("PKC_STREAMS", streams)
        if eager:
            monkeypatch.setenv("PKC_NO_GRAPH", "1")
        else:
            monkeypatch.delenv("PKC_NO_GRAPH", raising=False)
        m = pkc.Model(models[kind], devices=devices)
        try:
            r = {"a": m.encode_pcm_batch(a), "b": m.encode_pcm_batch(b),
                 "a_tm": m.encode_pcm_batch(a, layout=pkc.LAYOUT_TIME_MAJOR), "a_again": m.encode_pcm_batch(a)}
            if len(devices) == 1:
                flat = torch.from_numpy(np.concatenate(a)).cuda()
                out = torch.empty(m.out_floats(lens), device="cuda")
                m.encode_pcm_device(flat.data_ptr(), lens, out.data_ptr(), sync=True)
                r["device"] = [out.cpu().numpy()]
        finally:
            m.close()
        return r

    one = run("1")
    assert not np.array_equal(one["a"][0], one["b"][0])
    for variant in ({}, {"eager": True}, {"devices": (0, 0)}):
        two = run("2", **variant)
        for key, outs in two.items():
            assert len(outs) == len(one[key])
            for i, (x, y) in enumerate(zip(outs, one[key])):
                np.testing.assert_array_equal(x, y, err_msg=f"{variant} {key} clip {i}")


def test_ctc_head_matches_oracle_on_the_same_encoder_output(models, oracles):
    """CTC head (hybrid model): the GPU's split-f16 GEMM (~22-bit products) +
    log-softmax + argmax, fed the GPU's own encoder output, against the f64
    restatement of CTCDecoder::forward on that same output: log-probabilities
    within 1e-3, and the greedy tokens (ids, frames) identical to the oracle's
    ctc_greedy wherever no frame's top two classes are within 1e-3."""
    import oracle
    import pkc
    w = oracles("f32_bias")
    m = pkc.Model(models["f32_bias"])
    try:
        assert m.ctc_classes() == int(w.kv["parakeet.vocab_size"]) + 1
        pcm = clips([SR * 3 + 321, SR + 77, 9000], seed=41)
        toks, lps = m.ctc_greedy_pcm_batch(pcm, logprobs=True)
        xs = m.encode_pcm_batch(pcm, layout=pkc.LAYOUT_TIME_MAJOR)
    finally:
        m.close()
    blank = int(w.kv["parakeet.blank_id"])
    for tk, lp, x in zip(toks, lps, xs):
        ref = oracle.ctc_log_probs(w, x)
        assert np.abs(lp - ref).max() < 1e-3
        top2 = np.sort(ref, axis=1)[:, -2:]
        if (top2[:, 1] - top2[:, 0]).min() > 1e-3:
            want = oracle.ctc_greedy(ref, blank)
            assert [(t[0], t[1]) for t in tk] == [(t[0], t[1]) for t in want]
            for t, u in zip(tk, want):
                assert abs(t[2] - u[2]) < 1e-3


def test_ctc_end_to_end_matches_oracle(models, oracles):
    """PCM -> tokens through mel, encoder and CTC head against the oracle's
    encoder + head: log-probabilities within the encoder's bound, and the
    tokens equal the fold of the GPU's own per-frame results."""
    import oracle
    import pkc
    w = oracles("f32_bias")
    m = pkc.Model(models["f32_bias"])
    try:
        pcm = clips([SR * 2 + 5, 4000], seed=43)
        toks, lps = m.ctc_greedy_pcm_batch(pcm, logprobs=True)
    finally:
        m.close()
    ref = oracle.encode_pcm_batch(w, pcm)
    blank = int(w.kv["parakeet.blank_id"])
    for tk, lp, r in zip(toks, lps, ref.outs):
        want = oracle.ctc_log_probs(w, r)
        assert lp.shape == want.shape
        assert np.abs(lp - want).max() < 2e-2 * np.abs(want).max()
        am = lp.argmax(axis=1)
        folded = pkc.ctc_fold(am, lp.max(axis=1), lp.shape[1], blank)
        assert [(t[0], t[1]) for t in tk] == [(t[0], t[1]) for t in folded]


def test_ctc_without_head_is_unsupported(opened):
    import pkc
    m = opened("f16")   # TDT-only synthetic model: no CTC head
    assert m.ctc_classes() == 0
    with pytest.raises(pkc.PkcError) as e:
        m.ctc_greedy_pcm_batch(clips([SR], seed=1))
    assert e.value.status == 4   # PKC_ERR_UNSUPPORTED


@pytest.mark.parametrize("kind", ["f16", "q8_0"])
def test_transducer_greedy_matches_oracle(models, oracles, kind):
    """Greedy transducer decode on the GPU (f16 model: TDT with durations
    0..4; q8_0 model: RNN-T), fed the GPU's own encoder output, against the f64
    restatement of tdt_greedy / rnnt_greedy (prediction LSTM, joint, argmax,
    max_symbols, duration skips): token ids, frames and spans identical and
    confidences within 1e-4, on clips whose decisions never come within 1e-5
    of a tie (the synthetic weights make the joint logits nearly flat)."""
    import oracle
    import pkc
    w = oracles(kind)
    tr = oracle.Transducer(w)
    m = pkc.Model(models[kind])
    try:
        assert m.transducer_kind() == (2 if tr.durations else 1)
        pcm = clips([SR * 2 + 111, SR + 5, 7000, SR * 3], seed=51)
        toks = m.transducer_greedy_pcm_batch(pcm)
        xs = m.encode_pcm_batch(pcm, layout=pkc.LAYOUT_TIME_MAJOR)
    finally:
        m.close()
    compared = 0
    for tk, x in zip(toks, xs):
        want, gap = oracle.transducer_greedy(tr, x)
        if gap < 1e-5:
            continue
        compared += 1
        assert [(t[0], t[1], t[3]) for t in tk] == [(t[0], t[1], t[3]) for t in want]
        for t, u in zip(tk, want):
            assert abs(t[2] - u[2]) < 1e-4
    assert compared >= 2


def test_pack_cache_open_matches_packed_open(models, monkeypatch, tmp_path):
    """Pre-pack cache through pkc_model_open (PKC_PACK_CACHE): the first open
    packs and writes the cache, the second uploads from it; both give the same
    encoder output bit for bit, and so does a two-runner open (devices 0, 0:
    the host image uploaded concurrently to both, the batch sharded)."""
    import pkc
    monkeypatch.setenv("PKC_PACK_CACHE", str(tmp_path))
    pcm = clips([SR * 2 + 7, SR + 333, 9000, SR * 3 + 1], seed=61)
    outs, stats = [], []
    for devices in [(0,), (0,), (0, 0)]:
        m = pkc.Model(models["q8_0"], devices=devices)
        try:
            stats.append(m.load_stats())
            outs.append(m.encode_pcm_batch(pcm))
        finally:
            m.close()
    assert [s["from_cache"] for s in stats] == [False, True, True]
    assert len([f for f in os.listdir(tmp_path) if f.endswith(".pack")]) == 1
    for o in outs[1:]:
        for a, b in zip(outs[0], o):
            assert np.array_equal(a, b)


@pytest.mark.parametrize("variant", ["resident", "streamed", "groups", "joint_streamed"])
def test_transducer_two_layer_paths(models, oracles, monkeypatch, variant):
    """Two-layer prediction LSTM (H = 128, J = 96) through the decode kernel's
    three schedules: every layer resident in shared memory; one resident layer
    with the next one streamed in during the grid barrier
    (PKC_DECODE_STREAM=1); the batch decoded in groups of 2 utterances, one
    launch each (PKC_DECODE_GROUP=2). Tokens identical to the f64 oracle."""
    import oracle
    import pkc
    if variant == "streamed":
        monkeypatch.setenv("PKC_DECODE_STREAM", "1")
    if variant == "groups":
        monkeypatch.setenv("PKC_DECODE_GROUP", "2")
    if variant == "joint_streamed":
        monkeypatch.setenv("PKC_DECODE_JOINT_STREAM", "1")
    tr = oracle.Transducer(oracles("tdt2"))
    assert tr.L == 2
    m = pkc.Model(models["tdt2"])
    try:
        pcm = clips([SR * 2 + 111, SR + 5, 7000, SR * 3, 3300, SR // 2 + 13], seed=57)
        toks = m.transducer_greedy_pcm_batch(pcm)
        xs = m.encode_pcm_batch(pcm, layout=pkc.LAYOUT_TIME_MAJOR)
    finally:
        m.close()
    compared = 0
    for tk, x in zip(toks, xs):
        want, gap = oracle.transducer_greedy(tr, x)
        if gap < 1e-5:
            continue
        compared += 1
        assert [(t[0], t[1], t[3]) for t in tk] == [(t[0], t[1], t[3]) for t in want]
        for t, u in zip(tk, want):
            assert abs(t[2] - u[2]) < 1e-4
    assert compared >= 3


def test_transducer_large_vocabulary(models, oracles):
    """8192 tokens + 5 durations with J = 640: a CTA's joint rows (56 x 640
    f32) do not fit beside the resident LSTM / pred rows and the inputs, so
    the decode streams them through its two-slot ring. Tokens identical to
    the f64 oracle."""
    import oracle
    import pkc
    tr = oracle.Transducer(oracles("tdt_bigv"))
    m = pkc.Model(models["tdt_bigv"])
    try:
        pcm = clips([SR * 2 + 5, SR + 777, 9000], seed=71)
        toks = m.transducer_greedy_pcm_batch(pcm)
        xs = m.encode_pcm_batch(pcm, layout=pkc.LAYOUT_TIME_MAJOR)
    finally:
        m.close()
    compared = 0
    for tk, x in zip(toks, xs):
        want, gap = oracle.transducer_greedy(tr, x)
        if gap < 1e-5:
            continue
        compared += 1
        assert [(t[0], t[1], t[3]) for t in tk] == [(t[0], t[1], t[3]) for t in want]
        for t, u in zip(tk, want):
            assert abs(t[2] - u[2]) < 1e-4
    assert compared >= 2


def test_transducer_absent_is_unsupported(models):
    import pkc
    m = pkc.Model(models["f32_bias"])   # hybrid model: has a transducer too
    try:
        assert m.transducer_kind() == 2
    finally:
        m.close()
