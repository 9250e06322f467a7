"""GPU parity of the cache-aware streaming encoder (pkc_stream_*) against the
oracle's restatement of StreamingEncoder::step (src/streaming_encoder.cpp),
which is itself pinned to the offline causal encoder by the reference's
cache-aware equivalence (tests/test_oracle_cpu.py).

Tolerance: each chunk's output within 2e-2 relative error (max |gpu - oracle|
/ max |oracle|), the north star's bound for f16 / bf16 compute; q8_0 weights
are dequantised to the compute type inside the GEMM and use the same bound.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-2


@pytest.fixture(scope="module")
def stream_models(tmp_path_factory):
    import synth
    d = str(tmp_path_factory.mktemp("smodels"))
    small = dict(n_layers=2, d_model=256, n_heads=4, ff_dim=512, n_mels=64, vocab=16, pred_hidden=16,
                 joint_hidden=16)
    return {
        "f16": synth.ensure_gguf(synth.small_cfg("eou_120m_stream", **small), d),
        "q8_0": synth.ensure_gguf(synth.small_cfg("eou_120m_stream", dtype="q8_0", **small), d),
    }


def run_stream(s, sched, mel):
    outs = []
    for lo, hi, last in sched:
        outs.append(s.step(mel[:, lo:hi], last))
    return outs


def oracle_stream(w, mel):
    import oracle
    sc = oracle.StreamCfg(w)
    enc = oracle.StreamingEncoder(w)
    sched = oracle.stream_schedule(sc, mel.shape[1])
    return sched, [enc.step(mel[:, lo:hi], last) for lo, hi, last in sched]


@pytest.mark.parametrize("kind,T", [("f16", 300), ("f16", 701), ("q8_0", 300)])
def test_stream_matches_oracle(stream_models, kind, T):
    """Chunk by chunk against the oracle; 701 mel frames (88 encoder frames)
    fill the 70-frame attention cache and roll it."""
    import oracle
    import pkc
    w = oracle.Weights(stream_models[kind])
    mel = np.random.default_rng(T).standard_normal((64, T)).astype(np.float32)
    sched, want = oracle_stream(w, mel)
    m = pkc.Model(stream_models[kind])
    try:
        sch = m.stream_schedule()
        assert (sch["chunk_size_first"], sch["chunk_size"], sch["pre_encode_cache_size"], sch["valid_out_len"]) == \
            (9, 16, 9, 2)
        s = pkc.Stream(m)
        got = run_stream(s, sched, mel)
        assert s.step_num == len(sched)
        s.close()
    finally:
        m.close()
    assert [g.shape for g in got] == [x.shape for x in want]
    for g, x in zip(got, want):
        if len(x):
            assert np.abs(g - x).max() <= TOL * np.abs(x).max()
    total = np.concatenate(got)
    ref = np.concatenate(want)
    assert np.abs(total - ref).max() <= TOL * np.abs(ref).max()


def test_stream_reset_and_interleaved_streams(stream_models):
    """reset() replays a stream bit for bit, and two streams stepped in
    alternation keep separate caches: each equals itself run alone."""
    import oracle
    import pkc
    w = oracle.Weights(stream_models["f16"])
    sc = oracle.StreamCfg(w)
    a = np.random.default_rng(1).standard_normal((64, 260)).astype(np.float32)
    b = np.random.default_rng(2).standard_normal((64, 260)).astype(np.float32)
    sched = oracle.stream_schedule(sc, 260)
    m = pkc.Model(stream_models["f16"])
    try:
        s = pkc.Stream(m)
        alone_a = run_stream(s, sched, a)
        s.reset()
        assert s.step_num == 0
        again_a = run_stream(s, sched, a)
        s.reset()
        alone_b = run_stream(s, sched, b)
        s.reset()
        t = pkc.Stream(m)
        inter_a, inter_b = [], []
        for lo, hi, last in sched:
            inter_a.append(s.step(a[:, lo:hi], last))
            inter_b.append(t.step(b[:, lo:hi], last))
        s.close()
        t.close()
    finally:
        m.close()
    for x, y in zip(alone_a, again_a):
        assert np.array_equal(x, y)
    for x, y in zip(alone_a, inter_a):
        assert np.array_equal(x, y)
    for x, y in zip(alone_b, inter_b):
        assert np.array_equal(x, y)


def test_stream_needs_a_streaming_model(stream_models, tmp_path):
    """Offline models refuse a stream; streaming models refuse the offline
    encoder (its causal path is not implemented) with PKC_ERR_UNSUPPORTED."""
    import pkc
    import synth
    off = synth.ensure_gguf(synth.small_cfg("c2_0.6b_f16", n_layers=1, d_model=256, n_heads=4, ff_dim=256,
                                            n_mels=80, vocab=16, pred_hidden=16, joint_hidden=16), str(tmp_path))
    m = pkc.Model(off)
    try:
        with pytest.raises(pkc.PkcError) as e:
            pkc.Stream(m)
        assert e.value.status == 4
        with pytest.raises(pkc.PkcError) as e:
            m.stream_schedule()
        assert e.value.status == 4
    finally:
        m.close()
    m = pkc.Model(stream_models["f16"])
    try:
        with pytest.raises(pkc.PkcError) as e:
            m.encode_pcm_batch([synth.synth_audio(16000, 3)])
        assert e.value.status == 4
    finally:
        m.close()


def test_stream_graph_replay_matches_eager(stream_models, monkeypatch):
    """The chunk step replayed from captured CUDA graphs equals the eagerly
    issued step (PKC_NO_GRAPH=1) bit for bit, across a cache roll."""
    import oracle
    import pkc
    w = oracle.Weights(stream_models["f16"])
    sc = oracle.StreamCfg(w)
    mel = np.random.default_rng(9).standard_normal((64, 640)).astype(np.float32)
    sched = oracle.stream_schedule(sc, 640)
    res = []
    for eager in (False, True):
        if eager:
            monkeypatch.setenv("PKC_NO_GRAPH", "1")
        m = pkc.Model(stream_models["f16"])
        try:
            s = pkc.Stream(m)
            res.append(run_stream(s, sched, mel))
            s.close()
        finally:
            m.close()
    for x, y in zip(*res):
        assert np.array_equal(x, y)


def test_stream_batch_equals_streams_alone(stream_models):
    """pkc_stream_step_batch: three streams with different audio stepped as
    one batch (6 stacked frames, skinny GEMMs) equal each stream stepped alone
    bit for bit, final chunk included; 12 streams (24 frames, tcgen05 GEMMs)
    match the oracle's streaming restatement per stream and chunk."""
    import oracle
    import pkc
    w = oracle.Weights(stream_models["f16"])
    sc = oracle.StreamCfg(w)
    T = 330
    sched = oracle.stream_schedule(sc, T)
    mels = [np.random.default_rng(100 + i).standard_normal((64, T)).astype(np.float32) for i in range(12)]
    m = pkc.Model(stream_models["f16"])
    try:
        alone = []
        for i in range(3):
            s = pkc.Stream(m)
            alone.append(run_stream(s, sched, mels[i]))
            s.close()
        for S in (3, 12):
            streams = [pkc.Stream(m) for _ in range(S)]
            got = [[] for _ in range(S)]
            for lo, hi, last in sched:
                outs = pkc.stream_step_batch(streams, [mels[i][:, lo:hi] for i in range(S)], [last] * S)
                for i in range(S):
                    got[i].append(outs[i])
            assert all(s.step_num == len(sched) for s in streams)
            for s in streams:
                s.close()
            if S == 3:
                for i in range(3):
                    for x, y in zip(alone[i], got[i]):
                        assert np.array_equal(x, y)
            else:
                for i in (0, 5, 11):
                    _, want = oracle_stream(w, mels[i])
                    for g, x in zip(got[i], want):
                        assert g.shape == x.shape
                        if len(x):
                            assert np.abs(g - x).max() <= TOL * np.abs(x).max()
        # a batch mixing a stream at its first window with one past it is refused
        a, b = pkc.Stream(m), pkc.Stream(m)
        lo, hi, _ = sched[0]
        a.step(mels[0][:, lo:hi])
        lo, hi, _ = sched[1]
        with pytest.raises(pkc.PkcError) as e:
            pkc.stream_step_batch([a, b], [mels[0][:, lo:hi], mels[1][:, lo:hi]], [False, False])
        assert e.value.status == 1
        a.close()
        b.close()
    finally:
        m.close()
