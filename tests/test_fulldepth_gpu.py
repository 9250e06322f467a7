"""Full-depth parity at the benchmark architectures (GPU vs the float64
oracle), per element with the reference's comparator form (tests/parity.py):
the 110M-class model of configuration 1 (17 layers, d 512, biases, f32
weights: the f32-accurate split-f16 path) on its 10 s utterance within 1e-3,
and the 0.6B-class model of configuration 2 (24 layers, d 1024, f16 weights)
on a ragged pair of short clips within 2e-2 (the f16 compute path). Weights
are the seeded random init of the benchmark."""
import pytest

from parity import max_rel_err

pytestmark = pytest.mark.gpu


def _check(cfg_name, pcm, tol):
    import oracle
    import pkc
    import synth
    path = synth.ensure_gguf(synth.CONFIGS[cfg_name])
    m = pkc.Model(path)
    try:
        outs = m.encode_pcm_batch(pcm)
    finally:
        m.close()
    ref = oracle.encode_pcm_batch(oracle.Weights(path), pcm)
    errs = []
    for got, r in zip(outs, ref.outs):
        assert got.shape == r.T.shape
        errs.append(max_rel_err(got, r.T))
    print(f"{cfg_name}: per-element max rel err {[f'{e:.2e}' for e in errs]}")
    assert max(errs) <= tol, errs
    return errs


def test_config1_110m_f32_10s():
    import synth
    pcm = synth.synth_batch("c1_110m", seed=0)
    assert len(pcm) == 1 and len(pcm[0]) == 160000
    _check("c1_110m", pcm, 1e-3)


def test_config2_0p6b_f16_ragged_pair():
    import synth
    pcm = [synth.synth_audio(16000 * 3 + 211, 41), synth.synth_audio(16000 * 2 - 77, 42)]
    _check("c2_0.6b_f16", pcm, 2e-2)
