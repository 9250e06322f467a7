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


# ------------------------------------------------------------ decoded tokens
#
# Greedy decoding is exact arithmetic on top of the encoder output, so a
# token can only differ from the oracle's where the encoder's rounding moves a
# joint / CTC logit across the decision. The tests below therefore compare
# tokens on the prefix before the first decision (in the oracle's decode of
# its own encoder output) whose top-two margin is at most
# tau = max(1e-3, 2 * delta), where delta is the largest logit change that the
# GPU's encoder output causes along that decode path (measured, printed): the
# north star's 1e-3 margin, widened only by what the compute type's rounding
# can account for. A second, teacher-forced check follows the reference's
# decode path (its token history) and requires every decision on it whose
# margin exceeds tau to come out the same from the GPU's encoder output. The
# GPU decoder itself must reproduce the oracle's decode of the GPU's own
# encoder output exactly (near-ties below 1e-5 excepted).

def _transducer_prefix(tr, x_ref, x_gpu, gpu_tokens, max_decisions=3000):
    import numpy as np
    import oracle
    trace = []
    want, _ = oracle.transducer_greedy(tr, x_ref, trace=trace)
    own, own_gap = oracle.transducer_greedy(tr, x_gpu)
    if own_gap >= 1e-5:
        assert [(t[0], t[1], t[3]) for t in gpu_tokens] == [(t[0], t[1], t[3]) for t in own], \
            "GPU decode differs from the oracle's decode of the GPU's encoder output"
    dec = trace[:max_decisions]
    ts = np.array([d[2] for d in dec])
    G = np.stack([d[3] for d in dec])
    pred = G @ tr.w_pred.T + tr.b_pred
    ep_ref = x_ref.astype(np.float64) @ tr.w_enc.T + tr.b_enc
    ep_gpu = x_gpu.astype(np.float64) @ tr.w_enc.T + tr.b_enc
    f_ref = np.maximum(ep_ref[ts] + pred, 0.0)
    f_gpu = np.maximum(ep_gpu[ts] + pred, 0.0)
    l_ref = f_ref @ tr.w_out.T + tr.b_out
    l_gpu = f_gpu @ tr.w_out.T + tr.b_out
    delta = float(np.abs(l_ref - l_gpu).max())
    tau = max(1e-3, 2.0 * delta)
    # teacher-forced: every decision of the reference path (its token history,
    # so its prediction state) whose top-two margin exceeds tau takes the same
    # token (and TDT duration) from the GPU's encoder output
    gaps = np.array([d[1] for d in dec])
    safe = gaps > tau
    V1 = tr.V1
    assert (l_gpu[safe, :V1].argmax(1) == l_ref[safe, :V1].argmax(1)).all()
    if tr.durations:
        assert (l_gpu[safe, V1:].argmax(1) == l_ref[safe, V1:].argmax(1)).all()
    n_forced = int(safe.sum())
    # (reported, not asserted) at the bare 1e-3 margin: how many of those
    # decisions the GPU's encoder output leaves unchanged
    strict = gaps > 1e-3
    n_strict = int(strict.sum())
    n_strict_same = int((l_gpu[strict, :V1].argmax(1) == l_ref[strict, :V1].argmax(1)).sum())
    n_safe = dec[-1][0] if len(dec) < len(trace) else len(want)
    for n_before, gap, _, _ in dec:
        if gap <= tau:
            n_safe = n_before
            break
    got = [(t[0], t[1], t[3]) for t in gpu_tokens[:n_safe]]
    assert got == [(t[0], t[1], t[3]) for t in want[:n_safe]], (n_safe, tau)
    return n_safe, len(want), tau, delta, n_forced, len(dec), n_strict_same, n_strict


def _ctc_frames(lp_gpu, lp_ref):
    import numpy as np
    delta = float(np.abs(lp_gpu - lp_ref).max())
    tau = max(1e-3, 2.0 * delta)
    s = np.sort(lp_ref, axis=1)
    safe = (s[:, -1] - s[:, -2]) > tau
    assert (lp_gpu.argmax(axis=1)[safe] == lp_ref.argmax(axis=1)[safe]).all()
    return int(safe.sum()), lp_ref.shape[0], tau, delta


def _run_full(cfg_name, pcm, tol, decode):
    """Encoder (per element, tol) and decoded tokens of the full-size model."""
    import oracle
    import pkc
    import synth
    path = synth.ensure_gguf(synth.CONFIGS[cfg_name])
    m = pkc.Model(path)
    try:
        xs = m.encode_pcm_batch(pcm, layout=pkc.LAYOUT_TIME_MAJOR)
        toks = m.transducer_greedy_pcm_batch(pcm) if "transducer" in decode else None
        ctc = m.ctc_greedy_pcm_batch(pcm, logprobs=True) if "ctc" in decode else None
    finally:
        m.close()
    w = oracle.Weights(path)
    ref = oracle.encode_pcm_batch(w, pcm)
    errs = [max_rel_err(x, r) for x, r in zip(xs, ref.outs)]  # both time-major [T', d]
    print(f"{cfg_name}: encoder per-element max rel err {[f'{e:.2e}' for e in errs]}")
    assert max(errs) <= tol, errs
    if toks is not None:
        tr = oracle.Transducer(w)
        for b, (x, r) in enumerate(zip(xs, ref.outs)):
            T = min(x.shape[0], decode["transducer"])
            x_ref = r[:T]
            # tokens of frames < T (greedy decoding is causal over frames)
            gtk = [t for t in toks[b] if t[1] < T]
            n_safe, n_all, tau, delta, n_forced, n_dec, n_ss, n_s = _transducer_prefix(tr, x_ref, x[:T], gtk)
            print(f"{cfg_name} clip {b}: transducer tokens identical on the first {n_safe} of {n_all}; "
                  f"teacher-forced decisions identical on {n_forced} of {n_dec} "
                  f"(margin > tau {tau:.2e}; logit deviation {delta:.2e}); "
                  f"at margin > 1e-3: {n_ss} of {n_s} the same")
    if ctc is not None:
        tks, lps = ctc
        for b, (lp, r) in enumerate(zip(lps, ref.outs)):
            n_safe, n_all, tau, delta = _ctc_frames(lp, oracle.ctc_log_probs(w, r))
            print(f"{cfg_name} clip {b}: CTC argmax identical on {n_safe} of {n_all} frames "
                  f"(margin > tau {tau:.2e}; log-prob deviation {delta:.2e})")
    return errs


def test_config1_110m_f32_tokens():
    """C1 (f32 weights, the f32-accurate path): CTC and TDT tokens."""
    import synth
    pcm = synth.synth_batch("c1_110m", seed=0)
    _run_full("c1_110m", pcm, 1e-3, {"ctc": True, "transducer": 10 ** 9})


def test_config3_0p6b_q8_rnnt_full_depth():
    """C3: 24 layers, d 1024, q8_0 weights dequantised in the GEMM, RNN-T."""
    import synth
    pcm = [synth.synth_audio(int(16000 * 4.3), 301), synth.synth_audio(int(16000 * 2.1), 302),
           synth.synth_audio(16000 * 3 + 17, 303)]
    _run_full("c3_0.6b_q8", pcm, 2e-2, {"transducer": 10 ** 9})


def test_config4_1p1b_q4k_ctc_tdt_full_depth():
    """C4: 42 layers, d 1024, q4_k weights, hybrid TDT + CTC (both decoded)."""
    import synth
    pcm = [synth.synth_audio(16000 * 3 + 5, 401), synth.synth_audio(int(16000 * 2.2), 402)]
    _run_full("c4_1.1b_q4k", pcm, 2e-2, {"ctc": True, "transducer": 10 ** 9})


def test_config5_0p6b_bf16_120s_full_depth():
    """C5: one 120 s clip (T' = 1500 frames, full-context attention), bf16
    weights, 8192-token TDT joint; tokens compared over the first 300 frames
    (the encoder output itself over all 1500). The random-init joint makes
    nearly the same decision every step with a top-two margin of ~3.4e-3,
    below twice the logit deviation bf16 operands cause (~5e-3), so here the
    margin-safe prefix is empty and the check that binds is the GPU decoder
    reproducing the oracle's decode of the GPU's own encoder output."""
    import synth
    pcm = [synth.synth_audio(16000 * 120, 501)]
    _run_full("c5_0.6b_bf16_long", pcm, 2e-2, {"transducer": 300})
