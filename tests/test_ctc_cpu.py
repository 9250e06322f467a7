"""CPU: the greedy CTC fold of the C ABI (pkc_ctc_fold, host arithmetic)
against the oracle's restatement of the reference's ctc_greedy
(src/search.cpp:21-90): token ids and frames identical, confidences within
f32 rounding."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "oracle"))
sys.path.insert(0, os.path.join(HERE, "..", "parakeet.cpp_b200", "python"))


def _logp(argmax, maxlp, N):
    """log-probability rows whose argmax / max are the given ones (no ties)"""
    T = len(argmax)
    lp = np.repeat((np.asarray(maxlp, dtype=np.float64) - 4.0)[:, None], N, axis=1)
    lp[np.arange(T), argmax] = maxlp
    return lp


def _check(argmax, maxlp, N, blank):
    import oracle
    import pkc
    got = pkc.ctc_fold(argmax, maxlp, N, blank)
    want = oracle.ctc_greedy(_logp(argmax, maxlp, N), blank)
    assert [(g[0], g[1], g[3]) for g in got] == [(w[0], w[1], w[3]) for w in want]
    for g, w in zip(got, want):
        assert abs(g[2] - w[2]) < 1e-5 * max(1.0, abs(w[2]))
    return got


def test_fold_known_answer():
    # blank 3; frames: blank, 1, 1, blank, 2, 2 -> tokens 1 (frame 0), 2 (frame 1)
    lp = np.log(0.7)
    got = _check(np.array([3, 1, 1, 3, 2, 2]), np.full(6, lp), 4, 3)
    assert [(t[0], t[1], t[3]) for t in got] == [(1, 0, 1), (2, 1, 1)]
    assert abs(got[0][2] - 0.6) < 1e-6


@pytest.mark.parametrize("seed", range(6))
def test_fold_random_sequences(seed):
    rng = np.random.default_rng(seed)
    N = int(rng.integers(3, 1100))
    blank = N - 1 if seed % 2 == 0 else 0
    T = int(rng.integers(1, 600))
    # runs of repeated classes, many blanks
    seq, t = [], 0
    while t < T:
        run = int(rng.integers(1, 6))
        c = blank if rng.random() < 0.45 else int(rng.integers(0, N))
        seq += [c] * run
        t += run
    seq = np.array(seq[:T])
    maxlp = rng.uniform(-3.0, -1e-3, size=T)
    _check(seq, maxlp, N, blank)


def test_fold_edge_cases():
    import pkc
    assert pkc.ctc_fold(np.zeros(0, np.int32), np.zeros(0, np.float32), 5, 4) == []
    assert _check(np.full(7, 4), np.full(7, -0.1), 5, 4) == []          # all blank
    got = _check(np.array([2, 2, 2]), np.array([-0.5, -0.2, -0.9]), 5, 4)
    assert len(got) == 1 and got[0][1] == 0                              # first token at t=0
    lib = pkc.lib()
    out = (pkc.Token * 1)()
    a = np.array([1, 2, 3], np.int32)
    m = np.zeros(3, np.float32)
    assert lib.pkc_ctc_fold(a.ctypes.data, m.ctypes.data, 3, 5, 4, out, 1) == -1  # cap too small
    assert lib.pkc_ctc_fold(a.ctypes.data, m.ctypes.data, 3, 1, 0, out, 3) == -1  # bad class count
