"""Regenerate tests/golden/ref_frontend.npz from parakeet.cpp's own code.

Run where the reference checkout exists (its root in PKC_REFERENCE_DIR, see
oracle/Makefile.ref) and oracle/_ref has been built by oracle/Makefile.ref: it calls the reference's compiled
MelFrontend::compute (src/mel.cpp), pk::rfft (src/fft.cpp) and
pk::rel_pos_encoding (src/pos_enc.cpp) on seeded inputs and stores their
outputs, so tests on machines without the reference checkout (the GPU box)
still compare the oracle against the reference's numbers.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(REPO, "oracle"), os.path.join(REPO, "parakeet.cpp_b200", "python")]

import ref  # noqa: E402
import synth  # noqa: E402


def reference_test_signal(S=16000 * 4):
    """The seeded signal of the reference's GpuMel test (tests/test_mel_gpu.cpp:20-33):
    0.6 sin(220 Hz) + 0.3 sin(740 Hz) + 0.1 sin(3100 Hz) + 0.05 * LCG noise."""
    t = np.arange(S, dtype=np.float64) / 16000.0
    v = 0.6 * np.sin(2 * np.pi * 220 * t) + 0.3 * np.sin(2 * np.pi * 740 * t) + 0.1 * np.sin(2 * np.pi * 3100 * t)
    seed = 0x12345678
    noise = np.empty(S)
    for i in range(S):
        seed = (seed * 1664525 + 1013904223) & 0xFFFFFFFF
        noise[i] = (seed >> 9) / float(1 << 23) - 0.5
    return (v + 0.05 * noise).astype(np.float32)


def golden_clips():
    """The inputs the fixtures were made from (regenerated, not stored)."""
    return {"refsig": reference_test_signal(), "synth_a": synth.synth_audio(16000 * 3 + 77, 5),
            "synth_b": synth.synth_audio(1234, 6)}


def main():
    assert ref.available(), "build oracle/_ref first (make -C oracle -f Makefile.ref)"
    out = {}
    for n_mels in (80, 128):
        fb = synth.slaney_mel_fb(16000, 512, n_mels)
        win = synth.hann_symmetric(400)
        kw = dict(n_mels=n_mels, n_fft=512, hop=160, win_length=400, preemph=0.97, mag_power=2.0,
                  log_guard=2.0 ** -24, per_feature=True, window=win, fb=fb)
        clips = golden_clips()
        for name, c in clips.items():
            out[f"mel{n_mels}_{name}"] = ref.mel(c, **kw)
        out[f"fb{n_mels}"] = fb
    out["window"] = synth.hann_symmetric(400)
    for T, d in ((7, 64), (31, 128)):
        out[f"pe_{T}_{d}"] = ref.rel_pos_encoding(T, d)
    x = np.cos(2 * np.pi * 8 * np.arange(512) / 512).astype(np.float32)
    re, im = ref.rfft(x)
    out["rfft_cos8_re"], out["rfft_cos8_im"] = re, im
    np.savez_compressed(os.path.join(HERE, "ref_frontend.npz"), **out)
    print("wrote", os.path.join(HERE, "ref_frontend.npz"), {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
