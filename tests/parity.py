"""Per-element comparator of the parity tests.

The reference's comparator (tests/parity.hpp:44-70 of parakeet.cpp) passes an
output when every element satisfies |got - ref| <= atol + rtol * |ref|. The
encoder's output rows are LayerNorm'd (unit scale), so atol is tied to the
output's own scale: atol = rtol * rms(ref). The figure reported is the largest
per-element ratio |got - ref| / (rms(ref) + |ref|), which must not exceed rtol
(the north star's bound: 1e-3 for f32, 2e-2 for f16 / bf16 compute).
"""
import numpy as np


def max_rel_err(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    if ref.size == 0:
        return 0.0
    rms = float(np.sqrt(np.mean(ref * ref)))
    return float(np.max(np.abs(got - ref) / (rms + np.abs(ref) + 1e-30)))


def check(got, ref, rtol, what=""):
    e = max_rel_err(got, ref)
    assert e <= rtol, f"{what}: max per-element relative error {e:.3e} > {rtol:g}"
    return e
