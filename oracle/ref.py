"""ctypes binding of oracle/_ref/libpkref.so: parakeet.cpp's own CPU mel front
end, FFT and relative positional encoding, compiled from the reference sources
by oracle/Makefile.ref. TEST INFRASTRUCTURE ONLY (parity pins and the timed
CPU baseline of the front end)."""
from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int, c_long, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_ref", "libpkref.so")
_lib = None


def available() -> bool:
    return os.path.exists(LIB)


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(LIB)
        L.pkref_mel.restype = c_int
        L.pkref_mel.argtypes = [c_void_p, c_int, c_int, c_int, c_int, c_int, c_float, c_float, c_float,
                                c_int, c_void_p, c_void_p, c_void_p, c_long]
        L.pkref_rfft.restype = None
        L.pkref_rfft.argtypes = [c_void_p, c_int, c_void_p, c_void_p]
        L.pkref_rel_pos_encoding.restype = None
        L.pkref_rel_pos_encoding.argtypes = [c_int, c_int, c_void_p]
        _lib = L
    return _lib


def mel(samples, *, n_mels, n_fft, hop, win_length, preemph, mag_power, log_guard, per_feature,
        window, fb):
    """MelFrontend::compute -> feats [n_mels, T] f32. `window` is the raw
    win_length Hann window (the reference centre-pads it), fb [n_mels, n_fft/2+1]."""
    s = np.ascontiguousarray(samples, dtype=np.float32)
    win = np.ascontiguousarray(window, dtype=np.float32)
    fbm = np.ascontiguousarray(fb, dtype=np.float32)
    pad = n_fft // 2
    T = 1 + (len(s) + 2 * pad - n_fft) // hop
    out = np.zeros(n_mels * T, dtype=np.float32)
    got = lib().pkref_mel(s.ctypes.data, len(s), n_mels, n_fft, hop, win_length, preemph, mag_power,
                          log_guard, 1 if per_feature else 0, win.ctypes.data, fbm.ctypes.data,
                          out.ctypes.data, out.size)
    assert got == T, (got, T)
    return out.reshape(n_mels, T)


def rfft(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = len(x)
    re = np.zeros(n // 2 + 1, dtype=np.float32)
    im = np.zeros(n // 2 + 1, dtype=np.float32)
    lib().pkref_rfft(x.ctypes.data, n, re.ctypes.data, im.ctypes.data)
    return re, im


def rel_pos_encoding(T, d):
    out = np.zeros((2 * T - 1) * d, dtype=np.float32)
    lib().pkref_rel_pos_encoding(T, d, out.ctypes.data)
    return out.reshape(2 * T - 1, d)
