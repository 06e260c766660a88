"""TEST INFRASTRUCTURE: the reference's resampler, soxr 0.1.3 built from the
reference's own vendored sources by `make -C oracle ref` into oracle/_ref/,
called the way src/mel.rs:537-715 calls it: soxr_quality_spec(SOXR_HQ, 0)
(20-bit, linear phase), one thread, the input fed in blocks of 4096 samples
(`IN_BLOCK`, mel.rs:566), then flushed, and the result cut or zero-padded to
ceil(n * sr_out / sr_in) (librosa's fix_length, mel.rs:703-708).

Only the CPU tests use it, as the checker of qa_resample; nothing in the
library loads it.
"""
import ctypes
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SO = os.path.join(ROOT, "oracle", "_ref", "libsoxr.so")

SOXR_HQ = 4  # SOXR_20_BITQ
IN_BLOCK = 16 * 1024 // 4


class _QSpec(ctypes.Structure):
    _fields_ = [("precision", ctypes.c_double), ("phase_response", ctypes.c_double),
                ("passband_end", ctypes.c_double), ("stopband_begin", ctypes.c_double),
                ("e", ctypes.c_void_p), ("flags", ctypes.c_ulong)]


class _RSpec(ctypes.Structure):
    _fields_ = [("log2_min_dft_size", ctypes.c_uint), ("log2_large_dft_size", ctypes.c_uint),
                ("coef_size_kbytes", ctypes.c_uint), ("num_threads", ctypes.c_uint),
                ("e", ctypes.c_void_p), ("flags", ctypes.c_ulong)]


_lib = None


def available() -> bool:
    return os.path.exists(SO)


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(SO)
        L.soxr_quality_spec.restype = _QSpec
        L.soxr_quality_spec.argtypes = [ctypes.c_ulong, ctypes.c_ulong]
        L.soxr_runtime_spec.restype = _RSpec
        L.soxr_runtime_spec.argtypes = [ctypes.c_uint]
        L.soxr_create.restype = ctypes.c_void_p
        L.soxr_create.argtypes = [ctypes.c_double, ctypes.c_double, ctypes.c_uint,
                                  ctypes.POINTER(ctypes.c_char_p), ctypes.c_void_p,
                                  ctypes.POINTER(_QSpec), ctypes.POINTER(_RSpec)]
        L.soxr_process.restype = ctypes.c_char_p
        L.soxr_process.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                   ctypes.POINTER(ctypes.c_size_t), ctypes.c_void_p,
                                   ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]
        L.soxr_delete.argtypes = [ctypes.c_void_p]
        _lib = L
    return _lib


def resample(x, sr_in: int, sr_out: int) -> np.ndarray:
    """soxr HQ resampling of mono f32 samples, exactly as the reference feeds it."""
    L = lib()
    x = np.ascontiguousarray(x, dtype=np.float32)
    expected = int(np.ceil(len(x) * sr_out / sr_in))
    q = L.soxr_quality_spec(SOXR_HQ, 0)
    rt = L.soxr_runtime_spec(1)
    err = ctypes.c_char_p()
    h = L.soxr_create(float(sr_in), float(sr_out), 1, ctypes.byref(err), None,
                      ctypes.byref(q), ctypes.byref(rt))
    if err.value or not h:
        raise RuntimeError(f"soxr_create: {err.value}")
    out = np.zeros(expected + 8192, np.float32)
    written, off = 0, 0
    idone, odone = ctypes.c_size_t(), ctypes.c_size_t()
    try:
        while off < len(x):
            take = min(IN_BLOCK, len(x) - off)
            e = L.soxr_process(h, x[off:].ctypes.data, take, ctypes.byref(idone),
                               out[written:].ctypes.data, len(out) - written, ctypes.byref(odone))
            if e:
                raise RuntimeError(e)
            if idone.value == 0 and odone.value == 0:
                raise RuntimeError("soxr made no progress")
            off += idone.value
            written += odone.value
        while written < len(out):
            e = L.soxr_process(h, None, 0, ctypes.byref(idone), out[written:].ctypes.data,
                               len(out) - written, ctypes.byref(odone))
            if e:
                raise RuntimeError(e)
            if odone.value == 0:
                break
            written += odone.value
    finally:
        L.soxr_delete(h)
    y = out[:written]
    return y[:expected] if len(y) >= expected else np.pad(y, (0, expected - len(y)))
