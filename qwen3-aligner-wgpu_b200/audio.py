"""Audio file input: ``load_audio_wav`` (src/mel.rs:347-474), the step
``Aligner.align`` takes before the alignment path.

The decode, the downmix and the resampler are host C++ in libqa_b200.so
(``qa_decode_wav``, ``qa_resample``); this module reads the file and sizes the
buffers.  16 kHz sources are returned exactly as the reference decodes them;
other rates are converted to 16 kHz with the library's Kaiser-windowed sinc
(soxr HQ's band edges and librosa's output length, not soxr's bits).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import _lib

TARGET_SR = 16000


def decode_wav(data: bytes):
    """(mono f32 samples, sample rate, channels) of a WAV file's bytes."""
    buf = np.frombuffer(data, np.uint8)
    L = _lib.lib()
    n = ctypes.c_int64(0)
    sr = ctypes.c_int(0)
    ch = ctypes.c_int(0)
    _lib.check(L.qa_decode_wav(buf.ctypes.data, len(buf), None, 0, ctypes.byref(n),
                               ctypes.byref(sr), ctypes.byref(ch)))
    out = np.empty(n.value, np.float32)
    _lib.check(L.qa_decode_wav(buf.ctypes.data, len(buf), out.ctypes.data, len(out),
                               ctypes.byref(n), ctypes.byref(sr), ctypes.byref(ch)))
    return out, sr.value, ch.value


def resampled_length(n: int, sr_in: int, sr_out: int) -> int:
    return int(_lib.lib().qa_resampled_length(n, sr_in, sr_out))


def resample(x: np.ndarray, sr_in: int, sr_out: int) -> np.ndarray:
    """Mono f32 from sr_in to sr_out, ceil(n * sr_out / sr_in) samples."""
    x = np.ascontiguousarray(x, np.float32)
    if len(x) == 0:
        raise ValueError("nothing to resample")
    out = np.empty(resampled_length(len(x), sr_in, sr_out), np.float32)
    _lib.check(_lib.lib().qa_resample(x.ctypes.data, len(x), sr_in, sr_out, out.ctypes.data,
                                      len(out)))
    return out


def load_audio_wav(path: str | os.PathLike, target_sr: int = TARGET_SR) -> np.ndarray:
    """mel::load_audio_wav: read, decode, downmix to mono, resample to target_sr."""
    with open(path, "rb") as f:
        mono, sr, _ = decode_wav(f.read())
    return mono if sr == target_sr else resample(mono, sr, target_sr)
