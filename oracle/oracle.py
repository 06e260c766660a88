"""TEST INFRASTRUCTURE — ctypes binding of the CPU oracle (build/liboracle.so).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm import this module, and only as the checker or the timed CPU reference.
The oracle restates the reference crate's `--device cpu` path (see oracle.h
for the per-function citations); it is never part of the product path.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "build", "liboracle.so")

_lib = None


def build() -> str:
    """Compile the oracle (make in this directory); returns the library path."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        vp, i, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
        L.or_f32_to_f16.argtypes = [ctypes.c_float]
        L.or_f32_to_f16.restype = ctypes.c_uint16
        L.or_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.or_f16_to_f32.restype = ctypes.c_float
        L.or_f32_to_bf16.argtypes = [ctypes.c_float]
        L.or_f32_to_bf16.restype = ctypes.c_uint16
        for fn in ("or_conv3_length", "or_valid_mel_frames"):
            getattr(L, fn).argtypes = [i64]
            getattr(L, fn).restype = i64
        for fn in ("or_audio_token_count", "or_padded_mel_frames"):
            getattr(L, fn).argtypes = [i64, i64]
            getattr(L, fn).restype = i64
        L.or_mel.argtypes = [vp, i64, vp, i64, ctypes.POINTER(i)]
        L.or_hann_window.argtypes = [i, vp]
        L.or_reflection_pad.argtypes = [vp, i, i, vp]
        L.or_mel_filterbank.argtypes = [i, i, i, vp]
        L.or_rope_tables.argtypes = [i, i, ctypes.c_double, vp, vp]
        L.or_load.argtypes = [vp, i, vp, ctypes.c_char_p, i]
        L.or_load.restype = vp
        L.or_free.argtypes = [vp]
        L.or_set_threads.argtypes = [i]
        L.or_audio_embeds.argtypes = [vp, vp, i, vp, i64]
        L.or_gather.argtypes = [vp, vp, i, vp, i, vp]
        L.or_text_hidden.argtypes = [vp, vp, i, i, vp]
        L.or_head.argtypes = [vp, vp, i, vp, i, vp, vp, vp, vp]
        L.or_fix_timestamps.argtypes = [vp, i, vp]
        L.or_gemm.argtypes = [vp, i, vp, i, vp, i, i, i, i, i]
        L.or_lh_load.argtypes = [vp, i, vp, vp, ctypes.c_char_p, i]
        L.or_lh_load.restype = vp
        L.or_lh_free.argtypes = [vp]
        L.or_lh_hann.argtypes = [i, vp]
        L.or_lh_mel_bank.argtypes = [vp]
        L.or_lh_band_edges.argtypes = [i, vp]
        L.or_lh_valid_class_count.argtypes = [ctypes.c_double, i64]
        L.or_lh_valid_class_count.restype = i64
        L.or_lh_remove_overlaps.argtypes = [vp, i]
        L.or_lh_bound_to_duration.argtypes = [vp, i, ctypes.c_double]
        L.or_lh_features_one.argtypes = [vp, vp, i64, i64, vp]
        L.or_lh_endpoint_offset.argtypes = [vp, vp, vp, vp, i]
        L.or_lh_endpoint_offset.restype = ctypes.c_float
        L.or_lh_refine.argtypes = [vp, vp, i64, i, vp, i, vp, i, vp, vp, vp]
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data if a is not None else None


def f32_to_f16_bits(x: float) -> int:
    return lib().or_f32_to_f16(x)


def f32_to_bf16_bits(x: float) -> int:
    return lib().or_f32_to_bf16(x)


def mel(samples: np.ndarray) -> np.ndarray:
    s = np.ascontiguousarray(samples, np.float32)
    frames = len(s) // 160
    out = np.zeros((128, max(frames, 1)), np.float32)
    nf = ctypes.c_int(0)
    rc = lib().or_mel(_p(s), len(s), _p(out), out.size, ctypes.byref(nf))
    if rc != 0:
        raise ValueError(f"or_mel rc={rc}")
    return out[:, : nf.value].copy() if nf.value != out.shape[1] else out


def hann_window(n: int) -> np.ndarray:
    out = np.zeros(n, np.float32)
    lib().or_hann_window(n, _p(out))
    return out


def reflection_pad(x, pad: int) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(len(x) + 2 * pad, np.float32)
    k = lib().or_reflection_pad(_p(x), len(x), pad, _p(out))
    return out[:k]


def mel_filterbank(num_mels=128, n_fft=400, sr=16000) -> np.ndarray:
    out = np.zeros((num_mels, n_fft // 2 + 1), np.float32)
    lib().or_mel_filterbank(num_mels, n_fft, sr, _p(out))
    return out


def rope_tables(positions: int, head_dim: int, theta: float = 1e6):
    c = np.zeros((positions, head_dim), np.float32)
    s = np.zeros((positions, head_dim), np.float32)
    lib().or_rope_tables(positions, head_dim, theta, _p(c), _p(s))
    return c, s


def fix_timestamps(data) -> list:
    a = np.ascontiguousarray(data, np.int64)
    out = np.zeros_like(a)
    if len(a):
        lib().or_fix_timestamps(_p(a), len(a), _p(out))
    return out.tolist()


def gemm(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    M, K = A.shape
    N = B.shape[0]
    C = np.zeros((M, N), np.float32)
    lib().or_gemm(_p(A), K, _p(B), K, _p(C), N, M, N, K, 0)
    return C


def set_threads(n: int) -> None:
    lib().or_set_threads(n)


class Model:
    """The CPU model over a weights dict (name -> bf16 bits or (dtype, array))."""

    def __init__(self, weights: dict, mcfg):
        import importlib
        qa = importlib.import_module("qwen3-aligner-wgpu_b200")
        L = lib()
        self.cfg = mcfg
        self._qcfg = qa._lib.make_cfg(mcfg)
        tens, self._keep = qa._lib.make_tensors(weights)
        err = ctypes.create_string_buffer(512)
        self.h = L.or_load(ctypes.addressof(tens), len(tens), ctypes.addressof(self._qcfg), err, 512)
        self._keep = None  # the oracle copies what it needs
        if not self.h:
            raise ValueError(err.value.decode())

    def __del__(self):
        try:
            if getattr(self, "h", None):
                lib().or_free(self.h)
        except Exception:
            pass

    def audio_embeds(self, mel_: np.ndarray) -> np.ndarray:
        """[n_mels, valid] -> [n_audio_tokens, output_dim] f32."""
        mel_ = np.ascontiguousarray(mel_, np.float32)
        valid = mel_.shape[1]
        n_tok = audio_token_count(valid, self.cfg.n_window)
        out = np.zeros((n_tok, self.cfg.output_dim), np.float32)
        rc = lib().or_audio_embeds(self.h, _p(mel_), valid, _p(out), out.size)
        if rc != 0:
            raise ValueError(f"or_audio_embeds rc={rc}")
        return out

    def gather(self, ids, audio_f16_bits: np.ndarray) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.uint32)
        a = np.ascontiguousarray(audio_f16_bits, np.uint16)
        emb = np.zeros((len(ids), self.cfg.hidden_size), np.uint16)
        rc = lib().or_gather(self.h, _p(ids), len(ids), _p(a), a.shape[0], _p(emb))
        if rc != 0:
            raise ValueError(f"or_gather rc={rc}")
        return emb

    def text_hidden(self, emb_f16_bits: np.ndarray, n_layers: int = -1) -> np.ndarray:
        e = np.ascontiguousarray(emb_f16_bits, np.uint16)
        out = np.zeros_like(e)
        rc = lib().or_text_hidden(self.h, _p(e), e.shape[0], n_layers, _p(out))
        if rc != 0:
            raise ValueError(f"or_text_hidden rc={rc}")
        return out

    def head(self, hidden_f32: np.ndarray, rows, want_logits=True, want_normed=False):
        h = np.ascontiguousarray(hidden_f32, np.float32)
        r = np.ascontiguousarray(rows, np.int32)
        n = len(r)
        raw = np.zeros(n, np.int64)
        logits = np.zeros((n, self.cfg.num_labels), np.float32) if want_logits else None
        normed = np.zeros((n, self.cfg.hidden_size), np.float32) if want_normed else None
        margin = np.zeros(n, np.float32)
        rc = lib().or_head(self.h, _p(h), h.shape[0], _p(r), n, _p(raw), _p(logits), _p(normed),
                           _p(margin))
        if rc != 0:
            raise ValueError(f"or_head rc={rc}")
        return raw, logits, normed, margin

    def align_raw(self, samples: np.ndarray, input_ids, ts_positions):
        """The whole CPU path for one clip: samples -> raw_ms (+ intermediates)."""
        m = mel(samples)
        audio = self.audio_embeds(m)
        a16 = f32_to_f16_array(audio)
        emb = self.gather(input_ids, a16)
        hid = self.text_hidden(emb)
        hid32 = f16_bits_to_f32(hid)
        raw, logits, _, margin = self.head(hid32, ts_positions)
        return dict(mel=m, audio=audio, hidden=hid32, raw_ms=raw, logits=logits, margin=margin)


def audio_token_count(valid: int, n_window: int = 50) -> int:
    return int(lib().or_audio_token_count(valid, n_window))


def f32_to_f16_array(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f16 bits (numpy's float16 cast is RNE)."""
    return np.ascontiguousarray(x, np.float32).astype(np.float16).view(np.uint16)


def f16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(b, np.uint16).view(np.float16).astype(np.float32)


# ---------------------------------------------------------------- Local Head
def lh_hann(n: int) -> np.ndarray:
    out = np.zeros(n, np.float32)
    lib().or_lh_hann(n, _p(out))
    return out


def lh_mel_bank() -> np.ndarray:
    out = np.zeros((80, 257), np.float32)
    lib().or_lh_mel_bank(_p(out))
    return out


def lh_band_edges(bins: int) -> list:
    out = np.zeros(5, np.int32)
    lib().or_lh_band_edges(bins, _p(out))
    return out.tolist()


def lh_valid_class_count(duration_ms: float, class_count: int) -> int:
    return int(lib().or_lh_valid_class_count(duration_ms, class_count))


def lh_remove_overlaps(intervals) -> list:
    iv = np.ascontiguousarray(intervals, np.float64).reshape(-1, 2).copy()
    lib().or_lh_remove_overlaps(_p(iv), len(iv))
    return iv.tolist()


def lh_bound_to_duration(intervals, duration_ms: float) -> list:
    iv = np.ascontiguousarray(intervals, np.float64).reshape(-1, 2).copy()
    lib().or_lh_bound_to_duration(_p(iv), len(iv), duration_ms)
    return iv.tolist()


class LocalHead:
    """The CPU Local Head over a package (name -> (dtype, array)) and normalizer."""

    def __init__(self, tensors: dict, mean, std):
        import importlib
        qa = importlib.import_module("qwen3-aligner-wgpu_b200")
        tens, keep = qa._lib.make_tensors(tensors)
        self._mean = np.ascontiguousarray(mean, np.float32)
        self._std = np.ascontiguousarray(std, np.float32)
        err = ctypes.create_string_buffer(512)
        self.h = lib().or_lh_load(ctypes.addressof(tens), len(tens), _p(self._mean),
                                  _p(self._std), err, 512)
        del keep
        if not self.h:
            raise ValueError(err.value.decode())

    def __del__(self):
        try:
            if getattr(self, "h", None):
                lib().or_lh_free(self.h)
        except Exception:
            pass

    def features_one(self, samples: np.ndarray, center_ms: int) -> np.ndarray:
        s = np.ascontiguousarray(samples, np.float32)
        out = np.zeros((41, 91), np.float32)
        lib().or_lh_features_one(self.h, _p(s), len(s), int(center_ms), _p(out))
        return out

    def endpoint_offset(self, feat, ctx, mask, is_end: int) -> float:
        f = np.ascontiguousarray(feat, np.float32)
        c = np.ascontiguousarray(ctx, np.float32)
        m = np.ascontiguousarray(mask, np.float32)
        return float(lib().or_lh_endpoint_offset(self.h, _p(f), _p(c), _p(m), int(is_end)))

    def refine(self, samples, logits, hidden):
        """(intervals [W][2] seconds, fixed centres [2W] ms, offsets [2W] ms)."""
        s = np.ascontiguousarray(samples, np.float32)
        lg = np.ascontiguousarray(logits, np.float32)
        hd = np.ascontiguousarray(hidden, np.float32)
        slots, n_labels = lg.shape
        W = slots // 2
        out = np.zeros((W, 2), np.float64)
        fixed = np.zeros(slots, np.int64)
        off = np.zeros(slots, np.float32)
        rc = lib().or_lh_refine(self.h, _p(s), len(s), W, _p(lg), n_labels, _p(hd), hd.shape[1],
                                _p(out), _p(fixed), _p(off))
        if rc != 0:
            raise ValueError(f"or_lh_refine rc={rc}")
        return out, fixed, off
