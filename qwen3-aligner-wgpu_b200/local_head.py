"""The Local Head package (src/local_head.rs) on the host side: reading and
validating ``<model>/local_head/`` and the handle through which an
``Aligner`` runs ``LocalHead::refine`` on the device.

Validation follows the reference's contract line by line
(src/local_head.rs:109-160 for the files, 661-715 for config.json, 722-731
for the canonical prior, 810-916 for the tensors): every failure raises
``ValueError`` with the reference's wording, and nothing is computed on the
host — the refinement itself is the CUDA path behind
``qa_local_head_refine`` / the batched ``qa_result.intervals``.
"""
from __future__ import annotations

import ctypes
import json
import os

import numpy as np

from . import _lib
from . import synth
from .postprocess import AlignItem

DIR = "local_head"
SCHEMA = "qwen-fa-ultra.local-head.v1"
ARCHITECTURE = "IdentityConditionedBoundaryHead"
CONTEXT_ROLES = ["timestamp slot", "current avg", "prev avg", "next avg"]
OFFSETS_MS = [float(o) for o in range(-60, 61, 10)]
FEATURE_DIM = 91
FRAME_COUNT = 41


def package_dir(model_dir: str) -> str:
    """``<model>/local_head``, where the reference looks (src/local_head.rs:103-106)."""
    return os.path.join(model_dir, DIR)


def _close(a: float, b: float, what: str) -> None:
    if abs(float(a) - b) > 1e-6:
        raise ValueError(f"{what} {a} != the accepted head's {b}")


def validate_config(cfg: dict) -> None:
    """HeadFile::validate (src/local_head.rs:661-715)."""
    if cfg.get("schema") != SCHEMA:
        raise ValueError(f"local head schema {cfg.get('schema')!r} != {SCHEMA!r}")
    if cfg.get("architecture") != ARCHITECTURE:
        raise ValueError(f"local head architecture {cfg.get('architecture')!r} != {ARCHITECTURE!r}")
    if list(cfg.get("context_roles", [])) != CONTEXT_ROLES:
        raise ValueError(f"local head context_roles {cfg.get('context_roles')!r} != {CONTEXT_ROLES!r}")
    offs = cfg.get("offsets_ms", [])
    if len(offs) != len(OFFSETS_MS) or any(abs(a - b) > 1e-6 for a, b in zip(offs, OFFSETS_MS)):
        raise ValueError("local head offsets_ms must be ±60 ms in 10 ms steps")
    _close(cfg["decoder_temperature"], 1.5, "decoder_temperature")
    _close(cfg["decoder_amplitude"], 1.0, "decoder_amplitude")
    _close(cfg["inference_prior_scale"], 2.0, "inference_prior_scale")
    f = cfg["feature_contract"]
    if f["center_source"] != "fixed":
        raise ValueError('feature center_source must be "fixed"')
    for key, want in (("context_ms", 200), ("feature_dim", FEATURE_DIM),
                      ("frame_count", FRAME_COUNT), ("frame_ms", 25), ("hop_ms", 10),
                      ("n_fft", 512), ("n_mels", 80), ("sample_rate", 16000),
                      ("spectral_distance_bands", 4)):
        if int(f[key]) != want:
            raise ValueError(f"feature {key} must be {want}")
    m = cfg["model_config"]
    for key, want in (("acoustic_dim", FEATURE_DIM), ("qwen_dim", 1024), ("model_dim", 128),
                      ("heads", 4)):
        if int(m[key]) != want:
            raise ValueError(f"model_config.{key} must be {want}")
    _close(m["prior_sigma_ms"], 35.0, "model_config.prior_sigma_ms")
    _close(m["activity_weight"], 0.25, "model_config.activity_weight")


def load_package(model_dir: str):
    """(tensors, mean, std) of ``<model>/local_head``, or None when the
    checkpoint ships none; ValueError when it ships one that does not validate."""
    d = package_dir(model_dir)
    if not os.path.isdir(d):
        return None
    with open(os.path.join(d, "config.json")) as fh:
        validate_config(json.load(fh))
    with open(os.path.join(d, "normalizer.json")) as fh:
        norm = json.load(fh)
    mean = np.asarray(norm["mean"], np.float32)
    std = np.asarray(norm["std"], np.float32)
    if len(mean) != FEATURE_DIM or len(std) != FEATURE_DIM:
        raise ValueError(f"normalizer must hold {FEATURE_DIM} mean/std values, got "
                         f"{len(mean)}/{len(std)}")
    if not (np.all(np.isfinite(mean)) and np.all(np.isfinite(std)) and np.all(std > 0)):
        raise ValueError("normalizer must be finite with positive std")
    tensors = synth.load_safetensors(os.path.join(d, "model.safetensors"))
    check_prior(tensors)
    return tensors, mean, std


def check_prior(tensors: dict) -> None:
    """The package's qwen_prior must be the canonical production prior
    (src/local_head.rs:139-148)."""
    if "qwen_prior" not in tensors:
        return  # reported as a missing tensor by the device load
    got = np.asarray(tensors["qwen_prior"][1], np.float32).reshape(-1)
    want = synth.local_head_prior()
    if got.shape != want.shape or np.any(np.abs(got - want) > 1e-5):
        raise ValueError("local_head qwen_prior is not the canonical production prior "
                         "(σ=35 ms ×2)")


def num_parameters(tensors: dict) -> int:
    """Weights::numel (src/local_head.rs:774-808)."""
    return int(sum(np.asarray(v[1]).size for v in tensors.values()))


class LocalHead:
    """Handle of the Local Head loaded on an Aligner's device context."""

    def __init__(self, aligner, n_params: int):
        self._al = aligner
        self._n_params = n_params

    def num_parameters(self) -> int:
        return self._n_params

    def describe(self) -> str:
        return f"{self._n_params} parameters"

    def refine_raw(self, samples, logits, hidden, want_features: bool = False) -> dict:
        """The device refinement of one clip: intervals [W][2] seconds, the
        repaired coarse centres and the offsets (ms) of its 2W endpoints, and
        optionally the [2W][41][91] feature windows."""
        s = np.ascontiguousarray(samples, np.float32)
        lg = np.ascontiguousarray(logits, np.float32)
        hd = np.ascontiguousarray(hidden, np.float32)
        if lg.ndim != 2 or hd.ndim != 2 or lg.shape[0] != hd.shape[0] or lg.shape[0] % 2:
            raise ValueError(f"timestamp logits {lg.shape} and hidden rows {hd.shape} must hold "
                             f"the same even number of slots")
        slots = lg.shape[0]
        W = slots // 2
        iv = np.zeros((W, 2), np.float64)
        fixed = np.zeros(slots, np.int64)
        off = np.zeros(slots, np.float32)
        feat = np.zeros((slots, FRAME_COUNT, FEATURE_DIM), np.float32) if want_features else None
        ctx = self._al._ctx
        self._al._check(_lib.lib().qa_local_head_refine(
            ctx, s.ctypes.data, len(s), W, lg.ctypes.data, lg.shape[1], hd.ctypes.data,
            hd.shape[1], iv.ctypes.data, fixed.ctypes.data, off.ctypes.data,
            feat.ctypes.data if feat is not None else None))
        return {"intervals": iv, "fixed_ms": fixed, "offsets_ms": off, "features": feat}

    def refine(self, samples, words, logits, n_labels: int, hidden, hidden_size: int) -> list:
        """LocalHead::refine (src/local_head.rs:179-307): AlignItems per word."""
        slots = len(words) * 2
        lg = np.asarray(logits, np.float32).reshape(-1)
        hd = np.asarray(hidden, np.float32).reshape(-1)
        if lg.size != slots * n_labels:
            raise ValueError(f"timestamp logits are {lg.size} values, expected {slots}x{n_labels}")
        if hd.size != slots * hidden_size:
            raise ValueError(f"hidden rows are {hd.size} values, expected {slots}x{hidden_size}")
        if not words:
            return []
        r = self.refine_raw(samples, lg.reshape(slots, n_labels), hd.reshape(slots, hidden_size))
        return [AlignItem(w, float(a), float(b)) for w, (a, b) in zip(words, r["intervals"])]


def load_into(aligner, tensors: dict, mean, std) -> LocalHead:
    """Upload a package (name -> (dtype, array), [91] mean / std) to the
    aligner's device context; returns the handle."""
    check_prior(tensors)
    tens, keep = _lib.make_tensors(tensors)
    m = np.ascontiguousarray(mean, np.float32)
    sd = np.ascontiguousarray(std, np.float32)
    if m.size != FEATURE_DIM or sd.size != FEATURE_DIM:
        raise ValueError(f"normalizer must hold {FEATURE_DIM} mean/std values, got "
                         f"{m.size}/{sd.size}")
    rc = _lib.lib().qa_local_head_load(aligner._ctx, ctypes.addressof(tens), len(tens),
                                       m.ctypes.data, sd.ctypes.data)
    del keep
    aligner._check(rc)
    return LocalHead(aligner, num_parameters(tensors))
