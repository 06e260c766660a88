"""Shared, lazily built test environment: the seeded random-init model, the
CPU oracle over it, and GPU aligners (f16 / bf16) over the same weights."""
import functools
import importlib
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle  # noqa: E402

qa = importlib.import_module("qwen3-aligner-wgpu_b200")


@functools.lru_cache(maxsize=None)
def model(seed: int = 0):
    cfg = qa.synth.ModelConfig()
    return cfg, qa.synth.random_weights(cfg, seed)


@functools.lru_cache(maxsize=None)
def cpu_model(seed: int = 0):
    cfg, w = model(seed)
    oracle.build()
    return oracle.Model(w, cfg)


@functools.lru_cache(maxsize=None)
def gpu_aligner(half: str = "f16", seed: int = 0):
    cfg, w = model(seed)
    return qa.Aligner.load_backend_with_dtype(w, half, cfg=cfg)


def rel_err(got, ref) -> float:
    """max |got - ref| / max |ref| — the north star's max-abs relative error."""
    import numpy as np
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def bits_to_f32(bits, half: str):
    import numpy as np
    b = np.ascontiguousarray(bits, np.uint16)
    if half == "bf16":
        return (b.astype(np.uint32) << 16).view(np.float32)
    return b.view(np.float16).astype(np.float32)


@functools.lru_cache(maxsize=None)
def lh_package(seed: int = 0):
    """(tensors, mean, std) of the seeded random-init Local Head."""
    return qa.synth.random_local_head(seed)


@functools.lru_cache(maxsize=None)
def cpu_local_head(seed: int = 0):
    oracle.build()
    return oracle.LocalHead(*lh_package(seed))


@functools.lru_cache(maxsize=None)
def gpu_aligner_lh(half: str = "f16", seed: int = 0):
    """An aligner over the seeded model with the seeded Local Head loaded."""
    cfg, w = model(seed)
    return qa.Aligner.load_backend_with_dtype(w, half, cfg=cfg, local_head=lh_package(seed))
