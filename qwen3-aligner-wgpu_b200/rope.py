"""RoPE tables, restated from src/mrope.rs:15-89 (host side, f64 -> f32).

The aligner uses plain RoPE: section [head_dim/2, 0, 0] in the blocked layout
puts every frequency on the one position axis (src/align_inference.rs:315-328),
so the device kernels only ever see this table; the multi-axis map is kept
for parity with the reference's helper and its tests.
"""
from __future__ import annotations

import numpy as np


def build_dim_map(section, half: int, interleaved: bool) -> list:
    """src/mrope.rs:15-47."""
    if interleaved:
        nd = len(section)
        m, used = [], [0] * nd
        while len(m) < half:
            before = len(m)
            for d in range(nd):
                if len(m) >= half:
                    break
                if used[d] < section[d]:
                    m.append(d)
                    used[d] += 1
            if len(m) == before:
                break
        return m
    m = []
    for d, sz in enumerate(section):
        for _ in range(sz):
            if len(m) >= half:
                break
            m.append(d)
    while len(m) < half:
        m.append(len(section) - 1)
    return m


def compute_mrope_cos_sin(pos, head_dim: int, rope_theta: float, section, interleaved: bool):
    """src/mrope.rs:55-83: (cos, sin), each [seq_len, head_dim] f32."""
    half = head_dim // 2
    inv = 1.0 / rope_theta ** (2.0 * np.arange(half, dtype=np.float64) / head_dim)
    dm = build_dim_map(section, half, interleaved)
    p = np.stack([np.asarray(pos[dm[j]], dtype=np.float64) for j in range(half)], 1)
    ang = p * inv[None, :]
    c = np.cos(ang).astype(np.float32)
    s = np.sin(ang).astype(np.float32)
    return np.concatenate([c, c], 1), np.concatenate([s, s], 1)


def rope_tables(positions: int, head_dim: int, theta: float = 1e6):
    """Plain RoPE for positions 0..n (text_positions + section [half, 0, 0])."""
    p = np.arange(positions, dtype=np.int64)
    return compute_mrope_cos_sin([p, p, p], head_dim, theta, [head_dim // 2, 0, 0], False)
