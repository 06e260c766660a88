"""Timestamp repair and word pairing — host glue kept on the CPU, as in the
reference (src/postprocess.rs).  Restated from src/postprocess.rs:33-149:

1. longest non-decreasing subsequence by O(n^2) DP, ties to the earliest index;
2. runs of non-LIS positions: length <= 2 snap to the nearer neighbour by index
   distance; longer runs interpolate linearly in f64, truncated toward zero;
3. (2i, 2i+1) pairs per word, milliseconds / 1000.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(slots=True)
class AlignItem:
    text: str
    start_time: float
    end_time: float


def fix_timestamps(data) -> list:
    n = len(data)
    if n == 0:
        return []
    data = [int(x) for x in data]
    dp = [1] * n
    parent = [-1] * n
    for i in range(1, n):
        for j in range(i):
            if data[j] <= data[i] and dp[j] + 1 > dp[i]:
                dp[i] = dp[j] + 1
                parent[i] = j
    max_len = max(dp)
    idx = dp.index(max_len)
    normal = [False] * n
    while idx != -1:
        normal[idx] = True
        idx = parent[idx]
    result = list(data)
    bs = 0
    while bs < n:
        if normal[bs]:
            bs += 1
            continue
        be = bs
        while be < n and not normal[be]:
            be += 1
        cnt = be - bs
        left = next((result[k] for k in range(bs - 1, -1, -1) if normal[k]), None)
        right = next((result[k] for k in range(be, n) if normal[k]), None)
        if left is not None or right is not None:
            if cnt <= 2:
                for p in range(bs, be):
                    if left is not None and right is not None:
                        result[p] = left if p - (bs - 1) <= be - p else right
                    else:
                        result[p] = left if left is not None else right
            elif left is not None and right is not None:
                step = (right - left) / (cnt + 1)
                for p in range(bs, be):
                    result[p] = int(left + step * (p - bs + 1))  # int() truncates toward zero
            else:
                fill = left if left is not None else right
                for p in range(bs, be):
                    result[p] = fill
        bs = be
    return result


def pair_words(words, fixed_ms) -> list:
    if len(fixed_ms) != 2 * len(words):
        raise ValueError(f"expected {2 * len(words)} timestamps for {len(words)} words, "
                         f"got {len(fixed_ms)}")
    import numpy as np
    sec = (np.asarray(fixed_ms, dtype=np.int64) / 1000.0).tolist()  # IEEE division, as in Python
    return [AlignItem(w, sec[2 * i], sec[2 * i + 1]) for i, w in enumerate(words)]


def decode_timestamps(words, raw_ms) -> list:
    return pair_words(words, fix_timestamps(raw_ms))
