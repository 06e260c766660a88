"""Clip sharding across GPUs: one process per GPU, no data-path collective.

Clips are independent (the reference restarts the K/V cache at position 0 for
every clip, src/cpu_decoder.rs:267-269), so N GPUs align N disjoint sets of
clips.  Two assignment rules:

* ``contiguous_shard`` — rank r takes a fixed-size slice of a clip stream
  (the benchmark's weak scaling: per-GPU work is constant as N grows);
* ``lpt_assign`` — longest-processing-time-first over estimated FLOPs, for a
  fixed set of clips of very different lengths.

The only cross-rank traffic is host-side bookkeeping: a barrier and scalar
max/sum reductions of timings (``RankGroup``), over NCCL on GPUs or gloo on CPU.
"""
from __future__ import annotations

import heapq
import os


def clip_flops(n_audio_tokens: int, seq_len: int, n_ts: int, n_chunks: int) -> float:
    """Algorithmic FLOPs of one clip (tower + decoder + head), the per-clip
    figure the roofline divides: conv stem per 100-frame chunk, 18 tower layers
    per audio token (+ windowed attention, bounded by 104-token windows),
    28 decoder layers per token plus exact causal attention, 1024x5000 head per
    timestamp row."""
    f_enc = 4.2080256e9 * n_chunks + n_audio_tokens * (13.76256e6 + 18 * 19.267584e6 + 3.44064e6)
    f_enc += 18 * 4 * 896 * 104 * n_audio_tokens  # upper bound of the window term
    f_dec = 880_803_840.0 * seq_len + 114_688.0 * seq_len * (seq_len + 1)
    f_head = 10_240_000.0 * n_ts
    return f_enc + f_dec + f_head


def contiguous_shard(rank: int, world: int, per_rank: int) -> range:
    """Clip indices of `rank` when every rank takes `per_rank` consecutive clips."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    return range(rank * per_rank, (rank + 1) * per_rank)


def lpt_assign(costs, n_workers: int) -> list:
    """Longest-processing-time-first: each clip, in descending cost order, goes
    to the currently least-loaded worker (ties to the lower worker index).
    Returns one index list per worker, each in the clips' original order."""
    if n_workers <= 0:
        raise ValueError("need at least one worker")
    heap = [(0.0, w) for w in range(n_workers)]
    out = [[] for _ in range(n_workers)]
    for i in sorted(range(len(costs)), key=lambda k: (-costs[k], k)):
        load, w = heapq.heappop(heap)
        out[w].append(i)
        heapq.heappush(heap, (load + costs[i], w))
    return [sorted(x) for x in out]


class RankGroup:
    """Host-side rank bookkeeping from the torchrun environment."""

    def __init__(self, backend: str = "nccl", timeout_s: int = 300):
        import datetime
        import torch.distributed as dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.backend = backend
        self._dist = dist
        if self.world > 1 and not dist.is_initialized():
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))

    def _device(self):
        import torch
        return torch.device("cuda", self.local) if self.backend == "nccl" else torch.device("cpu")

    def barrier(self) -> None:
        if self.world > 1:
            self._dist.barrier()

    def _reduce(self, x: float, op) -> float:
        if self.world == 1:
            return float(x)
        import torch
        t = torch.tensor([float(x)], dtype=torch.float64, device=self._device())
        self._dist.all_reduce(t, op=op)
        return float(t.item())

    def max(self, x: float) -> float:
        return self._reduce(x, self._dist.ReduceOp.MAX)

    def sum(self, x: float) -> float:
        return self._reduce(x, self._dist.ReduceOp.SUM)

    def close(self) -> None:
        if self.world > 1 and self._dist.is_initialized():
            self._dist.destroy_process_group()
