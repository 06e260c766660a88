"""Aligning a large set of clips: the whole-box sweep of BASELINE config 4
(4096 clips of 5-60 s), one process per GPU.

The reference aligns one clip per call.  Here a set of clips is

* split across ranks longest-processing-time first by each clip's estimated
  FLOPs (``shard.lpt_assign`` over ``shard.clip_flops``), so the GPUs finish
  together even though clip lengths vary twelve-fold;
* packed, on each rank, into device passes whose decoder tokens stay under a
  budget (the paged K/V cache holds 112 KiB per token, so 65,536 tokens are
  7.3 GB), longest clips first, first fit;
* streamed through ``Aligner.align_inputs_stream`` (two passes in flight, the
  host building the next batch while the GPU runs the current one);
* journaled: every finished clip is appended to a JSON-lines file as soon as
  its pass returns (one file per rank), and a rerun with the same journal
  skips the clips already there (resume after a crash or a preempted job).

Nothing here computes: the alignment is the library's, and a missing CUDA
library fails loudly where the Aligner is created.
"""
from __future__ import annotations

import json
import os

from . import postprocess
from . import shard

DEFAULT_TOKEN_BUDGET = 65536
DEFAULT_MAX_CLIPS = 128


def pack_batches(seq_lens, token_budget: int = DEFAULT_TOKEN_BUDGET,
                 max_clips: int = DEFAULT_MAX_CLIPS) -> list:
    """Clip indices grouped into passes: longest first, each clip into the
    first pass with room (tokens and clip count); a clip longer than the
    budget gets a pass of its own."""
    if token_budget <= 0 or max_clips <= 0:
        raise ValueError("token budget and clips per pass must be positive")
    order = sorted(range(len(seq_lens)), key=lambda i: (-seq_lens[i], i))
    batches, used = [], []
    for i in order:
        for b, u in enumerate(used):
            if u + seq_lens[i] <= token_budget and len(batches[b]) < max_clips:
                batches[b].append(i)
                used[b] += seq_lens[i]
                break
        else:
            batches.append([i])
            used.append(seq_lens[i])
    return batches


def clip_cost(inp, n_samples: int, n_window: int = 50) -> float:
    """Estimated FLOPs of one clip, the LPT weight."""
    frames = n_samples // 160
    chunks = -(-frames // (2 * n_window))
    return shard.clip_flops(inp.n_audio_tokens, inp.seq_len(), len(inp.timestamp_positions), chunks)


class Journal:
    """JSON lines, one finished clip per line: {"id", "raw_ms", "items"}.

    Each rank appends only to its own file: `path` for a single process,
    `path.rank<r>` for rank r of several, so no two processes ever write one
    file.  Every rank reads the finished clips of all of them (`path` and
    every `path.rank*`), so a rerun skips them whatever the number of ranks
    was before.  A record cut short by a crash (no final newline) is dropped
    and the clip is redone; the writer trims it from its own file."""

    def __init__(self, path, rank: int = 0, world: int = 1):
        import glob
        base = os.fspath(path)
        self.path = base if world <= 1 else f"{base}.rank{rank}"
        self.done = {}
        for p in sorted({base, self.path, *glob.glob(glob.escape(base) + ".rank*")}):
            if os.path.exists(p):
                self._read(p, trim=p == self.path)

    def _read(self, path: str, trim: bool) -> None:
        with open(path, "rb") as f:
            data = f.read()
        keep = data.rfind(b"\n") + 1
        if trim and keep < len(data):
            # new records must start on a line of their own
            with open(path, "r+b") as f:
                f.truncate(keep)
        for line in data[:keep].decode().splitlines():
            line = line.strip()
            if not line:
                continue
            try:
                rec = json.loads(line)
            except json.JSONDecodeError:
                continue
            self.done[rec["id"]] = (rec["raw_ms"], [postprocess.AlignItem(*x) for x in rec["items"]])

    def append(self, results) -> None:
        """results: [(id, raw_ms, items)], written and flushed together."""
        with open(self.path, "a") as f:
            for cid, raw, items in results:
                rec = {"id": cid, "raw_ms": [int(v) for v in raw],
                       "items": [[i.text, i.start_time, i.end_time] for i in items]}
                f.write(json.dumps(rec) + "\n")
                self.done[cid] = (rec["raw_ms"], list(items))
            f.flush()
            os.fsync(f.fileno())


def estimate_cost(samples_len: int, words: list, n_window: int = 50) -> float:
    """clip_cost from the sample count and the words alone, before any
    tokenisation: the audio tokens are exact; the text tokens are taken as
    one per three characters of each word (exact for the synthetic
    tokenizer, an estimate for a BPE)."""
    from . import synth
    valid = synth.valid_mel_frames(samples_len)
    na = synth.audio_token_count(valid, n_window)
    seq = na + 2 + 2 * len(words) + sum(-(-len(w) // 3) for w in words)
    chunks = -(-valid // (2 * n_window))
    return shard.clip_flops(na, seq, 2 * len(words), chunks)


def rank_share(costs, rank: int, world: int) -> list:
    """The clip indices rank `rank` of `world` aligns (LPT over the costs)."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    return shard.lpt_assign(costs, world)[rank]


def sweep(aligner, clips, ids=None, journal=None, token_budget: int = DEFAULT_TOKEN_BUDGET,
          max_clips: int = DEFAULT_MAX_CLIPS, rank: int = 0, world: int = 1) -> dict:
    """Align `clips` ([(samples, text, language)]) on this rank's share.

    ids: one JSON-serialisable id per clip (default: the index).  journal: a
    path; clips already in it (or in another rank's `path.rank*`) are
    skipped, this rank's new ones are appended to its own file.  The share
    is chosen from estimated costs (estimate_cost: word split only), and only
    this rank's clips are tokenised.  Returns {id: (raw_ms, items)} for this
    rank's share, journaled clips included."""
    from . import synth
    ids = list(range(len(clips))) if ids is None else list(ids)
    if len(ids) != len(clips) or len(set(ids)) != len(ids):
        raise ValueError("one distinct id per clip")
    j = Journal(journal, rank, world) if journal is not None else None
    mine = list(range(len(clips)))
    if world > 1:
        n_window = aligner.cfg.n_window
        costs = [estimate_cost(len(c[0]), synth.split_words(c[1], c[2]), n_window) for c in clips]
        mine = rank_share(costs, rank, world)
    out = {}
    todo = []
    for i in mine:
        if j is not None and ids[i] in j.done:
            out[ids[i]] = j.done[ids[i]]
        else:
            todo.append(i)
    built = aligner.build_inputs([clips[i] for i in todo]) if todo else []
    inputs = dict(zip(todo, built))
    batches = [[todo[k] for k in b] for b in
               pack_batches([inputs[i].seq_len() for i in todo], token_budget, max_clips)]
    stream = aligner.align_inputs_stream(([clips[i][0] for i in b], [inputs[i] for i in b])
                                         for b in batches)
    for b, res in zip(batches, stream):
        done = [(ids[i], [int(v) for v in raw], items) for i, (raw, items) in zip(b, res)]
        if j is not None:
            j.append(done)
        for cid, raw, items in done:
            out[cid] = (raw, items)
    return out
