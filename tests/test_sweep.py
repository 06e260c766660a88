"""The clip-set driver (sweep.py) on CPU: token-budget packing, LPT shares
across ranks and the resumable journal, with a stand-in for the Aligner that
records what it is asked to align (the device path itself is covered by the
GPU tests through align_inputs_stream)."""
import json

import numpy as np
import pytest

from conftest import pkg


class _Input:
    def __init__(self, words, n_samples):
        self.words = words
        self.n_audio_tokens = max(1, n_samples // 1280)
        self.timestamp_positions = list(range(2 * len(words)))
        self._L = 3 + self.n_audio_tokens + 4 * len(words)

    def seq_len(self):
        return self._L


class FakeAligner:
    """build_input + align_inputs_stream with deterministic outputs; raises
    after `crash_after` passes to stand for a job that dies mid-sweep."""

    def __init__(self, crash_after=None):
        self.passes = []
        self.built = 0
        self.crash_after = crash_after
        self.cfg = pkg().synth.ModelConfig()

    def build_input(self, samples, text, language):
        return _Input(text.split(), len(samples))

    def build_inputs(self, clips):
        self.built += len(clips)
        return [self.build_input(*c) for c in clips]

    def align_inputs_stream(self, batches):
        post = pkg().postprocess
        for samples_list, inputs in batches:
            if self.crash_after is not None and len(self.passes) == self.crash_after:
                raise RuntimeError("worker died")
            self.passes.append([inp.seq_len() for inp in inputs])
            res = []
            for s, inp in zip(samples_list, inputs):
                raw = [int(len(s)) % 997 + 80 * k for k in range(len(inp.timestamp_positions))]
                res.append((np.array(raw, np.int64), post.decode_timestamps(inp.words, raw)))
            yield res


def _clips(n, seed=0):
    rng = np.random.default_rng(seed)
    out = []
    for k in range(n):
        sec = float(rng.uniform(0.5, 6.0))
        words = " ".join(f"w{k}x{j}" for j in range(int(rng.integers(1, 9))))
        out.append((np.zeros(int(sec * 16000), np.float32), words, "English"))
    return out


def test_pack_batches_respects_budget_and_covers():
    sw = pkg().sweep
    rng = np.random.default_rng(1)
    lens = [int(x) for x in rng.integers(50, 3000, 300)]
    for budget, cap in ((8192, 128), (4000, 16), (3000, 300)):
        b = sw.pack_batches(lens, budget, cap)
        assert sorted(i for x in b for i in x) == list(range(len(lens)))
        assert all(sum(lens[i] for i in x) <= budget and len(x) <= cap for x in b)
    assert sw.pack_batches([9000, 10, 20], 8192) == [[0], [2, 1]]  # an oversized clip alone
    with pytest.raises(ValueError):
        sw.pack_batches([1], 0)


def test_sweep_results_and_batches():
    sw = pkg().sweep
    clips = _clips(40)
    fa = FakeAligner()
    out = sw.sweep(fa, clips, token_budget=120, max_clips=8)
    assert sorted(out) == list(range(40))
    assert all(sum(p) <= 120 and len(p) <= 8 for p in fa.passes)
    assert sum(len(p) for p in fa.passes) == 40
    for k, (s, text, _) in enumerate(clips):
        raw, items = out[k]
        assert [i.text for i in items] == text.split()
        assert raw[0] == len(s) % 997


def test_journal_resume_after_a_crash(tmp_path):
    sw = pkg().sweep
    clips = _clips(30, seed=2)
    ids = [f"clip-{k:03d}" for k in range(30)]
    path = tmp_path / "sweep.jsonl"
    with pytest.raises(RuntimeError):
        sw.sweep(FakeAligner(crash_after=2), clips, ids=ids, journal=path, token_budget=100)
    done_first = len(path.read_text().splitlines())
    assert 0 < done_first < 30
    with open(path, "a") as f:
        f.write('{"id": "clip-9')  # a record cut short by the crash: redone
    fa = FakeAligner()
    out = sw.sweep(fa, clips, ids=ids, journal=path, token_budget=100)
    assert sum(len(p) for p in fa.passes) == 30 - done_first
    full = sw.sweep(FakeAligner(), clips, ids=ids, token_budget=100)
    assert sorted(out) == sorted(full) == sorted(ids)
    for cid in ids:
        assert out[cid][0] == full[cid][0]
        assert [(i.text, i.start_time, i.end_time) for i in out[cid][1]] == \
            [(i.text, i.start_time, i.end_time) for i in full[cid][1]]
    # a third run aligns nothing
    fa3 = FakeAligner()
    sw.sweep(fa3, clips, ids=ids, journal=path, token_budget=100)
    assert fa3.passes == []


def test_rank_shares_cover_once_and_balance():
    sw = pkg().sweep
    clips = _clips(64, seed=3)
    shares = [sw.sweep(FakeAligner(), clips, rank=r, world=4, token_budget=200) for r in range(4)]
    got = sorted(k for s in shares for k in s)
    assert got == list(range(64))
    S = pkg().synth
    costs = [sw.estimate_cost(len(c[0]), S.split_words(c[1], c[2])) for c in clips]
    loads = [sum(costs[k] for k in s) for s in shares]
    assert max(loads) <= sum(costs) / 4 + max(costs)
    # a rank tokenises its own share only
    fa = FakeAligner()
    sw.sweep(fa, clips, rank=1, world=4, token_budget=200)
    assert fa.built == len(shares[1])
    with pytest.raises(ValueError):
        sw.rank_share(costs, 4, 4)
    with pytest.raises(ValueError):
        sw.sweep(FakeAligner(), clips[:2], ids=["a", "a"])


def test_rank_journals_are_separate_and_shared_on_resume(tmp_path):
    """Each rank writes its own journal file; a rerun with another number of
    ranks skips every clip any rank finished."""
    sw = pkg().sweep
    clips = _clips(48, seed=4)
    path = tmp_path / "j.jsonl"
    for r in range(3):
        sw.sweep(FakeAligner(), clips, journal=path, rank=r, world=3, token_budget=150)
    files = sorted(p.name for p in tmp_path.iterdir())
    assert files == ["j.jsonl.rank0", "j.jsonl.rank1", "j.jsonl.rank2"]
    assert sum(len((tmp_path / f).read_text().splitlines()) for f in files) == 48
    for r in range(2):  # resumed on two ranks: nothing left to align
        fa = FakeAligner()
        out = sw.sweep(fa, clips, journal=path, rank=r, world=2, token_budget=150)
        assert fa.passes == [] and fa.built == 0 and len(out) > 0
    fa = FakeAligner()
    assert len(sw.sweep(fa, clips, journal=path, token_budget=150)) == 48
    assert fa.passes == []
