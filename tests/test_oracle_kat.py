"""The CPU oracle and the host-side glue against the reference's own
known-answer tests (tests/golden/kat.json, extracted from the reference's
test modules by tests/golden/make_kat.py), plus independent pins of the
oracle's building blocks (f16/bf16 rounding, GEMM, FFT)."""
import json
import os

import numpy as np
import pytest

from conftest import pkg

HERE = os.path.dirname(os.path.abspath(__file__))
KAT = json.load(open(os.path.join(HERE, "golden", "kat.json"), encoding="utf-8"))


@pytest.fixture(scope="module")
def orc():
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))
    import oracle
    oracle.build()
    return oracle


def test_bookkeeping_kats(orc):
    synth = pkg().synth
    for n, want in KAT["conv3_length"]:
        assert orc.lib().or_conv3_length(n) == want
        assert synth.conv3_length(n) == want
    assert len(KAT["audio_token_count_samples"]) == 9
    for samples, want in KAT["audio_token_count_samples"]:
        v = orc.lib().or_valid_mel_frames(samples)
        assert v == synth.valid_mel_frames(samples)
        assert orc.lib().or_audio_token_count(v, 50) == want
        assert synth.audio_token_count(v, 50) == want
    for valid, nw, want in KAT["padded_mel_frames"]:
        assert orc.lib().or_padded_mel_frames(valid, nw) == want
        assert synth.padded_mel_frames(valid, nw) == want
    assert synth.audio_token_count(0, 50) == 0


def test_fix_timestamps_kats(orc):
    post = pkg().postprocess
    assert len(KAT["fix_timestamps"]) == 9
    for case in KAT["fix_timestamps"]:
        for impl in (orc.fix_timestamps, post.fix_timestamps):
            got = impl(case["data"])
            if "want" in case:
                assert got == case["want"], (case, got)
            else:
                assert all(a <= b for a, b in zip(got, got[1:]))
    assert orc.fix_timestamps([]) == [] and post.fix_timestamps([]) == []


def test_library_fix_timestamps_kats():
    """The compiled repair in libqa_b200.so (the Aligner's host path) against
    the reference's own cases and the Python restatement on random streams."""
    import random
    lib = pkg()._lib
    post = pkg().postprocess
    for case in KAT["fix_timestamps"]:
        got = lib.fix_timestamps(case["data"])
        if "want" in case:
            assert got == case["want"], (case, got)
        else:
            assert all(a <= b for a, b in zip(got, got[1:]))
    rnd = random.Random(3)
    for _ in range(300):
        n = rnd.randint(0, 40)
        data = [rnd.choice([rnd.randint(0, 30) * 80, rnd.randint(0, 4000)]) for _ in range(n)]
        assert lib.fix_timestamps(data) == post.fix_timestamps(data)


def test_library_fix_timestamps_long_streams(orc):
    """The library's O(n log n) chain search against the oracle's O(n^2) scan
    of the reference (src/postprocess.rs:39-48) on long streams: many equal
    values (the tie rules pick the parent), runs that fall, constant and
    reversed streams, and the 1,800 slots of a 300 s clip."""
    lib = pkg()._lib
    rng = np.random.default_rng(11)
    cases = [list(range(2000, 0, -1)), [480] * 1500, [0, 80] * 700]
    for n in (1, 2, 3, 17, 300, 1800, 4000):
        cases.append((rng.integers(0, 12, n) * 80).tolist())        # heavy ties
        cases.append(rng.integers(0, 400000, n).tolist())            # distinct-ish
        ramp = np.sort(rng.integers(0, 5000, n)) * 80
        flips = rng.random(n) < 0.1
        ramp[flips] = rng.integers(0, 5000, int(flips.sum())) * 80  # anomalies
        cases.append(ramp.tolist())
    for data in cases:
        got = lib.fix_timestamps(data)
        assert got == orc.fix_timestamps(data), len(data)
        assert all(a <= b for a, b in zip(got, got[1:]))


def test_pairing_kat():
    post = pkg().postprocess
    k = KAT["pair_words"]
    items = post.decode_timestamps(k["words"], k["raw"])
    assert [(i.text, i.start_time, i.end_time) for i in items] == [tuple(w) for w in k["want"]]
    with pytest.raises(ValueError):
        post.decode_timestamps(["a"], [0, 1, 2])


def test_mel_helper_kats(orc):
    for case in KAT["reflection_pad"]:
        got = orc.reflection_pad(case["signal"], case["pad"])
        assert got.tolist() == case["want"]
    assert len(orc.reflection_pad([], 3)) == 0
    w = orc.hann_window(4)
    assert abs(w[0] - KAT["hann4"]["w0"]) < 1e-6 and abs(w[2] - KAT["hann4"]["w2"]) < 1e-6
    fb = orc.mel_filterbank()
    assert fb.shape == (128, 201) and (fb >= 0).all()
    silent = orc.mel(np.zeros(16000, np.float32))
    assert silent.shape == (128, 100) and np.isfinite(silent).all()


def test_split_words_kats():
    synth = pkg().synth
    assert len(KAT["split_words"]) >= 15
    for case in KAT["split_words"]:
        assert synth.split_words(case["text"], case["language"]) == case["want"], case


def test_half_carriers(orc):
    import torch
    for x, bits in KAT["bf16_bits"]:
        assert orc.f32_to_bf16_bits(x) == bits
    # f16: every f32 whose top bits sweep the f16 range, vs numpy's RNE cast
    rng = np.random.default_rng(0)
    u = np.concatenate([rng.integers(0x30000000, 0x48000000, 20000, dtype=np.uint32),
                        np.arange(0x33000000, 0x33000000 + 4096, dtype=np.uint32) * 1,
                        np.array([0x38800000, 0x387FFFFF, 0x477FEFFF, 0x477FF000, 0x477FF001],
                                 dtype=np.uint32)])
    x = u.view(np.float32)
    want = x.astype(np.float16).view(np.uint16)
    got = np.array([orc.f32_to_f16_bits(float(v)) for v in x], dtype=np.uint16)
    assert (got == want).all()
    # bf16: the halfway sweep of src/shaders.rs (low 16 bits at and around 0x8000)
    tops = [0, 1, 2, 0x3F, 0x40, 0x7E, 0x7F]
    lows = [0, 1, 0x7FFE, 0x7FFF, 0x8000, 0x8001, 0xFFFE, 0xFFFF]
    vals = np.array([(0x3F80 + t) << 16 | lo for t in tops for lo in lows], dtype=np.uint32)
    xs = vals.view(np.float32)
    want = torch.from_numpy(xs.copy()).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    got = np.array([orc.f32_to_bf16_bits(float(v)) for v in xs], dtype=np.uint16)
    assert (got == want).all()


def test_dim_map_kats():
    post = pkg().synth  # noqa: F841  (the map lives with the rope tables below)
    from importlib import import_module
    rope = import_module("qwen3-aligner-wgpu_b200.rope")
    for case in KAT["dim_map"]:
        m = rope.build_dim_map(case["section"], case["half"], case["interleaved"])
        if "want" in case:
            assert m == case["want"]
        else:
            assert m[:6] == case["prefix"]
            assert [m.count(d) for d in range(3)] == case["counts"]


def test_rope_tables(orc):
    from importlib import import_module
    rope = import_module("qwen3-aligner-wgpu_b200.rope")
    c, s = orc.rope_tables(64, 128)
    c2, s2 = rope.rope_tables(64, 128)
    assert np.array_equal(c, c2) and np.array_equal(s, s2)
    assert np.array_equal(c[:, :64], c[:, 64:])  # halves duplicate (src/mrope.rs:110-116)


@pytest.mark.parametrize("m,n,k", [(3, 5, 4), (8, 8, 8), (4, 64, 32), (210, 1280, 1024),
                                   (64, 3072, 1024), (64, 1024, 3072)])
def test_oracle_gemm_matches_naive(orc, m, n, k):
    """src/cpu_decoder.rs:620-646: the GEMM at toy and production shapes, |Δ| < 1e-3."""
    x = np.array([((i * 13 % 61) * 0.03 - 0.9) for i in range(m * k)], np.float32).reshape(m, k)
    w = np.array([((i * 7 % 53) * 0.02 - 0.5) for i in range(n * k)], np.float32).reshape(n, k)
    got = orc.gemm(x, w)
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    assert np.abs(got - ref).max() < 1e-3


def test_oracle_mel_matches_float64_numpy(orc):
    """The oracle's f32 mixed-radix FFT mel vs an independent float64 numpy mel
    built from the same published steps (parity of the FFT is unpinned against
    rustfft; this bounds the restatement's own error)."""
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(16000 * 3 + 77) * 0.1).astype(np.float32)
    got = orc.mel(x)
    xp = np.pad(x.astype(np.float64), 200, mode="reflect")
    n = len(x) // 160
    win = orc.hann_window(400).astype(np.float64)
    frames = np.stack([xp[i * 160:i * 160 + 400] * win for i in range(n)])
    pw = np.abs(np.fft.rfft(frames, axis=1)) ** 2
    mel = orc.mel_filterbank().astype(np.float64) @ pw.T
    lg = np.log10(np.maximum(mel, 1e-10))
    ref = (np.maximum(lg, lg.max() - 8.0) + 4.0) / 4.0
    assert got.shape == ref.shape
    assert np.abs(got - ref).max() < 2e-5
