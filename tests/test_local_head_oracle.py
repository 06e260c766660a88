"""The CPU restatement of the Local Head refinement stage (src/local_head.rs)
against the reference's own unit tests (tests/golden/kat.json) and against an
independent numpy (features) / PyTorch fp32 (boundary network) restatement of
the same algorithm.

The reference's model-level gold for this stage (tools/gold/local_head/, a
frozen run of the Python trainer) is not in its tree, so features, offsets
and refined intervals are pinned here by the primitive KATs plus the
independent restatement, at the reference's own tolerances: features within
2e-3, offsets within 0.05 ms, intervals within 0.5 ms
(src/local_head.rs:1268,1307,1366)."""
import json
import math
import os

import numpy as np
import pytest

from conftest import pkg

HERE = os.path.dirname(os.path.abspath(__file__))
KAT = json.load(open(os.path.join(HERE, "golden", "kat.json"), encoding="utf-8"))

FEATURE_TOL = 2e-3
OFFSET_TOL_MS = 0.05
INTERVAL_TOL_MS = 0.5


@pytest.fixture(scope="module")
def orc():
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))
    import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="module")
def package():
    return pkg().synth.random_local_head(seed=0)


@pytest.fixture(scope="module")
def head(orc, package):
    tensors, mean, std = package
    return orc.LocalHead(tensors, mean, std)


# ---------------------------------------------------------------- KATs

def test_hann_kat(orc):
    k = KAT["lh_hann"]
    w = orc.lh_hann(k["n"])
    for i, want in zip(k["index"], k["want"]):
        assert abs(float(w[i]) - want) < k["tol"], (i, w[i], want)
    assert w[0] == 0.0 and w[-1] == 0.0
    assert np.all((w >= 0) & (w <= 1))
    a, b = k["symmetric"]
    assert abs(float(w[a]) - float(w[b])) < k["tol"]


def test_mel_bank_kat(orc):
    k = KAT["lh_mel_bank"]
    bank = orc.lh_mel_bank()
    assert bank.shape == (k["rows"], k["bins"])
    assert np.all(np.abs(bank.sum(1, dtype=np.float32) - 1.0) < k["row_sum_tol"])
    assert np.all(bank >= 0)


def test_band_edges_kat(orc):
    k = KAT["lh_band_edges"]
    assert orc.lh_band_edges(k["bins"]) == k["want"]


def test_valid_class_count_kat(orc):
    assert len(KAT["lh_valid_class_count"]) == 3
    for dur, classes, want in KAT["lh_valid_class_count"]:
        assert orc.lh_valid_class_count(dur, classes) == want


def test_overlap_repair_kat(orc):
    assert len(KAT["lh_remove_overlaps"]) == 2
    for case in KAT["lh_remove_overlaps"]:
        assert orc.lh_remove_overlaps(case["intervals"]) == case["want"]


def test_duration_bound_kat(orc):
    exact, pulled = KAT["lh_bound_to_duration"]
    assert orc.lh_bound_to_duration(exact["intervals"], exact["duration_ms"]) == exact["want"]
    v = orc.lh_bound_to_duration(pulled["intervals"], pulled["duration_ms"])
    tol = pulled["tol"]
    assert abs(v[1][1] - pulled["last_end"]) < tol
    assert v[0][1] <= v[1][0] + tol
    assert v[0][1] - v[0][0] >= pulled["min_len"] - tol


def test_duration_bound_non_finite_and_empty(orc):
    assert orc.lh_bound_to_duration(np.zeros((0, 2)), 100.0) == []
    v = orc.lh_bound_to_duration([[float("nan"), 5.0], [20.0, float("inf")]], 100.0)
    assert v[0][0] >= 0 and v[-1][1] <= 100.0
    assert all(b - a >= 10.0 - 1e-9 for a, b in v)


def test_package_validation(orc, package):
    tensors, mean, std = package
    bad = dict(tensors)
    bad["audio.0.weight"] = ("F32", np.zeros((128, 90, 5), np.float32))
    with pytest.raises(ValueError):
        orc.LocalHead(bad, mean, std)
    missing = {k: v for k, v in tensors.items() if k != "derivative_scale"}
    with pytest.raises(ValueError):
        orc.LocalHead(missing, mean, std)


# ---------------------------------------------------------------- independent restatement

def np_hann(n):
    i = np.arange(n, dtype=np.float64)
    return (0.5 - 0.5 * np.cos(2 * np.pi * i / (n - 1))).astype(np.float32)


def np_mel_bank():
    hz_to_mel = lambda hz: 2595.0 * np.log10(1.0 + hz / 700.0)
    mel_to_hz = lambda m: 700.0 * (10.0 ** (m / 2595.0) - 1.0)
    pts = mel_to_hz(np.linspace(hz_to_mel(0.0), hz_to_mel(8000.0), 82))
    edges = np.maximum(np.floor(513 * pts / 16000).astype(np.int64), 0)
    bank = np.zeros((80, 257), np.float32)
    for m in range(80):
        l, c = edges[m], max(edges[m + 1], edges[m] + 1)
        r = min(max(edges[m + 2], c + 1), 256)
        if c >= 257:
            continue
        if c > l:
            bank[m, l:c] = np.arange(c - l, dtype=np.float32) / np.float32(c - l)
        if r > c:
            bank[m, c:r] = 1 - np.arange(r - c, dtype=np.float32) / np.float32(r - c)
        t = bank[m].sum(dtype=np.float32)
        if t > 0:
            bank[m] /= t
    return bank


def np_features(samples, center_ms, mean, std):
    """[41][91]: the feature window of the Python trainer (numpy rfft, f64)."""
    center = center_ms * 16000 // 1000
    win = np_hann(400)
    frames = np.zeros((41, 400), np.float32)
    for f in range(41):
        start = center + (f - 20) * 160 - 200
        idx = np.arange(start, start + 400)
        ok = (idx >= 0) & (idx < len(samples))
        frames[f, ok] = samples[idx[ok]] * win[ok]
    mag = np.abs(np.fft.rfft(frames.astype(np.float64), n=512, axis=1)).astype(np.float32)
    power = mag * mag
    log_mel = np.log(np.maximum(power @ np_mel_bank().T, 1e-6))
    log_rms = np.log(np.maximum(np.sqrt((frames * frames).sum(1) / 400 + 1e-6), 1e-6))
    delta = np.concatenate([[0.0], np.diff(log_rms)]).astype(np.float32)
    nrm = np.log(np.maximum(mag, 1e-6))
    nrm = nrm - nrm.mean(1, keepdims=True)
    flux = np.zeros(41, np.float32)
    flux[1:] = np.maximum(mag[1:] - mag[:-1], 0).sum(1) / (mag[:-1].sum(1) + 1e-6)
    edges = [1, 65, 129, 193, 257]
    dist = np.zeros((41, 8), np.float32)
    for b in range(4):
        seg = nrm[:, edges[b]:edges[b + 1]]
        left = np.concatenate([seg[:1], seg[:-1]])
        right = np.concatenate([seg[1:], seg[-1:]])
        dist[:, b] = np.abs(seg - left).mean(1)
        dist[:, 4 + b] = np.abs(seg - right).mean(1)
    feat = np.concatenate([log_mel, log_rms[:, None], delta[:, None], flux[:, None], dist], 1)
    return ((feat - mean) / std).astype(np.float32)


class TorchHead:
    """IdentityConditionedBoundaryHead in PyTorch fp32 modules, loaded from
    the package's tensors (nn.Conv1d, nn.MultiheadAttention, nn.LayerNorm)."""

    def __init__(self, tensors):
        import torch
        import torch.nn as nn
        self.torch = torch
        t = {k: torch.from_numpy(np.array(v[1], np.float32)) for k, v in tensors.items()}
        self.conv1 = nn.Conv1d(91, 128, 5, padding=2)
        self.conv2 = nn.Conv1d(128, 128, 5, padding=2)
        self.ctx = nn.Linear(1024, 128)
        self.catt = nn.MultiheadAttention(128, 4, batch_first=True)
        self.aatt = nn.MultiheadAttention(128, 4, batch_first=True)
        self.qn = nn.LayerNorm(128)
        self.an = nn.LayerNorm(128)
        with torch.no_grad():
            for mod, pre in ((self.conv1, "audio.0"), (self.conv2, "audio.2"),
                             (self.ctx, "context_projection"), (self.qn, "query_norm"),
                             (self.an, "audio_norm")):
                mod.weight.copy_(t[pre + ".weight"])
                mod.bias.copy_(t[pre + ".bias"])
            for mod, pre in ((self.catt, "context_attention"), (self.aatt, "audio_attention")):
                mod.in_proj_weight.copy_(t[pre + ".in_proj_weight"])
                mod.in_proj_bias.copy_(t[pre + ".in_proj_bias"])
                mod.out_proj.weight.copy_(t[pre + ".out_proj.weight"])
                mod.out_proj.bias.copy_(t[pre + ".out_proj.bias"])
        self.t = t

    def offset(self, feat, ctx, mask, is_end):
        torch, t = self.torch, self.t
        F = torch.nn.functional
        with torch.no_grad():
            x = torch.from_numpy(np.ascontiguousarray(feat.T))[None]
            a = F.gelu(self.conv2(F.gelu(self.conv1(x))))[0].T[None]  # [1, 41, 128]
            tok = self.ctx(torch.from_numpy(ctx)[None]) + t["role_embedding.weight"][None]
            base = tok[:, :1] + t["endpoint_embedding.weight"][is_end]
            pad = torch.from_numpy(np.asarray(mask) == 0)[None]
            o, _ = self.catt(base, tok, tok, key_padding_mask=pad, need_weights=False)
            q = self.qn(o + base)
            o, _ = self.aatt(q, a, a, need_weights=False)
            q = self.qn(o + q)[0, 0]
            an = self.an(a[0])
            root = math.sqrt(128.0)
            act = an @ q / root + an @ t["activity_bias.weight"][0] + t["activity_bias.bias"][0]
            seg = an[14:27]
            local = seg @ q / root + seg @ t["boundary_bias.weight"][0] + t["boundary_bias.bias"][0]
            der = act[14:27] - act[13:26]
            direction = der if is_end == 0 else -der
            logits = local + t["derivative_scale"] * direction + t["qwen_prior"]
            p = torch.softmax(logits / 1.5, 0)
            return float((p * torch.arange(-60.0, 61.0, 10.0)).sum())


def speechlike(seconds, seed):
    return pkg().synth.synth_audio(seconds, seed)


def test_features_match_numpy(orc, head, package):
    _, mean, std = package
    s = speechlike(3.0, 11)
    worst = 0.0
    # centres inside, at the start (left zero padding) and past the end
    for c in (0, 35, 1000, 1480, 2960, 3100):
        got = head.features_one(s, c)
        want = np_features(s, c, mean, std)
        # the flux of a frame after an all-zero frame is sum / 1e-6 (about
        # 1e6): there the summation order moves the f32 value by a few ulp,
        # so the bound is absolute plus 1e-5 relative (allclose semantics)
        excess = np.abs(got - want) - (FEATURE_TOL + 1e-5 * np.abs(want))
        worst = max(worst, float(excess.max()))
    assert worst <= 0.0, worst


def test_features_of_silence(orc, head, package):
    _, mean, std = package
    got = head.features_one(np.zeros(16000, np.float32), 500)
    want = np_features(np.zeros(16000, np.float32), 500, mean, std)
    assert np.abs(got - want).max() < FEATURE_TOL


def test_endpoint_offset_matches_torch(orc, head, package):
    tensors, mean, std = package
    th = TorchHead(tensors)
    rng = np.random.default_rng(3)
    s = speechlike(2.0, 5)
    worst = 0.0
    for k, (c, mask, e) in enumerate(((400, [1, 1, 0, 1], 0), (800, [1, 1, 1, 1], 1),
                                      (1200, [1, 1, 1, 0], 0), (30, [1, 1, 0, 0], 1))):
        feat = head.features_one(s, c)
        ctx = rng.standard_normal((4, 1024)).astype(np.float32)
        got = head.endpoint_offset(feat, ctx, np.array(mask, np.float32), e)
        want = th.offset(feat, ctx, mask, e)
        assert -60.0 <= got <= 60.0
        worst = max(worst, abs(got - want))
    assert worst < OFFSET_TOL_MS, worst


def np_refine(head, th, samples, logits, hidden, orc):
    """Steps 1-5 of LocalHead::refine over the numpy / torch restatement."""
    slots, n_labels = logits.shape
    W = slots // 2
    dur = len(samples) * 1000.0 / 16000
    valid = orc.lh_valid_class_count(dur, n_labels)
    raw = [int(np.argmax(logits[s, :valid]) * 80.0) for s in range(slots)]
    fixed = orc.fix_timestamps(raw)
    offsets = []
    for w in range(W):
        cur = hidden[2 * w:2 * w + 2].mean(0)
        prev = hidden[2 * w - 2:2 * w].mean(0) if w > 0 else np.zeros(1024, np.float32)
        nxt = hidden[2 * w + 2:2 * w + 4].mean(0) if w + 1 < W else np.zeros(1024, np.float32)
        mask = [1, 1, 1 if w > 0 else 0, 1 if w + 1 < W else 0]
        for e in range(2):
            ctx = np.stack([hidden[2 * w + e], cur, prev, nxt]).astype(np.float32)
            feat = head.features_one(samples, fixed[2 * w + e])
            offsets.append(th.offset(feat, ctx, mask, e))
    iv = []
    for i in range(W):
        s, e = fixed[2 * i] + offsets[2 * i], fixed[2 * i + 1] + offsets[2 * i + 1]
        if e - s < 10.0:
            mid = (s + e) / 2
            s, e = (0.0, 10.0) if mid < 5.0 else (mid - 5.0, mid + 5.0)
        elif s < 0:
            e, s = e - s, 0.0
        if s < 0 or e < 0 or e - s < 10.0:
            s, e = 0.0, 10.0
        iv.append([s, e])
    iv = orc.lh_remove_overlaps(iv)
    iv = orc.lh_bound_to_duration(iv, dur)
    return np.array(iv) / 1000.0, np.array(fixed), np.array(offsets)


@pytest.mark.parametrize("words,seconds,labels", [(5, 3.0, 64), (1, 0.7, 64), (8, 2.0, 20)])
def test_refine_matches_restatement(orc, head, package, words, seconds, labels):
    tensors, _, _ = package
    th = TorchHead(tensors)
    rng = np.random.default_rng(words)
    samples = speechlike(seconds, words)
    # coarse logits that favour an increasing, slightly jittered path
    logits = rng.standard_normal((2 * words, labels)).astype(np.float32)
    valid = orc.lh_valid_class_count(len(samples) * 1000.0 / 16000, labels)
    for s in range(2 * words):
        logits[s, min(valid - 1, int((s + 1) * valid / (2 * words + 2)))] += 6.0
    hidden = rng.standard_normal((2 * words, 1024)).astype(np.float32)
    got, fixed, off = head.refine(samples, logits, hidden)
    want, wfixed, woff = np_refine(head, th, samples, logits, hidden, orc)
    assert list(fixed) == list(wfixed)
    assert np.abs(off - woff).max() < OFFSET_TOL_MS
    assert np.abs(got - want).max() * 1000.0 < INTERVAL_TOL_MS
    dur = len(samples) / 16000.0
    assert np.all(got[:, 0] >= 0) and np.all(got[:, 1] <= dur + 1e-12)
    assert np.all(got[:, 1] > got[:, 0])
    assert np.all(got[1:, 0] >= got[:-1, 1] - 1e-12)
