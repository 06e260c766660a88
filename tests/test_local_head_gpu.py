"""Parity of the CUDA Local Head (qa_local_head_refine and the batched
qa_result.intervals) against the CPU oracle's restatement of
src/local_head.rs, on the seeded random-init head.

Bars, the reference's own tolerances for this stage (src/local_head.rs:1268,
1307, 1366): features within 2e-3 (plus 1e-5 relative, for the flux of a
frame after silence, about 1e6), offsets within 0.05 ms, refined intervals
within 0.5 ms; the repaired coarse centres (an integer stream) identical."""
import numpy as np
import pytest

from conftest import cuda_ok

pytestmark = pytest.mark.gpu

FEATURE_TOL = 2e-3
OFFSET_TOL_MS = 0.05
INTERVAL_TOL_MS = 0.5


@pytest.fixture(scope="module")
def env():
    if not cuda_ok():
        pytest.skip("no CUDA device")
    import pipeline_env as E
    return E


def _case(E, words, seconds, labels, seed):
    rng = np.random.default_rng(seed)
    samples = E.qa.synth.synth_audio(seconds, seed)
    logits = rng.standard_normal((2 * words, labels)).astype(np.float32)
    valid = min(int(np.floor(len(samples) * 1000.0 / 16000 / 80.0)) + 1, labels)
    for s in range(2 * words):  # an increasing path with some outliers
        logits[s, min(valid - 1, int((s + 1) * valid / (2 * words + 2)))] += 6.0
    if 2 * words > 6:
        logits[3, valid - 1] += 12.0  # an anomaly for fix_timestamps
    hidden = rng.standard_normal((2 * words, 1024)).astype(np.float32)
    return samples, logits, hidden


def _check_intervals(iv, seconds):
    assert np.all(np.isfinite(iv))
    assert np.all(iv[:, 0] >= 0) and np.all(iv[:, 1] <= seconds + 1e-9)
    assert np.all(iv[:, 1] > iv[:, 0])
    assert np.all(iv[1:, 0] >= iv[:-1, 1] - 1e-9)


@pytest.mark.parametrize("words,seconds,labels,seed", [
    (5, 3.0, 64, 1), (1, 0.7, 64, 2), (8, 2.0, 20, 3), (60, 20.0, 400, 4), (180, 60.0, 5000, 5)])
def test_refine_matches_oracle(env, words, seconds, labels, seed):
    E = env
    al = E.gpu_aligner_lh()
    head = al.local_head()
    samples, logits, hidden = _case(E, words, seconds, labels, seed)
    got = head.refine_raw(samples, logits, hidden, want_features=True)
    want_iv, want_fixed, want_off = E.cpu_local_head().refine(samples, logits, hidden)
    assert list(got["fixed_ms"]) == list(want_fixed)
    # features of every endpoint against the oracle's window at the same centre
    cpu = E.cpu_local_head()
    for e in range(0, 2 * words, max(1, (2 * words) // 12)):
        ref = cpu.features_one(samples, int(want_fixed[e]))
        excess = np.abs(got["features"][e] - ref) - (FEATURE_TOL + 1e-5 * np.abs(ref))
        assert excess.max() <= 0.0, (e, float(excess.max()))
    assert np.abs(got["offsets_ms"] - want_off).max() < OFFSET_TOL_MS
    assert np.abs(got["intervals"] - want_iv).max() * 1000.0 < INTERVAL_TOL_MS
    _check_intervals(got["intervals"], seconds)


def test_refine_items_and_timing(env):
    E = env
    al = E.gpu_aligner_lh()
    samples, logits, hidden = _case(E, 4, 2.0, 40, 9)
    words = ["aa", "bb", "cc", "dd"]
    items = al.local_head().refine(samples, words, logits, 40, hidden, 1024)
    assert [i.text for i in items] == words
    want_iv, _, _ = E.cpu_local_head().refine(samples, logits, hidden)
    for it, (a, b) in zip(items, want_iv):
        assert abs(it.start_time - a) * 1000 < INTERVAL_TOL_MS
        assert abs(it.end_time - b) * 1000 < INTERVAL_TOL_MS
    assert al.local_head().num_parameters() == 405264


def test_batch_intervals_match_oracle(env):
    """align_batch with the Local Head on: the device pass's intervals against
    the oracle's refine over the same pass's logits and unfolded rows."""
    E = env
    al = E.gpu_aligner_lh()
    assert al.local_head_enabled()
    rng = np.random.default_rng(7)
    clips = []
    for k, (sec, nw) in enumerate(((4.0, 9), (7.5, 20), (2.2, 5), (12.0, 33))):
        s = E.qa.synth.synth_audio(sec, 300 + k)
        clips.append((s, " ".join(E.qa.synth.english_words(nw, rng)), "English"))
    res = al.align_batch(clips, want_logits=True, want_normed=True)
    cpu = E.cpu_local_head()
    for (samples, text, _), (raw, items, extra) in zip(clips, res):
        iv = extra["intervals"]
        assert iv is not None and len(items) == len(iv)
        want_iv, _, _ = cpu.refine(samples, extra["logits"], extra["normed"])
        assert np.abs(iv - want_iv).max() * 1000.0 < INTERVAL_TOL_MS
        _check_intervals(iv, len(samples) / 16000.0)
        for it, (a, b) in zip(items, iv):
            assert (it.start_time, it.end_time) == (float(a), float(b))
    t = al.timings
    assert t["local_ms"] > 0.0


def test_batch_without_local_head_keeps_the_coarse_items(env):
    E = env
    al = E.gpu_aligner_lh()
    rng = np.random.default_rng(8)
    s = E.qa.synth.synth_audio(3.0, 77)
    clip = (s, " ".join(E.qa.synth.english_words(7, rng)), "English")
    al.set_local_head_enabled(False)
    try:
        (raw, items), = al.align_batch([clip])
        want = E.qa.postprocess.pair_words(al.build_input(*clip).words,
                                           E.qa._lib.fix_timestamps(raw))
        assert [(i.text, i.start_time, i.end_time) for i in items] == \
            [(i.text, i.start_time, i.end_time) for i in want]
        assert al.timings["local_ms"] == 0.0
    finally:
        al.set_local_head_enabled(True)


def test_local_head_state_and_shape_errors(env):
    E = env
    qa = E.qa
    plain = E.gpu_aligner()
    assert plain.local_head() is None and not plain.local_head_enabled()
    with pytest.raises(ValueError):
        plain.set_local_head_enabled(True)
    rc = qa._lib.lib().qa_set_local_head_enabled(plain._ctx, 1)
    assert rc == qa._lib.QA_ERR_STATE
    al = E.gpu_aligner_lh()
    samples, logits, hidden = _case(E, 3, 1.5, 30, 11)
    with pytest.raises(qa.QaError) as ei:  # the head's context width is 1024
        al.local_head().refine_raw(samples, logits, hidden[:, :512])
    assert ei.value.code == qa._lib.QA_ERR_SHAPE
    with pytest.raises(qa.QaError) as ei:  # empty audio
        al.local_head().refine_raw(np.zeros(0, np.float32), logits, hidden)
    assert ei.value.code == qa._lib.QA_ERR_SHAPE
    with pytest.raises(ValueError):  # odd slot count
        al.local_head().refine_raw(samples, logits[:5], hidden[:5])


def test_bad_package_is_refused(env):
    E = env
    qa = E.qa
    cfg, w = E.model()
    tensors, mean, std = E.lh_package()
    bad = dict(tensors)
    bad["audio.2.weight"] = ("F32", np.zeros((128, 128, 3), np.float32))
    with pytest.raises(qa.QaError) as ei:
        qa.Aligner.load_backend_with_dtype(w, "f16", cfg=cfg, local_head=(bad, mean, std))
    assert ei.value.code == qa._lib.QA_ERR_WEIGHTS
    prior = dict(tensors)
    prior["qwen_prior"] = ("F32", np.zeros(13, np.float32))
    with pytest.raises(ValueError):
        qa.Aligner.load_backend_with_dtype(w, "f16", cfg=cfg, local_head=(prior, mean, std))


def test_many_clips_properties(env):
    """A config-4-like batch (the 405k head on, 3 words/s): every interval is
    finite, ordered and inside its clip; a sample of clips matches the oracle."""
    E = env
    al = E.gpu_aligner_lh()
    rng = np.random.default_rng(12)
    clips = []
    for k in range(24):
        sec = float(rng.uniform(5.0, 20.0))
        s = E.qa.synth.synth_audio(sec, 500 + k)
        clips.append((s, " ".join(E.qa.synth.english_words(int(round(3 * sec)), rng)), "English"))
    res = al.align_batch(clips, want_logits=True, want_normed=True)
    cpu = E.cpu_local_head()
    for k, ((samples, _, _), (raw, items, extra)) in enumerate(zip(clips, res)):
        _check_intervals(extra["intervals"], len(samples) / 16000.0)
        if k % 8 == 0:
            want_iv, _, _ = cpu.refine(samples, extra["logits"], extra["normed"])
            assert np.abs(extra["intervals"] - want_iv).max() * 1000.0 < INTERVAL_TOL_MS
