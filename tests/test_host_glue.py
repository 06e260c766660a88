"""Host glue of the aligner (input building, tokenizer contract) on CPU."""
import numpy as np
import pytest

from conftest import pkg


def test_input_builder_matches_whole_string_tokenization():
    """InputBuilder emits the marker run directly; the ids must equal those of
    tokenizing the reference's whole assembled string (src/align_input.rs:197-213)."""
    synth = pkg().synth
    tok = synth.SyntheticTokenizer()
    b = synth.InputBuilder(tok)
    rng = np.random.default_rng(3)
    for i in range(12):
        words = synth.english_words(int(rng.integers(1, 20)), rng)
        if i % 2:
            words += synth.chinese_words(int(rng.integers(1, 9)), rng)
        valid = int(rng.integers(1, 4000))
        inp = b.build(words, valid)
        text = (synth.AUDIO_START + synth.AUDIO_PAD * inp.n_audio_tokens + synth.AUDIO_END
                + "".join((synth.TIMESTAMP * 2 if k else "") + w for k, w in enumerate(words))
                + synth.TIMESTAMP * 2)
        assert tok.encode(text) == inp.input_ids
        assert inp.n_audio_tokens == synth.audio_token_count(valid)
        assert len(inp.timestamp_positions) == 2 * len(words)
        assert inp.input_ids[0] == synth.AUDIO_START_ID
        assert inp.input_ids[inp.n_audio_tokens + 1] == synth.AUDIO_END_ID


def test_input_builder_rejects_zero_audio_tokens():
    synth = pkg().synth
    with pytest.raises(ValueError):
        synth.InputBuilder().build(["a"], 0)


def test_language_check_and_split():
    qa = pkg()
    langs = qa.Aligner.supported_languages(None)  # no instance state is read
    assert langs == sorted(langs) and len(langs) == 11 and "english" in langs
    with pytest.raises(ValueError):
        qa.synth.split_words("x", "ja")


def test_workload_shards_are_prefix_consistent():
    """Shard r of config 2 is clips [64r, 64r+64) of one stream."""
    synth = pkg().synth
    whole = synth.workload(2, n_clips=6)
    part = synth.workload(2, n_clips=3, start=3)
    for a, b in zip(whole[3:], part):
        assert a.text == b.text and np.array_equal(a.samples, b.samples)


def test_align_batch_host_phases_and_items(tmp_path):
    """align_batch's host side (word split, input build, repair + pairing, and
    the host phase timings of the reference's Timings) with the device pass
    replaced by a stand-in; align_with_raw adds wav_ms."""
    import struct
    import numpy as np
    qa = pkg()
    cfg = qa.synth.ModelConfig()
    al = qa.Aligner(None, cfg, "f16", qa.synth.InputBuilder(None, n_window=cfg.n_window))

    def fake_align_inputs(samples_list, inputs, want_logits=False, want_normed=False):
        al.timings = {"mel_ms": 0.5, "enc_ms": 1.0}
        return [(np.array([80 * (len(inp.timestamp_positions) - k) for k in
                           range(len(inp.timestamp_positions))], np.int64), {})
                for inp in inputs]

    al.align_inputs = fake_align_inputs
    clips = [(np.zeros(32000, np.float32), "alpha beta gamma", "English"),
             (np.zeros(16000, np.float32), "delta", None)]
    res = al.align_batch(clips)
    assert [[i.text for i in items] for _, items in res] == [["alpha", "beta", "gamma"], ["delta"]]
    for raw, items in res:
        assert all(a.end_time <= b.start_time for a, b in zip(items, items[1:]))
    t = al.timings
    assert t["mel_ms"] == 0.5 and all(t[k] >= 0.0 for k in ("words_ms", "build_ms", "post_ms"))
    with pytest.raises(ValueError):
        al.align_batch([(np.zeros(1600, np.float32), "x", "Klingon")])
    pcm = np.zeros(8000, "<i2").tobytes()
    fmt = struct.pack("<HHIIHH", 1, 1, 16000, 32000, 2, 16)
    body = b"WAVE" + b"fmt " + struct.pack("<I", 16) + fmt + b"data" + struct.pack("<I", len(pcm)) + pcm
    p = tmp_path / "z.wav"
    p.write_bytes(b"RIFF" + struct.pack("<I", len(body)) + body)
    raw, items = al.align_with_raw(p, "one two", "English")
    assert [i.text for i in items] == ["one", "two"] and al.timings["wav_ms"] >= 0.0
