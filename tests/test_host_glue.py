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
