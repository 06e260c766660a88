"""The input builder on a real tokenizer.json through the `tokenizers`
binding (0.22.2, the version of the crate the reference links), CPU.

The reference loads tokenizer.json + tokenizer_config.json from the model
directory (src/align_input.rs:131-171) and tokenises one assembled string per
clip with no special tokens added (:180-186).  No checkpoint tokenizer exists
here, so synth.write_tokenizer_dir writes a real tokenizer.json whose markers
carry the checkpoint's ids (151669, 151670, 151676, 151705) and whose
ordinary pieces are SyntheticTokenizer's; these tests check that the two
tokenizers give the same ids, that batch building equals one-clip building,
and that Aligner picks the model directory's tokenizer as the reference does.
"""
import numpy as np
import pytest

from conftest import pkg

tokenizers = pytest.importorskip("tokenizers")


@pytest.fixture(scope="module")
def tokdir(tmp_path_factory):
    d = tmp_path_factory.mktemp("tok")
    pkg().synth.write_tokenizer_dir(str(d))
    return str(d)


def test_tokenizer_json_markers_and_ids(tokdir):
    S = pkg().synth
    hf = S.HFTokenizer.from_file(tokdir + "/tokenizer.json")
    for m, i in ((S.AUDIO_START, S.AUDIO_START_ID), (S.AUDIO_END, S.AUDIO_END_ID),
                 (S.AUDIO_PAD, S.AUDIO_PAD_ID), (S.TIMESTAMP, S.TIMESTAMP_ID)):
        assert hf.token_to_id(m) == i
    st = S.SyntheticTokenizer()
    rng = np.random.default_rng(5)
    texts = []
    for i in range(40):
        words = S.english_words(int(rng.integers(1, 30)), rng)
        if i % 2:
            words += S.chinese_words(int(rng.integers(1, 12)), rng)
            rng.shuffle(words)
        texts.append(S.InputBuilder._words_text(words))
    # the whole assembled string of the reference, markers included
    texts.append(S.AUDIO_START + S.AUDIO_PAD * 7 + S.AUDIO_END + texts[3])
    for t in texts:
        assert hf.encode(t) == st.encode(t)
    assert hf.encode_batch(texts) == [st.encode(t) for t in texts]


def test_builder_load_matches_synthetic_builder(tokdir):
    S = pkg().synth
    a = S.InputBuilder.load(tokdir)
    b = S.InputBuilder()
    assert (a.audio_start_token_id, a.audio_end_token_id, a.audio_token_id,
            a.timestamp_token_id) == (S.AUDIO_START_ID, S.AUDIO_END_ID, S.AUDIO_PAD_ID,
                                      S.TIMESTAMP_ID)
    clips = S.workload(2, n_clips=16)
    words = [S.split_words(c.text, c.language) for c in clips]
    vm = [S.valid_mel_frames(len(c.samples)) for c in clips]
    xa, xb = a.build_batch(words, vm), b.build_batch(words, vm)
    for p, q, w, v in zip(xa, xb, words, vm):
        assert np.array_equal(p.input_ids, q.input_ids)
        assert np.array_equal(p.timestamp_positions, q.timestamp_positions)
        one = a.build(w, v)  # one clip at a time: the same input
        assert list(p.input_ids) == one.input_ids
        assert list(p.timestamp_positions) == one.timestamp_positions
        assert p.n_audio_tokens == one.n_audio_tokens == S.audio_token_count(v)


def test_builder_load_reads_marker_strings(tmp_path):
    """tokenizer_config.json names the markers; absent keys take the defaults."""
    import json
    S = pkg().synth
    S.write_tokenizer_dir(str(tmp_path))
    with open(tmp_path / "tokenizer_config.json", "w") as f:
        json.dump({"audio_token": S.TIMESTAMP}, f)  # a deliberately odd choice
    b = S.InputBuilder.load(str(tmp_path))
    assert b.audio_token_id == S.TIMESTAMP_ID and b.audio_start_token_id == S.AUDIO_START_ID
    with open(tmp_path / "tokenizer_config.json", "w") as f:
        json.dump({"audio_bos_token": "<no such token>"}, f)
    with pytest.raises(ValueError):
        S.InputBuilder.load(str(tmp_path))


def test_builder_rejects_pads_inside_the_words(tokdir):
    S = pkg().synth
    b = S.InputBuilder.load(tokdir)
    with pytest.raises(ValueError):
        b.build(["ab" + S.AUDIO_PAD], 500)
    with pytest.raises(ValueError):  # a word that holds a timestamp marker
        b.build(["ab", "c" + S.TIMESTAMP], 500)


def test_aligner_uses_the_model_directory_tokenizer(tmp_path):
    qa = pkg()
    S = qa.synth
    cfg = S.ModelConfig(encoder_layers=1, num_layers=1)
    S.write_tokenizer_dir(str(tmp_path))
    b = qa.Aligner._input_builder(str(tmp_path), None, cfg)
    assert isinstance(b.tok, S.HFTokenizer)
    b2 = qa.Aligner._input_builder({}, str(tmp_path / "tokenizer.json"), cfg)
    assert isinstance(b2.tok, S.HFTokenizer)
    b3 = qa.Aligner._input_builder({}, None, cfg)
    assert isinstance(b3.tok, S.SyntheticTokenizer)
    raw = tokenizers.Tokenizer.from_file(str(tmp_path / "tokenizer.json"))
    assert isinstance(qa.Aligner._input_builder({}, raw, cfg).tok, S.HFTokenizer)
