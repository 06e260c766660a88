"""WAV decode + downmix and resampling (qa_decode_wav, qa_resample): the host
step of Aligner.align before the alignment path (src/mel.rs:347-474, 537-715).

The decode is checked bit for bit against the reference's rules restated in
numpy float32 arithmetic (16-bit PCM: i16 / 32768 with channels summed in
order from 0 and divided by their count; other PCM depths and 32-bit float as
the hound crate decodes them).  The resampler is checked through properties
that hold for soxr's HQ recipe: the reference's own length test
(src/mel.rs:291-301), DC and pass-band gain, and the stop band."""
import struct

import numpy as np
import pytest

from conftest import pkg

F32 = np.float32


def wav_bytes(tag, channels, rate, bits, data, extra=(), ext_sub=None, data_size=None):
    """A RIFF/WAVE file: optional extra (id, body) chunks before fmt, the fmt
    chunk (extensible when ext_sub is a subformat tag) and the data chunk."""
    block = channels * bits // 8
    fmt = struct.pack("<HHIIHH", 0xFFFE if ext_sub is not None else tag, channels, rate,
                      rate * block, block, bits)
    if ext_sub is not None:
        guid_tail = b"\x00\x00\x00\x00\x10\x00\x80\x00\x00\xaa\x00\x38\x9b\x71"
        fmt += struct.pack("<HHI", 22, bits, 0) + struct.pack("<H", ext_sub) + guid_tail
    chunks = b""
    for cid, body in extra:
        chunks += cid + struct.pack("<I", len(body)) + body + (b"\x00" if len(body) % 2 else b"")
    f = b"fmt " + struct.pack("<I", len(fmt)) + fmt
    d = b"data" + struct.pack("<I", len(data) if data_size is None else data_size) + data
    body = b"WAVE" + chunks + f + d
    return b"RIFF" + struct.pack("<I", len(body)) + body


def mix(samples_f32, ch):
    """Sum each frame's channels in order from 0.0f, then divide (f32)."""
    s = np.asarray(samples_f32, F32)
    frames = -(-len(s) // ch)
    out = np.empty(frames, F32)
    for f in range(frames):
        acc = F32(0.0)
        for v in s[f * ch:(f + 1) * ch]:
            acc = F32(acc + v)
        out[f] = F32(acc / F32(ch))
    return out


@pytest.fixture(scope="module")
def audio():
    return pkg().audio


@pytest.mark.parametrize("ch", [1, 2, 3, 8])
def test_pcm16_matches_reference_rules(audio, ch):
    rng = np.random.default_rng(ch)
    x = rng.integers(-32768, 32768, (1001, ch), dtype=np.int16)
    got, sr, c = audio.decode_wav(wav_bytes(1, ch, 16000, 16, x.tobytes()))
    assert (sr, c) == (16000, ch)
    want = mix((x.reshape(-1).astype(F32) / F32(32768.0)), ch)
    assert got.dtype == F32 and np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_pcm16_drops_a_partial_frame_and_honours_pad_bytes(audio):
    x = np.arange(-50, 51, dtype=np.int16)  # 101 samples: 50 stereo frames + 1
    extra = [(b"LIST", b"abc"), (b"junk", b"12345")]  # odd sizes: pad bytes follow
    got, _, _ = audio.decode_wav(wav_bytes(1, 2, 16000, 16, x.tobytes(), extra=extra))
    assert len(got) == 50
    assert np.array_equal(got, mix(x[:100].astype(F32) / F32(32768.0), 2))


@pytest.mark.parametrize("bits", [8, 24, 32])
def test_other_pcm_depths_as_hound_decodes_them(audio, bits):
    rng = np.random.default_rng(bits)
    n, ch = 777, 2
    if bits == 8:
        raw = rng.integers(0, 256, n * ch, dtype=np.uint8)
        vals = raw.astype(np.int64) - 128
        data = raw.tobytes()
    elif bits == 24:
        vals = rng.integers(-(1 << 23), 1 << 23, n * ch)
        data = b"".join(int(v & 0xFFFFFF).to_bytes(3, "little") for v in vals)
    else:
        vals = rng.integers(-(1 << 31), 1 << 31, n * ch)
        data = vals.astype("<i4").tobytes()
    got, _, c = audio.decode_wav(wav_bytes(1, ch, 16000, bits, data))
    assert c == ch
    want = mix(vals.astype(F32) / F32(1 << (bits - 1)), ch)
    assert np.array_equal(got, want)


def test_float32_and_extensible(audio):
    rng = np.random.default_rng(4)
    x = rng.standard_normal(999 * 3).astype(F32) * F32(0.3)
    got, _, _ = audio.decode_wav(wav_bytes(3, 3, 16000, 32, x.tobytes()))
    assert np.array_equal(got, mix(x, 3))
    got, _, _ = audio.decode_wav(wav_bytes(3, 3, 16000, 32, x.tobytes(), ext_sub=3))
    assert np.array_equal(got, mix(x, 3))
    pcm = rng.integers(-32768, 32768, 600, dtype=np.int16)
    got, _, _ = audio.decode_wav(wav_bytes(1, 2, 16000, 16, pcm.tobytes(), ext_sub=1))
    assert np.array_equal(got, mix(pcm.astype(F32) / F32(32768.0), 2))


def test_truncated_data_keeps_what_is_there(audio):
    # hound path (24-bit stereo): a partial last frame is kept, divided by 2
    vals = np.arange(-7, 8) * 1000  # 15 samples: 7 frames + 1
    data = b"".join(int(v & 0xFFFFFF).to_bytes(3, "little") for v in vals)
    got, _, _ = audio.decode_wav(wav_bytes(1, 2, 16000, 24, data, data_size=len(data) + 3000))
    assert np.array_equal(got, mix(vals.astype(F32) / F32(1 << 23), 2))
    assert len(got) == 8


def test_rejections(audio):
    qa = pkg()
    with pytest.raises(qa.QaError) as e:
        audio.decode_wav(b"RIFX" + b"\x00" * 40)
    assert e.value.code == qa._lib.QA_ERR_SHAPE
    with pytest.raises(qa.QaError):  # ADPCM
        audio.decode_wav(wav_bytes(2, 1, 16000, 4, b"\x00" * 64))
    with pytest.raises(qa.QaError):  # no samples
        audio.decode_wav(wav_bytes(1, 1, 16000, 16, b""))


def test_resample_length_kat(audio):
    """src/mel.rs:291-301: 44.1 kHz -> 16 kHz gives ceil(n * 16000 / 44100)
    samples, finite and not all zero."""
    n = 44100
    x = np.sin(np.arange(n, dtype=F32) * F32(0.01)).astype(F32)
    y = audio.resample(x, 44100, 16000)
    assert len(y) == int(np.ceil(n * 16000.0 / 44100.0)) == 16000
    assert np.isfinite(y).all() and (y != 0).any()
    for sr in (48000, 22050, 8000, 11025, 32000):
        assert len(audio.resample(x[:12345], sr, 16000)) == -(-12345 * 16000 // sr)
    assert np.array_equal(audio.resample(x, 16000, 16000), x)


@pytest.mark.parametrize("sr_in", [44100, 48000, 22050, 8000, 44101])
def test_resample_pass_band_and_dc(audio, sr_in):
    t_in = np.arange(sr_in) / sr_in  # 1 s
    lo, hi = 0.2, 0.8  # interior of the output, away from the edges' transients
    for freq in (0.0, 440.0, 3000.0, 7000.0):
        if freq >= 0.913 * min(sr_in, 16000) / 2:
            continue
        x = (0.5 * np.cos(2 * np.pi * freq * t_in)).astype(F32)
        y = audio.resample(x, sr_in, 16000)
        t = np.arange(len(y)) / 16000.0
        want = 0.5 * np.cos(2 * np.pi * freq * t)
        sl = slice(int(lo * len(y)), int(hi * len(y)))
        assert np.abs(y[sl] - want[sl]).max() < 2e-5, (sr_in, freq)


def test_resample_stop_band(audio):
    """Tones above the 8 kHz output Nyquist frequency do not alias back."""
    sr_in = 48000
    t_in = np.arange(sr_in) / sr_in
    for freq in (8200.0, 10000.0, 15000.0, 21000.0):
        x = (0.5 * np.sin(2 * np.pi * freq * t_in)).astype(F32)
        y = audio.resample(x, sr_in, 16000)
        sl = slice(len(y) // 5, 4 * len(y) // 5)
        assert np.sqrt(np.mean(y[sl].astype(np.float64) ** 2)) < 5e-6, freq


def test_load_audio_wav(audio, tmp_path):
    rng = np.random.default_rng(9)
    x = rng.integers(-20000, 20000, 4410, dtype=np.int16)
    p16 = tmp_path / "a16.wav"
    p16.write_bytes(wav_bytes(1, 1, 16000, 16, x.tobytes()))
    assert np.array_equal(audio.load_audio_wav(p16), x.astype(F32) / F32(32768.0))
    p44 = tmp_path / "a44.wav"
    p44.write_bytes(wav_bytes(1, 1, 44100, 16, x.tobytes()))
    y = audio.load_audio_wav(p44)
    assert len(y) == 1600
    assert np.array_equal(y, audio.resample(x.astype(F32) / F32(32768.0), 44100, 16000))
