"""qa_resample against the reference's own resampler (CPU).

The reference resamples non-16 kHz audio with soxr 0.1.3 HQ
(src/mel.rs:537-715), a multi-stage design with FFT-based filtering in f32.
The library's qa_resample is its own design: one linear-phase Kaiser-windowed
sinc with soxr HQ's band edges, evaluated in f64.  Here soxr is built from the
reference's vendored sources (`make -C oracle ref`, tests/soxr_ref.py) and the
two are compared, fed as the reference feeds soxr.  Measured (this container):

  - tones in the pass band (DC, 440 Hz, 3 kHz), away from the first and last
    10 % of the output: max |diff| 5e-7 at amplitude 0.5, i.e. f32 rounding.
    A 7 kHz tone (0.875 of the output Nyquist frequency) differs by 3.7e-4
    (0.0065 dB) at 44.1 and 22.05 kHz: soxr HQ lets its pass band roll off by
    up to 0.01 dB near the edge (SOXR_ROLLOFF_SMALL, soxr.h:248), the library's
    filter is flat there;
  - the workload's audio (bursts of noise low-passed at 3.4 kHz, RMS 0.1),
    generated at 8 / 11.025 / 22.05 / 32 / 44.1 / 48 kHz: max |diff| 8e-5 over
    the whole clip; the log-mel of the two 16 kHz signals differs by at most
    5.4e-3 (in the bins far above 3.4 kHz where the signal is close to the
    mel floor);
  - white noise (energy up to the source Nyquist frequency): max |diff| 9e-4
    in the interior at RMS 0.1, because the two filters' transition bands
    (7.3-8 kHz at a 16 kHz output) are shaped differently.

The bounds below sit a little above those figures.  Skipped when the soxr
build is absent (the reference tree is not on this machine).
"""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import soxr_ref  # noqa: E402
from conftest import pkg  # noqa: E402

pytestmark = pytest.mark.skipif(not soxr_ref.available(),
                                reason="oracle/_ref/libsoxr.so not built (make -C oracle ref)")

RATES = [44100, 48000, 22050, 8000, 11025, 32000]


@pytest.fixture(scope="module")
def qa():
    return pkg()


def _interior(y):
    n = len(y)
    return y[n // 10: 9 * n // 10]


@pytest.mark.parametrize("sr", RATES)
def test_tones_match_soxr(qa, sr):
    t = np.arange(2 * sr) / sr
    # bound: f32 rounding inside the band; soxr's 0.01 dB roll-off of a
    # 0.5-amplitude tone (5.8e-4) near the band edge
    for freq, bound in ((0.0, 2e-6), (440.0, 2e-6), (3000.0, 2e-6), (7000.0, 6e-4)):
        if freq >= 0.9 * min(sr, 16000) / 2:
            continue
        x = (0.5 * np.cos(2 * np.pi * freq * t)).astype(np.float32)
        a = soxr_ref.resample(x, sr, 16000)
        b = qa.audio.resample(x, sr, 16000)
        assert len(a) == len(b) == -(-len(x) * 16000 // sr)
        assert np.abs(_interior(a) - _interior(b)).max() <= bound, (sr, freq)


@pytest.mark.parametrize("sr", RATES)
def test_workload_audio_and_log_mel_match_soxr(qa, sr):
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle"))
    import oracle
    x = qa.synth.synth_audio(6.0, 11, rate=sr)
    a = soxr_ref.resample(x, sr, 16000)
    b = qa.audio.resample(x, sr, 16000)
    assert np.abs(a - b).max() <= 1.5e-4, sr
    assert np.abs(oracle.mel(a) - oracle.mel(b)).max() <= 1e-2, sr


@pytest.mark.parametrize("sr", [44100, 22050, 8000])
def test_white_noise_difference_is_bounded(qa, sr):
    rng = np.random.default_rng(sr)
    x = (0.1 * rng.standard_normal(3 * sr)).astype(np.float32)
    a = soxr_ref.resample(x, sr, 16000)
    b = qa.audio.resample(x, sr, 16000)
    assert np.abs(_interior(a) - _interior(b)).max() <= 2e-3, sr
    # the difference is a transition-band effect: it is small against the signal
    assert np.sqrt(np.mean((a - b) ** 2)) <= 0.02 * np.sqrt(np.mean(a ** 2)), sr
