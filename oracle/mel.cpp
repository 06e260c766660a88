// TEST INFRASTRUCTURE (parity oracle / CPU baseline).
//
// Log-mel restated from src/mel.rs:15-242 (MelExtractor::extract): reflect-pad
// n_fft/2, periodic Hann, f32 400-point FFT, |X|², slaney mel filterbank built
// in f64 (src/mel.rs:101-164), log10 with a 1e-10 floor, clamp at max - 8,
// (x + 4) / 4, trailing frame dropped.
//
// The FFT: the reference calls rustfft 6.4.1 (Cargo.lock:1442), whose source is
// not in the reference tree.  Restated here as a mixed-radix decimation-in-time
// DFT (400 = 2^4 · 5^2) in f32 with f64-computed twiddles rounded to f32, which
// is the published algorithm family rustfft plans for composite sizes.  Its
// rounding differs from rustfft's in the last bits (parity unpinned, as the
// reference's own mel tests check only shape and finiteness, src/mel.rs:249-289).
#include <omp.h>

#include <algorithm>
#include <complex>

#include "common.h"

namespace {

constexpr int kNfft = 400;
constexpr int kHop = 160;
constexpr int kMels = 128;
constexpr int kSr = 16000;

using cf = std::complex<float>;

// src/mel.rs:19-27: periodic Hann in f32 arithmetic.
std::vector<float> hann(int n) {
  std::vector<float> w(n);
  for (int i = 0; i < n; ++i) {
    const float x = 2.0f * static_cast<float>(M_PI) * static_cast<float>(i) / static_cast<float>(n);
    w[i] = 0.5f * (1.0f - std::cos(x));
  }
  return w;
}

// src/mel.rs:31-46: reflection index, edge not repeated; n <= 1 gives 0.
int64_t reflect_index(int64_t i, int64_t n) {
  if (n <= 1) return 0;
  const int64_t period = 2 * (n - 1);
  int64_t x = i % period;
  if (x < 0) x += period;
  return x > n - 1 ? period - x : x;
}

// src/mel.rs:101-164, f64 build, f32 storage.
std::vector<float> mel_filterbank(int num_mels, int n_fft, int sample_rate, double fmin,
                                  double fmax) {
  const int n_freqs = n_fft / 2 + 1;
  const double sr = sample_rate;
  const double f_sp = 200.0 / 3.0;
  const double min_log_hz = 1000.0;
  const double min_log_mel = min_log_hz / f_sp;
  const double logstep = std::log(6.4) / 27.0;
  auto hz_to_mel = [&](double f) {
    return f < min_log_hz ? f / f_sp : min_log_mel + std::log(f / min_log_hz) / logstep;
  };
  auto mel_to_hz = [&](double m) {
    return m < min_log_mel ? f_sp * m : min_log_hz * std::exp(logstep * (m - min_log_mel));
  };
  const double mel_min = hz_to_mel(fmin), mel_max = hz_to_mel(fmax);
  std::vector<double> ff(num_mels + 2);
  for (int i = 0; i < num_mels + 2; ++i)
    ff[i] = mel_to_hz(mel_min + (mel_max - mel_min) * i / static_cast<double>(num_mels + 1));
  std::vector<double> fd(num_mels + 1);
  for (int i = 0; i < num_mels + 1; ++i) fd[i] = ff[i + 1] - ff[i];
  std::vector<float> filt(static_cast<size_t>(num_mels) * n_freqs, 0.0f);
  for (int j = 0; j < n_freqs; ++j) {
    const double f = j * sr / n_fft;
    for (int i = 0; i < num_mels; ++i) {
      const double down = (f - ff[i]) / fd[i];
      const double up = (ff[i + 2] - f) / fd[i + 1];
      filt[static_cast<size_t>(i) * n_freqs + j] = static_cast<float>(std::max(std::min(down, up), 0.0));
    }
  }
  for (int i = 0; i < num_mels; ++i) {
    const double enorm = 2.0 / (ff[i + 2] - ff[i]);
    for (int j = 0; j < n_freqs; ++j) filt[static_cast<size_t>(i) * n_freqs + j] *= static_cast<float>(enorm);
  }
  return filt;
}

// Mixed-radix DIT DFT of length n (n = product of small radices), f32.
struct Fft {
  int n;
  std::vector<int> radices;
  std::vector<cf> tw;  // tw[k] = exp(-2πi k / n), f64 -> f32
  explicit Fft(int n_) : n(n_) {
    int m = n;
    for (int r : {4, 2, 5, 3}) {
      while (m % r == 0) {
        radices.push_back(r);
        m /= r;
      }
    }
    tw.resize(n);
    for (int k = 0; k < n; ++k) {
      const double a = -2.0 * M_PI * k / n;
      tw[k] = cf(static_cast<float>(std::cos(a)), static_cast<float>(std::sin(a)));
    }
  }
  // out[k] = Σ_j in[j*stride] · w^(jk), len = remaining length, level = radix index
  void rec(const cf* in, int stride, cf* out, int len, size_t level, cf* scratch) const {
    if (len == 1) {
      out[0] = in[0];
      return;
    }
    const int p = radices[level];
    const int m = len / p;
    // sub-transforms of the p decimated sequences
    for (int q = 0; q < p; ++q) rec(in + q * stride, stride * p, out + q * m, m, level + 1, scratch);
    // butterflies: X[k + m t] = Σ_q W_len^{q(k + m t)} Y_q[k]
    const int tstep = n / len;  // twiddle index unit for W_len
    for (int k = 0; k < m; ++k) {
      cf y[5];
      for (int q = 0; q < p; ++q) {
        const cf v = out[q * m + k];
        y[q] = q == 0 ? v : v * tw[(static_cast<int64_t>(q) * k * tstep) % n];
      }
      for (int t = 0; t < p; ++t) {
        cf s = y[0];
        for (int q = 1; q < p; ++q) s += y[q] * tw[(static_cast<int64_t>(q) * t * m * tstep) % n];
        scratch[k + m * t] = s;
      }
    }
    for (int i = 0; i < len; ++i) out[i] = scratch[i];
  }
  void forward(const cf* in, cf* out) const {
    std::vector<cf> scratch(n);
    rec(in, 1, out, n, 0, scratch.data());
  }
};

}  // namespace

extern "C" {

void or_hann_window(int n, float* out) {
  auto w = hann(n);
  std::copy(w.begin(), w.end(), out);
}

int or_reflection_pad(const float* x, int n, int pad, float* out) {
  // src/mel.rs:48-64; returns the padded length.
  if (n == 0 || pad == 0) {
    for (int i = 0; i < n; ++i) out[i] = x[i];
    return n;
  }
  int o = 0;
  for (int k = 0; k < pad; ++k) out[o++] = x[reflect_index(-static_cast<int64_t>(pad) + k, n)];
  for (int i = 0; i < n; ++i) out[o++] = x[i];
  for (int k = 0; k < pad; ++k) out[o++] = x[reflect_index(static_cast<int64_t>(n) + k, n)];
  return o;
}

void or_mel_filterbank(int num_mels, int n_fft, int sr, float* out) {
  auto f = mel_filterbank(num_mels, n_fft, sr, 0.0, sr / 2.0);
  std::copy(f.begin(), f.end(), out);
}

int or_mel(const float* samples, int64_t n, float* out, int64_t out_len, int* n_frames_out) {
  if (n <= 0) return QA_ERR_SHAPE;  // "empty audio" (src/mel.rs:199)
  const int pad = kNfft / 2;
  std::vector<float> padded(static_cast<size_t>(n) + 2 * pad);
  const int64_t plen = or_reflection_pad(samples, static_cast<int>(n), pad, padded.data());
  const auto window = hann(kNfft);
  const int n_freqs = kNfft / 2 + 1;
  const int64_t with_last = plen >= kNfft ? (plen - kNfft) / kHop + 1 : 0;
  const int64_t frames = with_last > 0 ? with_last - 1 : 0;
  if (out_len < frames * kMels) return QA_ERR_SHAPE;
  static const auto filt = mel_filterbank(kMels, kNfft, kSr, 0.0, kSr / 2.0);
  static const Fft fft(kNfft);

  // power[f][t] then mel[m][t] (src/mel.rs:66-99, 215-227)
  std::vector<float> power(static_cast<size_t>(n_freqs) * frames);
#pragma omp parallel
  {
    std::vector<cf> buf(kNfft), spec(kNfft);
#pragma omp for schedule(static)
    for (int64_t i = 0; i < frames; ++i) {
      const int64_t start = i * kHop;
      for (int j = 0; j < kNfft; ++j) buf[j] = cf(padded[start + j] * window[j], 0.0f);
      fft.forward(buf.data(), spec.data());
      for (int k = 0; k < n_freqs; ++k) {
        const float re = spec[k].real(), im = spec[k].imag();
        power[static_cast<size_t>(k) * frames + i] = re * re + im * im;
      }
    }
  }
  std::fill(out, out + frames * kMels, 0.0f);
#pragma omp parallel for schedule(static)
  for (int m = 0; m < kMels; ++m) {
    float* orow = out + static_cast<size_t>(m) * frames;
    for (int f = 0; f < n_freqs; ++f) {
      const float w = filt[static_cast<size_t>(m) * n_freqs + f];
      if (w == 0.0f) continue;  // src/mel.rs:221
      const float* prow = &power[static_cast<size_t>(f) * frames];
      for (int64_t t = 0; t < frames; ++t) orow[t] += w * prow[t];
    }
  }
  const float log10_factor = 1.0f / std::log(10.0f);
  float mx = -INFINITY;
  for (int64_t i = 0; i < frames * kMels; ++i) {
    const float v = std::log(std::max(out[i], 1e-10f)) * log10_factor;
    out[i] = v;
    mx = v > mx ? v : mx;
  }
  const float mn = mx - 8.0f;
  for (int64_t i = 0; i < frames * kMels; ++i) out[i] = (std::max(out[i], mn) + 4.0f) / 4.0f;
  if (n_frames_out) *n_frames_out = static_cast<int>(frames);
  return QA_OK;
}

}  // extern "C"
