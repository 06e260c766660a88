// Audio file input on the host: WAV decode + downmix (src/mel.rs:347-465,
// `load_audio_wav`) and the sample-rate conversion that follows it for
// sources that are not 16 kHz (src/mel.rs:467-474, 537-715).
//
// Decode rules, as the reference applies them:
//  * 16-bit PCM (format tag 1) with 1..8 channels: the reference's own reader
//    (`read_pcm16_fast`, :351-403): chunk walk from byte 12, unknown chunks
//    skipped, an odd chunk size followed by a pad byte, the data chunk clipped
//    to the file, only whole frames; a sample is i16 / 32768.0f; several
//    channels are summed in order from 0.0f and divided by the channel count;
//  * everything else goes through the `hound` 3.5.1 crate (:404-465): 8-bit
//    PCM (unsigned bytes, value - 128), 24- and 32-bit PCM (sign-extended),
//    each as (float)v / 2^(bits-1); 32-bit IEEE float as is; the extensible
//    header (tag 0xFFFE) with a PCM or IEEE-float subformat GUID.  A data
//    chunk cut short by the end of the file keeps the samples it holds (a
//    trailing partial frame included: its sum is still divided by the channel
//    count).
//
// Resampling: the reference calls soxr (HQ recipe: 20-bit precision, pass
// band to 0.913 of the lower Nyquist frequency, linear phase) and then
// librosa's fix_length to ceil(n * target / source) samples.  soxr is built
// only through CMake with a generated configuration header, so it is not
// compiled here; this file designs its own linear-phase low-pass with the
// same band edges instead: a Kaiser-windowed sinc (Kaiser's window design
// formulas for the stop-band attenuation and the transition width),
// evaluated as a polyphase filter at output time t = k * source / target,
// with f64 coefficients and accumulation.  A rate pair whose reduced ratio
// has more than 4096 output phases interpolates the taps between 4096
// tabulated ones.  The tables are built on the host cores and kept for the
// last few rate pairs.  Results match soxr's in band edges and length, not
// bit for bit.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include "qa_b200.h"

namespace {

uint16_t rd16(const uint8_t* p) { return static_cast<uint16_t>(p[0] | (p[1] << 8)); }
uint32_t rd32(const uint8_t* p) {
  return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) |
         (static_cast<uint32_t>(p[2]) << 16) | (static_cast<uint32_t>(p[3]) << 24);
}

struct WavInfo {
  int format = 0;  // 1 PCM, 3 IEEE float (after resolving the extensible subformat)
  int tag = 0;     // the fmt chunk's own format tag
  int channels = 0;
  uint32_t rate = 0;
  int bits = 0;
  const uint8_t* data = nullptr;
  size_t data_len = 0;
  bool has_fmt = false, has_data = false;
};

// The RIFF chunk walk (src/mel.rs:357-383).  Returns false when the buffer is
// not RIFF/WAVE.
bool walk(const uint8_t* b, size_t n, WavInfo& w) {
  if (n < 12 || std::memcmp(b, "RIFF", 4) != 0 || std::memcmp(b + 8, "WAVE", 4) != 0) return false;
  size_t pos = 12;
  while (pos + 8 <= n) {
    const uint8_t* id = b + pos;
    const size_t size = rd32(b + pos + 4);
    const size_t body = pos + 8;
    const size_t end = std::min(body + size, n);
    if (std::memcmp(id, "fmt ", 4) == 0 && size >= 16 && body + 16 <= n) {
      w.tag = rd16(b + body);
      w.channels = rd16(b + body + 2);
      w.rate = rd32(b + body + 4);
      w.bits = rd16(b + body + 14);
      w.format = w.tag;
      // WAVE_FORMAT_EXTENSIBLE: the subformat GUID's first two bytes carry the tag
      if (w.tag == 0xFFFE && size >= 40 && body + 40 <= n) {
        const int valid = rd16(b + body + 18);
        w.format = rd16(b + body + 24);
        if (valid != 0 && valid != w.bits) w.format = -1;  // padded containers: unsupported
      }
      w.has_fmt = true;
    } else if (std::memcmp(id, "data", 4) == 0) {
      w.data = b + body;
      w.data_len = end > body ? end - body : 0;
      w.has_data = true;
    }
    const size_t next = body + size + (size & 1);
    if (next <= body) break;
    pos = next;
  }
  return true;
}

// Decoded mono samples, or a status code.
int decode(const uint8_t* b, size_t n, std::vector<float>& mono, int* rate, int* channels) {
  WavInfo w;
  if (!walk(b, n, w)) return QA_ERR_SHAPE;
  if (!w.has_fmt || !w.has_data || w.channels <= 0) return QA_ERR_SHAPE;
  *rate = static_cast<int>(w.rate);
  *channels = w.channels;
  const int ch = w.channels;
  mono.clear();
  if (w.tag == 1 && w.bits == 16 && ch <= 8) {  // the reference's own PCM16 reader
    const size_t frames = w.data_len / (2 * static_cast<size_t>(ch));
    mono.resize(frames);
    for (size_t f = 0; f < frames; ++f) {
      const uint8_t* fr = w.data + f * 2 * ch;
      if (ch == 1) {
        mono[f] = static_cast<float>(static_cast<int16_t>(rd16(fr))) / 32768.0f;
      } else {
        float acc = 0.0f;
        for (int c = 0; c < ch; ++c) acc += static_cast<float>(static_cast<int16_t>(rd16(fr + 2 * c))) / 32768.0f;
        mono[f] = acc / static_cast<float>(ch);
      }
    }
    return mono.empty() ? QA_ERR_SHAPE : QA_OK;
  }
  // the hound path: interleaved samples, then chunks of `ch` summed and divided
  std::vector<float> s;
  if (w.format == 3 && w.bits == 32) {
    const size_t cnt = w.data_len / 4;
    s.resize(cnt);
    for (size_t i = 0; i < cnt; ++i) {
      const uint32_t u = rd32(w.data + 4 * i);
      std::memcpy(&s[i], &u, 4);
    }
  } else if (w.format == 1 && (w.bits == 8 || w.bits == 16 || w.bits == 24 || w.bits == 32)) {
    const int bytes = w.bits / 8;
    const size_t cnt = w.data_len / bytes;
    const float max_val = static_cast<float>(1LL << (w.bits - 1));
    s.resize(cnt);
    for (size_t i = 0; i < cnt; ++i) {
      const uint8_t* p = w.data + i * bytes;
      int32_t v;
      if (bytes == 1) v = static_cast<int32_t>(p[0]) - 128;
      else if (bytes == 2) v = static_cast<int16_t>(rd16(p));
      else if (bytes == 3) v = static_cast<int32_t>((static_cast<uint32_t>(p[0]) << 8) |
                                                    (static_cast<uint32_t>(p[1]) << 16) |
                                                    (static_cast<uint32_t>(p[2]) << 24)) >> 8;
      else v = static_cast<int32_t>(rd32(p));
      s[i] = static_cast<float>(v) / max_val;
    }
  } else {
    return QA_ERR_SHAPE;  // a format the reference's readers do not take either
  }
  if (s.empty()) return QA_ERR_SHAPE;
  if (ch == 1) {
    mono.swap(s);
    return QA_OK;
  }
  const size_t frames = (s.size() + ch - 1) / ch;
  mono.resize(frames);
  for (size_t f = 0; f < frames; ++f) {
    float acc = 0.0f;
    for (size_t i = f * ch; i < std::min(s.size(), (f + 1) * static_cast<size_t>(ch)); ++i) acc += s[i];
    mono[f] = acc / static_cast<float>(ch);
  }
  return QA_OK;
}

// ------------------------------------------------------------------ resampler

constexpr double kPassEnd = 0.913;   // of the lower Nyquist frequency (soxr HQ)
constexpr double kStopBegin = 1.0;
constexpr double kAttenDb = 125.0;   // 20-bit quality
constexpr int kMaxRows = 4096;        // exact polyphase rows up to this many phases

double bessel_i0(double x) {  // power series, converges for every x used here
  double sum = 1.0, term = 1.0;
  const double q = 0.25 * x * x;
  for (int k = 1; k < 200; ++k) {
    term *= q / (static_cast<double>(k) * k);
    sum += term;
    if (term < 1e-17 * sum) break;
  }
  return sum;
}

struct Filter {
  long long up = 1, down = 1;  // output time k * down / up, in input samples
  int half = 0;                // taps on each side of the output time
  double cut = 1.0;            // cutoff, fraction of the input Nyquist frequency
  double beta = 0.0;
  double i0_beta = 1.0;
  // [rows][2 * half] taps: one row per output phase p / up when up <= kMaxRows
  // (exact), else kMaxRows + 1 rows at phases r / kMaxRows between which the
  // taps are interpolated linearly
  std::vector<double> table;
  int rows = 0;
  bool exact = true;

  double tap(double tau) const {  // tau: distance in input samples
    const double r = tau / half;
    if (r <= -1.0 || r >= 1.0) return 0.0;
    const double w = bessel_i0(beta * std::sqrt(1.0 - r * r)) / i0_beta;
    const double x = cut * tau;
    const double s = x == 0.0 ? 1.0 : std::sin(M_PI * x) / (M_PI * x);
    return cut * s * w;
  }
};

Filter design(int sr_in, int sr_out) {
  Filter f;
  long long a = sr_in, b = sr_out;
  while (b) {
    const long long t = a % b;
    a = b;
    b = t;
  }
  f.up = sr_out / a;
  f.down = sr_in / a;
  const double lower = std::min(sr_in, sr_out) / static_cast<double>(sr_in);  // <= 1
  f.cut = lower * 0.5 * (kPassEnd + kStopBegin);
  // Kaiser: beta from the attenuation, length from the transition width
  // (in radians per input sample)
  f.beta = 0.1102 * (kAttenDb - 8.7);
  f.i0_beta = bessel_i0(f.beta);
  const double dw = M_PI * lower * (kStopBegin - kPassEnd);
  const double taps = (kAttenDb - 7.95) / (2.285 * dw) + 1.0;
  f.half = static_cast<int>(std::ceil(taps / 2.0));
  f.exact = f.up <= kMaxRows;
  f.rows = f.exact ? static_cast<int>(f.up) : kMaxRows + 1;
  const double den = f.exact ? static_cast<double>(f.up) : static_cast<double>(kMaxRows);
  f.table.resize(static_cast<size_t>(f.rows) * 2 * f.half);
  std::atomic<int> next{0};
  auto rows = [&] {
    for (int r = next++; r < f.rows; r = next++)
      for (int j = 0; j < 2 * f.half; ++j)
        f.table[static_cast<size_t>(r) * 2 * f.half + j] = f.tap(r / den + (f.half - 1 - j));
  };
  const int nt = std::max(1, std::min<int>(f.rows / 16, static_cast<int>(std::min(16u, std::thread::hardware_concurrency()))));
  std::vector<std::thread> th;
  for (int t = 1; t < nt; ++t) th.emplace_back(rows);
  rows();
  for (auto& t : th) t.join();
  return f;
}

// The filters of the last few rate pairs (a file set usually has one or two
// source rates), shared by every call.
std::shared_ptr<const Filter> filter_for(int sr_in, int sr_out) {
  static std::mutex mu;
  static std::vector<std::pair<std::pair<int, int>, std::shared_ptr<const Filter>>> cache;
  std::lock_guard<std::mutex> lock(mu);
  for (auto& e : cache)
    if (e.first == std::make_pair(sr_in, sr_out)) return e.second;
  auto f = std::make_shared<const Filter>(design(sr_in, sr_out));
  if (cache.size() >= 4) cache.erase(cache.begin());
  cache.emplace_back(std::make_pair(sr_in, sr_out), f);
  return f;
}

}  // namespace

extern "C" {

int qa_decode_wav(const uint8_t* bytes, int64_t n_bytes, float* out, int64_t out_cap,
                  int64_t* n_out, int* sample_rate, int* channels) {
  if (!bytes || n_bytes < 0 || !n_out || !sample_rate || !channels) return QA_ERR_ARG;
  std::vector<float> mono;
  int rate = 0, ch = 0;
  const int rc = decode(bytes, static_cast<size_t>(n_bytes), mono, &rate, &ch);
  if (rc) return rc;
  *n_out = static_cast<int64_t>(mono.size());
  *sample_rate = rate;
  *channels = ch;
  if (!out) return QA_OK;  // size query
  if (out_cap < static_cast<int64_t>(mono.size())) return QA_ERR_SHAPE;
  std::copy(mono.begin(), mono.end(), out);
  return QA_OK;
}

int64_t qa_resampled_length(int64_t n, int sr_in, int sr_out) {
  if (n < 0 || sr_in <= 0 || sr_out <= 0) return -1;
  // ceil(n * out / in) in integers (librosa fix_length after soxr)
  return (n * static_cast<int64_t>(sr_out) + sr_in - 1) / sr_in;
}

int qa_resample(const float* in, int64_t n, int sr_in, int sr_out, float* out, int64_t out_len) {
  if (!in || !out || n <= 0 || sr_in <= 0 || sr_out <= 0) return QA_ERR_ARG;
  if (out_len != qa_resampled_length(n, sr_in, sr_out)) return QA_ERR_SHAPE;
  if (sr_in == sr_out) {
    std::copy(in, in + n, out);
    return QA_OK;
  }
  const std::shared_ptr<const Filter> fp = filter_for(sr_in, sr_out);
  const Filter& f = *fp;
  const int width = 2 * f.half;
  auto one = [&](int64_t k) {
    // output k sits at input time t = k * down / up = n0 + p / up
    const long long num = k * f.down;
    const long long n0 = num / f.up, p = num % f.up;
    const long long first = n0 - f.half + 1;
    double acc = 0.0;
    const long long j0 = std::max<long long>(0, -first), j1 = std::min<long long>(width, n - first);
    if (f.exact) {
      const double* row = &f.table[static_cast<size_t>(p) * width];
      for (long long j = j0; j < j1; ++j) acc += row[j] * static_cast<double>(in[first + j]);
    } else {
      const double pos = static_cast<double>(p) / f.up * kMaxRows;
      const int r = std::min(static_cast<int>(pos), kMaxRows - 1);
      const double w = pos - r;
      const double* a = &f.table[static_cast<size_t>(r) * width];
      const double* b = a + width;
      for (long long j = j0; j < j1; ++j)
        acc += (a[j] + w * (b[j] - a[j])) * static_cast<double>(in[first + j]);
    }
    out[k] = static_cast<float>(acc);
  };
  const unsigned hw = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
  const int64_t chunk = 4096;
  std::atomic<int64_t> next{0};
  auto worker = [&] {
    for (int64_t s = next.fetch_add(chunk); s < out_len; s = next.fetch_add(chunk))
      for (int64_t k = s; k < std::min(out_len, s + chunk); ++k) one(k);
  };
  std::vector<std::thread> th;
  const unsigned nt = static_cast<unsigned>(std::min<int64_t>(hw, (out_len + chunk - 1) / chunk));
  for (unsigned t = 1; t < nt; ++t) th.emplace_back(worker);
  worker();
  for (auto& t : th) t.join();
  return QA_OK;
}

}  // extern "C"
