// TEST INFRASTRUCTURE (parity oracle) — the Local Head refinement stage
// (src/local_head.rs), restated on the CPU.  Every function cites the
// reference lines it follows; the arithmetic is f32 where the reference's is,
// the frame FFT is f64 as the reference's (numpy's rfft widens to f64), and
// sums run in the reference's order.
#include <algorithm>
#include <cmath>
#include <complex>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "common.h"

namespace {

// src/local_head.rs:55-77
constexpr int kSampleRate = 16000;
constexpr int kFrameLen = 25 * kSampleRate / 1000;  // 400
constexpr int kHop = 10 * kSampleRate / 1000;       // 160
constexpr int kContextFrames = 200 / 10;            // frames either side of the centre
constexpr int kFrames = 41;
constexpr int kNfft = 512;
constexpr int kBins = kNfft / 2 + 1;  // 257
constexpr int kMels = 80;
constexpr int kBands = 4;
constexpr int kFeat = kMels + 3 + 2 * kBands;  // 91
constexpr float kLogEps = 1e-6f;
constexpr double kSegmentMs = 80.0;
constexpr double kMinWordMs = 10.0;
constexpr float kTemperature = 1.5f;
constexpr int kOffsets = 13;
constexpr float kOffsetsMs[kOffsets] = {-60, -50, -40, -30, -20, -10, 0, 10, 20, 30, 40, 50, 60};
constexpr int kDim = 128, kHeads = 4, kQwen = 1024;

// src/local_head.rs:917-925: symmetric Hann, phase over length - 1, f64 then f32
std::vector<float> hann(int length) {
  std::vector<float> w(length);
  for (int i = 0; i < length; ++i) {
    const double phase = 2.0 * M_PI * i / (length - 1);
    w[i] = static_cast<float>(0.5 - 0.5 * std::cos(phase));
  }
  return w;
}

// src/local_head.rs:927-973: HTK mel points, floored bin edges, triangles,
// each row normalised to unit sum
std::vector<float> mel_bank() {
  auto hz_to_mel = [](double hz) { return 2595.0 * std::log10(1.0 + hz / 700.0); };
  auto mel_to_hz = [](double mel) { return 700.0 * (std::pow(10.0, mel / 2595.0) - 1.0); };
  const double low = hz_to_mel(0.0), high = hz_to_mel(kSampleRate / 2.0);
  std::vector<int> edges(kMels + 2);
  for (int i = 0; i < kMels + 2; ++i) {
    const double p = mel_to_hz(low + (high - low) * i / (kMels + 1));
    edges[i] = static_cast<int>(std::max<long long>(
        static_cast<long long>(std::floor((kNfft + 1) * p / kSampleRate)), 0));
  }
  std::vector<float> bank(static_cast<size_t>(kMels) * kBins, 0.0f);
  for (int m = 0; m < kMels; ++m) {
    const int left = edges[m];
    const int center = std::max(edges[m + 1], left + 1);
    const int right = std::min(std::max(edges[m + 2], center + 1), kBins - 1);
    if (center >= kBins) continue;
    float* row = &bank[static_cast<size_t>(m) * kBins];
    if (center > left) {
      const int n = center - left;
      for (int i = 0; i < n; ++i) row[left + i] = static_cast<float>(i) / n;
    }
    if (right > center) {
      const int n = right - center;
      for (int i = 0; i < n; ++i) row[center + i] = 1.0f - static_cast<float>(i) / n;
    }
    float total = 0.0f;
    for (int b = 0; b < kBins; ++b) total += row[b];
    if (total > 0.0f)
      for (int b = 0; b < kBins; ++b) row[b] /= total;
  }
  return bank;
}

// src/local_head.rs:975-982
void band_edges(int bins, int* edges) {
  for (int i = 0; i <= kBands; ++i)
    edges[i] = static_cast<int>(1.0 + (bins - 1.0) * i / kBands);
}

// src/local_head.rs:984-986 (libm erff)
float gelu(float x) { return 0.5f * x * (1.0f + erff(x * static_cast<float>(M_SQRT1_2))); }

// src/local_head.rs:988-994
float dot(const float* a, const float* b, int n) {
  float acc = 0.0f;
  for (int i = 0; i < n; ++i) acc += a[i] * b[i];
  return acc;
}

// src/local_head.rs:996-1004
void layer_norm(float* x, int n, const float* w, const float* b) {
  float s = 0.0f;
  for (int i = 0; i < n; ++i) s += x[i];
  const float mean = s / n;
  float v = 0.0f;
  for (int i = 0; i < n; ++i) v += (x[i] - mean) * (x[i] - mean);
  const float var = v / n;
  const float inv = 1.0f / std::sqrt(var + 1e-5f);
  for (int i = 0; i < n; ++i) x[i] = (x[i] - mean) * inv * w[i] + b[i];
}

// src/local_head.rs:1006-1012
void softmax(float* s, int n) {
  float mx = -INFINITY;
  for (int i = 0; i < n; ++i) mx = std::max(mx, s[i]);
  float total = 0.0f;
  for (int i = 0; i < n; ++i) {
    s[i] = std::exp(s[i] - mx);
    total += s[i];
  }
  for (int i = 0; i < n; ++i) s[i] /= total;
}

// src/local_head.rs:1021-1064: one query, n keys, all heads; keys / values
// [n][dim]; mask[r] == 0 removes key r
void attention(const float* q, const float* keys, const float* values, int n, const float* mask,
               float* out) {
  const int hd = kDim / kHeads;
  const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
  std::vector<float> scores(n);
  for (int h = 0; h < kHeads; ++h) {
    for (int r = 0; r < n; ++r) {
      float acc = 0.0f;
      for (int d = 0; d < hd; ++d) acc += q[h * hd + d] * keys[r * kDim + h * hd + d];
      scores[r] = acc * scale;
      if (mask && mask[r] == 0.0f) scores[r] = -INFINITY;
    }
    softmax(scores.data(), n);
    for (int d = 0; d < hd; ++d) {
      float acc = 0.0f;
      for (int r = 0; r < n; ++r) acc += scores[r] * values[r * kDim + h * hd + d];
      out[h * hd + d] = acc;
    }
  }
}

// in-place radix-2 FFT (512 points), f64
void fft512(std::complex<double>* a) {
  for (int i = 1, j = 0; i < kNfft; ++i) {
    int bit = kNfft >> 1;
    for (; j & bit; bit >>= 1) j ^= bit;
    j ^= bit;
    if (i < j) std::swap(a[i], a[j]);
  }
  for (int len = 2; len <= kNfft; len <<= 1) {
    const double ang = -2.0 * M_PI / len;
    for (int i = 0; i < kNfft; i += len)
      for (int k = 0; k < len / 2; ++k) {
        const std::complex<double> w(std::cos(ang * k), std::sin(ang * k));
        const std::complex<double> u = a[i + k], v = a[i + k + len / 2] * w;
        a[i + k] = u + v;
        a[i + k + len / 2] = u - v;
      }
  }
}

}  // namespace

struct or_local_head {
  std::vector<float> conv1_w, conv1_b, conv2_w, conv2_b, ctx_w, ctx_b, role, endpoint;
  std::vector<float> cq, ck, cv, cbq, cbk, cbv, co_w, co_b;
  std::vector<float> aq, ak, av, abq, abk, abv, ao_w, ao_b;
  std::vector<float> qn_w, qn_b, an_w, an_b, act_w, bnd_w, prior;
  float act_b = 0, bnd_b = 0, derivative_scale = 0;
  std::vector<float> mean, stdv, hann, bank;
};

extern "C" {

// src/local_head.rs:810-916: the package's F32 tensors by name and shape
or_local_head* or_lh_load(const qa_tensor* t, int n, const float* mean, const float* stdv,
                          char* err, int err_len) {
  auto fail = [&](const std::string& m) -> or_local_head* {
    if (err && err_len > 0) std::snprintf(err, err_len, "%s", m.c_str());
    return nullptr;
  };
  auto find = [&](const char* name, std::vector<int64_t> shape,
                  std::vector<float>& dst) -> bool {
    for (int i = 0; i < n; ++i) {
      if (std::strcmp(t[i].name, name)) continue;
      if (t[i].dtype != QA_DTYPE_F32 || t[i].ndim != static_cast<int>(shape.size())) return false;
      size_t count = 1;
      for (int d = 0; d < t[i].ndim; ++d) {
        if (t[i].shape[d] != shape[d]) return false;
        count *= static_cast<size_t>(shape[d]);
      }
      const float* p = static_cast<const float*>(t[i].data);
      dst.assign(p, p + count);
      return true;
    }
    return false;
  };
  auto* h = new or_local_head();
  std::vector<float> w, b, s;
  bool ok = find("audio.0.weight", {kDim, kFeat, 5}, h->conv1_w) &&
            find("audio.0.bias", {kDim}, h->conv1_b) &&
            find("audio.2.weight", {kDim, kDim, 5}, h->conv2_w) &&
            find("audio.2.bias", {kDim}, h->conv2_b) &&
            find("context_projection.weight", {kDim, kQwen}, h->ctx_w) &&
            find("context_projection.bias", {kDim}, h->ctx_b) &&
            find("role_embedding.weight", {4, kDim}, h->role) &&
            find("endpoint_embedding.weight", {2, kDim}, h->endpoint) &&
            find("context_attention.out_proj.weight", {kDim, kDim}, h->co_w) &&
            find("context_attention.out_proj.bias", {kDim}, h->co_b) &&
            find("audio_attention.out_proj.weight", {kDim, kDim}, h->ao_w) &&
            find("audio_attention.out_proj.bias", {kDim}, h->ao_b) &&
            find("query_norm.weight", {kDim}, h->qn_w) && find("query_norm.bias", {kDim}, h->qn_b) &&
            find("audio_norm.weight", {kDim}, h->an_w) && find("audio_norm.bias", {kDim}, h->an_b) &&
            find("activity_bias.weight", {1, kDim}, h->act_w) &&
            find("boundary_bias.weight", {1, kDim}, h->bnd_w) &&
            find("qwen_prior", {kOffsets}, h->prior);
  // nn.MultiheadAttention packs q, k, v in one [3 dim, dim] matrix
  auto split = [&](const char* name, std::vector<float>& q, std::vector<float>& k,
                   std::vector<float>& v, std::vector<float>& bq, std::vector<float>& bk,
                   std::vector<float>& bv) -> bool {
    const std::string pw = std::string(name) + ".in_proj_weight";
    const std::string pb = std::string(name) + ".in_proj_bias";
    if (!find(pw.c_str(), {3 * kDim, kDim}, w) || !find(pb.c_str(), {3 * kDim}, b)) return false;
    const size_t blk = static_cast<size_t>(kDim) * kDim;
    q.assign(w.begin(), w.begin() + blk);
    k.assign(w.begin() + blk, w.begin() + 2 * blk);
    v.assign(w.begin() + 2 * blk, w.end());
    bq.assign(b.begin(), b.begin() + kDim);
    bk.assign(b.begin() + kDim, b.begin() + 2 * kDim);
    bv.assign(b.begin() + 2 * kDim, b.end());
    return true;
  };
  ok = ok && split("context_attention", h->cq, h->ck, h->cv, h->cbq, h->cbk, h->cbv) &&
       split("audio_attention", h->aq, h->ak, h->av, h->abq, h->abk, h->abv);
  ok = ok && find("activity_bias.bias", {1}, s);
  if (ok) h->act_b = s[0];
  ok = ok && find("boundary_bias.bias", {1}, s);
  if (ok) h->bnd_b = s[0];
  // derivative_scale: an F32 tensor of one element, whatever its rank
  // (src/local_head.rs:834-846 checks the byte count only)
  bool found_scale = false;
  for (int i = 0; ok && i < n; ++i) {
    if (std::strcmp(t[i].name, "derivative_scale") || t[i].dtype != QA_DTYPE_F32) continue;
    long long count = 1;
    for (int d = 0; d < t[i].ndim; ++d) count *= t[i].shape[d];
    if (count != 1) continue;
    h->derivative_scale = *static_cast<const float*>(t[i].data);
    found_scale = true;
  }
  if (!ok || !found_scale) {
    delete h;
    return fail("local head package: missing or mis-shaped tensor");
  }
  h->mean.assign(mean, mean + kFeat);
  h->stdv.assign(stdv, stdv + kFeat);
  h->hann = hann(kFrameLen);
  h->bank = mel_bank();
  return h;
}

void or_lh_free(or_local_head* h) { delete h; }

// --- primitives exposed for the reference's unit tests (src/local_head.rs:1136-1207)
void or_lh_hann(int n, float* out) {
  const std::vector<float> w = hann(n);
  std::copy(w.begin(), w.end(), out);
}
void or_lh_mel_bank(float* out) {
  const std::vector<float> b = mel_bank();
  std::copy(b.begin(), b.end(), out);
}
void or_lh_band_edges(int bins, int* out) { band_edges(bins, out); }

// src/local_head.rs:1066-1069
int64_t or_lh_valid_class_count(double duration_ms, int64_t class_count) {
  const long long by_audio = static_cast<long long>(std::floor(duration_ms / kSegmentMs)) + 1;
  return std::min<long long>(std::max<long long>(by_audio, 1), class_count);
}

// src/local_head.rs:1084-1100
void or_lh_remove_overlaps(double* iv, int n) {
  for (int i = 0; i + 1 < n; ++i) {
    if (iv[2 * i + 1] <= iv[2 * (i + 1)]) continue;
    double cut = iv[2 * (i + 1)];
    const double minimum_cut = iv[2 * i] + kMinWordMs;
    if (cut < minimum_cut) {
      cut = minimum_cut;
      iv[2 * (i + 1)] = cut;
      iv[2 * (i + 1) + 1] = std::max(iv[2 * (i + 1) + 1], cut + kMinWordMs);
    }
    iv[2 * i + 1] = cut;
  }
}

// src/local_head.rs:1102-1130
void or_lh_bound_to_duration(double* iv, int n, double duration_ms) {
  if (n <= 0) return;
  const double minimum = std::min(kMinWordMs, duration_ms / n);
  bool inside = true;
  for (int i = 0; i < n; ++i) {
    const double s = iv[2 * i], e = iv[2 * i + 1];
    if (!(std::isfinite(s) && std::isfinite(e) && s >= 0.0 && s < e && e <= duration_ms))
      inside = false;
  }
  if (inside) return;
  double cursor = 0.0;
  for (int i = 0; i < n; ++i) {
    double s = iv[2 * i], e = iv[2 * i + 1];
    if (!std::isfinite(s) || !std::isfinite(e)) {
      s = 0.0;
      e = duration_ms;
    }
    const double remaining = static_cast<double>(n - i - 1);
    const double latest_start = duration_ms - minimum * (remaining + 1.0);
    s = std::min(std::max(s, cursor), latest_start);
    const double earliest_end = s + minimum;
    const double latest_end = duration_ms - minimum * remaining;
    e = std::min(std::max(e, earliest_end), latest_end);
    iv[2 * i] = s;
    iv[2 * i + 1] = e;
    cursor = e;
  }
}

// src/local_head.rs:359-507 (features_one): [41][91], normalised
void or_lh_features_one(const or_local_head* h, const float* samples, int64_t n, int64_t center_ms,
                        float* dst) {
  const int64_t center = center_ms * kSampleRate / 1000;
  std::vector<float> frames(static_cast<size_t>(kFrames) * kFrameLen, 0.0f);
  for (int f = 0; f < kFrames; ++f) {
    const int64_t start =
        center + static_cast<int64_t>(f - kContextFrames) * kHop - kFrameLen / 2;
    for (int i = 0; i < kFrameLen; ++i) {
      const int64_t idx = start + i;
      if (idx >= 0 && idx < n) frames[static_cast<size_t>(f) * kFrameLen + i] = samples[idx] * h->hann[i];
    }
  }
  std::vector<float> mag(static_cast<size_t>(kFrames) * kBins);
  std::vector<std::complex<double>> buf(kNfft);
  for (int f = 0; f < kFrames; ++f) {
    std::fill(buf.begin(), buf.end(), std::complex<double>(0.0, 0.0));
    for (int i = 0; i < kFrameLen; ++i) buf[i] = frames[static_cast<size_t>(f) * kFrameLen + i];
    fft512(buf.data());
    for (int b = 0; b < kBins; ++b) mag[static_cast<size_t>(f) * kBins + b] = static_cast<float>(std::abs(buf[b]));
  }
  std::vector<float> power(mag.size());
  for (size_t i = 0; i < mag.size(); ++i) power[i] = mag[i] * mag[i];
  std::vector<float> log_mel(static_cast<size_t>(kFrames) * kMels);
  for (int f = 0; f < kFrames; ++f)
    for (int m = 0; m < kMels; ++m) {
      float acc = 0.0f;
      for (int b = 0; b < kBins; ++b) acc += h->bank[static_cast<size_t>(m) * kBins + b] * power[static_cast<size_t>(f) * kBins + b];
      log_mel[static_cast<size_t>(f) * kMels + m] = std::log(std::max(acc, kLogEps));
    }
  float log_rms[kFrames], delta_rms[kFrames];
  for (int f = 0; f < kFrames; ++f) {
    float acc = 0.0f;
    for (int i = 0; i < kFrameLen; ++i) {
      const float v = frames[static_cast<size_t>(f) * kFrameLen + i];
      acc += v * v;
    }
    log_rms[f] = std::log(std::max(std::sqrt(acc / kFrameLen + kLogEps), kLogEps));
    delta_rms[f] = f == 0 ? 0.0f : log_rms[f] - log_rms[f - 1];
  }
  std::vector<float> nrm(static_cast<size_t>(kFrames) * kBins);
  for (int f = 0; f < kFrames; ++f) {
    float mean = 0.0f;
    for (int b = 0; b < kBins; ++b) {
      const float v = std::log(std::max(mag[static_cast<size_t>(f) * kBins + b], kLogEps));
      nrm[static_cast<size_t>(f) * kBins + b] = v;
      mean += v;
    }
    mean /= kBins;
    for (int b = 0; b < kBins; ++b) nrm[static_cast<size_t>(f) * kBins + b] -= mean;
  }
  float flux[kFrames];
  flux[0] = 0.0f;
  for (int f = 1; f < kFrames; ++f) {
    float positive = 0.0f, total = 0.0f;
    for (int b = 0; b < kBins; ++b) {
      const float cur = mag[static_cast<size_t>(f) * kBins + b], prev = mag[static_cast<size_t>(f - 1) * kBins + b];
      positive += std::max(cur - prev, 0.0f);
      total += prev;
    }
    flux[f] = positive / (total + kLogEps);
  }
  int edges[kBands + 1];
  band_edges(kBins, edges);
  float dist[kFrames][2 * kBands];
  for (int band = 0; band < kBands; ++band) {
    const int left = edges[band], right = std::max(edges[band + 1], left + 1);
    for (int f = 0; f < kFrames; ++f) {
      const float* cur = &nrm[static_cast<size_t>(f) * kBins + left];
      const float* nl = f == 0 ? cur : &nrm[static_cast<size_t>(f - 1) * kBins + left];
      const float* nr = f + 1 == kFrames ? cur : &nrm[static_cast<size_t>(f + 1) * kBins + left];
      float al = 0.0f, ar = 0.0f;
      for (int i = 0; i < right - left; ++i) {
        al += std::fabs(cur[i] - nl[i]);
        ar += std::fabs(cur[i] - nr[i]);
      }
      const float width = static_cast<float>(right - left);
      dist[f][band] = al / width;
      dist[f][kBands + band] = ar / width;
    }
  }
  for (int f = 0; f < kFrames; ++f) {
    float* row = dst + static_cast<size_t>(f) * kFeat;
    for (int m = 0; m < kMels; ++m) row[m] = log_mel[static_cast<size_t>(f) * kMels + m];
    row[kMels] = log_rms[f];
    row[kMels + 1] = delta_rms[f];
    row[kMels + 2] = flux[f];
    for (int k = 0; k < 2 * kBands; ++k) row[kMels + 3 + k] = dist[f][k];
    for (int c = 0; c < kFeat; ++c) row[c] = (row[c] - h->mean[c]) / h->stdv[c];
  }
}

// src/local_head.rs:509-611 (endpoint_offset): feat [41][91], ctx [4][1024]
float or_lh_endpoint_offset(const or_local_head* h, const float* feat, const float* ctx,
                            const float* mask, int is_end) {
  std::vector<float> ha(static_cast<size_t>(kDim) * kFrames), hb(static_cast<size_t>(kDim) * kFrames);
  for (int c = 0; c < kDim; ++c)
    for (int t = 0; t < kFrames; ++t) {
      float acc = h->conv1_b[c];
      for (int k = 0; k < 5; ++k) {
        const int tt = t + k - 2;
        if (tt < 0 || tt >= kFrames) continue;
        for (int ic = 0; ic < kFeat; ++ic)
          acc += h->conv1_w[(static_cast<size_t>(c) * kFeat + ic) * 5 + k] * feat[static_cast<size_t>(tt) * kFeat + ic];
      }
      ha[static_cast<size_t>(c) * kFrames + t] = gelu(acc);
    }
  for (int c = 0; c < kDim; ++c)
    for (int t = 0; t < kFrames; ++t) {
      float acc = h->conv2_b[c];
      for (int k = 0; k < 5; ++k) {
        const int tt = t + k - 2;
        if (tt < 0 || tt >= kFrames) continue;
        for (int ic = 0; ic < kDim; ++ic)
          acc += h->conv2_w[(static_cast<size_t>(c) * kDim + ic) * 5 + k] * ha[static_cast<size_t>(ic) * kFrames + tt];
      }
      hb[static_cast<size_t>(c) * kFrames + t] = gelu(acc);
    }
  std::vector<float> audio(static_cast<size_t>(kFrames) * kDim);
  for (int t = 0; t < kFrames; ++t)
    for (int d = 0; d < kDim; ++d) audio[static_cast<size_t>(t) * kDim + d] = hb[static_cast<size_t>(d) * kFrames + t];

  std::vector<float> tokens(4 * kDim);
  for (int r = 0; r < 4; ++r)
    for (int d = 0; d < kDim; ++d) {
      float acc = h->ctx_b[d] + h->role[r * kDim + d];
      for (int j = 0; j < kQwen; ++j) acc += h->ctx_w[static_cast<size_t>(d) * kQwen + j] * ctx[r * kQwen + j];
      tokens[r * kDim + d] = acc;
    }
  std::vector<float> base(kDim);
  for (int d = 0; d < kDim; ++d) base[d] = tokens[d] + h->endpoint[is_end * kDim + d];
  auto proj = [&](const float* x, const std::vector<float>& w, const std::vector<float>& b,
                  float* out) {
    for (int d = 0; d < kDim; ++d) {
      float acc = b[d];
      for (int j = 0; j < kDim; ++j) acc += w[static_cast<size_t>(d) * kDim + j] * x[j];
      out[d] = acc;
    }
  };
  std::vector<float> q(kDim), att(kDim), projd(kDim), keys(static_cast<size_t>(kFrames) * kDim),
      vals(static_cast<size_t>(kFrames) * kDim);
  proj(base.data(), h->cq, h->cbq, q.data());
  for (int r = 0; r < 4; ++r) {
    proj(&tokens[r * kDim], h->ck, h->cbk, &keys[r * kDim]);
    proj(&tokens[r * kDim], h->cv, h->cbv, &vals[r * kDim]);
  }
  attention(q.data(), keys.data(), vals.data(), 4, mask, att.data());
  proj(att.data(), h->co_w, h->co_b, projd.data());
  std::vector<float> query(kDim);
  for (int d = 0; d < kDim; ++d) query[d] = projd[d] + base[d];
  layer_norm(query.data(), kDim, h->qn_w.data(), h->qn_b.data());

  proj(query.data(), h->aq, h->abq, q.data());
  for (int t = 0; t < kFrames; ++t) {
    proj(&audio[static_cast<size_t>(t) * kDim], h->ak, h->abk, &keys[static_cast<size_t>(t) * kDim]);
    proj(&audio[static_cast<size_t>(t) * kDim], h->av, h->abv, &vals[static_cast<size_t>(t) * kDim]);
  }
  attention(q.data(), keys.data(), vals.data(), kFrames, nullptr, att.data());
  proj(att.data(), h->ao_w, h->ao_b, projd.data());
  for (int d = 0; d < kDim; ++d) query[d] = projd[d] + query[d];
  layer_norm(query.data(), kDim, h->qn_w.data(), h->qn_b.data());
  for (int t = 0; t < kFrames; ++t)
    layer_norm(&audio[static_cast<size_t>(t) * kDim], kDim, h->an_w.data(), h->an_b.data());

  const float root = std::sqrt(static_cast<float>(kDim));
  float activity[kFrames];
  for (int t = 0; t < kFrames; ++t) {
    const float* row = &audio[static_cast<size_t>(t) * kDim];
    activity[t] = dot(row, query.data(), kDim) / root + dot(h->act_w.data(), row, kDim) + h->act_b;
  }
  float logits[kOffsets];
  for (int j = 0; j < kOffsets; ++j) {
    const float* row = &audio[static_cast<size_t>(14 + j) * kDim];
    const float local = dot(row, query.data(), kDim) / root + dot(h->bnd_w.data(), row, kDim) + h->bnd_b;
    const float derivative = activity[14 + j] - activity[14 + j - 1];
    const float direction = is_end == 0 ? derivative : -derivative;
    logits[j] = local + h->derivative_scale * direction + h->prior[j];
  }
  // softmax_scaled (src/local_head.rs:1014-1017), then the expected offset
  for (int j = 0; j < kOffsets; ++j) logits[j] = logits[j] / kTemperature;
  softmax(logits, kOffsets);
  float off = 0.0f;
  for (int j = 0; j < kOffsets; ++j) off += logits[j] * kOffsetsMs[j];
  return off;
}

// src/local_head.rs:189-307 (refine): W words; logits [2W][n_labels], hidden
// [2W][1024] (the unfolded final-norm rows); out [W][2] seconds; also the
// fixed centres and the offsets when the pointers are non-null
int or_lh_refine(const or_local_head* h, const float* samples, int64_t n, int W,
                 const float* logits, int n_labels, const float* hidden, int hidden_size,
                 double* out, int64_t* fixed_out, float* offsets_out) {
  if (W <= 0 || n <= 0 || n_labels <= 0 || hidden_size != kQwen) return 1;
  const int slots = 2 * W;
  const double duration_ms = static_cast<double>(n) * 1000.0 / kSampleRate;
  const int64_t valid = or_lh_valid_class_count(duration_ms, n_labels);
  std::vector<int64_t> raw(slots), fixed(slots);
  for (int s = 0; s < slots; ++s) {
    const float* row = logits + static_cast<size_t>(s) * n_labels;
    int best = 0;
    float bv = -INFINITY;
    for (int i = 0; i < valid; ++i)
      if (row[i] > bv) {
        bv = row[i];
        best = i;
      }
    raw[s] = static_cast<int64_t>(best * kSegmentMs);
  }
  or_fix_timestamps(raw.data(), slots, fixed.data());
  // context rows: [slot, current avg, prev avg, next avg] (src/local_head.rs:309-346)
  auto mean = [&](int a, int b, float* dst) {
    for (int d = 0; d < kQwen; ++d) dst[d] = 0.0f;
    for (int i = a; i < b; ++i)
      for (int d = 0; d < kQwen; ++d) dst[d] += hidden[static_cast<size_t>(i) * kQwen + d];
    const float cnt = static_cast<float>(b - a);
    for (int d = 0; d < kQwen; ++d) dst[d] /= cnt;
  };
  std::vector<float> offsets(slots);
  std::vector<float> cur(kQwen), prev(kQwen), next(kQwen), ctx(4 * kQwen),
      feat(static_cast<size_t>(kFrames) * kFeat);
  for (int w = 0; w < W; ++w) {
    mean(2 * w, 2 * w + 2, cur.data());
    if (w > 0) mean(2 * w - 2, 2 * w, prev.data()); else std::fill(prev.begin(), prev.end(), 0.0f);
    if (w + 1 < W) mean(2 * w + 2, 2 * w + 4, next.data()); else std::fill(next.begin(), next.end(), 0.0f);
    for (int e = 0; e < 2; ++e) {
      const int slot = 2 * w + e;
      std::memcpy(&ctx[0], hidden + static_cast<size_t>(slot) * kQwen, kQwen * 4);
      std::memcpy(&ctx[kQwen], cur.data(), kQwen * 4);
      std::memcpy(&ctx[2 * kQwen], prev.data(), kQwen * 4);
      std::memcpy(&ctx[3 * kQwen], next.data(), kQwen * 4);
      const float mask[4] = {1.0f, 1.0f, w > 0 ? 1.0f : 0.0f, w + 1 < W ? 1.0f : 0.0f};
      or_lh_features_one(h, samples, n, fixed[slot], feat.data());
      offsets[slot] = or_lh_endpoint_offset(h, feat.data(), ctx.data(), mask, e);
    }
  }
  // corrected intervals, in the reference's order (src/local_head.rs:256-296)
  std::vector<double> iv(2 * static_cast<size_t>(W));
  for (int i = 0; i < W; ++i) {
    const double fs = static_cast<double>(fixed[2 * i]), fe = static_cast<double>(fixed[2 * i + 1]);
    double s = fs + offsets[2 * i], e = fe + offsets[2 * i + 1];
    if (!std::isfinite(s) || !std::isfinite(e)) {
      s = fs;
      e = fe;
    } else if (e - s < kMinWordMs) {
      const double mid = (s + e) / 2.0;
      if (mid < kMinWordMs / 2.0) {
        s = 0.0;
        e = kMinWordMs;
      } else {
        s = mid - kMinWordMs / 2.0;
        e = mid + kMinWordMs / 2.0;
      }
    } else if (s < 0.0) {
      e -= s;
      s = 0.0;
    }
    if (!std::isfinite(s) || !std::isfinite(e) || s < 0.0 || e < 0.0 || e - s < kMinWordMs) {
      s = 0.0;
      e = kMinWordMs;
    }
    iv[2 * i] = s;
    iv[2 * i + 1] = e;
  }
  or_lh_remove_overlaps(iv.data(), W);
  or_lh_bound_to_duration(iv.data(), W, duration_ms);
  for (int i = 0; i < 2 * W; ++i) out[i] = iv[i] / 1000.0;
  if (fixed_out) std::copy(fixed.begin(), fixed.end(), fixed_out);
  if (offsets_out) std::copy(offsets.begin(), offsets.end(), offsets_out);
  return 0;
}

}  // extern "C"
