// TEST INFRASTRUCTURE (parity oracle / CPU baseline).
//
// The CPU audio tower, restated from src/audio_encoder.rs (CpuAudioEncoder):
// chunking (:754-790), conv stem of three 3x3/s2/p1 convolutions via im2col +
// GEMM + bias + erf-GELU (:207-236, :361-447), permute + conv_out + sinusoidal
// PE (:295-357), packing of valid tokens (:797-804), 18 pre-LN layers with
// windowed attention (:466-690) and ln_post + proj1 + GELU + proj2
// (:816-821).  All f32, as in the reference.
#include <omp.h>

#include <algorithm>

#include "model.h"

namespace {

// src/audio_encoder.rs:693-696
int64_t feo(int64_t ifr) {
  auto f = [](int64_t l) { return (l - 1) / 2 + 1; };
  return f(f(f(ifr)));
}

// src/audio_encoder.rs:207-236: cols [b*ho*wo][c_in*9], k = ic*9 + kh*3 + kw
void im2col(const float* x, int b, int c_in, int h, int w, std::vector<float>& cols, int& ho,
            int& wo) {
  ho = (h + 2 - 3) / 2 + 1;
  wo = (w + 2 - 3) / 2 + 1;
  const int64_t count = static_cast<int64_t>(b) * ho * wo;
  const int k = c_in * 9;
  cols.assign(static_cast<size_t>(count) * k, 0.0f);
#pragma omp parallel for schedule(static)
  for (int64_t ci = 0; ci < count; ++ci) {
    const int ib = static_cast<int>(ci / (ho * wo));
    const int rem = static_cast<int>(ci % (ho * wo));
    const int oh = rem / wo, ow = rem % wo;
    float* col = &cols[static_cast<size_t>(ci) * k];
    for (int ic = 0; ic < c_in; ++ic)
      for (int kh = 0; kh < 3; ++kh)
        for (int kw = 0; kw < 3; ++kw) {
          const int ih = oh * 2 + kh - 1, iw = ow * 2 + kw - 1;
          col[ic * 9 + kh * 3 + kw] =
              (ih < 0 || ih >= h || iw < 0 || iw >= w)
                  ? 0.0f
                  : x[((static_cast<size_t>(ib) * c_in + ic) * h + ih) * w + iw];
        }
  }
}

// src/audio_encoder.rs:361-447 (conv_block): act [b][c_out][ho*wo] =
// gelu(W · col + bias), processed in batch tiles of 8 chunks (CONV_TILE).
std::vector<float> conv_block(const float* x, int b, int c_in, int h, int w,
                              const std::vector<float>& W, const std::vector<float>& bias,
                              int c_out, int& ho, int& wo) {
  ho = (h + 2 - 3) / 2 + 1;
  wo = (w + 2 - 3) / 2 + 1;
  const int plane = ho * wo;
  const int k = c_in * 9;
  const int64_t in_plane = static_cast<int64_t>(c_in) * h * w;
  std::vector<float> act(static_cast<size_t>(b) * c_out * plane);
  const int tile = 8;
  std::vector<float> cols, scratch;
  for (int b0 = 0; b0 < b; b0 += tile) {
    const int nb = std::min(tile, b - b0);
    int h2, w2;
    im2col(x + b0 * in_plane, nb, c_in, h, w, cols, h2, w2);
    const int count = nb * plane;
    scratch.assign(static_cast<size_t>(c_out) * count, 0.0f);
    // raw[c_out][count] = W[c_out][k] · cols[count][k]ᵀ
    orc::gemm(W.data(), k, cols.data(), k, scratch.data(), count, c_out, count, k, false);
#pragma omp parallel for schedule(static)
    for (int pi = 0; pi < nb * c_out; ++pi) {
      const int ib = pi / c_out, oc = pi % c_out;
      const float bv = bias[oc];
      const float* src = &scratch[static_cast<size_t>(oc) * count + static_cast<size_t>(ib) * plane];
      float* dst = &act[(static_cast<size_t>(b0 + ib) * c_out + oc) * plane];
      for (int i = 0; i < plane; ++i) dst[i] = orc::gelu_erf(src[i] + bv);
    }
  }
  return act;
}

// CpuAudioLinear::forward (src/audio_encoder.rs:133-143): y = x·Wᵀ + b
std::vector<float> linear(const std::vector<float>& x, int rows, int in, const std::vector<float>& W,
                          int out, const std::vector<float>* b) {
  std::vector<float> y(static_cast<size_t>(rows) * out);
  orc::gemm(x.data(), in, W.data(), in, y.data(), out, rows, out, in, false);
  if (b && !b->empty()) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r)
      for (int j = 0; j < out; ++j) y[static_cast<size_t>(r) * out + j] += (*b)[j];
  }
  return y;
}

// CpuAudioLayerNorm::forward (src/audio_encoder.rs:170-191): serial sums
std::vector<float> layer_norm(const std::vector<float>& x, int rows, int d,
                              const std::vector<float>& w, const std::vector<float>& b) {
  std::vector<float> o(x.size());
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    const float* xr = &x[static_cast<size_t>(r) * d];
    float mean = 0.0f;
    for (int j = 0; j < d; ++j) mean += xr[j];
    mean /= static_cast<float>(d);
    float var = 0.0f;
    for (int j = 0; j < d; ++j) {
      const float t = xr[j] - mean;
      var += t * t;
    }
    var /= static_cast<float>(d);
    const float inv = 1.0f / std::sqrt(var + 1e-5f);
    float* orow = &o[static_cast<size_t>(r) * d];
    for (int j = 0; j < d; ++j) orow[j] = (xr[j] - mean) * inv * w[j] + b[j];
  }
  return o;
}

// attention_window (src/audio_encoder.rs:574-627) over every window of `ws`
// tokens (the last one short), flattened back to [s, nh*hd] (:495-555).
std::vector<float> windowed_attention(const std::vector<float>& q, const std::vector<float>& k,
                                      const std::vector<float>& v, int s, int dm, int nh, int ws) {
  const int hd = dm / nh;
  const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
  const int window = (ws > 0 && ws < s) ? ws : s;
  std::vector<float> out(static_cast<size_t>(s) * dm, 0.0f);
  const int nwin = (s + window - 1) / window;
#pragma omp parallel
  {
    std::vector<float> scores(window);
#pragma omp for collapse(2) schedule(dynamic)
    for (int wi = 0; wi < nwin; ++wi)
      for (int h = 0; h < nh; ++h) {
        const int st = wi * window, len = std::min(window, s - st);
        for (int qi = 0; qi < len; ++qi) {
          const float* qr = &q[static_cast<size_t>(st + qi) * dm + h * hd];
          float mx = -INFINITY;
          for (int ki = 0; ki < len; ++ki) {
            const float* kr = &k[static_cast<size_t>(st + ki) * dm + h * hd];
            float dot = 0.0f;
            for (int j = 0; j < hd; ++j) dot += qr[j] * kr[j];
            const float sc = dot * scale;
            scores[ki] = sc;
            mx = sc > mx ? sc : mx;
          }
          float sum = 0.0f;
          for (int ki = 0; ki < len; ++ki) {
            scores[ki] = std::exp(scores[ki] - mx);
            sum += scores[ki];
          }
          const float inv = 1.0f / sum;
          float* orow = &out[static_cast<size_t>(st + qi) * dm + h * hd];
          for (int ki = 0; ki < len; ++ki) {
            const float wgt = scores[ki] * inv;
            const float* vr = &v[static_cast<size_t>(st + ki) * dm + h * hd];
            for (int j = 0; j < hd; ++j) orow[j] += wgt * vr[j];
          }
        }
      }
  }
  return out;
}

}  // namespace

extern "C" int or_audio_embeds(or_model* m, const float* mel, int mel_len, float* out,
                               int64_t out_len) {
  const qa_cfg& c = m->cfg;
  const int n_mels = c.num_mel_bins;
  const int cs = c.n_window * 2;
  const int64_t tpc = feo(cs);
  const int nfull = mel_len / cs, tail = mel_len % cs;
  const int n_chunks = nfull + (tail > 0 ? 1 : 0);
  if (n_chunks == 0) return QA_ERR_SHAPE;
  std::vector<int64_t> chunk_tokens;
  // chunked [n_chunks][n_mels][cs], zero padded (src/audio_encoder.rs:763-790)
  std::vector<float> chunked(static_cast<size_t>(n_chunks) * n_mels * cs, 0.0f);
  for (int i = 0; i < n_chunks; ++i) {
    const int len = i < nfull ? cs : tail;
    for (int mm = 0; mm < n_mels; ++mm)
      for (int j = 0; j < len; ++j)
        chunked[(static_cast<size_t>(i) * n_mels + mm) * cs + j] =
            mel[static_cast<size_t>(mm) * mel_len + static_cast<size_t>(i) * cs + j];
    chunk_tokens.push_back(i < nfull ? tpc : feo(tail));
  }
  int64_t n_total = 0;
  for (auto t : chunk_tokens) n_total += t;
  if (out_len < n_total * c.output_dim) return QA_ERR_SHAPE;

  int h1, w1, h2, w2, h3, w3;
  auto x1 = conv_block(chunked.data(), n_chunks, 1, n_mels, cs, m->c1w, m->c1b, m->c1_out, h1, w1);
  auto x2 = conv_block(x1.data(), n_chunks, m->c1_out, h1, w1, m->c2w, m->c2b, m->c2_out, h2, w2);
  auto x3 = conv_block(x2.data(), n_chunks, m->c2_out, h2, w2, m->c3w, m->c3b, m->c3_out, h3, w3);
  const int t2 = w3, cdim = m->c3_out, fdim = h3, row = cdim * fdim;
  if (row != m->co_in) return QA_ERR_WEIGHTS;
  // permute [b, c, f, t] -> [b, t, c*f] (src/audio_encoder.rs:318-335)
  std::vector<float> perm(static_cast<size_t>(n_chunks) * t2 * row);
#pragma omp parallel for schedule(static)
  for (int idx = 0; idx < n_chunks * t2; ++idx) {
    const int ib = idx / t2, it = idx % t2;
    for (int ic = 0; ic < cdim; ++ic)
      for (int f = 0; f < fdim; ++f)
        perm[static_cast<size_t>(idx) * row + ic * fdim + f] =
            x3[((static_cast<size_t>(ib) * cdim + ic) * fdim + f) * t2 + it];
  }
  const int dm = c.d_model;
  auto co = linear(perm, n_chunks * t2, row, m->co_w, dm, m->co_b.empty() ? nullptr : &m->co_b);
  for (int idx = 0; idx < n_chunks * t2; ++idx) {
    const int it = idx % t2;
    for (int j = 0; j < dm; ++j) co[static_cast<size_t>(idx) * dm + j] += m->pe[static_cast<size_t>(it) * dm + j];
  }
  // pack valid tokens (src/audio_encoder.rs:797-804)
  std::vector<float> h;
  h.reserve(static_cast<size_t>(n_total) * dm);
  for (int i = 0; i < n_chunks; ++i) {
    const size_t base = static_cast<size_t>(i) * t2 * dm;
    h.insert(h.end(), co.begin() + base, co.begin() + base + chunk_tokens[i] * dm);
  }
  const int s = static_cast<int>(n_total);
  const int ws = static_cast<int>(tpc * (c.n_window_infer / cs));
  for (const EncLayer& L : m->enc) {
    auto nrm = layer_norm(h, s, dm, L.ln1_w, L.ln1_b);
    auto q = linear(nrm, s, dm, L.q_w, dm, &L.q_b);
    auto k = linear(nrm, s, dm, L.k_w, dm, &L.k_b);
    auto v = linear(nrm, s, dm, L.v_w, dm, &L.v_b);
    auto att = windowed_attention(q, k, v, s, dm, c.encoder_heads, ws);
    auto o = linear(att, s, dm, L.o_w, dm, &L.o_b);
    for (size_t i = 0; i < h.size(); ++i) h[i] += o[i];
    auto nrm2 = layer_norm(h, s, dm, L.ln2_w, L.ln2_b);
    auto f1 = linear(nrm2, s, dm, L.fc1_w, c.encoder_ffn_dim, &L.fc1_b);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < static_cast<int64_t>(f1.size()); ++i) f1[i] = orc::gelu_erf(f1[i]);
    auto f2 = linear(f1, s, c.encoder_ffn_dim, L.fc2_w, dm, &L.fc2_b);
    for (size_t i = 0; i < h.size(); ++i) h[i] += f2[i];
  }
  auto hp = layer_norm(h, s, dm, m->lnp_w, m->lnp_b);
  auto p1 = linear(hp, s, dm, m->p1_w, dm, &m->p1_b);
  for (auto& x : p1) x = orc::gelu_erf(x);
  auto p2 = linear(p1, s, dm, m->p2_w, c.output_dim, &m->p2_b);
  std::copy(p2.begin(), p2.end(), out);
  return QA_OK;
}
