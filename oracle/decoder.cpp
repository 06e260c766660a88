// TEST INFRASTRUCTURE (parity oracle / CPU baseline).
//
// The CPU text decoder, restated from src/cpu_decoder.rs:283-547
// (CpuTextDecoder::forward / prefill_hidden) with its f16 rounding points:
// norm output, each of q/k/v, the normed+roped q and k, v, the attention
// output, f16(h + acc) after o_proj and after down_proj, gate, up and
// silu(gate)·up.  Accumulation is f32.  Prefill starts at position 0
// (src/align_inference.rs:156,168).
#include <omp.h>

#include <algorithm>

#include "model.h"

namespace {

// Mat::batch_dot (src/cpu_decoder.rs:59-76): f16(x · Wᵀ)
void batch_dot(const std::vector<float>& x, int rows, const std::vector<float>& W, int out, int in,
               std::vector<float>& y) {
  y.assign(static_cast<size_t>(rows) * out, 0.0f);
  orc::gemm(x.data(), in, W.data(), in, y.data(), out, rows, out, in, false);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < static_cast<int64_t>(y.size()); ++i) y[i] = orc::r16(y[i]);
}

// Mat::batch_dot_acc (src/cpu_decoder.rs:80-97): h = f16(h + x · Wᵀ)
void batch_dot_acc(const std::vector<float>& x, int rows, const std::vector<float>& W, int out,
                   int in, std::vector<float>& h) {
  std::vector<float> acc(static_cast<size_t>(rows) * out, 0.0f);
  orc::gemm(x.data(), in, W.data(), in, acc.data(), out, rows, out, in, false);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < static_cast<int64_t>(h.size()); ++i) h[i] = orc::r16(h[i] + acc[i]);
}

// rms_norm_row (src/cpu_decoder.rs:289-300)
void rms_norm_rows(const std::vector<float>& x, int rows, int n, const std::vector<float>& w,
                   float eps, std::vector<float>& out) {
  out.resize(x.size());
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    const float* xr = &x[static_cast<size_t>(r) * n];
    float s2 = 0.0f;
    for (int i = 0; i < n; ++i) s2 += xr[i] * xr[i];
    const float inv = 1.0f / std::sqrt(s2 / static_cast<float>(n) + eps);
    float* o = &out[static_cast<size_t>(r) * n];
    for (int i = 0; i < n; ++i) o[i] = orc::r16(xr[i] * inv * w[i]);
  }
}

// norm_rope_head (src/cpu_decoder.rs:305-321)
void norm_rope_head(const float* raw, const float* nw, const float* cosr, const float* sinr, int hd,
                    float eps, float* out) {
  const int half = hd / 2;
  float s2 = 0.0f;
  for (int j = 0; j < hd; ++j) s2 += raw[j] * raw[j];
  const float inv = 1.0f / std::sqrt(s2 / static_cast<float>(hd) + eps);
  for (int j = 0; j < hd; ++j) {
    const float xj = raw[j] * inv * nw[j];
    const int pj = j < half ? j + half : j - half;
    const float sign = j < half ? -1.0f : 1.0f;
    const float xp = raw[pj] * inv * nw[pj];
    out[j] = orc::r16(xj * cosr[j] + sign * xp * sinr[j]);
  }
}

}  // namespace

extern "C" int or_text_hidden(or_model* m, const uint16_t* emb, int seq, int n_layers,
                              uint16_t* out) {
  const qa_cfg& c = m->cfg;
  if (seq <= 0) return QA_ERR_SHAPE;
  if (seq > c.max_seq) return QA_ERR_CAP;  // src/cpu_decoder.rs:527-532
  const int hs = c.hidden_size, nqh = c.num_heads, nkvh = c.num_kv_heads, hd = c.head_dim;
  const int qd = nqh * hd, kvd = nkvh * hd, inter = c.intermediate_size;
  const float eps = static_cast<float>(c.rms_norm_eps);
  const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
  const int rep = nqh / nkvh;
  const int nl = n_layers < 0 ? static_cast<int>(m->dec.size()) : std::min<int>(n_layers, m->dec.size());

  std::vector<float> x(static_cast<size_t>(seq) * hs);
  for (size_t i = 0; i < x.size(); ++i) x[i] = orc::f16_to_f32(emb[i]);
  std::vector<float> normed, q, k, v, attn(static_cast<size_t>(seq) * qd), norm2, gate, up;
  // per-layer K/V "cache" [nkvh][seq][hd] holding f16 values widened to f32
  std::vector<float> kc(static_cast<size_t>(nkvh) * seq * hd), vc(kc.size());

  for (int li = 0; li < nl; ++li) {
    const DecLayer& L = m->dec[li];
    rms_norm_rows(x, seq, hs, L.iln, eps, normed);
    batch_dot(normed, seq, L.q, qd, hs, q);
    batch_dot(normed, seq, L.k, kvd, hs, k);
    batch_dot(normed, seq, L.v, kvd, hs, v);
    // q/k norm + rope, v into the cache (src/cpu_decoder.rs:449-475)
#pragma omp parallel
    {
      std::vector<float> tmp(hd);
#pragma omp for schedule(static)
      for (int r = 0; r < seq; ++r) {
        const float* cr = &m->cos[static_cast<size_t>(r) * hd];
        const float* sr = &m->sin[static_cast<size_t>(r) * hd];
        for (int h = 0; h < nqh; ++h) {
          float* qh = &q[static_cast<size_t>(r) * qd + h * hd];
          norm_rope_head(qh, L.qn.data(), cr, sr, hd, eps, tmp.data());
          std::copy(tmp.begin(), tmp.end(), qh);
        }
        for (int h = 0; h < nkvh; ++h) {
          const float* kh = &k[static_cast<size_t>(r) * kvd + h * hd];
          norm_rope_head(kh, L.kn.data(), cr, sr, hd, eps,
                         &kc[(static_cast<size_t>(h) * seq + r) * hd]);
          std::copy(&v[static_cast<size_t>(r) * kvd + h * hd],
                    &v[static_cast<size_t>(r) * kvd + h * hd] + hd,
                    &vc[(static_cast<size_t>(h) * seq + r) * hd]);
        }
      }
    }
    // causal attention per (row, head) (src/cpu_decoder.rs:327-412)
#pragma omp parallel
    {
      std::vector<float> scores(seq), acc(hd);
#pragma omp for schedule(dynamic, 16)
      for (int64_t hi = 0; hi < static_cast<int64_t>(seq) * nqh; ++hi) {
        const int r = static_cast<int>(hi / nqh), h = static_cast<int>(hi % nqh);
        const int valid = r + 1;
        const float* qr = &q[static_cast<size_t>(r) * qd + h * hd];
        const int kh = h / rep;
        const float* kb = &kc[static_cast<size_t>(kh) * seq * hd];
        const float* vb = &vc[static_cast<size_t>(kh) * seq * hd];
        float best = -INFINITY;
        for (int t = 0; t < valid; ++t) {
          const float* kr = kb + static_cast<size_t>(t) * hd;
          float a0 = 0, a1 = 0, a2 = 0, a3 = 0;
          for (int j = 0; j < hd; j += 4) {
            a0 += qr[j] * kr[j];
            a1 += qr[j + 1] * kr[j + 1];
            a2 += qr[j + 2] * kr[j + 2];
            a3 += qr[j + 3] * kr[j + 3];
          }
          const float s = ((a0 + a1) + (a2 + a3)) * scale;
          scores[t] = s;
          best = s > best ? s : best;
        }
        float sum = 0.0f;
        for (int t = 0; t < valid; ++t) {
          scores[t] = std::exp(scores[t] - best);
          sum += scores[t];
        }
        const float inv = 1.0f / sum;
        std::fill(acc.begin(), acc.end(), 0.0f);
        for (int t = 0; t < valid; ++t) {
          const float w = scores[t] * inv;
          const float* vr = vb + static_cast<size_t>(t) * hd;
          for (int j = 0; j < hd; ++j) acc[j] += w * vr[j];
        }
        float* o = &attn[static_cast<size_t>(r) * qd + h * hd];
        for (int j = 0; j < hd; ++j) o[j] = orc::r16(acc[j]);
      }
    }
    batch_dot_acc(attn, seq, L.o, hs, qd, x);
    rms_norm_rows(x, seq, hs, L.pln, eps, norm2);
    batch_dot(norm2, seq, L.gate, inter, hs, gate);
    batch_dot(norm2, seq, L.up, inter, hs, up);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < static_cast<int64_t>(gate.size()); ++i) {
      const float g = gate[i];
      const float silu = g / (1.0f + std::exp(-g));
      gate[i] = orc::r16(silu * up[i]);
    }
    batch_dot_acc(gate, seq, L.down, hs, inter, x);
  }
  for (size_t i = 0; i < x.size(); ++i) out[i] = orc::f32_to_f16(x[i]);
  return QA_OK;
}

// Host gather + scatter (src/align_inference.rs:685-715), CPU path: f16 rows.
extern "C" int or_gather(or_model* m, const uint32_t* ids, int seq, const uint16_t* audio,
                         int n_audio, uint16_t* emb) {
  const qa_cfg& c = m->cfg;
  const int hs = c.hidden_size;
  int cursor = 0;
  for (int p = 0; p < seq; ++p) {
    uint16_t* dst = emb + static_cast<size_t>(p) * hs;
    if (static_cast<int>(ids[p]) == c.audio_token_id) {
      if (cursor >= n_audio) return QA_ERR_SHAPE;
      std::copy(audio + static_cast<size_t>(cursor) * hs, audio + static_cast<size_t>(cursor + 1) * hs, dst);
      ++cursor;
    } else {
      if (ids[p] >= static_cast<uint32_t>(c.vocab_size)) return QA_ERR_SHAPE;
      std::copy(&m->embed[static_cast<size_t>(ids[p]) * hs], &m->embed[static_cast<size_t>(ids[p] + 1) * hs], dst);
    }
  }
  return cursor == n_audio ? QA_OK : QA_ERR_SHAPE;
}
