// TEST INFRASTRUCTURE (parity oracle / CPU baseline).
//
// Final norm + timestamp head + argmax (src/align_inference.rs:737-805),
// timestamp repair (src/postprocess.rs:33-113) and the token/frame
// bookkeeping (src/align_input.rs:49-87).
#include <omp.h>

#include <algorithm>

#include "model.h"

extern "C" int or_head(or_model* m, const float* hidden, int seq, const int* rows, int n_rows,
                       int64_t* raw_ms, float* logits_out, float* normed_out, float* margin) {
  const qa_cfg& c = m->cfg;
  const int hs = c.hidden_size, nl = c.num_labels;
  const float eps = static_cast<float>(c.rms_norm_eps);
  for (int i = 0; i < n_rows; ++i)
    if (rows[i] < 0 || rows[i] >= seq) return QA_ERR_SHAPE;
  // folded norm: x·w / sqrt(mean((x·w)²) + eps) (:766-783)
  std::vector<float> normed(static_cast<size_t>(n_rows) * hs);
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n_rows; ++i) {
    const float* row = hidden + static_cast<size_t>(rows[i]) * hs;
    float acc = 0.0f;
    for (int j = 0; j < hs; ++j) {
      const float xf = row[j] * m->final_norm[j];
      acc += xf * xf;
    }
    const float inv = 1.0f / std::sqrt(acc / static_cast<float>(hs) + eps);
    for (int j = 0; j < hs; ++j) normed[static_cast<size_t>(i) * hs + j] = row[j] * m->final_norm[j] * inv;
    if (normed_out) {  // the Local Head's unfolded form (:748-765)
      float a2 = 0.0f;
      for (int j = 0; j < hs; ++j) a2 += row[j] * row[j];
      const float inv2 = 1.0f / std::sqrt(a2 / static_cast<float>(hs) + eps);
      for (int j = 0; j < hs; ++j)
        normed_out[static_cast<size_t>(i) * hs + j] = row[j] * inv2 * m->final_norm[j];
    }
  }
  std::vector<float> logits(static_cast<size_t>(n_rows) * nl);
  orc::gemm(normed.data(), hs, m->score.data(), hs, logits.data(), nl, n_rows, nl, hs, false);
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n_rows; ++i) {
    const float* r = &logits[static_cast<size_t>(i) * nl];
    int best = 0;
    float bv = -INFINITY, second = -INFINITY;
    for (int l = 0; l < nl; ++l) {
      if (r[l] > bv) {
        second = bv;
        bv = r[l];
        best = l;
      } else if (r[l] > second) {
        second = r[l];
      }
    }
    if (raw_ms) raw_ms[i] = static_cast<int64_t>(static_cast<double>(best) * c.timestamp_segment_time_ms);
    if (margin) margin[i] = bv - second;
  }
  if (logits_out) std::copy(logits.begin(), logits.end(), logits_out);
  return QA_OK;
}

// src/postprocess.rs:33-113 (_fix_timestamps)
extern "C" void or_fix_timestamps(const int64_t* data, int n, int64_t* out) {
  if (n <= 0) return;
  std::vector<int> dp(n, 1);
  std::vector<int64_t> parent(n, -1);
  for (int i = 1; i < n; ++i)
    for (int j = 0; j < i; ++j)
      if (data[j] <= data[i] && dp[j] + 1 > dp[i]) {
        dp[i] = dp[j] + 1;
        parent[i] = j;
      }
  const int max_len = *std::max_element(dp.begin(), dp.end());
  const int max_idx = static_cast<int>(std::find(dp.begin(), dp.end(), max_len) - dp.begin());
  std::vector<char> normal(n, 0);
  for (int64_t idx = max_idx; idx != -1; idx = parent[idx]) normal[idx] = 1;
  for (int i = 0; i < n; ++i) out[i] = data[i];
  int bs = 0;
  while (bs < n) {
    if (normal[bs]) {
      ++bs;
      continue;
    }
    int be = bs;
    while (be < n && !normal[be]) ++be;
    const int cnt = be - bs;
    bool hl = false, hr = false;
    int64_t lv = 0, rv = 0;
    for (int k = bs - 1; k >= 0; --k)
      if (normal[k]) {
        hl = true;
        lv = out[k];
        break;
      }
    for (int k = be; k < n; ++k)
      if (normal[k]) {
        hr = true;
        rv = out[k];
        break;
      }
    if (hl || hr) {
      if (cnt <= 2) {
        for (int p = bs; p < be; ++p) {
          if (hl && hr)
            out[p] = (p - (bs - 1) <= be - p) ? lv : rv;
          else
            out[p] = hl ? lv : rv;
        }
      } else if (hl && hr) {
        const double step = static_cast<double>(rv - lv) / static_cast<double>(cnt + 1);
        for (int p = bs; p < be; ++p)
          out[p] = static_cast<int64_t>(static_cast<double>(lv) + step * static_cast<double>(p - bs + 1));
      } else {
        for (int p = bs; p < be; ++p) out[p] = hl ? lv : rv;
      }
    }
    bs = be;
  }
}

// src/align_input.rs:49-87
extern "C" int64_t or_conv3_length(int64_t len) {
  int64_t l = len;
  for (int i = 0; i < 3; ++i) l = l > 0 ? (l - 1) / 2 + 1 : 0;
  return l;
}
extern "C" int64_t or_audio_token_count(int64_t valid, int64_t n_window) {
  const int64_t cl = n_window * 2;
  return (valid / cl) * 13 + or_conv3_length(valid % cl);
}
extern "C" int64_t or_padded_mel_frames(int64_t valid, int64_t n_window) {
  const int64_t mult = n_window * 2, rem = valid % mult;
  return rem == 0 ? valid : valid + (mult - rem);
}
extern "C" int64_t or_valid_mel_frames(int64_t n_samples) { return n_samples / 160; }
