// Timestamp repair on the host (src/postprocess.rs:33-113), the one piece of
// post-processing the reference keeps in compiled code after the argmax.
#include <algorithm>
#include <cstdint>
#include <vector>

#include "qa_b200.h"

namespace {

// The longest non-decreasing subsequence of the reference's repair
// (src/postprocess.rs:39-48): dp[i] = 1 + max dp[j] over j < i with
// v[j] <= v[i], and parent[i] = the first j (smallest index) that reaches
// that maximum, since the reference scans j upwards and updates only on a
// strictly longer chain.  The O(n^2) scan is replaced by a Fenwick tree over
// the ranks of the distinct values: each node keeps the best (longest chain,
// then smallest index) entry of its range, so one prefix query over the
// values <= v[i] gives the same dp and parent in O(log n).
struct Chain {
  int len = 0;  // 0: empty
  int at = -1;
};

inline bool longer(const Chain& a, const Chain& b) {
  return a.len > b.len || (a.len == b.len && a.len > 0 && a.at < b.at);
}

void lis_parents(const std::vector<int64_t>& v, std::vector<int>& dp, std::vector<int>& parent) {
  const int n = static_cast<int>(v.size());
  std::vector<int64_t> keys(v);
  std::sort(keys.begin(), keys.end());
  keys.erase(std::unique(keys.begin(), keys.end()), keys.end());
  const int m = static_cast<int>(keys.size());
  std::vector<Chain> tree(m + 1);
  for (int i = 0; i < n; ++i) {
    // 1-based rank of v[i]: the prefix [1, r] holds every value <= v[i]
    const int r = static_cast<int>(std::upper_bound(keys.begin(), keys.end(), v[i]) - keys.begin());
    Chain best;
    for (int p = r; p > 0; p -= p & -p)
      if (longer(tree[p], best)) best = tree[p];
    dp[i] = best.len + 1;
    parent[i] = best.len > 0 ? best.at : -1;
    const Chain me{dp[i], i};
    for (int p = r; p <= m; p += p & -p)
      if (longer(me, tree[p])) tree[p] = me;
  }
}

}  // namespace

extern "C" int qa_fix_timestamps(const int64_t* data, int n, int64_t* out) {
  if (n < 0 || (n > 0 && (!data || !out))) return QA_ERR_ARG;
  if (n == 0) return QA_OK;
  std::vector<int64_t> v(data, data + n);
  std::vector<int> dp(n, 1), parent(n, -1);
  lis_parents(v, dp, parent);
  const int best = static_cast<int>(std::max_element(dp.begin(), dp.end()) - dp.begin());
  std::vector<char> normal(n, 0);
  for (int i = best; i != -1; i = parent[i]) normal[i] = 1;
  std::vector<int64_t> r(v);
  for (int bs = 0; bs < n;) {
    if (normal[bs]) {
      ++bs;
      continue;
    }
    int be = bs;
    while (be < n && !normal[be]) ++be;
    const int cnt = be - bs;
    int li = bs - 1, ri = be;
    while (li >= 0 && !normal[li]) --li;
    while (ri < n && !normal[ri]) ++ri;
    const bool hl = li >= 0, hr = ri < n;
    if (hl || hr) {
      const int64_t lv = hl ? r[li] : 0, rv = hr ? r[ri] : 0;
      if (cnt <= 2) {
        for (int p = bs; p < be; ++p)
          r[p] = (hl && hr) ? ((p - (bs - 1) <= be - p) ? lv : rv) : (hl ? lv : rv);
      } else if (hl && hr) {
        const double step = static_cast<double>(rv - lv) / static_cast<double>(cnt + 1);
        for (int p = bs; p < be; ++p)
          r[p] = static_cast<int64_t>(static_cast<double>(lv) + step * static_cast<double>(p - bs + 1));
      } else {
        for (int p = bs; p < be; ++p) r[p] = hl ? lv : rv;
      }
    }
    bs = be;
  }
  std::copy(r.begin(), r.end(), out);
  return QA_OK;
}
