// Timestamp repair on the host (src/postprocess.rs:33-113), the one piece of
// post-processing the reference keeps in compiled code after the argmax.
#include <algorithm>
#include <cstdint>
#include <vector>

#include "qa_b200.h"

extern "C" int qa_fix_timestamps(const int64_t* data, int n, int64_t* out) {
  if (n < 0 || (n > 0 && (!data || !out))) return QA_ERR_ARG;
  if (n == 0) return QA_OK;
  std::vector<int64_t> v(data, data + n);
  std::vector<int> dp(n, 1), parent(n, -1);
  for (int i = 1; i < n; ++i)
    for (int j = 0; j < i; ++j)
      if (v[j] <= v[i] && dp[j] + 1 > dp[i]) {
        dp[i] = dp[j] + 1;
        parent[i] = j;
      }
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
