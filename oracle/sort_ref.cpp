// Descending argsort as torch.sort(descending=True) orders a CPU row, equal
// values included -- TEST INFRASTRUCTURE ONLY (the oracle of the host sampler).
// torch's CPU sort runs std::sort over (value, index) with a comparator that
// puts NaN first and then larger values; the tie order is that introsort's, so
// the oracle calls the same library sort rather than a stable one.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <utility>
#include <vector>

extern "C" void oracle_desc_argsort(const float* x, int n, int32_t* out) {
  std::vector<std::pair<float, int32_t>> a(n);
  for (int i = 0; i < n; ++i) a[i] = {x[i], i};
  std::sort(a.begin(), a.end(), [](const std::pair<float, int32_t>& l, const std::pair<float, int32_t>& r) {
    return (std::isnan(l.first) && !std::isnan(r.first)) || l.first > r.first;
  });
  for (int i = 0; i < n; ++i) out[i] = a[i].second;
}
