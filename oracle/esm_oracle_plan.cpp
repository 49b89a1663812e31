/* PlanBatches restated -- TEST INFRASTRUCTURE ONLY (see esm_oracle.h).
 *
 * scheduler.cpp:13-50 PlanChunk: a chunk with max/mean length above the
 * threshold is sorted by length with std::sort (ties in the order that call
 * leaves them) and split into halves, recursively; scheduler.cpp:54-75
 * PlanBatches first chunks the caller's indices by max_batch. */
#include <algorithm>
#include <vector>

#include "esm_oracle.h"

namespace {
void plan_chunk(std::vector<int> idx, const int* lengths, float threshold,
                std::vector<std::vector<int>>& out) {
  if (idx.empty()) return;
  if (idx.size() > 1) {
    int max_len = 0;
    long total = 0;
    for (int i : idx) {
      max_len = std::max(max_len, lengths[i]);
      total += lengths[i];
    }
    const float mean = static_cast<float>(total) / static_cast<float>(idx.size());
    if (mean > 0.0f && static_cast<float>(max_len) / mean > threshold) {
      std::sort(idx.begin(), idx.end(), [&](int a, int b) { return lengths[a] < lengths[b]; });
      const size_t mid = idx.size() / 2;
      plan_chunk(std::vector<int>(idx.begin(), idx.begin() + static_cast<long>(mid)), lengths,
                 threshold, out);
      plan_chunk(std::vector<int>(idx.begin() + static_cast<long>(mid), idx.end()), lengths,
                 threshold, out);
      return;
    }
  }
  out.push_back(std::move(idx));
}
}  // namespace

extern "C" int orc_plan_batches(const int* lengths, int n, float threshold, int max_batch,
                                int* order_out, int* group_sizes_out) {
  if (n <= 0) return 0;
  const int mb = max_batch > 0 ? max_batch : n;
  std::vector<std::vector<int>> out;
  for (int s = 0; s < n; s += mb) {
    std::vector<int> chunk;
    for (int i = s; i < std::min(n, s + mb); ++i) chunk.push_back(i);
    plan_chunk(std::move(chunk), lengths, threshold, out);
  }
  int pos = 0;
  for (size_t g = 0; g < out.size(); ++g) {
    group_sizes_out[g] = static_cast<int>(out[g].size());
    for (int i : out[g]) order_out[pos++] = i;
  }
  return static_cast<int>(out.size());
}
