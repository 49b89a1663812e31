// Host-side packing logic kept from the reference's engine:
//  * PlanBatches / PlanChunk (scheduler.cpp:13-75): chunk the caller's
//    sequences by max_batch_size, then split any chunk whose max/mean length
//    exceeds the threshold into sorted halves, recursively.  The split sorts
//    with std::sort and the same comparator so the plan -- including how
//    equal lengths are divided -- is the reference's (per-tensor activation
//    scales make a sequence's INT8 numerics depend on its group).
//  * BatchView validation (batch.cpp:8-45) with the same messages.
//  * RopeBuildTables (rope_tables.cpp:14-29) with the same float expressions,
//    so the device tables are bit-identical to the reference's.
#include "scheduler.h"

#include <algorithm>
#include <cmath>
#include <numeric>
#include <stdexcept>
#include <string>

#include "context.h"
#include "esm_b200.h"

namespace esmb200 {

namespace {

void PlanChunk(std::vector<int>& indices, const std::vector<int>& lengths, float threshold,
               std::vector<std::vector<int>>* out) {
  if (indices.empty()) return;
  if (indices.size() == 1) {
    out->push_back(std::move(indices));
    return;
  }
  int max_len = 0;
  long total = 0;
  for (int i : indices) {
    const int L = lengths[static_cast<size_t>(i)];
    max_len = std::max(max_len, L);
    total += L;
  }
  const float mean_len = static_cast<float>(total) / static_cast<float>(indices.size());
  if (mean_len > 0.0f && static_cast<float>(max_len) / mean_len > threshold) {
    std::sort(indices.begin(), indices.end(), [&](int a, int b) {
      return lengths[static_cast<size_t>(a)] < lengths[static_cast<size_t>(b)];
    });
    const size_t mid = indices.size() / 2;
    std::vector<int> lo(indices.begin(), indices.begin() + static_cast<long>(mid));
    std::vector<int> hi(indices.begin() + static_cast<long>(mid), indices.end());
    PlanChunk(lo, lengths, threshold, out);
    PlanChunk(hi, lengths, threshold, out);
    return;
  }
  out->push_back(std::move(indices));
}

}  // namespace

std::vector<std::vector<int>> PlanBatches(const std::vector<int>& lengths, float threshold,
                                          int max_batch_size) {
  std::vector<std::vector<int>> out;
  if (lengths.empty()) return out;
  const int mb = max_batch_size > 0 ? max_batch_size : static_cast<int>(lengths.size());
  std::vector<int> all(lengths.size());
  std::iota(all.begin(), all.end(), 0);
  for (size_t s = 0; s < all.size(); s += static_cast<size_t>(mb)) {
    const size_t e = std::min(s + static_cast<size_t>(mb), all.size());
    std::vector<int> chunk(all.begin() + static_cast<long>(s), all.begin() + static_cast<long>(e));
    PlanChunk(chunk, lengths, threshold, &out);
  }
  return out;
}

std::string ValidateBatchView(int T, int n_masks, const int* cu, int n_cu, int batch_size) {
  if (batch_size < 1) return "BatchView: batch_size must be >= 1";
  if (n_cu != batch_size + 1)
    return "BatchView: cu_seqlens.size() (" + std::to_string(n_cu) +
           ") must equal batch_size + 1 (" + std::to_string(batch_size + 1) + ")";
  if (cu[0] != 0) return "BatchView: cu_seqlens[0] must be 0";
  for (int i = 1; i < n_cu; ++i)
    if (cu[i] < cu[i - 1]) return "BatchView: cu_seqlens must be non-decreasing";
  if (cu[n_cu - 1] != T)
    return "BatchView: cu_seqlens.back() (" + std::to_string(cu[n_cu - 1]) +
           ") must equal packed_ids.size() (" + std::to_string(T) + ")";
  if (n_masks != 0 && n_masks != T)
    return "BatchView: packed_masks must be empty or match packed_ids size";
  return {};
}

void RopeBuildTables(int seq_len, int head_dim, float* cos_t, float* sin_t) {
  const int half = head_dim / 2;
  for (int i = 0; i < half; ++i) {
    const float exponent = static_cast<float>(2 * i) / static_cast<float>(head_dim);
    const float inv_freq = std::pow(10000.0f, -exponent);
    for (int t = 0; t < seq_len; ++t) {
      const float angle = static_cast<float>(t) * inv_freq;
      const float c = std::cos(angle);
      const float s = std::sin(angle);
      cos_t[t * head_dim + i] = c;
      cos_t[t * head_dim + i + half] = c;
      sin_t[t * head_dim + i] = s;
      sin_t[t * head_dim + i + half] = s;
    }
  }
}

}  // namespace esmb200

extern "C" {

int esmcu_plan_batches(const int* lengths, int n, float threshold, int max_batch,
                       int* order_out, int* group_sizes_out) {
  if (n < 0 || (n > 0 && (lengths == nullptr || order_out == nullptr || group_sizes_out == nullptr))) {
    esmb200::set_error("esmcu_plan_batches: bad arguments");
    return -1;
  }
  std::vector<int> lens(lengths, lengths + n);
  auto plan = esmb200::PlanBatches(lens, threshold, max_batch);
  int pos = 0;
  for (size_t g = 0; g < plan.size(); ++g) {
    group_sizes_out[g] = static_cast<int>(plan[g].size());
    for (int idx : plan[g]) order_out[pos++] = idx;
  }
  return static_cast<int>(plan.size());
}

int esmcu_batch_view_check(int T, int n_masks, const int* cu, int n_cu, int batch_size) {
  if (cu == nullptr && n_cu > 0) return esmb200::fail(ESMCU_ERR_INVALID_ARGUMENT, "cu_seqlens is null");
  std::string msg = esmb200::ValidateBatchView(T, n_masks, cu, n_cu, batch_size);
  if (!msg.empty()) return esmb200::fail(ESMCU_ERR_INVALID_ARGUMENT, msg);
  return ESMCU_OK;
}

int esmcu_rope_build_tables(int seq_len, int head_dim, float* cos_out, float* sin_out) {
  if (seq_len < 0 || head_dim <= 0 || (head_dim & 1) || (seq_len > 0 && (!cos_out || !sin_out)))
    return esmb200::fail(ESMCU_ERR_INVALID_ARGUMENT, "bad RoPE table arguments");
  esmb200::RopeBuildTables(seq_len, head_dim, cos_out, sin_out);
  return ESMCU_OK;
}

}  // extern "C"
