// Host-side packing helpers (see scheduler.cpp).
#pragma once

#include <string>
#include <vector>

namespace esmb200 {

std::vector<std::vector<int>> PlanBatches(const std::vector<int>& lengths, float threshold,
                                          int max_batch_size);
// Empty string when valid, else the reference's BatchView message.
std::string ValidateBatchView(int T, int n_masks, const int* cu, int n_cu, int batch_size);
void RopeBuildTables(int seq_len, int head_dim, float* cos_t, float* sin_t);

}  // namespace esmb200
