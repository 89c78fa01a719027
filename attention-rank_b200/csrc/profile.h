// Host-side profile accumulator and attention-basin pick.
//
// Same semantics as the reference's host code in attnrank/src/attnrank.cpp:
//   profile_from_accumulated      <- AttentionProfile::from_accumulated (:151-169)
//   stable_descending_order       <- AttentionProfile::recompute_position_order (:171-177)
//   basin_statistics              <- basin_statistics (:236-255)
//   select_shallowest_basin_layer <- select_shallowest_basin_layer (:257-265)
//   resolve_position_order        <- resolve_position_order (:377-392)
//   normalize_to_unit_sum         <- normalize_to_unit_sum (model.cu:503-508)
// These run once per scan on a few hundred numbers; they stay scalar C++.
#pragma once

#include <algorithm>
#include <cstdint>
#include <limits>
#include <numeric>
#include <vector>

namespace arb {

constexpr int kMinimumBasinSlots = 3;

inline void normalize_to_unit_sum(double* values, int count) {
  double sum = 0.0;
  for (int i = 0; i < count; ++i) sum += values[i];
  if (sum <= 0.0) return;
  for (int i = 0; i < count; ++i) values[i] /= sum;
}

// Slots ordered by attention, largest first; ties keep slot order.
inline void stable_descending_order(const double* attention, int slots, int* order) {
  std::vector<int> index(slots);
  std::iota(index.begin(), index.end(), 0);
  std::stable_sort(index.begin(), index.end(), [attention](int a, int b) { return attention[a] > attention[b]; });
  std::copy(index.begin(), index.end(), order);
}

inline void profile_from_accumulated(const double* accumulated, int slots, int64_t sample_count, double* attention,
                                     int* position_order) {
  double total = 0.0;
  for (int s = 0; s < slots; ++s) {
    attention[s] = accumulated[s] / static_cast<double>(sample_count);
    total += attention[s];
  }
  if (total > 0.0) {
    for (int s = 0; s < slots; ++s) attention[s] /= total;
  }
  if (position_order != nullptr) stable_descending_order(attention, slots, position_order);
}

struct BasinStatistics {
  double first = 0.0;
  double last = 0.0;
  double interior_mean = 0.0;
  double edge_ratio = 0.0;
  bool is_basin = false;
};

inline BasinStatistics basin_statistics(const double* attention, int slots, double min_edge_ratio) {
  BasinStatistics stats;
  if (slots < kMinimumBasinSlots) return stats;
  stats.first = attention[0];
  stats.last = attention[slots - 1];
  double interior = 0.0;
  for (int s = 1; s + 1 < slots; ++s) interior += attention[s];
  stats.interior_mean = interior / static_cast<double>(slots - 2);
  const double weakest = std::min(stats.first, stats.last);
  if (stats.interior_mean > 0.0) {
    stats.edge_ratio = weakest / stats.interior_mean;
  } else {
    stats.edge_ratio = weakest > 0.0 ? std::numeric_limits<double>::infinity() : 0.0;
  }
  stats.is_basin = stats.edge_ratio >= min_edge_ratio;
  return stats;
}

inline int select_shallowest_basin_layer(const double* attention, const int* layer_indices, int profiles, int slots,
                                         double min_edge_ratio) {
  int selected = -1;
  for (int p = 0; p < profiles; ++p) {
    if (!basin_statistics(attention + static_cast<size_t>(p) * slots, slots, min_edge_ratio).is_basin) continue;
    const int layer = layer_indices[p];
    if (selected < 0 || layer < selected) selected = layer;
  }
  return selected;
}

inline void resolve_position_order(const int* preferred, int preferred_count, int count, int* order) {
  std::vector<bool> taken(count, false);
  int written = 0;
  for (int i = 0; i < preferred_count; ++i) {
    const int slot = preferred[i];
    if (slot < 0 || slot >= count || taken[slot]) continue;
    taken[slot] = true;
    order[written++] = slot;
  }
  for (int slot = 0; slot < count; ++slot) {
    if (!taken[slot]) order[written++] = slot;
  }
}

}  // namespace arb
