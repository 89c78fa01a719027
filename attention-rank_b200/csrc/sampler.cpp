// Host token samplers (declarations and reference mapping in sampler.h).
#include "sampler.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>

#include "engine.h"

namespace arb {

namespace {

// float -> unsigned key whose ascending order is the descending order of the floats
// (-0.0 and 0.0 compare equal as floats; NaN is not expected in logits)
inline uint32_t descending_key(float value) {
  uint32_t bits;
  std::memcpy(&bits, &value, sizeof(bits));
  if (value == 0.0f) bits = 0u;  // +0 and -0 are one value, as for the reference's comparator
  const uint32_t ascending = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
  return ~ascending;
}

}  // namespace

// GreedySampler::select (model.cpp:70-73): the first index holding the largest logit.
int GreedyTokenSampler::select(const float* logits, int count) {
  if (logits == nullptr || count <= 0) throw Error("cannot sample from empty logits");
  return static_cast<int>(std::max_element(logits, logits + count) - logits);
}

NucleusTokenSampler::NucleusTokenSampler(const SamplerConfig& config) : config_(config), random_(config.seed) {
  if (!(config_.temperature > 0.0f)) throw Error("nucleus sampling needs a positive temperature");
}

// Stable sort of all logits by descending value (radix sort of 32-bit keys, 8 bits a pass):
// order_ holds the ids, keys_ their keys.
void NucleusTokenSampler::sort_descending(const float* logits, int count) {
  const size_t n = static_cast<size_t>(count);
  keys_.resize(n);
  order_.resize(n);
  spare_keys_.resize(n);
  spare_order_.resize(n);
  for (size_t i = 0; i < n; ++i) {
    keys_[i] = descending_key(logits[i]);
    order_[i] = static_cast<int>(i);
  }
  for (int shift = 0; shift < 32; shift += 8) {
    size_t counts[257] = {0};
    for (size_t i = 0; i < n; ++i) ++counts[((keys_[i] >> shift) & 0xFFu) + 1];
    if (counts[1] == n || counts[256] == n) continue;  // one bucket: this pass keeps the order
    for (int b = 0; b < 256; ++b) counts[b + 1] += counts[b];
    for (size_t i = 0; i < n; ++i) {
      const size_t at = counts[(keys_[i] >> shift) & 0xFFu]++;
      spare_keys_[at] = keys_[i];
      spare_order_[at] = order_[i];
    }
    keys_.swap(spare_keys_);
    order_.swap(spare_order_);
  }
}

// NucleusSampler::select (model.cpp:79-122):
//   1. candidates: the top_k ids (all when top_k == 0) by descending logit (std::partial_sort);
//   2. weights w_i = exp((logit_i - logit_0) / temperature) in double, total = sum w_i;
//   3. the nucleus is the shortest prefix whose running sum of w_i / total reaches top_p;
//   4. a uniform draw in [0, nucleus weight) walks the prefix; the candidate where it reaches 0
//      is returned (the last nucleus candidate if rounding leaves it above 0).
// Steps 2-4 depend only on the sequence of candidate VALUES, which every correct descending sort
// yields (equal logits have equal weights). So the values come from a radix sort here, the weights
// are computed in parallel (each exp is independent), and the sums, the cut and the walk run in
// the reference's order. Only the id at the chosen position can depend on how std::partial_sort
// orders equal logits: when the chosen value occurs more than once, the id is taken from the
// reference's own partial_sort order; otherwise it is unique and identical by construction.
int NucleusTokenSampler::select(const float* logits, int count) {
  if (logits == nullptr || count <= 0) throw Error("cannot sample from empty logits");
  sort_descending(logits, count);
  const size_t n = static_cast<size_t>(count);
  const size_t keep = config_.top_k > 0 ? std::min<size_t>(static_cast<size_t>(config_.top_k), n) : n;
  const double top = logits[order_[0]];
  const double temperature = static_cast<double>(config_.temperature);
  weights_.resize(keep);
  const long long parallel_keep = static_cast<long long>(keep);
#pragma omp parallel for schedule(static) if (parallel_keep > 32768)
  for (long long i = 0; i < parallel_keep; ++i) {
    weights_[i] = std::exp((static_cast<double>(logits[order_[i]]) - top) / temperature);
  }
  double total = 0.0;
  for (size_t i = 0; i < keep; ++i) total += weights_[i];
  size_t nucleus = keep;
  double running = 0.0;
  for (size_t i = 0; i < keep; ++i) {
    running += weights_[i] / total;
    if (running >= static_cast<double>(config_.top_p)) {
      nucleus = i + 1;
      break;
    }
  }
  double nucleus_weight = 0.0;
  for (size_t i = 0; i < nucleus; ++i) nucleus_weight += weights_[i];
  std::uniform_real_distribution<double> draw(0.0, nucleus_weight);
  double remaining = draw(random_);
  size_t chosen = nucleus - 1;
  for (size_t i = 0; i < nucleus; ++i) {
    remaining -= weights_[i];
    if (remaining <= 0.0) {
      chosen = i;
      break;
    }
  }
  const uint32_t key = keys_[chosen];
  const bool tied = (chosen > 0 && keys_[chosen - 1] == key) || (chosen + 1 < n && keys_[chosen + 1] == key);
  if (!tied) return order_[chosen];
  // equal logits around the chosen position: the reference's order decides which id it is
  exact_.resize(n);
  std::iota(exact_.begin(), exact_.end(), 0);
  std::partial_sort(exact_.begin(), exact_.begin() + static_cast<long>(keep), exact_.end(),
                    [logits](int a, int b) { return logits[a] > logits[b]; });
  return exact_[chosen];
}

std::unique_ptr<TokenSampler> make_token_sampler(const SamplerConfig& config) {
  if (config.temperature <= 0.0f) return std::make_unique<GreedyTokenSampler>();
  return std::make_unique<NucleusTokenSampler>(config);
}

}  // namespace arb
