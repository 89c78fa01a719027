// Host token samplers (declarations and reference mapping in sampler.h).
#include "sampler.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>

#include <omp.h>

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

// the logit of a key (+0.0 for the zero key, which -0.0 shares)
inline double key_value(uint32_t key) {
  const uint32_t ascending = ~key;
  const uint32_t bits = (ascending & 0x80000000u) ? (ascending & 0x7FFFFFFFu) : ~ascending;
  float value;
  std::memcpy(&value, &bits, sizeof(value));
  return value;
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

// The order keys of the `keep` largest logits, ascending (so the logits descend), in keys_; keys
// of equal logits are equal. One parallel most-significant-digit pass puts every key into one of
// 4096 buckets by its top 12 bits (sign, exponent, three mantissa bits). Only the buckets that
// hold the first `keep` keys are filled, and each is then sorted on its own. id_keys_ keeps every
// id's key, so an id can be found again from its key.
void NucleusTokenSampler::sort_keys(const float* logits, int count, size_t keep) {
  constexpr int kBits = 12;
  constexpr int kBuckets = 1 << kBits;
  constexpr int kShift = 32 - kBits;
  static_assert(kShift % 10 == 0 && (kShift / 10) % 2 == 0, "an even number of 10-bit passes per bucket");
  const size_t n = static_cast<size_t>(count);
  const int threads = n >= 32768 ? std::max(1, std::min(omp_get_max_threads(), 16)) : 1;
  id_keys_.resize(n);
  counts_.assign(static_cast<size_t>(threads) * kBuckets, 0u);
  starts_.resize(kBuckets + 1);
#pragma omp parallel num_threads(threads)
  {
    const int t = omp_get_thread_num();
    uint32_t* histogram = counts_.data() + static_cast<size_t>(t) * kBuckets;
    for (size_t i = n * t / threads, end = n * (t + 1) / threads; i < end; ++i) {
      const uint32_t key = descending_key(logits[i]);
      id_keys_[i] = key;
      ++histogram[key >> kShift];
    }
  }
  // bucket starts; `needed` buckets hold at least `keep` keys
  int needed = kBuckets;
  uint32_t total = 0;
  for (int b = 0; b < kBuckets; ++b) {
    starts_[b] = total;
    for (int t = 0; t < threads; ++t) {
      uint32_t& slot = counts_[static_cast<size_t>(t) * kBuckets + b];
      const uint32_t here = slot;
      slot = total;  // this thread's first position in bucket b
      total += here;
    }
    if (total >= keep && needed == kBuckets) needed = b + 1;
  }
  starts_[kBuckets] = total;
  keys_.resize(starts_[needed]);
#pragma omp parallel num_threads(threads)
  {
    const int t = omp_get_thread_num();
    uint32_t* offset = counts_.data() + static_cast<size_t>(t) * kBuckets;
    for (size_t i = n * t / threads, end = n * (t + 1) / threads; i < end; ++i) {
      const uint32_t key = id_keys_[i];
      const uint32_t bucket = key >> kShift;
      if (bucket < static_cast<uint32_t>(needed)) keys_[offset[bucket]++] = key;
    }
  }
  // each bucket: its keys share the top 12 bits; large buckets take two counting passes over the
  // low 20 bits (10 bits a pass, through a per-thread scratch buffer), small ones std::sort
  if (scratch_.size() < static_cast<size_t>(threads)) scratch_.resize(threads);
#pragma omp parallel num_threads(threads)
  {
    std::vector<uint32_t>& scratch = scratch_[omp_get_thread_num()];
#pragma omp for schedule(dynamic, 1)
    for (int b = 0; b < needed; ++b) {
      uint32_t* first = keys_.data() + starts_[b];
      const uint32_t size = starts_[b + 1] - starts_[b];
      if (size <= 256) {
        std::sort(first, first + size);
        continue;
      }
      if (scratch.size() < size) scratch.resize(size);
      uint32_t* from = first;
      uint32_t* to = scratch.data();
      for (int shift = 0; shift < kShift; shift += 10) {
        uint32_t digits[1025] = {0};
        for (uint32_t i = 0; i < size; ++i) ++digits[((from[i] >> shift) & 0x3FFu) + 1];
        for (int d = 0; d < 1024; ++d) digits[d + 1] += digits[d];
        for (uint32_t i = 0; i < size; ++i) to[digits[(from[i] >> shift) & 0x3FFu]++] = from[i];
        std::swap(from, to);
      }
      // an even number of passes: the sorted keys are back in the bucket
    }
  }
}

// NucleusSampler::select (model.cpp:79-122):
//   1. candidates: the top_k ids (all when top_k == 0) by descending logit (std::partial_sort);
//   2. weights w_i = exp((logit_i - logit_0) / temperature) in double, total = sum w_i;
//   3. the nucleus is the shortest prefix whose running sum of w_i / total reaches top_p;
//   4. a uniform draw in [0, nucleus weight) walks the prefix; the candidate where it reaches 0
//      is returned (the last nucleus candidate if rounding leaves it above 0).
// Steps 2-4 depend only on the sequence of candidate VALUES, which every correct descending sort
// yields (equal logits have equal weights). So the values come from a sort of order keys
// (sort_keys), the weights are computed in parallel (each exp is independent), and the sums, the
// cut and the walk run in the reference's order. Only the id at the chosen position can depend on
// how std::partial_sort orders equal logits: when the chosen value occurs more than once, the id
// is taken from the reference's own partial_sort order; otherwise exactly one id has its key.
int NucleusTokenSampler::select(const float* logits, int count) {
  if (logits == nullptr || count <= 0) throw Error("cannot sample from empty logits");
  const size_t n = static_cast<size_t>(count);
  const size_t keep = config_.top_k > 0 ? std::min<size_t>(static_cast<size_t>(config_.top_k), n) : n;
  sort_keys(logits, count, keep);
  const double top = key_value(keys_[0]);
  const double temperature = static_cast<double>(config_.temperature);
  weights_.resize(keep);
  const long long parallel_keep = static_cast<long long>(keep);
#pragma omp parallel for schedule(static) if (parallel_keep > 32768)
  for (long long i = 0; i < parallel_keep; ++i) {
    weights_[i] = std::exp((key_value(keys_[i]) - top) / temperature);
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
  // equal keys share a bucket, and every filled bucket lies whole in keys_: the neighbours there
  // tell whether the chosen logit occurs more than once among all ids
  const uint32_t key = keys_[chosen];
  const bool tied = (chosen > 0 && keys_[chosen - 1] == key) || (chosen + 1 < keys_.size() && keys_[chosen + 1] == key);
  if (!tied) return static_cast<int>(std::find(id_keys_.begin(), id_keys_.end(), key) - id_keys_.begin());
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
