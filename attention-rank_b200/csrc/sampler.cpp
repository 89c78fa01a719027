// Host token samplers (declarations and reference mapping in sampler.h).
#include "sampler.h"

#include <algorithm>
#include <cmath>
#include <numeric>

#include "engine.h"

namespace arb {

// GreedySampler::select (model.cpp:70-73): the first index holding the largest logit.
int GreedyTokenSampler::select(const float* logits, int count) {
  if (logits == nullptr || count <= 0) throw Error("cannot sample from empty logits");
  return static_cast<int>(std::max_element(logits, logits + count) - logits);
}

NucleusTokenSampler::NucleusTokenSampler(const SamplerConfig& config) : config_(config), random_(config.seed) {
  if (!(config_.temperature > 0.0f)) throw Error("nucleus sampling needs a positive temperature");
}

// NucleusSampler::select (model.cpp:79-122):
//   1. candidates: the top_k ids (all when top_k == 0) by descending logit (std::partial_sort);
//   2. weights w_i = exp((logit_i - logit_0) / temperature) in double, total = sum w_i;
//   3. the nucleus is the shortest prefix whose running sum of w_i / total reaches top_p;
//   4. a uniform draw in [0, nucleus weight) walks the prefix; the candidate where it reaches 0
//      is returned (the last nucleus candidate if rounding leaves it above 0).
int NucleusTokenSampler::select(const float* logits, int count) {
  if (logits == nullptr || count <= 0) throw Error("cannot sample from empty logits");
  order_.resize(static_cast<size_t>(count));
  std::iota(order_.begin(), order_.end(), 0);
  const size_t keep = config_.top_k > 0 ? std::min<size_t>(static_cast<size_t>(config_.top_k), order_.size())
                                         : order_.size();
  std::partial_sort(order_.begin(), order_.begin() + static_cast<long>(keep), order_.end(),
                    [logits](int a, int b) { return logits[a] > logits[b]; });

  const double top = logits[order_[0]];
  const double temperature = static_cast<double>(config_.temperature);
  weights_.resize(keep);
  double total = 0.0;
  for (size_t i = 0; i < keep; ++i) {
    weights_[i] = std::exp((static_cast<double>(logits[order_[i]]) - top) / temperature);
    total += weights_[i];
  }
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
  for (size_t i = 0; i < nucleus; ++i) {
    remaining -= weights_[i];
    if (remaining <= 0.0) return order_[i];
  }
  return order_[nucleus - 1];
}

std::unique_ptr<TokenSampler> make_token_sampler(const SamplerConfig& config) {
  if (config.temperature <= 0.0f) return std::make_unique<GreedyTokenSampler>();
  return std::make_unique<NucleusTokenSampler>(config);
}

}  // namespace arb
