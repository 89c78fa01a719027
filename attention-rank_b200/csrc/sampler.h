// Token selection for generation: the samplers of include/attnrank/model.hpp:88-116
// (GreedySampler, NucleusSampler, make_sampler; attnrank/src/model.cpp:70-127).
//
// Selection runs on the host over fp32 logits, as in the reference, so that the same logits and
// seed give the same token ids: the nucleus sampler weighs candidates in double precision in the
// reference's order, draws from std::mt19937_64 through std::uniform_real_distribution<double>,
// and where equal logits make the order matter, takes it from std::partial_sort under the
// reference's "larger logit first" predicate. (The engine's greedy path does not come through
// here: it takes the first maximum on the device.)
#pragma once

#include <cstdint>
#include <memory>
#include <random>
#include <vector>

namespace arb {

struct SamplerConfig {
  float temperature = 0.0f;  // <= 0: greedy (make_sampler, model.cpp:124-127)
  float top_p = 0.9f;
  int top_k = 0;             // 0: every token is a candidate
  uint64_t seed = 1234;
};

class TokenSampler {
 public:
  virtual ~TokenSampler() = default;
  // The selected token id; throws arb::Error on empty logits.
  virtual int select(const float* logits, int count) = 0;
  virtual bool greedy() const = 0;
};

class GreedyTokenSampler final : public TokenSampler {
 public:
  int select(const float* logits, int count) override;
  bool greedy() const override { return true; }
};

class NucleusTokenSampler final : public TokenSampler {
 public:
  explicit NucleusTokenSampler(const SamplerConfig& config);  // throws for temperature <= 0
  int select(const float* logits, int count) override;
  bool greedy() const override { return false; }

 private:
  void sort_keys(const float* logits, int count, size_t keep);

  SamplerConfig config_;
  std::mt19937_64 random_;
  // buffers reused between calls
  std::vector<uint32_t> id_keys_;     // order key of every id
  std::vector<uint32_t> keys_;        // ascending keys (descending logits), at least the first keep
  std::vector<uint32_t> counts_;      // per-thread bucket counts, then per-thread scatter offsets
  std::vector<uint32_t> starts_;      // bucket starts in keys_
  std::vector<std::vector<uint32_t>> scratch_;  // one buffer per sorting thread
  std::vector<int> exact_;            // the reference's partial_sort order, built only on ties
  std::vector<double> weights_;
};

std::unique_ptr<TokenSampler> make_token_sampler(const SamplerConfig& config);

}  // namespace arb
