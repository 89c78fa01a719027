// Harness around the reference's own implementation. Test / benchmark infrastructure only.
//
// Compiled (oracle/Makefile) together with the reference's unmodified sources, read in place
// from the reference checkout: attnrank/src/{core,checkpoint,model,attnrank}.cpp and
// attnrank/src/{kernels,model}.cu. Outputs go to oracle/_ref/ only. It gives the checker and the
// reference benchmark arm a C entry point to:
//   * the reference model (CudaLlamaModel, include/attnrank/model.hpp:144-165) built from the seeded
//     synthetic checkpoint, held in host memory and handed over as a WeightRegistry
//     (checkpoint.hpp:27-39) through an in-memory IWeightSource, exactly as the safetensors
//     loader would hand it over;
//   * its measure_attention_by_layer (model.cu:593-617) and the stock layer-scan path
//     AttentionLayerScanner::scan (attnrank.cpp:364-375) + select_shallowest_basin_layer
//     (attnrank.cpp:257-265), fed token-id prompts through an IPromptBuilder (prompt.hpp:25-30)
//     that returns the given StructuredPrompt for each sample;
//   * its generate (model.cu:532-565), the answering step, with the reference's samplers;
//   * the reference's host functions (profile, basin statistics, position order, the rerankers of
//     attnrank.cpp:394-456, the samplers of model.cpp:70-127), which run without a GPU and produce
//     the golden fixtures under tests/golden/.
#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "attnrank/attnrank.hpp"
#include "attnrank/checkpoint.hpp"
#include "attnrank/model.hpp"
#include "attnrank/prompt.hpp"
#include "attnrank/tokenizer.hpp"
#include "ref_abi.h"

extern "C" {
void oracle_fill_bf16(uint16_t* out, int64_t first, int64_t count, uint64_t seed, int layer, int kind,
                      double standard_deviation);
}

namespace {

using namespace attnrank;

thread_local std::string g_error;

enum Kind { kEmbedding = 0, kQuery, kKey, kValue, kOutput, kQueryBias, kKeyBias, kValueBias, kGate, kUp, kDown,
            kInputNorm, kPostNorm, kFinalNorm };

class MemoryWeightSource : public IWeightSource {
 public:
  const std::string& origin() const override { return origin_; }
  const std::vector<TensorView>& tensors() const override { return tensors_; }

  void add(const std::string& name, std::vector<int64_t> shape, std::vector<uint16_t> bf16) {
    storage_.push_back(std::move(bf16));
    TensorView view;
    view.name = name;
    view.dtype = DType::BF16;
    view.shape = std::move(shape);
    view.data = reinterpret_cast<const std::uint8_t*>(storage_.back().data());
    view.byte_size = storage_.back().size() * sizeof(uint16_t);
    tensors_.push_back(std::move(view));
  }

 private:
  std::string origin_ = "synthetic";
  std::vector<TensorView> tensors_;
  std::vector<std::vector<uint16_t>> storage_;
};

class StubTokenizer : public ITokenizer {
 public:
  explicit StubTokenizer(int vocab) : vocab_(vocab) {}
  TokenSequence encode(std::string_view, const EncodeOptions&) const override { return {}; }
  std::string decode(const TokenSequence&) const override { return {}; }
  std::string token_text(int) const override { return {}; }
  int vocab_size() const override { return vocab_; }
  int bos_id() const override { return -1; }
  int eos_id() const override { return -1; }
  int unk_id() const override { return 0; }

 private:
  int vocab_;
};

// Returns the prepared StructuredPrompt whose index is the sample's question text.
class TokenPromptBuilder : public IPromptBuilder {
 public:
  explicit TokenPromptBuilder(const std::vector<StructuredPrompt>* prompts) : prompts_(prompts) {}
  StructuredPrompt build(const PromptRequest& request) const override {
    return prompts_->at(static_cast<size_t>(std::stoul(request.question)));
  }
  std::vector<std::string> stop_sequences() const override { return {}; }

 private:
  const std::vector<StructuredPrompt>* prompts_;
};

std::vector<uint16_t> generate(int64_t count, uint64_t seed, int layer, int kind, double std) {
  std::vector<uint16_t> out(static_cast<size_t>(count));
  oracle_fill_bf16(out.data(), 0, count, seed, layer, kind, std);
  return out;
}

std::vector<uint16_t> ones(int64_t count) { return std::vector<uint16_t>(static_cast<size_t>(count), 0x3F80u); }

struct Holder {
  LlamaConfig config;
  std::unique_ptr<CudaLlamaModel> model;
  std::shared_ptr<CudaLlamaModel> shared;
};

StructuredPrompt make_prompt(const int32_t* tokens, int token_count, int query_begin, int query_end,
                             const int32_t* spans, int span_count) {
  StructuredPrompt prompt;
  prompt.tokens.assign(tokens, tokens + token_count);
  prompt.query_span.begin = query_begin;
  prompt.query_span.end = query_end;
  for (int s = 0; s < span_count; ++s) {
    TokenSpan span;
    span.begin = spans[2 * s];
    span.end = spans[2 * s + 1];
    prompt.document_spans.push_back(span);
  }
  return prompt;
}

// The seeded synthetic checkpoint of `config`, as the safetensors loader would hand it over.
void add_synthetic_weights(WeightRegistry& registry, const LlamaConfig& config, bool attention_bias, uint64_t seed,
                           double std) {
  const int64_t H = config.hidden_size, I = config.intermediate_size, V = config.vocab_size;
  const int64_t QD = static_cast<int64_t>(config.num_attention_heads) * config.head_dim();
  const int64_t KV = config.kv_hidden_size();
  auto source = std::make_unique<MemoryWeightSource>();
  source->add("model.embed_tokens.weight", {V, H}, generate(V * H, seed, -1, kEmbedding, std));
  source->add("model.norm.weight", {H}, ones(H));
  for (int l = 0; l < config.num_hidden_layers; ++l) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    source->add(p + "self_attn.q_proj.weight", {QD, H}, generate(QD * H, seed, l, kQuery, std));
    source->add(p + "self_attn.k_proj.weight", {KV, H}, generate(KV * H, seed, l, kKey, std));
    source->add(p + "self_attn.v_proj.weight", {KV, H}, generate(KV * H, seed, l, kValue, std));
    source->add(p + "self_attn.o_proj.weight", {H, QD}, generate(H * QD, seed, l, kOutput, std));
    if (attention_bias) {
      source->add(p + "self_attn.q_proj.bias", {QD}, generate(QD, seed, l, kQueryBias, std));
      source->add(p + "self_attn.k_proj.bias", {KV}, generate(KV, seed, l, kKeyBias, std));
      source->add(p + "self_attn.v_proj.bias", {KV}, generate(KV, seed, l, kValueBias, std));
    }
    source->add(p + "mlp.gate_proj.weight", {I, H}, generate(I * H, seed, l, kGate, std));
    source->add(p + "mlp.up_proj.weight", {I, H}, generate(I * H, seed, l, kUp, std));
    source->add(p + "mlp.down_proj.weight", {H, I}, generate(H * I, seed, l, kDown, std));
    source->add(p + "input_layernorm.weight", {H}, ones(H));
    source->add(p + "post_attention_layernorm.weight", {H}, ones(H));
  }
  registry.add_source(std::move(source));
}

}  // namespace

extern "C" {


const char* ref_last_error() { return g_error.c_str(); }

void* ref_create(const ref_config* c, uint64_t seed, double std, int max_sequence_length, int prefill_chunk_tokens,
                 int device_index) {
  try {
    auto holder = std::make_unique<Holder>();
    LlamaConfig& config = holder->config;
    config.hidden_size = c->hidden_size;
    config.intermediate_size = c->intermediate_size;
    config.num_hidden_layers = c->num_hidden_layers;
    config.num_attention_heads = c->num_attention_heads;
    config.num_key_value_heads = c->num_key_value_heads;
    config.vocab_size = c->vocab_size;
    config.max_position_embeddings = max_sequence_length;
    config.rms_norm_eps = c->rms_norm_eps;
    config.rope_theta = c->rope_theta;
    config.sliding_window = c->sliding_window;
    config.tie_word_embeddings = true;  // the output head is never used by probing

    WeightRegistry registry;
    add_synthetic_weights(registry, config, c->attention_bias != 0, seed, std);
    LlamaRuntimeOptions options;
    options.device_index = device_index;
    options.max_sequence_length = max_sequence_length;
    options.prefill_chunk_tokens = prefill_chunk_tokens;
    holder->shared = std::make_shared<CudaLlamaModel>(config, registry, std::make_shared<StubTokenizer>(c->vocab_size),
                                                      options);
    return holder.release();
  } catch (const std::exception& error) {
    g_error = error.what();
    return nullptr;
  }
}

void ref_destroy(void* handle) { delete static_cast<Holder*>(handle); }

int ref_measure_attention_by_layer(void* handle, const ref_prompt* prompt, int span_count, int layer_begin,
                                   int layer_end, int normalize_by_length, double* rows_out, int* layer_begin_out,
                                   int* layer_count_out) {
  try {
    auto* holder = static_cast<Holder*>(handle);
    const StructuredPrompt structured = make_prompt(prompt->tokens, prompt->token_count, prompt->query_begin,
                                                    prompt->query_end, prompt->spans, span_count);
    AttentionLayerProbeRequest request;
    request.layer_begin = layer_begin;
    request.layer_end = layer_end;
    request.query_span = structured.query_span;
    request.document_spans = structured.document_spans;
    request.normalize_by_document_length = normalize_by_length != 0;
    const AttentionLayerProbeResult result = holder->shared->measure_attention_by_layer(structured.tokens, request);
    for (size_t l = 0; l < result.attention_by_layer.size(); ++l) {
      for (int s = 0; s < span_count; ++s) rows_out[l * span_count + s] = result.attention_by_layer[l][s];
    }
    if (layer_begin_out) *layer_begin_out = result.layer_begin;
    if (layer_count_out) *layer_count_out = static_cast<int>(result.attention_by_layer.size());
    return 0;
  } catch (const std::exception& error) {
    g_error = error.what();
    return 1;
  }
}

int ref_measure_attention(void* handle, const ref_prompt* prompt, int span_count, int layer_begin, int layer_end,
                          int normalize_by_length, double* attention_out) {
  try {
    auto* holder = static_cast<Holder*>(handle);
    const StructuredPrompt structured = make_prompt(prompt->tokens, prompt->token_count, prompt->query_begin,
                                                    prompt->query_end, prompt->spans, span_count);
    AttentionProbeRequest request;
    request.layer_span_begin = layer_begin;
    request.layer_span_end = layer_end;
    request.query_span = structured.query_span;
    request.document_spans = structured.document_spans;
    request.normalize_by_document_length = normalize_by_length != 0;
    const AttentionProbeResult result = holder->shared->measure_attention(structured.tokens, request);
    for (int s = 0; s < span_count; ++s) attention_out[s] = result.document_attention[s];
    return 0;
  } catch (const std::exception& error) {
    g_error = error.what();
    return 1;
  }
}

// The stock scan: AttentionLayerScanner over a StaticProbeSampleSource, then the basin pick, with
// any IAttentionProvider behind it (the reference's CudaLlamaModel, or a provider of another
// library built against the reference's headers).
// attention_out / order_out: [layers][span_count]; seconds_out: wall time of the scan call
// (synchronous in the reference: every prompt ends with a device-to-host copy).
static int scan_with(std::shared_ptr<IAttentionProvider> provider, const ref_prompt* prompts, int prompt_count,
                     int span_count, int layer_begin, int layer_end, int normalize_by_length, double min_edge_ratio,
                     double* attention_out, int* order_out, int* layer_index_out, int* layer_count_out,
                     int* selected_out, double* seconds_out) {
  try {
    std::vector<StructuredPrompt> structured;
    std::vector<ProbeSample> samples;
    structured.reserve(prompt_count);
    for (int i = 0; i < prompt_count; ++i) {
      structured.push_back(make_prompt(prompts[i].tokens, prompts[i].token_count, prompts[i].query_begin,
                                       prompts[i].query_end, prompts[i].spans, span_count));
      ProbeSample sample;
      sample.question = std::to_string(i);
      sample.documents.resize(static_cast<size_t>(span_count));
      samples.push_back(std::move(sample));
    }
    ProbeDependencies dependencies;
    dependencies.attention_provider = std::move(provider);
    dependencies.prompt_builder = std::make_shared<TokenPromptBuilder>(&structured);
    dependencies.progress = std::make_shared<NullProgressObserver>();
    LayerScanConfig config;
    config.model_id = "synthetic";
    config.layer_begin = layer_begin;
    config.layer_end = layer_end;
    config.normalize_by_document_length = normalize_by_length != 0;
    AttentionLayerScanner scanner(dependencies, config);
    const StaticProbeSampleSource source(samples);
    cudaDeviceSynchronize();
    const auto start = std::chrono::steady_clock::now();
    const std::vector<AttentionProfile> profiles = scanner.scan(source);
    cudaDeviceSynchronize();
    const auto stop = std::chrono::steady_clock::now();
    BasinCriterion criterion;
    criterion.min_edge_ratio = min_edge_ratio;
    *selected_out = select_shallowest_basin_layer(profiles, criterion);
    for (size_t l = 0; l < profiles.size(); ++l) {
      for (int s = 0; s < span_count; ++s) {
        attention_out[l * span_count + s] = profiles[l].attention[s];
        order_out[l * span_count + s] = profiles[l].position_order[s];
      }
      layer_index_out[l] = profiles[l].layer_index;
    }
    *layer_count_out = static_cast<int>(profiles.size());
    *seconds_out = std::chrono::duration<double>(stop - start).count();
    return 0;
  } catch (const std::exception& error) {
    g_error = error.what();
    return 1;
  }
}

int ref_scan(void* handle, const ref_prompt* prompts, int prompt_count, int span_count, int layer_begin,
             int layer_end, int normalize_by_length, double min_edge_ratio, double* attention_out, int* order_out,
             int* layer_index_out, int* layer_count_out, int* selected_out, double* seconds_out) {
  return scan_with(static_cast<Holder*>(handle)->shared, prompts, prompt_count, span_count, layer_begin, layer_end,
                   normalize_by_length, min_edge_ratio, attention_out, order_out, layer_index_out, layer_count_out,
                   selected_out, seconds_out);
}

// The same stock scan over a caller's provider: `provider` is a std::shared_ptr<IAttentionProvider>*.
int ref_scan_provider(void* provider, const ref_prompt* prompts, int prompt_count, int span_count, int layer_begin,
                      int layer_end, int normalize_by_length, double min_edge_ratio, double* attention_out,
                      int* order_out, int* layer_index_out, int* layer_count_out, int* selected_out,
                      double* seconds_out) {
  return scan_with(*static_cast<std::shared_ptr<IAttentionProvider>*>(provider), prompts, prompt_count, span_count,
                   layer_begin, layer_end, normalize_by_length, min_edge_ratio, attention_out, order_out,
                   layer_index_out, layer_count_out, selected_out, seconds_out);
}

// The seeded synthetic checkpoint as a WeightRegistry with its LlamaConfig, for a caller that
// builds its own provider from them (ref_weights_registry / ref_weights_config give the objects).
struct SyntheticWeights {
  LlamaConfig config;
  WeightRegistry registry;
};

void* ref_weights_create(const ref_config* c, uint64_t seed, double std, int max_sequence_length) {
  try {
    auto weights = std::make_unique<SyntheticWeights>();
    LlamaConfig& config = weights->config;
    config.hidden_size = c->hidden_size;
    config.intermediate_size = c->intermediate_size;
    config.num_hidden_layers = c->num_hidden_layers;
    config.num_attention_heads = c->num_attention_heads;
    config.num_key_value_heads = c->num_key_value_heads;
    config.vocab_size = c->vocab_size;
    config.max_position_embeddings = max_sequence_length;
    config.rms_norm_eps = c->rms_norm_eps;
    config.rope_theta = c->rope_theta;
    config.sliding_window = c->sliding_window;
    config.tie_word_embeddings = true;
    add_synthetic_weights(weights->registry, config, c->attention_bias != 0, seed, std);
    return weights.release();
  } catch (const std::exception& error) {
    g_error = error.what();
    return nullptr;
  }
}

void ref_weights_destroy(void* weights) { delete static_cast<SyntheticWeights*>(weights); }
const void* ref_weights_registry(void* weights) { return &static_cast<SyntheticWeights*>(weights)->registry; }
const void* ref_weights_config(void* weights) { return &static_cast<SyntheticWeights*>(weights)->config; }

// CudaLlamaModel::generate (model.cu:532-565) with the sampler of make_sampler (model.cpp:124-127).
// tokens_out has room for max_new_tokens ids; seconds_out: wall time of the generate call.
int ref_generate(void* handle, const int32_t* prompt, int prompt_count, int max_new_tokens, float temperature,
                 float top_p, int top_k, uint64_t seed, int32_t* tokens_out, int* token_count_out,
                 double* seconds_out) {
  try {
    auto* holder = static_cast<Holder*>(handle);
    GenerationRequest request;
    request.prompt_tokens.assign(prompt, prompt + prompt_count);
    request.max_new_tokens = max_new_tokens;
    NucleusSamplerConfig config;
    config.temperature = temperature;
    config.top_p = top_p;
    config.top_k = top_k;
    config.seed = seed;
    const std::unique_ptr<ISampler> sampler = make_sampler(config);
    cudaDeviceSynchronize();
    const auto start = std::chrono::steady_clock::now();
    const GenerationResult result = holder->shared->generate(request, *sampler);
    cudaDeviceSynchronize();
    const auto stop = std::chrono::steady_clock::now();
    for (size_t i = 0; i < result.generated_tokens.size(); ++i) tokens_out[i] = result.generated_tokens[i];
    *token_count_out = static_cast<int>(result.generated_tokens.size());
    if (seconds_out) *seconds_out = std::chrono::duration<double>(stop - start).count();
    return 0;
  } catch (const std::exception& error) {
    g_error = error.what();
    return 1;
  }
}

// The logits the reference's generate hands its sampler after the prefill (model.cu:541-542,
// read_logits :341-350): a sampler that records them, run for one new token.
namespace {
class RecordingSampler : public ISampler {
 public:
  int select(const std::vector<float>& logits) override {
    recorded = logits;
    return GreedySampler().select(logits);
  }
  std::vector<float> recorded;
};
}  // namespace

int ref_prefill_logits(void* handle, const int32_t* prompt, int prompt_count, float* logits_out) {
  try {
    auto* holder = static_cast<Holder*>(handle);
    GenerationRequest request;
    request.prompt_tokens.assign(prompt, prompt + prompt_count);
    request.max_new_tokens = 1;
    RecordingSampler sampler;
    holder->shared->generate(request, sampler);
    std::copy(sampler.recorded.begin(), sampler.recorded.end(), logits_out);
    return 0;
  } catch (const std::exception& error) {
    g_error = error.what();
    return 1;
  }
}

// ---- host-only entry points (no GPU) --------------------------------------------------------

// make_sampler (model.cpp:124-127) + select (model.cpp:70-122): `draws` selections by one sampler
// (its generator advances between them), draw d over logits[d * count, (d + 1) * count).
int ref_sample(float temperature, float top_p, int top_k, uint64_t seed, const float* logits, int count, int draws,
               int* out) {
  try {
    NucleusSamplerConfig config;
    config.temperature = temperature;
    config.top_p = top_p;
    config.top_k = top_k;
    config.seed = seed;
    const std::unique_ptr<ISampler> sampler = make_sampler(config);
    for (int d = 0; d < draws; ++d) {
      const std::vector<float> row(logits + static_cast<size_t>(d) * count, logits + static_cast<size_t>(d + 1) * count);
      out[d] = sampler->select(row);
    }
    return 0;
  } catch (const std::exception& error) {
    g_error = error.what();
    return 1;
  }
}

int ref_from_accumulated(const double* accumulated, int slots, int64_t sample_count, double* attention_out,
                         int* order_out) {
  const AttentionProfile profile = AttentionProfile::from_accumulated(
      "fixture", 0, static_cast<size_t>(sample_count), std::vector<double>(accumulated, accumulated + slots));
  for (int s = 0; s < slots; ++s) {
    attention_out[s] = profile.attention[s];
    order_out[s] = profile.position_order[s];
  }
  return 0;
}

int ref_basin_statistics(const double* attention, int slots, double min_edge_ratio, double* out5) {
  BasinCriterion criterion;
  criterion.min_edge_ratio = min_edge_ratio;
  const BasinStatistics stats = basin_statistics(std::vector<double>(attention, attention + slots), criterion);
  out5[0] = stats.first;
  out5[1] = stats.last;
  out5[2] = stats.interior_mean;
  out5[3] = stats.edge_ratio;
  out5[4] = stats.is_basin ? 1.0 : 0.0;
  return 0;
}

int ref_select_shallowest(const double* attention, const int* layer_indices, int profile_count, int slots,
                          double min_edge_ratio) {
  std::vector<AttentionProfile> profiles(static_cast<size_t>(profile_count));
  for (int p = 0; p < profile_count; ++p) {
    profiles[p].layer_index = layer_indices[p];
    profiles[p].attention.assign(attention + static_cast<size_t>(p) * slots, attention + static_cast<size_t>(p + 1) * slots);
  }
  BasinCriterion criterion;
  criterion.min_edge_ratio = min_edge_ratio;
  return select_shallowest_basin_layer(profiles, criterion);
}

int ref_resolve_position_order(const int* preferred, int preferred_count, int count, int* order_out) {
  const std::vector<int> order = resolve_position_order(std::vector<int>(preferred, preferred + preferred_count),
                                                        static_cast<size_t>(count));
  for (int i = 0; i < count; ++i) order_out[i] = order[i];
  return 0;
}

// One reranker of RerankerFactory::create (attnrank.cpp:445-456) applied `calls` times to the
// ranking 0 .. count-1 (score count - i, as engine.py's rerank_baseline builds it): out[c][i] is
// the index at position i after call c. The random reranker's state carries across calls.
int ref_rerank(const char* strategy, uint64_t seed, int lim_start_first, const int* position_order, int order_count,
               int count, int calls, int* out) {
  try {
    AttentionProfile profile;
    profile.position_order.assign(position_order, position_order + order_count);
    RerankerOptions options;
    options.profile = &profile;
    options.seed = seed;
    options.lim_start_first = lim_start_first != 0;
    const std::shared_ptr<IReranker> reranker = RerankerFactory::create(strategy, options);
    std::vector<ScoredDocument> ranked(static_cast<size_t>(count));
    for (int i = 0; i < count; ++i) {
      ranked[i].index = static_cast<size_t>(i);
      ranked[i].score = static_cast<double>(count - i);
    }
    for (int c = 0; c < calls; ++c) {
      const std::vector<ScoredDocument> result = reranker->rerank(ranked);
      for (int i = 0; i < count; ++i) out[static_cast<size_t>(c) * count + i] = static_cast<int>(result[i].index);
    }
    return 0;
  } catch (const std::exception& error) {
    g_error = error.what();
    return 1;
  }
}

}  // extern "C"
