// The drop-in, run: the reference's own AttentionLayerScanner (attnrank/src/attnrank.cpp:347-375)
// over the B200AttentionProvider that INTEGRATION.md gives a reference maintainer, compiled from
// that document's code (oracle/extract_adapter.py) against the reference's headers and linked with
// libattnrank_b200.so and the reference's compiled sources (libattnrank_ref.so). The provider is
// built from the same seeded synthetic checkpoint as the reference's CudaLlamaModel, handed over as
// a WeightRegistry. Test infrastructure only: outputs go to oracle/_ref/.
#include <memory>
#include <string>

#include "b200_provider.cpp"  // generated into oracle/_ref/ from INTEGRATION.md
#include "ref_abi.h"

namespace {
thread_local std::string g_error;
}

extern "C" {

const char* prov_last_error(void) { return g_error.c_str(); }

// A std::shared_ptr<IAttentionProvider>* owning a B200AttentionProvider over the synthetic weights.
void* prov_create(const ref_config* c, uint64_t seed, double std, int max_sequence_length, int prefill_chunk_tokens,
                  int device_index) {
  void* weights = ref_weights_create(c, seed, std, max_sequence_length);
  if (weights == nullptr) {
    g_error = ref_last_error();
    return nullptr;
  }
  try {
    const auto& registry = *static_cast<const attnrank::WeightRegistry*>(ref_weights_registry(weights));
    const auto& config = *static_cast<const attnrank::LlamaConfig*>(ref_weights_config(weights));
    attnrank::LlamaRuntimeOptions options;
    options.device_index = device_index;
    options.max_sequence_length = max_sequence_length;
    options.prefill_chunk_tokens = prefill_chunk_tokens;
    auto* provider = new std::shared_ptr<attnrank::IAttentionProvider>(
        std::make_shared<attnrank::B200AttentionProvider>(config, registry, options));
    ref_weights_destroy(weights);  // the provider holds its own device copy of every tensor
    return provider;
  } catch (const std::exception& error) {
    g_error = error.what();
    ref_weights_destroy(weights);
    return nullptr;
  }
}

void prov_destroy(void* provider) { delete static_cast<std::shared_ptr<attnrank::IAttentionProvider>*>(provider); }

int prov_scan(void* provider, const ref_prompt* prompts, int prompt_count, int span_count, int layer_begin,
              int layer_end, int normalize_by_length, double min_edge_ratio, double* attention_out, int* order_out,
              int* layer_index_out, int* layer_count_out, int* selected_out, double* seconds_out) {
  const int status = ref_scan_provider(provider, prompts, prompt_count, span_count, layer_begin, layer_end,
                                       normalize_by_length, min_edge_ratio, attention_out, order_out, layer_index_out,
                                       layer_count_out, selected_out, seconds_out);
  if (status != 0) g_error = ref_last_error();
  return status;
}

}  // extern "C"
