/* C entry points of oracle/_ref/libattnrank_ref.so (ref_harness.cpp) that another harness links
 * against. Test infrastructure only. */
#ifndef ATTNRANK_ORACLE_REF_ABI_H
#define ATTNRANK_ORACLE_REF_ABI_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct ref_config {
  int hidden_size;
  int intermediate_size;
  int num_hidden_layers;
  int num_attention_heads;
  int num_key_value_heads;
  int vocab_size;
  float rms_norm_eps;
  float rope_theta;
  int sliding_window;
  int attention_bias;
};

struct ref_prompt {
  const int32_t* tokens;
  int token_count;
  int query_begin;
  int query_end;
  const int32_t* spans;
};

const char* ref_last_error(void);

/* The seeded synthetic checkpoint: a heap object holding a LlamaConfig and a WeightRegistry
 * (attnrank/checkpoint.hpp:27-39); the accessors return pointers to those two objects. */
void* ref_weights_create(const struct ref_config* c, uint64_t seed, double std, int max_sequence_length);
void ref_weights_destroy(void* weights);
const void* ref_weights_registry(void* weights);
const void* ref_weights_config(void* weights);

/* AttentionLayerScanner::scan + select_shallowest_basin_layer over `provider`, a
 * std::shared_ptr<attnrank::IAttentionProvider>*. Outputs as ref_scan. */
int ref_scan_provider(void* provider, const struct ref_prompt* prompts, int prompt_count, int span_count,
                      int layer_begin, int layer_end, int normalize_by_length, double min_edge_ratio,
                      double* attention_out, int* order_out, int* layer_index_out, int* layer_count_out,
                      int* selected_out, double* seconds_out);

#ifdef __cplusplus
}
#endif

#endif
