// extern "C" boundary of libattnrank_b200.so (declarations and reference citations in
// include/attnrank_b200.h). Every entry point converts C++ exceptions into an error code and a
// thread-local message, the way the reference's pybind layer maps attnrank::Error to
// AttnRankError (attnrank/src/bindings.cpp:134).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <numeric>
#include <utility>
#include <string>
#include <vector>

#include "../../include/attnrank_b200.h"
#include "capi_guard.h"
#include "decode.h"
#include "engine.h"
#include "layer_kernels.h"
#include "mass_call.h"
#include "mass_plan.h"
#include "profile.h"
#include "synthetic.h"

struct ar_engine {
  std::unique_ptr<arb::Engine> engine;
};

struct ar_prepared_scan {
  std::unique_ptr<arb::PreparedScan> scan;
};

struct ar_sampler {
  std::unique_ptr<arb::TokenSampler> sampler;
};

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& message) {
  g_last_error = message;
  return code;
}

template <typename F>
int guarded(F&& body) {
  return arb::guarded_call(std::forward<F>(body));
}

int cuda_result(cudaError_t status, const char* what) {
  if (status == cudaSuccess) return AR_OK;
  return fail(status == cudaErrorInvalidValue ? AR_ERR_INVALID : AR_ERR_CUDA,
              std::string(what) + ": " + cudaGetErrorString(status));
}

cudaStream_t as_stream(void* stream) { return static_cast<cudaStream_t>(stream); }

std::vector<arb::PromptView> prompt_views(const ar_prompt* prompts, int count) {
  if (prompts == nullptr || count <= 0) throw arb::Error("at least one probe prompt is required");
  std::vector<arb::PromptView> views(count);
  for (int i = 0; i < count; ++i) {
    if (prompts[i].tokens == nullptr || prompts[i].spans == nullptr) throw arb::Error("probe prompt has null arrays");
    views[i].tokens = prompts[i].tokens;
    views[i].token_count = prompts[i].token_count;
    views[i].query_begin = prompts[i].query_begin;
    views[i].query_end = prompts[i].query_end;
    views[i].spans = prompts[i].spans;
  }
  return views;
}

// Device scratch owned by one kernel-level call (released on the call's stream).
struct StreamScratch {
  cudaStream_t stream;
  std::vector<void*> blocks;
  explicit StreamScratch(cudaStream_t s) : stream(s) {}
  void* get(size_t bytes) {
    void* pointer = nullptr;
    arb::check_cuda(cudaMallocAsync(&pointer, std::max<size_t>(bytes, 16), stream), "scratch allocation");
    blocks.push_back(pointer);
    return pointer;
  }
  ~StreamScratch() {
    for (void* pointer : blocks) cudaFreeAsync(pointer, stream);
  }
};

}  // namespace

namespace arb {
void set_last_error(const std::string& message) { g_last_error = message; }
}  // namespace arb

extern "C" {

const char* ar_last_error(void) { return g_last_error.c_str(); }

const char* ar_version(void) { return "attnrank-b200 0.1.0 (sm_100a)"; }

int ar_embedding_rms_norm(const int32_t* token_ids, int token_count, const void* table, int vocab_size,
                          int hidden_size, const float* gamma, float eps, float* residual, void* normed,
                          int* device_status, int dtype, void* stream) {
  if (token_count < 0 || hidden_size <= 0 || hidden_size % 8 != 0 || vocab_size <= 0) {
    return fail(AR_ERR_INVALID, "embedding: invalid sizes (hidden_size must be a positive multiple of 8)");
  }
  return cuda_result(arb::launch_embed_rms_norm(token_ids, token_count, table, vocab_size, hidden_size, gamma, eps,
                                                residual, normed, device_status, dtype, as_stream(stream)),
                     "embedding_rms_norm");
}

int ar_rms_norm_residual(float* residual, const void* delta, const float* gamma, int token_count, int hidden_size,
                         float eps, void* normed, int dtype, void* stream) {
  if (token_count < 0 || hidden_size <= 0 || hidden_size % 8 != 0) {
    return fail(AR_ERR_INVALID, "rms_norm_residual: hidden_size must be a positive multiple of 8");
  }
  return cuda_result(arb::launch_rms_norm_residual(residual, delta, gamma, token_count, hidden_size, eps, normed, dtype,
                                                   as_stream(stream)),
                     "rms_norm_residual");
}

int ar_rotary_embedding(void* qkv, const float* bias, const int32_t* positions, int token_count, int query_heads,
                        int kv_heads, int head_dim, const float* cos_table, const float* sin_table,
                        int table_positions, int* device_status, int dtype, void* stream) {
  if (token_count < 0 || query_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || head_dim % 16 != 0) {
    return fail(AR_ERR_INVALID, "rotary_embedding: head_dim must be a positive multiple of 16");
  }
  return cuda_result(arb::launch_rotary_bias(qkv, bias, positions, token_count, query_heads, kv_heads, head_dim,
                                             cos_table, sin_table, table_positions, device_status, dtype,
                                             as_stream(stream)),
                     "rotary_embedding");
}

int ar_rope_table(float* cos_table, float* sin_table, int positions, int head_dim, float theta, void* stream) {
  if (positions < 0 || head_dim <= 0 || head_dim % 2 != 0) return fail(AR_ERR_INVALID, "rope_table: invalid sizes");
  return cuda_result(arb::launch_rope_table(cos_table, sin_table, positions, head_dim, theta, as_stream(stream)),
                     "rope_table");
}

int ar_silu_multiply(const void* gate, const void* up, int64_t in_row_stride, void* out, int64_t out_row_stride,
                     int token_count, int width, int dtype, void* stream) {
  if (token_count < 0 || width <= 0 || width % 8 != 0 || in_row_stride % 8 != 0 || out_row_stride % 8 != 0) {
    return fail(AR_ERR_INVALID, "silu_multiply: width and strides must be multiples of 8");
  }
  return cuda_result(arb::launch_silu_multiply(gate, up, in_row_stride, out, out_row_stride, token_count, width, dtype,
                                               as_stream(stream)),
                     "silu_multiply");
}

}  // extern "C"

namespace {

int causal_attention_call(bool tcgen05, const void* qkv, void* out, float* lse, const int32_t* prompt_offsets_host,
                          const int32_t* prompt_offsets_device, int prompt_count, int query_heads, int kv_heads,
                          int head_dim, int sliding_window, int dtype, void* stream) {
  return guarded([&] {
    if (prompt_count <= 0 || head_dim != 128 || kv_heads <= 0 || query_heads % kv_heads != 0) {
      throw arb::Error("causal_attention: head_dim must be 128 and query_heads a multiple of kv_heads");
    }
    if (dtype != arb::kActFp16 && dtype != arb::kActBf16) throw arb::Error("causal_attention: dtype must be fp16 or bf16");
    std::vector<int32_t> tiles;
    int max_tiles = 0;
    for (int p = 0; p < prompt_count; ++p) {
      const int length = prompt_offsets_host[p + 1] - prompt_offsets_host[p];
      if (length < 0) throw arb::Error("causal_attention: prompt offsets must be non-decreasing");
      max_tiles = std::max(max_tiles, (length + arb::kAttentionQueryTile - 1) / arb::kAttentionQueryTile);
    }
    for (int t = max_tiles - 1; t >= 0; --t) {
      for (int p = 0; p < prompt_count; ++p) {
        if (t * arb::kAttentionQueryTile < prompt_offsets_host[p + 1] - prompt_offsets_host[p]) {
          tiles.push_back(p);
          tiles.push_back(t);
        }
      }
    }
    if (tiles.empty()) return AR_OK;
    cudaStream_t s = as_stream(stream);
    StreamScratch scratch(s);
    auto* tiles_device = static_cast<int32_t*>(scratch.get(tiles.size() * sizeof(int32_t)));
    auto* status = static_cast<int*>(scratch.get(sizeof(int)));
    arb::check_cuda(cudaMemsetAsync(status, 0, sizeof(int), s), "status reset");
    arb::check_cuda(cudaMemcpyAsync(tiles_device, tiles.data(), tiles.size() * sizeof(int32_t), cudaMemcpyHostToDevice, s),
                    "tile upload");
    arb::AttentionArgs args;
    args.qkv = qkv;
    args.out = out;
    args.lse = lse;
    args.prompt_offsets = prompt_offsets_device;
    args.tiles = tiles_device;
    args.tile_count = static_cast<int>(tiles.size() / 2);
    args.query_heads = query_heads;
    args.kv_heads = kv_heads;
    args.head_dim = head_dim;
    args.sliding_window = sliding_window;
    args.dtype = dtype;
    args.rows = prompt_offsets_host[prompt_count];
    args.status = status;
    arb::check_cuda(tcgen05 ? arb::launch_causal_attention_tc(args, s) : arb::launch_causal_attention(args, s),
                    "causal_attention");
    int device_status = 0;
    arb::check_cuda(cudaMemcpyAsync(&device_status, status, sizeof(int), cudaMemcpyDeviceToHost, s), "status read");
    arb::check_cuda(cudaStreamSynchronize(s), "causal_attention");  // host tile list lifetime
    if (device_status != 0) {
      throw arb::Error("causal_attention: device reported status " + std::to_string(device_status));
    }
    return AR_OK;
  });
}

}  // namespace

extern "C" {

int ar_causal_attention(const void* qkv, void* out, float* lse, const int32_t* prompt_offsets_host,
                        const int32_t* prompt_offsets_device, int prompt_count, int query_heads, int kv_heads,
                        int head_dim, int sliding_window, int dtype, void* stream) {
  return causal_attention_call(true, qkv, out, lse, prompt_offsets_host, prompt_offsets_device, prompt_count,
                               query_heads, kv_heads, head_dim, sliding_window, dtype, stream);
}

int ar_causal_attention_mma(const void* qkv, void* out, float* lse, const int32_t* prompt_offsets_host,
                            const int32_t* prompt_offsets_device, int prompt_count, int query_heads, int kv_heads,
                            int head_dim, int sliding_window, int dtype, void* stream) {
  return causal_attention_call(false, qkv, out, lse, prompt_offsets_host, prompt_offsets_device, prompt_count,
                               query_heads, kv_heads, head_dim, sliding_window, dtype, stream);
}

int ar_document_attention_mass(const void* qkv, int qkv_rows, const float* lse, const int32_t* prompt_offsets_host,
                               int prompt_count, const int32_t* query_spans_host, const int32_t* spans_host,
                               int span_count, int query_heads, int kv_heads, int head_dim, int sliding_window,
                               int prefill_chunk_tokens, int normalize_by_length, double* mass_out, int dtype,
                               void* stream) {
  return guarded([&] {
    const char* who = "document_attention_mass";
    arb::MassCallArgs call{qkv, qkv_rows, lse, prompt_offsets_host, prompt_count, query_spans_host, spans_host,
                           span_count, query_heads, kv_heads, head_dim, sliding_window, prefill_chunk_tokens,
                           normalize_by_length, mass_out, dtype};
    const arb::MassBatch batch = arb::plan_mass_batch(who, call);
    const arb::MassScratchLayout layout = arb::mass_scratch_layout(batch);
    cudaStream_t s = as_stream(stream);
    StreamScratch scratch(s);
    arb::run_mass_batch(who, call, batch, layout, scratch.get(layout.total), s);
    return AR_OK;
  });
}

int ar_synthetic_fill(void* dst, int64_t count, uint64_t seed, int layer, int kind, float standard_deviation,
                      int dtype, void* stream) {
  if (count < 0) return fail(AR_ERR_INVALID, "synthetic_fill: negative count");
  return cuda_result(arb::launch_synthetic_fill(dst, count, arb::synthetic_tensor_key(seed, layer, kind),
                                                arb::synthetic_scale(standard_deviation), dtype, as_stream(stream)),
                     "synthetic_fill");
}

int ar_engine_create(const ar_llama_config* config, const ar_runtime_options* options, ar_engine** engine) {
  return guarded([&] {
    if (config == nullptr || engine == nullptr) throw arb::Error("engine_create: null argument");
    arb::ModelConfig c;
    c.hidden_size = config->hidden_size;
    c.intermediate_size = config->intermediate_size;
    c.num_hidden_layers = config->num_hidden_layers;
    c.num_attention_heads = config->num_attention_heads;
    c.num_key_value_heads = config->num_key_value_heads;
    c.vocab_size = config->vocab_size;
    c.max_position_embeddings = config->max_position_embeddings;
    c.rms_norm_eps = config->rms_norm_eps;
    c.rope_theta = config->rope_theta;
    c.sliding_window = config->sliding_window;
    c.attention_bias = config->attention_bias != 0;
    c.tie_word_embeddings = config->tie_word_embeddings != 0;
    arb::RuntimeOptions o;
    if (options != nullptr) {
      o.device_index = options->device_index;
      if (options->max_sequence_length > 0) o.max_sequence_length = options->max_sequence_length;
      if (options->prefill_chunk_tokens > 0) o.prefill_chunk_tokens = options->prefill_chunk_tokens;
      if (options->max_batch_tokens > 0) o.max_batch_tokens = options->max_batch_tokens;
      if (options->max_batch_prompts > 0) o.max_batch_prompts = options->max_batch_prompts;
      if (options->activation_dtype != 0) o.activation_dtype = options->activation_dtype;
      o.attention_kernel = options->attention_kernel;
    }
    auto holder = std::make_unique<ar_engine>();
    holder->engine = std::make_unique<arb::Engine>(c, o);
    *engine = holder.release();
    return AR_OK;
  });
}

void ar_engine_destroy(ar_engine* engine) { delete engine; }

int ar_engine_load_tensor(ar_engine* engine, const char* name, int dtype, const int64_t* shape, int rank,
                          const void* host_data) {
  return guarded([&] {
    if (engine == nullptr || name == nullptr || host_data == nullptr || rank < 0) throw arb::Error("load_tensor: null argument");
    engine->engine->load_tensor(name, dtype, std::vector<int64_t>(shape, shape + rank), host_data);
    return AR_OK;
  });
}

int ar_engine_init_synthetic(ar_engine* engine, uint64_t seed, float standard_deviation) {
  return guarded([&] {
    if (engine == nullptr) throw arb::Error("init_synthetic: null engine");
    engine->engine->init_synthetic(seed, standard_deviation);
    return AR_OK;
  });
}

int ar_engine_measure_attention_by_layer(ar_engine* engine, const ar_prompt* prompts, int prompt_count, int span_count,
                                         int layer_begin, int layer_end, int normalize_by_length, double* rows_out,
                                         int* layer_begin_out, int* layer_count_out) {
  return guarded([&] {
    if (engine == nullptr || rows_out == nullptr) throw arb::Error("measure_attention_by_layer: null argument");
    const arb::LayerRange range = engine->engine->resolve_layers(layer_begin, layer_end);
    engine->engine->probe(prompt_views(prompts, prompt_count), span_count, range, normalize_by_length != 0, rows_out,
                          nullptr, nullptr);
    if (layer_begin_out) *layer_begin_out = range.begin;
    if (layer_count_out) *layer_count_out = range.count();
    return AR_OK;
  });
}

int ar_engine_measure_attention(ar_engine* engine, const ar_prompt* prompt, int span_count, int layer_begin,
                                int layer_end, int normalize_by_length, double* attention_out) {
  return guarded([&] {
    if (engine == nullptr || attention_out == nullptr) throw arb::Error("measure_attention: null argument");
    if (layer_begin < 0 || layer_end <= layer_begin) throw arb::Error("measure_attention: invalid layer range");
    const arb::LayerRange range = engine->engine->resolve_layers(layer_begin, layer_end);
    std::vector<double> raw(static_cast<size_t>(range.count()) * span_count);
    engine->engine->probe(prompt_views(prompt, 1), span_count, range, normalize_by_length != 0, nullptr, raw.data(),
                          nullptr);
    // model.cu:576-589: totals / (query_rows * Hq * layers), summed over layers, unit-sum.
    for (int s = 0; s < span_count; ++s) attention_out[s] = 0.0;
    for (int l = 0; l < range.count(); ++l) {
      for (int s = 0; s < span_count; ++s) attention_out[s] += raw[static_cast<size_t>(l) * span_count + s] / range.count();
    }
    arb::normalize_to_unit_sum(attention_out, span_count);
    return AR_OK;
  });
}

int ar_engine_scan(ar_engine* engine, const ar_prompt* prompts, int prompt_count, int span_count, int layer_begin,
                   int layer_end, int normalize_by_length, float* device_accumulator, double* host_accumulator) {
  return guarded([&] {
    if (engine == nullptr || device_accumulator == nullptr) throw arb::Error("scan: null argument");
    const arb::LayerRange range = engine->engine->resolve_layers(layer_begin, layer_end);
    engine->engine->probe(prompt_views(prompts, prompt_count), span_count, range, normalize_by_length != 0, nullptr,
                          nullptr, device_accumulator);
    if (host_accumulator != nullptr) {
      const size_t n = static_cast<size_t>(range.count()) * span_count;
      std::vector<float> values(n);
      arb::check_cuda(cudaMemcpyAsync(values.data(), device_accumulator, n * sizeof(float), cudaMemcpyDeviceToHost,
                                      engine->engine->stream()),
                      "accumulator download");
      engine->engine->synchronize();
      for (size_t i = 0; i < n; ++i) host_accumulator[i] = values[i];
    }
    return AR_OK;
  });
}

int ar_engine_prepare_scan(ar_engine* engine, const ar_prompt* prompts, int prompt_count, int span_count,
                           int layer_begin, int layer_end, int normalize_by_length, ar_prepared_scan** prepared) {
  return guarded([&] {
    if (engine == nullptr || prepared == nullptr) throw arb::Error("prepare_scan: null argument");
    const arb::LayerRange range = engine->engine->resolve_layers(layer_begin, layer_end);
    auto holder = std::make_unique<ar_prepared_scan>();
    holder->scan = engine->engine->prepare_scan(prompt_views(prompts, prompt_count), span_count, range,
                                                normalize_by_length != 0);
    *prepared = holder.release();
    return AR_OK;
  });
}

int ar_engine_run_prepared_scan(ar_engine* engine, const ar_prepared_scan* prepared, float* device_accumulator,
                                int synchronize) {
  return guarded([&] {
    if (engine == nullptr || prepared == nullptr || device_accumulator == nullptr) {
      throw arb::Error("run_prepared_scan: null argument");
    }
    engine->engine->run_prepared(*prepared->scan, device_accumulator);
    if (synchronize) arb::Engine::raise_on_status(engine->engine->read_status());
    return AR_OK;
  });
}

void ar_prepared_scan_destroy(ar_prepared_scan* prepared) { delete prepared; }

int64_t ar_prepared_scan_bytes(const ar_prepared_scan* prepared) {
  return prepared ? static_cast<int64_t>(prepared->scan->device_bytes) : 0;
}

int ar_engine_synchronize(ar_engine* engine) {
  return guarded([&] {
    if (engine == nullptr) throw arb::Error("synchronize: null engine");
    const int status = engine->engine->read_status();
    engine->engine->reset_status();
    arb::Engine::raise_on_status(status);
    return AR_OK;
  });
}

void* ar_engine_stream(ar_engine* engine) { return engine ? static_cast<void*>(engine->engine->stream()) : nullptr; }

int ar_engine_device(ar_engine* engine) { return engine ? engine->engine->options().device_index : -1; }

int ar_engine_set_kernel_timing(ar_engine* engine, int enabled) {
  return guarded([&] {
    if (engine == nullptr) throw arb::Error("set_kernel_timing: null engine");
    engine->engine->set_kernel_timing(enabled != 0);
    return AR_OK;
  });
}

int ar_engine_kernel_timing(ar_engine* engine, double* milliseconds, double* work, int64_t* launches) {
  return guarded([&] {
    if (engine == nullptr) throw arb::Error("kernel_timing: null engine");
    static_assert(arb::kKernelClassCount == AR_KERNEL_CLASS_COUNT, "kernel class count");
    engine->engine->kernel_timing(milliseconds, work, launches);
    return AR_OK;
  });
}

const char* ar_kernel_class_name(int kernel_class) { return arb::kernel_class_name(kernel_class); }

int ar_kernel_class_is_tensor(int kernel_class) { return arb::kernel_class_is_tensor(kernel_class) ? 1 : 0; }

// ---- generation ----------------------------------------------------------------------------

namespace {
arb::SamplerConfig sampler_config(const ar_sampler_config* config) {
  arb::SamplerConfig c;
  if (config != nullptr) {
    c.temperature = config->temperature;
    c.top_p = config->top_p;
    c.top_k = config->top_k;
    c.seed = config->seed;
  }
  return c;
}
}  // namespace

int ar_engine_generate(ar_engine* engine, const int32_t* prompt, int prompt_count, int max_new_tokens,
                       int eos_token_id, const ar_sampler_config* sampler, int32_t* tokens_out, int* token_count_out) {
  return guarded([&] {
    if (engine == nullptr || token_count_out == nullptr || (max_new_tokens > 0 && tokens_out == nullptr)) {
      throw arb::Error("generate: null argument");
    }
    const std::vector<int32_t> tokens = engine->engine->generate(prompt, prompt_count, max_new_tokens, eos_token_id,
                                                                 sampler_config(sampler));
    std::copy(tokens.begin(), tokens.end(), tokens_out);
    *token_count_out = static_cast<int>(tokens.size());
    return AR_OK;
  });
}

int ar_engine_generation_begin(ar_engine* engine, const int32_t* prompt, int prompt_count, float* logits_out) {
  return guarded([&] {
    if (engine == nullptr) throw arb::Error("generation_begin: null engine");
    engine->engine->begin_generation(prompt, prompt_count);
    if (logits_out != nullptr) engine->engine->read_logits(logits_out);
    return AR_OK;
  });
}

int ar_engine_generation_step(ar_engine* engine, int32_t token, float* logits_out) {
  return guarded([&] {
    if (engine == nullptr) throw arb::Error("generation_step: null engine");
    engine->engine->decode_token(token);
    if (logits_out != nullptr) {
      engine->engine->read_logits(logits_out);
    } else {
      const int status = engine->engine->read_status();  // synchronises
      if (status != 0) {
        engine->engine->reset_status();
        arb::Engine::raise_on_status(status);
      }
    }
    return AR_OK;
  });
}

int ar_engine_generation_position(ar_engine* engine) {
  return engine ? engine->engine->generation_position() : -1;
}

int ar_engine_decode_mode(ar_engine* engine) { return engine != nullptr ? engine->engine->decode_mode() : -1; }

int ar_sampler_create(const ar_sampler_config* config, ar_sampler** sampler) {
  return guarded([&] {
    if (config == nullptr || sampler == nullptr) throw arb::Error("sampler_create: null argument");
    auto holder = std::make_unique<ar_sampler>();
    holder->sampler = arb::make_token_sampler(sampler_config(config));
    *sampler = holder.release();
    return AR_OK;
  });
}

int ar_sampler_select(ar_sampler* sampler, const float* logits, int count, int32_t* token_out) {
  return guarded([&] {
    if (sampler == nullptr || token_out == nullptr) throw arb::Error("sampler_select: null argument");
    *token_out = sampler->sampler->select(logits, count);
    return AR_OK;
  });
}

void ar_sampler_destroy(ar_sampler* sampler) { delete sampler; }

int ar_decode_gemv(const void* w, const void* x, int rows, int k, void* y, int f32_out, int dtype, void* stream) {
  if (rows <= 0 || k <= 0 || k % 8 != 0) return fail(AR_ERR_INVALID, "decode_gemv: k must be a positive multiple of 8");
  arb::DecodeGemvArgs args;
  args.kind = f32_out ? arb::kDecodeLogits : arb::kDecodePlain;
  args.w = w;
  args.rows = rows;
  args.k = k;
  args.x = x;
  args.y = y;
  args.dtype = dtype;
  return cuda_result(arb::launch_decode_gemv(args, false, as_stream(stream)), "decode_gemv");
}

int ar_decode_gate_up(const void* w, const void* x, int inter, int k, void* act, int dtype, void* stream) {
  if (inter <= 0 || k <= 0 || k % 8 != 0) {
    return fail(AR_ERR_INVALID, "decode_gate_up: k must be a positive multiple of 8");
  }
  arb::DecodeGemvArgs args;
  args.kind = arb::kDecodeGateUp;
  args.w = w;
  args.rows = inter;
  args.k = k;
  args.x = x;
  args.y = act;
  args.dtype = dtype;
  return cuda_result(arb::launch_decode_gemv(args, false, as_stream(stream)), "decode_gate_up");
}

int ar_decode_attention(const void* q, const void* k_cache, const void* v_cache, int context, int position,
                        int query_heads, int kv_heads, int head_dim, int sliding_window, void* out, int dtype,
                        void* stream) {
  return guarded([&] {
    if (head_dim != 128 || kv_heads <= 0 || query_heads % kv_heads != 0 ||
        query_heads / kv_heads > arb::kDecodeMaxGroup) {
      throw arb::Error("decode_attention: head_dim must be 128 and query_heads a multiple (<= 16x) of kv_heads");
    }
    if (position < 0 || position >= context) throw arb::Error("decode_attention: position outside the cache");
    cudaStream_t s = as_stream(stream);
    StreamScratch scratch(s);
    auto* state = static_cast<int32_t*>(scratch.get(2 * sizeof(int32_t)));
    const int32_t host_state[2] = {0, position};
    arb::check_cuda(cudaMemcpyAsync(state, host_state, sizeof(host_state), cudaMemcpyHostToDevice, s), "state upload");
    arb::DecodeAttentionArgs args;
    args.q = q;
    args.k_cache = k_cache;
    args.v_cache = v_cache;
    args.context = context;
    args.state = state;
    args.query_heads = query_heads;
    args.kv_heads = kv_heads;
    args.head_dim = head_dim;
    args.sliding_window = sliding_window;
    args.partials = static_cast<float*>(scratch.get(static_cast<size_t>(query_heads) * arb::kDecodeSplits * head_dim * 4));
    args.stats = static_cast<float*>(scratch.get(static_cast<size_t>(query_heads) * arb::kDecodeSplits * 2 * 4));
    args.tickets = static_cast<unsigned*>(scratch.get(static_cast<size_t>(kv_heads) * sizeof(unsigned)));
    arb::check_cuda(cudaMemsetAsync(args.tickets, 0, static_cast<size_t>(kv_heads) * sizeof(unsigned), s), "tickets");
    args.out = out;
    args.dtype = dtype;
    arb::check_cuda(arb::launch_decode_attention(args, false, s), "decode_attention");
    arb::check_cuda(cudaStreamSynchronize(s), "decode_attention");  // host_state outlives the copy
    return AR_OK;
  });
}

int ar_bounded_wait_selftest(int ctas, uint32_t spin_limit, void* stream) {
  return guarded([&] {
    if (ctas <= 0 || ctas > 1024 || spin_limit == 0 || spin_limit > (1u << 22)) {
      throw arb::Error("bounded_wait_selftest: ctas must be 1..1024 and spin_limit 1..4194304");
    }
    cudaStream_t s = as_stream(stream);
    StreamScratch scratch(s);
    auto* words = static_cast<unsigned*>(scratch.get(2 * sizeof(unsigned)));  // counter | status
    arb::check_cuda(cudaMemsetAsync(words, 0, 2 * sizeof(unsigned), s), "selftest reset");
    arb::check_cuda(arb::launch_bounded_wait_selftest(words, reinterpret_cast<int*>(words + 1), ctas, spin_limit, s),
                    "bounded_wait_selftest");
    unsigned status = 0;
    arb::check_cuda(cudaMemcpyAsync(&status, words + 1, sizeof(unsigned), cudaMemcpyDeviceToHost, s), "status read");
    arb::check_cuda(cudaStreamSynchronize(s), "bounded_wait_selftest");
    if (status != static_cast<unsigned>(arb::kStatusWaitTimeout)) {
      throw arb::Error("bounded_wait_selftest: the unreachable wait ended with status " + std::to_string(status) +
                       " instead of a wait timeout");
    }
    throw arb::Error("device reported a wait timeout (status " + std::to_string(status) +
                     "): the bounded wait gave up as designed");
    return AR_OK;
  });
}

int ar_profile_from_accumulated(const double* accumulated, int slots, int64_t sample_count, double* attention_out,
                                int* position_order_out) {
  return guarded([&] {
    if (slots < 0 || (slots > 0 && (accumulated == nullptr || attention_out == nullptr))) {
      throw arb::Error("profile_from_accumulated: invalid arguments");
    }
    arb::profile_from_accumulated(accumulated, slots, sample_count, attention_out, position_order_out);
    return AR_OK;
  });
}

int ar_position_order(const double* attention, int slots, int* position_order_out) {
  return guarded([&] {
    if (slots < 0) throw arb::Error("position_order: negative slot count");
    arb::stable_descending_order(attention, slots, position_order_out);
    return AR_OK;
  });
}

int ar_basin_statistics(const double* attention, int slots, double min_edge_ratio, ar_basin_stats* out) {
  return guarded([&] {
    if (out == nullptr || slots < 0) throw arb::Error("basin_statistics: invalid arguments");
    const arb::BasinStatistics stats = arb::basin_statistics(attention, slots, min_edge_ratio);
    out->first = stats.first;
    out->last = stats.last;
    out->interior_mean = stats.interior_mean;
    out->edge_ratio = stats.edge_ratio;
    out->is_basin = stats.is_basin ? 1 : 0;
    return AR_OK;
  });
}

int ar_select_shallowest_basin_layer(const double* attention, const int* layer_indices, int profile_count, int slots,
                                     double min_edge_ratio, int* selected_out) {
  return guarded([&] {
    if (selected_out == nullptr || profile_count < 0 || slots < 0) throw arb::Error("select_shallowest_basin_layer: invalid arguments");
    *selected_out = arb::select_shallowest_basin_layer(attention, layer_indices, profile_count, slots, min_edge_ratio);
    return AR_OK;
  });
}

int ar_resolve_position_order(const int* preferred, int preferred_count, int count, int* order_out) {
  return guarded([&] {
    if (count < 0 || preferred_count < 0 || (count > 0 && order_out == nullptr)) {
      throw arb::Error("resolve_position_order: invalid arguments");
    }
    arb::resolve_position_order(preferred, preferred_count, count, order_out);
    return AR_OK;
  });
}

}  // extern "C"
