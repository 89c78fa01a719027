/*
 * attnrank_b200.h -- C ABI of the B200 attention-profiling library (libattnrank_b200.so).
 *
 * Drop-in boundary for the hot path of AttnRank (Syun1208/attention-rank): the layer-kernel
 * library, the attention-capture forward pass, the profile accumulator and the basin pick.
 * Plain pointers and sizes only. Every function returns AR_OK (0) or an AR_ERR_* code; the
 * message of the last failure on the calling thread is available from ar_last_error().
 *
 * Citations are to files of the reference project (path:line).
 */
#ifndef ATTNRANK_B200_H
#define ATTNRANK_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AR_OK 0
#define AR_ERR_INVALID 1   /* bad argument (the reference throws attnrank::Error)              */
#define AR_ERR_CUDA 2      /* CUDA runtime / cuBLASLt failure (kernels.cu:244-254)               */
#define AR_ERR_DEVICE 3    /* a kernel reported a bad input (token id, position) or a wait timeout */
#define AR_ERR_INTERNAL 4

#define AR_DTYPE_F32 0
#define AR_DTYPE_F16 1
#define AR_DTYPE_BF16 2

/* Message of the last error raised on this thread ("" if none). */
const char* ar_last_error(void);
/* Library version string. */
const char* ar_version(void);

/* ------------------------------------------------------------------------------------------
 * Layer kernels. Device pointers, asynchronous on `stream` (a cudaStream_t, NULL = default).
 * They replace the reference's kernels:: launchers (attnrank/src/cuda_runtime.hpp:115-144).
 * Activations are 16-bit -- `dtype` AR_DTYPE_F16 (the reference's GEMM operand type,
 * model.cu:353-365) or AR_DTYPE_BF16 -- the residual stream fp32, norm weights and biases fp32.
 * ------------------------------------------------------------------------------------------ */

/* Replaces kernels::embedding_lookup (cuda_runtime.hpp:123-124, kernels.cu:424-430) fused with
 * the first kernels::rms_norm (kernels.cu:432-439): residual[t] = table[ids[t]] (fp32),
 * normed[t] = 16-bit(residual[t] * rsqrt(mean(residual[t]^2) + eps) * gamma).
 * Out-of-range ids set *device_status (nullable) to 1 and produce a zero row. */
int ar_embedding_rms_norm(const int32_t* token_ids, int token_count, const void* table, int vocab_size,
                          int hidden_size, const float* gamma, float eps, float* residual, void* normed,
                          int* device_status, int dtype, void* stream);

/* Replaces kernels::add_in_place + kernels::rms_norm (cuda_runtime.hpp:126-127, :135;
 * model.cu:398 then :408-409): residual += delta; normed = 16-bit(rms(residual) * gamma).
 * delta may be NULL (kernels::rms_norm alone, cuda_runtime.hpp:126-127): the residual is then
 * only read, and left unchanged. */
int ar_rms_norm_residual(float* residual, const void* delta, const float* gamma, int token_count,
                         int hidden_size, float eps, void* normed, int dtype, void* stream);

/* Replaces kernels::add_row_bias (cuda_runtime.hpp:137) + kernels::rotary_embedding
 * (cuda_runtime.hpp:129, kernels.cu:85-115), in place on the fused q|k|v projection output
 * [token_count, (Hq + 2 Hkv) * head_dim] 16-bit. bias (nullable) is fp32 [(Hq + 2 Hkv) * head_dim];
 * positions are int32 per token; cos/sin tables come from ar_rope_table. */
int ar_rotary_embedding(void* qkv, const float* bias, const int32_t* positions, int token_count,
                        int query_heads, int kv_heads, int head_dim, const float* cos_table,
                        const float* sin_table, int table_positions, int* device_status, int dtype, void* stream);

/* cos/sin of position * theta^(-2i/head_dim), fp32 [positions, head_dim / 2] each; the values of
 * the reference's per-element computation (kernels.cu:95-98). */
int ar_rope_table(float* cos_table, float* sin_table, int positions, int head_dim, float theta, void* stream);

/* Replaces kernels::silu_multiply (cuda_runtime.hpp:131, kernels.cu:164-170):
 * out[t, i] = silu(gate[t, i]) * up[t, i], 16-bit, rows addressed with the given strides (elements). */
int ar_silu_multiply(const void* gate, const void* up, int64_t in_row_stride, void* out,
                     int64_t out_row_stride, int token_count, int width, int dtype, void* stream);

/* Replaces the materialised attention of LlamaForwardPass::attend (model.cu:426-480:
 * scatter_kv_cache, SGEMM Q K^T, softmax_causal_kernel, SGEMM P V) for packed prompts.
 * qkv: 16-bit [tokens, (Hq + 2 Hkv) * 128]; out: 16-bit [tokens, Hq * 128];
 * lse: fp32 [tokens, Hq], log2-domain log-sum-exp of the scaled scores of each row.
 * prompt_offsets: int32 [prompt_count + 1] (host copy and device copy). head_dim must be 128.
 * Runs the tcgen05/TMEM kernel; synchronises the stream and reports a device-side wait timeout
 * as AR_ERR_DEVICE. */
int ar_causal_attention(const void* qkv, void* out, float* lse, const int32_t* prompt_offsets_host,
                        const int32_t* prompt_offsets_device, int prompt_count, int query_heads, int kv_heads,
                        int head_dim, int sliding_window, int dtype, void* stream);

/* The same contract computed by the mma.sync (warp-level tensor core) kernel; kept as the
 * engine's alternative (ar_runtime_options.attention_kernel = 1) and as a cross-check. */
int ar_causal_attention_mma(const void* qkv, void* out, float* lse, const int32_t* prompt_offsets_host,
                            const int32_t* prompt_offsets_device, int prompt_count, int query_heads, int kv_heads,
                            int head_dim, int sliding_window, int dtype, void* stream);

/* Replaces kernels::reduce_document_attention (cuda_runtime.hpp:139, kernels.cu:202-236) over
 * the output of softmax_causal_kernel, without any score matrix. For each prompt p and span s,
 *   mass[p][s] = sum over heads h and query rows q of sum_{k in span s} softmax(q.k / sqrt(D))
 * (each (h, q) term divided by the span length when normalize_by_length), i.e. the value the
 * reference accumulates for one layer. mass_out[p][s] = mass[p][s] / (query_rows * Hq), the row
 * of model.cu:613 before its unit-sum step (fp64 host, [prompt_count][span_count]).
 * Host arrays (prompt-relative): query_spans [prompt_count][2], spans [prompt_count][span_count][2].
 * lse is the output of ar_causal_attention on the same qkv. Allocates its scratch (metadata and
 * per-CTA partial sums) with cudaMallocAsync on `stream` and synchronises the stream. */
int ar_document_attention_mass(const void* qkv, int qkv_rows, const float* lse, const int32_t* prompt_offsets_host,
                               int prompt_count, const int32_t* query_spans_host, const int32_t* spans_host,
                               int span_count, int query_heads, int kv_heads, int head_dim, int sliding_window,
                               int prefill_chunk_tokens, int normalize_by_length, double* mass_out, int dtype,
                               void* stream);

/* The same computation as ar_document_attention_mass for callers that cannot let the library
 * allocate device memory while they run (a process holding the whole GPU under a fixed memory
 * budget, a latency-critical serving loop where an allocator call may block or synchronise, a
 * host framework that owns every device allocation). No counterpart in the reference. Its scratch
 * (metadata, per-CTA partials, rows, status) comes from one fixed 8 MiB device array that every
 * GPU loading the library keeps until the process exits; it calls no cudaMalloc, cudaFree or
 * other allocating routine. Batches that need more than 8 MiB of scratch are rejected with
 * AR_ERR_INVALID, as are the bad arguments ar_document_attention_mass rejects (same checks).
 * The array's device address is looked up once per device by the first call made on that device
 * (make that call before any stream capture) and cached; the cache is not refreshed after a
 * cudaDeviceReset, so do not call this entry point on a device after resetting it. Every call
 * shares the array, and calls whose work overlapped on the GPU would race on it: the library
 * holds a per-device lock from the first copy until `stream` has drained, so calls from several
 * host threads of one process run one after another. The stream is synchronised before return. */
int ar_document_attention_mass_noalloc(const void* qkv, int qkv_rows, const float* lse,
                                       const int32_t* prompt_offsets_host, int prompt_count,
                                       const int32_t* query_spans_host, const int32_t* spans_host, int span_count,
                                       int query_heads, int kv_heads, int head_dim, int sliding_window,
                                       int prefill_chunk_tokens, int normalize_by_length, double* mass_out,
                                       int dtype, void* stream);

/* Seeded synthetic weights: fills count 16-bit values of tensor (layer, kind) with the generator
 * documented in csrc/synthetic.h (Irwin-Hall, bf16 round-to-nearest-even); with AR_DTYPE_F16
 * each bf16 value is stored converted to fp16 (round to nearest even). */
int ar_synthetic_fill(void* dst, int64_t count, uint64_t seed, int layer, int kind, float standard_deviation,
                      int dtype, void* stream);

/* ------------------------------------------------------------------------------------------
 * Engine: the IAttentionProvider role of CudaLlamaModel (include/attnrank/model.hpp:79-86,
 * :144-165) plus the layer-scan loop of AttentionLayerScanner (attnrank/src/attnrank.cpp:350-375).
 * ------------------------------------------------------------------------------------------ */

typedef struct ar_engine ar_engine;

/* LlamaConfig (include/attnrank/model.hpp:16-38) fields the path uses. */
typedef struct {
  int hidden_size;
  int intermediate_size;
  int num_hidden_layers;
  int num_attention_heads;
  int num_key_value_heads;
  int vocab_size;
  int max_position_embeddings;
  float rms_norm_eps;
  float rope_theta;
  int sliding_window;    /* 0 = none (kernels.cu:125-126) */
  int attention_bias;    /* 1 when q/k/v projections have biases (Qwen2) */
  int tie_word_embeddings; /* 1: the output head is the embedding (model.cu:140-146); generation only */
} ar_llama_config;

/* LlamaRuntimeOptions (model.hpp:138-142) plus the batching limits of this build. */
typedef struct {
  int device_index;          /* -1 = device 0 */
  int max_sequence_length;   /* longest prompt */
  int prefill_chunk_tokens;  /* the reference's chunk length; only bounds normalize_by_length divisors */
  int max_batch_tokens;      /* packed tokens per forward (>= max_sequence_length) */
  int max_batch_prompts;
  int activation_dtype;      /* AR_DTYPE_F16 (default when 0) or AR_DTYPE_BF16 */
  int attention_kernel;      /* 0 = tcgen05 (default), 1 = mma.sync */
} ar_runtime_options;

/* One probe prompt: StructuredPrompt (include/attnrank/prompt.hpp:12-17) as token ids + spans. */
typedef struct {
  const int32_t* tokens;
  int token_count;
  int query_begin;       /* TokenSpan query_span (core.hpp:54-60), half-open */
  int query_end;
  const int32_t* spans;  /* document_spans: [span_count][2] half-open */
} ar_prompt;

/* Creates the model on a device (CudaLlamaModel::CudaLlamaModel, model.hpp:146-149). */
int ar_engine_create(const ar_llama_config* config, const ar_runtime_options* options, ar_engine** engine);
void ar_engine_destroy(ar_engine* engine);

/* Uploads one checkpoint tensor by its Hugging Face name (DeviceWeights, model.cu:113-174).
 * lm_head.weight is kept for generation; unknown names (rotary buffers) are accepted and ignored. */
int ar_engine_load_tensor(ar_engine* engine, const char* name, int dtype, const int64_t* shape, int rank,
                          const void* host_data);

/* Fills every weight with the seeded synthetic checkpoint (norm weights 1.0). */
int ar_engine_init_synthetic(ar_engine* engine, uint64_t seed, float standard_deviation);

/* CudaLlamaModel::measure_attention_by_layer (model.hpp:159-160, model.cu:593-617) for a batch
 * of prompts with the same span count: rows_out (host, fp64) [prompt_count][layers][span_count],
 * each row divided by query_rows * Hq and normalised to unit sum. layer_begin/layer_end follow
 * AttentionLayerProbeRequest::resolve_layers (model.cpp:66-68). *layer_begin_out (nullable)
 * receives the resolved first layer and *layer_count_out (nullable) the layer count. */
int ar_engine_measure_attention_by_layer(ar_engine* engine, const ar_prompt* prompts, int prompt_count, int span_count,
                                         int layer_begin, int layer_end, int normalize_by_length, double* rows_out,
                                         int* layer_begin_out, int* layer_count_out);

/* CudaLlamaModel::measure_attention (model.hpp:157-158, model.cu:567-591) for one prompt:
 * the per-layer totals over [layer_begin, layer_end) divided by query_rows * Hq * layers,
 * summed, and normalised to unit sum. attention_out: host fp64 [span_count]. */
int ar_engine_measure_attention(ar_engine* engine, const ar_prompt* prompt, int span_count, int layer_begin,
                                int layer_end, int normalize_by_length, double* attention_out);

/* The device half of AttentionLayerScanner::scan (attnrank.cpp:350-375): probes all prompts in
 * packed batches and adds, for every resolved layer, the sum of the prompts' unit-sum rows into
 * device_accumulator (fp32, device, [layers][span_count]; NOT cleared). host_accumulator (nullable,
 * fp64 [layers][span_count]) receives the accumulator's value after the scan. Returns after the
 * device work is complete. */
int ar_engine_scan(ar_engine* engine, const ar_prompt* prompts, int prompt_count, int span_count, int layer_begin,
                   int layer_end, int normalize_by_length, float* device_accumulator, double* host_accumulator);

/* Scan with HBM-resident inputs (no counterpart in the reference, whose scan re-uploads every
 * prompt): prepare once -- validates, packs the prompts into batches and uploads all batch
 * metadata -- then run as often as needed. Running enqueues the whole scan on the engine's stream
 * and returns without waiting unless `synchronize` is set (then it waits and reports device
 * errors). The accumulator is as in ar_engine_scan (not cleared). */
typedef struct ar_prepared_scan ar_prepared_scan;
int ar_engine_prepare_scan(ar_engine* engine, const ar_prompt* prompts, int prompt_count, int span_count,
                           int layer_begin, int layer_end, int normalize_by_length, ar_prepared_scan** prepared);
int ar_engine_run_prepared_scan(ar_engine* engine, const ar_prepared_scan* prepared, float* device_accumulator,
                                int synchronize);
void ar_prepared_scan_destroy(ar_prepared_scan* prepared);
/* Bytes of batch metadata the prepared scan keeps on the device (tokens + spans + work lists). */
int64_t ar_prepared_scan_bytes(const ar_prepared_scan* prepared);

/* Waits for the engine's stream and reports any device-side error since the last probe. */
int ar_engine_synchronize(ar_engine* engine);

/* The engine's CUDA stream (cudaStream_t) and device index. */
void* ar_engine_stream(ar_engine* engine);
int ar_engine_device(ar_engine* engine);

/* Per-launch kernel timing (no reference counterpart; the reference has no device profiler).
 * While enabled, every engine launch is bracketed by CUDA events on the engine stream.
 * ar_engine_kernel_timing synchronises and returns, per kernel class, the summed milliseconds,
 * the summed algorithmic work (FLOPs for tensor classes, HBM bytes otherwise) and the launch
 * count since the previous call (arrays of AR_KERNEL_CLASS_COUNT, each nullable), then clears. */
#define AR_KERNEL_CLASS_COUNT 12
int ar_engine_set_kernel_timing(ar_engine* engine, int enabled);
int ar_engine_kernel_timing(ar_engine* engine, double* milliseconds, double* work, int64_t* launches);
const char* ar_kernel_class_name(int kernel_class);
int ar_kernel_class_is_tensor(int kernel_class);

/* ------------------------------------------------------------------------------------------
 * Generation: CudaLlamaModel::generate (include/attnrank/model.hpp:118-136, :156;
 * attnrank/src/model.cu:532-565), the answering step after reranking, and the samplers of
 * model.hpp:88-116 (attnrank/src/model.cpp:70-127).
 * ------------------------------------------------------------------------------------------ */

/* NucleusSamplerConfig (model.hpp:99-104). temperature <= 0 selects greedily (make_sampler,
 * model.cpp:124-127): the first index of the largest logit. */
typedef struct {
  float temperature;
  float top_p;
  int top_k;       /* 0 = every token is a candidate */
  uint64_t seed;
} ar_sampler_config;

/* The generate loop for one prompt (GenerationRequest / GenerationResult, model.hpp:118-129):
 * prefill, then select -> stop at eos_token_id (not returned) -> decode, until max_new_tokens or
 * the end of the context (max_sequence_length). Stop strings need a tokenizer and stay with the
 * caller (ar_engine_generation_begin/_step hand out the logits step by step). tokens_out has
 * room for max_new_tokens ids; *token_count_out receives the count. The prompt must fit one
 * forward (max_batch_tokens). */
int ar_engine_generate(ar_engine* engine, const int32_t* prompt, int prompt_count, int max_new_tokens,
                       int eos_token_id, const ar_sampler_config* sampler, int32_t* tokens_out, int* token_count_out);

/* Step-wise generation. _begin prefills the prompt (restarting the position at its length);
 * _step feeds one token at the next position. Both leave the next-token logits on the device
 * and copy them to logits_out (host fp32 [vocab]) when it is not NULL. */
int ar_engine_generation_begin(ar_engine* engine, const int32_t* prompt, int prompt_count, float* logits_out);
int ar_engine_generation_step(ar_engine* engine, int32_t token, float* logits_out);
/* Position of the next token fed (prompt length + steps), -1 before a prompt. */
int ar_engine_generation_position(ar_engine* engine);
/* How decode steps run (-1 before the first generation): 2 = one persistent kernel per step (a
 * cooperative launch whose phases meet at a grid barrier), 1 = one kernel per phase with
 * programmatic dependent launch (the default), 0 = one kernel per phase, serialised.
 * ATTNRANK_DECODE_PERSISTENT=1 and ATTNRANK_DECODE_PDL=0 in the environment select modes 2 and 0;
 * a launch or graph capture that the device refuses falls back to the next mode down. */
int ar_engine_decode_mode(ar_engine* engine);

/* Host samplers: GreedySampler / NucleusSampler (model.cpp:70-127). The same logits and
 * config give the reference's token ids; a nucleus sampler's draws advance its own
 * std::mt19937_64 seeded with config->seed. */
typedef struct ar_sampler ar_sampler;
int ar_sampler_create(const ar_sampler_config* config, ar_sampler** sampler);
int ar_sampler_select(ar_sampler* sampler, const float* logits, int count, int32_t* token_out);
void ar_sampler_destroy(ar_sampler* sampler);

/* Decode kernels (device pointers, asynchronous on `stream`); the single-token forms of the
 * reference's cuBLAS projections at m = 1 (LlamaForwardPass::matmul, model.cu:353-365).
 * y[n] = w[n, :] . x for n < rows: w 16-bit [rows, k] row-major, x 16-bit [k], k % 8 == 0;
 * y 16-bit, or fp32 when f32_out (the lm_head logits, model.cu:341-350). */
int ar_decode_gemv(const void* w, const void* x, int rows, int k, void* y, int f32_out, int dtype, void* stream);
/* act[j] = silu(g_j) * u_j over the fused gate|up matrix w [2 inter, k] (model.cu:410-415). */
int ar_decode_gate_up(const void* w, const void* x, int inter, int k, void* act, int dtype, void* stream);
/* Attention of one query token at `position` over a KV cache (keys 0 .. position, or the last
 * sliding_window of them): q 16-bit [Hq, 128]; k_cache, v_cache 16-bit [Hkv, context, 128];
 * out 16-bit [Hq, 128]. The decode form of LlamaForwardPass::attend (model.cu:426-480).
 * Allocates its scratch with cudaMallocAsync on `stream` and synchronises the stream. */
int ar_decode_attention(const void* q, const void* k_cache, const void* v_cache, int context, int position,
                        int query_heads, int kv_heads, int head_dim, int sliding_window, void* out, int dtype,
                        void* stream);

/* Self-test of the library's bounded device waits. No counterpart in the reference: its kernels
 * never wait on one another. `ctas` CTAs (1..1024) wait on the grid barrier of the persistent
 * decode step for a counter value that nothing writes; the wait gives up after `spin_limit` polls
 * (each at least 64 ns; 1..4194304, the production limit) and the call returns AR_ERR_DEVICE with a
 * wait-timeout message. The device stays usable afterwards: a deployment can check that a stalled
 * wait ends in an error, not a hang. Allocates 8 bytes with cudaMallocAsync on `stream` and
 * synchronises the stream. */
int ar_bounded_wait_selftest(int ctas, uint32_t spin_limit, void* stream);

/* ------------------------------------------------------------------------------------------
 * Profile accumulator and basin pick (host functions of attnrank/src/attnrank.cpp).
 * ------------------------------------------------------------------------------------------ */

typedef struct {
  double first;
  double last;
  double interior_mean;
  double edge_ratio;
  int is_basin;
} ar_basin_stats;

/* AttentionProfile::from_accumulated (attnrank.cpp:151-169) + recompute_position_order (:171-177):
 * attention_out[s] = accumulated[s] / sample_count, renormalised to unit sum; position_order_out
 * is the stable descending argsort of attention_out. */
int ar_profile_from_accumulated(const double* accumulated, int slots, int64_t sample_count, double* attention_out,
                                int* position_order_out);

/* AttentionProfile::recompute_position_order (attnrank.cpp:171-177). */
int ar_position_order(const double* attention, int slots, int* position_order_out);

/* basin_statistics (attnrank.cpp:236-255). */
int ar_basin_statistics(const double* attention, int slots, double min_edge_ratio, ar_basin_stats* out);

/* select_shallowest_basin_layer (attnrank.cpp:257-265) over profiles given as a
 * [profile_count][slots] attention matrix and their layer indices. Writes the layer or -1. */
int ar_select_shallowest_basin_layer(const double* attention, const int* layer_indices, int profile_count, int slots,
                                     double min_edge_ratio, int* selected_out);

/* resolve_position_order (attnrank.cpp:377-392): preferred slots first (deduplicated, in range),
 * then the remaining slots ascending. order_out has `count` entries. */
int ar_resolve_position_order(const int* preferred, int preferred_count, int count, int* order_out);

#ifdef __cplusplus
}
#endif

#endif /* ATTNRANK_B200_H */
