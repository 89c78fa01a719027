// B200 attention-profiling engine: a Llama-family prefill that captures per-layer
// query->document attention mass for batches of packed prompts.
//
// It is the B200 counterpart of the reference's CudaLlamaModel in its IAttentionProvider role
// (include/attnrank/model.hpp:79-86, :144-165; attnrank/src/model.cu:512-679). Differences that
// are design, not semantics:
//   * many prompts run in one forward (packed, variable length), so the projection GEMMs see
//     thousands of rows instead of one prompt's chunk;
//   * weights stay 16-bit in HBM (q|k|v and gate|up fused into one matrix each); activations
//     are 16-bit except the fp32 residual stream. The 16-bit type is fp16 by default -- the
//     reference's own GEMM operand type (model.cu:353-365) -- or bf16;
//   * attention never materialises scores; mass is captured by a tcgen05 kernel per layer and
//     reduced on the device, with no host synchronisation until the caller asks for results.
#pragma once

#include <cublasLt.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

#include "sampler.h"

namespace arb {

class Error : public std::runtime_error {
 public:
  explicit Error(const std::string& message) : std::runtime_error(message) {}
};

void check_cuda(cudaError_t status, const char* what);

struct ModelConfig {
  int hidden_size = 0;
  int intermediate_size = 0;
  int num_hidden_layers = 0;
  int num_attention_heads = 0;
  int num_key_value_heads = 0;
  int vocab_size = 0;
  int max_position_embeddings = 0;
  float rms_norm_eps = 1e-6f;
  float rope_theta = 10000.0f;
  int sliding_window = 0;
  bool attention_bias = false;
  bool tie_word_embeddings = false;  // the output head is the embedding table (no lm_head.weight)

  int head_dim() const { return hidden_size / num_attention_heads; }
  int kv_width() const { return num_key_value_heads * head_dim(); }
  int qkv_width() const { return (num_attention_heads + 2 * num_key_value_heads) * head_dim(); }
};

struct RuntimeOptions {
  int device_index = 0;
  int max_sequence_length = 32768;   // longest prompt (size of the RoPE table)
  int prefill_chunk_tokens = 512;    // the reference's chunk length (normalize_by_length divisors)
  int max_batch_tokens = 16384;      // packed tokens per forward
  int max_batch_prompts = 256;
  int activation_dtype = 1;          // 1 = fp16 (default), 2 = bf16: weights, GEMM operands, activations
  int attention_kernel = 0;          // 0 = tcgen05 (attention_tc.cu), 1 = mma.sync (attention.cu)
};

// Kernel classes timed by the engine's optional per-launch timing (CUDA events on stream()).
enum KernelClass : int {
  kClassEmbedding = 0,
  kClassGemmQkv,
  kClassRotary,
  kClassAttention,
  kClassMass,
  kClassGemmOut,
  kClassNorm,
  kClassGemmGateUp,
  kClassSilu,
  kClassGemmDown,
  kClassPositions,
  kClassFinalize,
  kKernelClassCount
};
const char* kernel_class_name(int klass);
bool kernel_class_is_tensor(int klass);  // work unit: FLOPs (tensor) or bytes (HBM)

// One probe prompt as the host hands it over: token ids plus prompt-relative spans.
struct PromptView {
  const int32_t* tokens = nullptr;
  int token_count = 0;
  int query_begin = 0;
  int query_end = 0;
  const int32_t* spans = nullptr;  // [span_count][2] half-open [begin, end)
};

struct LayerRange {
  int begin = 0;
  int end = 0;
  int count() const { return end - begin; }
};

// Offsets (int32 elements) of one batch's metadata inside a metadata buffer.
struct BatchLayout {
  size_t tokens_at = 0, offsets_at = 0, queries_at = 0, spans_at = 0, tiles_at = 0, items_at = 0, fused_items_at = 0,
         size = 0;
  int first = 0;       // index of the batch's first prompt
  int prompts = 0;
  int tokens = 0;
  int tile_count = 0;  // attention query tiles
  int item_count = 0;  // mass CTAs (separate mass kernel)
  int fused_item_count = 0;  // mass partial slots of the fused attention (Hq x query tiles in the span)
  double attention_flops = 0;  // 4 D Hq x visible causal (query, key) pairs
  double mass_flops = 0;       // 2 D Hq x sum over prompts of query rows x document-span keys
};

// A scan whose batch metadata is resident in HBM: running it launches kernels only.
struct PreparedScan {
  std::vector<BatchLayout> batches;
  int32_t* device = nullptr;
  size_t device_bytes = 0;
  int span_count = 0;
  int prompt_count = 0;
  LayerRange range;
  bool normalize_by_length = false;
  ~PreparedScan();
};

// Buffers of generation, allocated at the first begin_generation. Device arrays are engine
// allocations (freed with the engine); pinned host memory, events and graphs are freed here.
struct GenerationState {
  int context = 0;                // positions the KV cache holds (max_sequence_length)
  size_t layer_elements = 0;      // Hkv * context * D: one layer's K (or V) cache
  void* k_cache = nullptr;        // 16-bit [layers][Hkv][context][D]
  void* v_cache = nullptr;
  void* q = nullptr;              // 16-bit [Hq D]: the step's rotated query
  float* partials = nullptr;      // fp32 [Hq][kDecodeSplits][D]
  float* stats = nullptr;         // fp32 [Hq][kDecodeSplits][2]
  float* logits = nullptr;        // fp32 [vocab]
  float* pick_values = nullptr;   // greedy pick: per-CTA candidates [kDecodePickSlots]
  int32_t* pick_indices = nullptr;
  unsigned* tickets = nullptr;    // [2 + Hkv]: the pick's and the attention's last-CTA tickets, the step barrier
  void* layer_table = nullptr;    // DecodeLayerWeights [layers] for the persistent step kernel
  int32_t* state = nullptr;       // device {token, position}
  int32_t* meta = nullptr;        // device: prompt tokens | offsets [2] | attention tiles
  size_t meta_capacity = 0;       // int32 elements of meta (and of the staging area behind the slots)
  int32_t* staging = nullptr;     // pinned: state upload [2], two download slots [2][2], metadata
  float* logits_host = nullptr;   // pinned [vocab], allocated by the first host read
  cudaEvent_t slot_ready[2] = {nullptr, nullptr};
  cudaGraphExec_t graphs[2] = {nullptr, nullptr};  // decode step: [0] logits only, [1] + greedy pick
  bool warmed[2] = {false, false};  // the first step of each kind runs eagerly, later ones replay
  bool programmatic = true;       // per-phase kernels use programmatic dependent launch
  bool persistent = true;         // one persistent kernel per step (falls back to per-phase kernels)
  int position = -1;              // position of the next token fed; -1: no prompt
  ~GenerationState();
};

class Engine {
 public:
  Engine(const ModelConfig& config, const RuntimeOptions& options);
  ~Engine();
  Engine(const Engine&) = delete;
  Engine& operator=(const Engine&) = delete;

  const ModelConfig& config() const { return config_; }
  const RuntimeOptions& options() const { return options_; }
  cudaStream_t stream() const { return stream_; }

  // Weights. Names are the Hugging Face Llama/Qwen2 tensor names (reference model.cu:120-166).
  // dtype: 0 = fp32, 1 = fp16, 2 = bf16. Host data is converted to the resident layout.
  void load_tensor(const std::string& name, int dtype, const std::vector<int64_t>& shape, const void* host);
  void init_synthetic(uint64_t seed, float standard_deviation);
  bool weights_complete(std::string* missing) const;

  LayerRange resolve_layers(int layer_begin, int layer_end) const;

  // Probe prompts through layers [0, range.end), capturing mass for layers in `range`.
  //   rows_host:      optional [prompts][range.count()][span_count] unit-sum rows (fp64)
  //   raw_rows_host:  optional [prompts][range.count()][span_count] mass / observations before
  //                   the unit-sum step (the input of the reference's measure_attention)
  //   device_accumulator: optional fp32 [range.count()][span_count], += sum of the rows
  // Prompts are packed into batches of at most max_batch_tokens tokens. The call returns after
  // every requested host output is written (one stream synchronisation at the end).
  void probe(const std::vector<PromptView>& prompts, int span_count, LayerRange range, bool normalize_by_length,
             double* rows_host, double* raw_rows_host, float* device_accumulator);

  // Scan with HBM-resident inputs: prepare once (validates, plans batches, uploads all metadata),
  // then run_prepared enqueues the whole scan on stream() without any host synchronisation.
  std::unique_ptr<PreparedScan> prepare_scan(const std::vector<PromptView>& prompts, int span_count, LayerRange range,
                                             bool normalize_by_length);
  void run_prepared(const PreparedScan& prepared, float* device_accumulator);

  // Device-side status word (0 = ok): reset, read (synchronises the stream), raise on error.
  void reset_status();
  int read_status();
  static void raise_on_status(int status);
  int last_device_status() const { return last_status_; }

  // Per-launch timing of the engine's kernels: while enabled every launch is bracketed by CUDA
  // events; kernel_timing() synchronises, adds up milliseconds, algorithmic work and launches
  // per KernelClass since the last call, and clears the record.
  void set_kernel_timing(bool enabled);
  void kernel_timing(double* milliseconds, double* work, int64_t* launches);

  // ---- generation: CudaLlamaModel::generate (model.hpp:131-136, 156; model.cu:532-565) ----
  // The KV cache ([layers][Hkv][context][D] 16-bit K and V, context = max_sequence_length) and
  // the decode buffers are allocated at the first call.
  // Prefills `prompt` through every layer (the probe's batched kernels, K/V stored into the
  // cache) and computes the next-token logits (fp32 [vocab], on the device). The prompt must be
  // non-empty, fit one forward (max_batch_tokens) and leave room in the context.
  void begin_generation(const int32_t* prompt, int count);
  // Feeds `token` at the next position through one decode step: every layer on one token, the
  // KV cache extended by one row, new logits. Replays a captured CUDA graph of the step.
  void decode_token(int32_t token);
  // Copies the current logits to host memory (fp32 [vocab]); synchronises.
  void read_logits(float* host);
  // The generate loop (model.cu:537-562 without the text/stop-sequence part, which needs a
  // tokenizer): select a token from the logits, stop at eos_token_id (not returned), else keep
  // it and decode it, up to max_new_tokens or the end of the context. temperature <= 0 selects
  // greedily on the device (the first maximum, GreedySampler::select) with one step in flight;
  // otherwise NucleusTokenSampler selects on the host.
  std::vector<int32_t> generate(const int32_t* prompt, int count, int max_new_tokens, int eos_token_id,
                                const SamplerConfig& sampler);
  // Position the next decoded token takes (prompt length + tokens fed so far); -1 before a prompt.
  int generation_position() const;
  int generation_context() const { return options_.max_sequence_length; }
  // How decode steps run: 2 = one persistent kernel per step, 1 = per-phase kernels with
  // programmatic dependent launch, 0 = per-phase kernels serialised (set by the environment, or
  // by a launch or graph capture the device refused).
  int decode_mode() const;

  // Raw access for the kernel-level tests: the device buffers of the last batch.
  const void* qkv_buffer() const { return qkv_; }
  int qkv_capacity_rows() const { return capacity_tokens_; }

  void synchronize();

 private:
  void ensure_generation();
  void prefill_generation(int tokens);  // metadata already uploaded
  void launch_decode_step(bool greedy);  // the step's kernels, in order, on stream_
  bool launch_persistent_step(bool greedy);  // false: the device refused the cooperative launch
  void run_decode_step(bool greedy);     // eager on first use, then a CUDA graph replay
  void release_decode_graphs();
  const void* output_head() const;

  struct LayerWeights {
    void* qkv = nullptr;     // 16-bit [(Hq + 2 Hkv) D, H]
    float* qkv_bias = nullptr;  // fp32 [(Hq + 2 Hkv) D] or null
    void* qkv_bias_half = nullptr;  // the same in the 16-bit type (the GEMM's bias epilogue) or null
    void* out = nullptr;     // 16-bit [H, Hq D]
    void* gate_up = nullptr;  // 16-bit [2 I, H]
    void* down = nullptr;    // 16-bit [H, I]
    float* input_norm = nullptr;  // fp32 [H]
    float* post_norm = nullptr;   // fp32 [H]
  };

  struct Batch {
    int first = 0;
    int count = 0;
    int tokens = 0;
  };

  void allocate();
  void ensure_partials(size_t items, int span_count, int layers);
  // y[m, n] = x[m, k] w[n, k]^T (+ bias[n], 16-bit like y, when given and cuBLASLt offers the
  // epilogue; returns whether the bias was applied)
  bool gemm(const void* x, const void* w, void* y, int m, int n, int k, const void* bias = nullptr);
  void gemm_residual(const void* x, const void* w, float* residual, int m, int n, int k);
  bool gemm_plan_and_run(const void* x, const void* w, void* y, int m, int n, int k, const void* bias,
                         bool accumulate);
  void refresh_half_bias(int layer);
  void run_batch(const std::vector<PromptView>& prompts, const Batch& batch, int span_count, LayerRange range,
                 bool normalize_by_length, double* rows_device, double* raw_rows_device, float* device_accumulator,
                 int slot);
  BatchLayout build_metadata(const std::vector<PromptView>& prompts, const Batch& batch, int span_count, int32_t* host,
                             size_t capacity) const;
  void execute_batch(const BatchLayout& layout, const int32_t* device_metadata, int span_count, LayerRange range,
                     bool normalize_by_length, double* rows_device, double* raw_rows_device,
                     float* device_accumulator);
  void validate(const std::vector<PromptView>& prompts, int span_count, LayerRange range) const;
  std::vector<Batch> plan_batches(const std::vector<PromptView>& prompts) const;
  void* device_alloc(size_t bytes);
  void upload_matrix(void* dst, const void* host, int dtype, size_t count);
  template <typename Launch>
  void timed(int klass, double work, Launch&& launch);
  struct KernelTimer;
  std::unique_ptr<KernelTimer> timer_;

  ModelConfig config_;
  RuntimeOptions options_;
  int capacity_tokens_ = 0;
  cudaStream_t stream_ = nullptr;
  cublasLtHandle_t lt_ = nullptr;
  void* lt_workspace_ = nullptr;
  size_t lt_workspace_bytes_ = 0;
  struct GemmPlans;
  std::unique_ptr<GemmPlans> plans_;  // cuBLASLt descriptors + algorithm per (m, n, k)

  std::vector<void*> allocations_;
  void* embedding_ = nullptr;  // 16-bit [V, H]
  void* lm_head_ = nullptr;    // 16-bit [V, H] when loaded or synthesised; else the embedding is the head
  std::unique_ptr<GenerationState> generation_;
  std::vector<LayerWeights> layers_;
  float* final_norm_ = nullptr;
  std::vector<std::vector<bool>> loaded_;  // per layer, per tensor kind
  bool embedding_loaded_ = false;

  // workspace
  float* residual_ = nullptr;
  void* normed_ = nullptr;
  void* qkv_ = nullptr;
  void* attn_ = nullptr;
  void* delta_ = nullptr;       // 16-bit [2, H]: the decode step's o_proj and down_proj rows
  size_t gate_up_bytes_ = 0;    // also the scratch on which accumulating GEMMs are autotuned
  void* gate_up_ = nullptr;
  void* act_ = nullptr;
  float* lse_ = nullptr;
  int32_t* positions_ = nullptr;
  float* cos_table_ = nullptr;
  float* sin_table_ = nullptr;
  int* status_ = nullptr;
  int32_t* meta_device_[2] = {nullptr, nullptr};
  int32_t* meta_host_[2] = {nullptr, nullptr};
  size_t meta_capacity_ = 0;  // int32 elements per metadata buffer
  cudaEvent_t meta_free_[2] = {nullptr, nullptr};
  float* partials_ = nullptr;
  size_t partials_capacity_ = 0;  // floats
  double* rows_device_ = nullptr;
  size_t rows_capacity_ = 0;      // doubles per rows buffer (two buffers: rows, raw rows)
  int* status_host_ = nullptr;
  int last_status_ = 0;
};

}  // namespace arb
