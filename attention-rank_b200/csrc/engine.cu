// B200 attention-profiling engine (see engine.h). Host orchestration of one packed batch:
//
//   positions, embed+norm                                         (layer_kernels.cu)
//   for layer in [0, probe_end):
//     qkv   = normed @ Wqkv^T                 cuBLASLt, fp16 (or bf16) operands, fp32 accumulation
//     qkv  += bias; RoPE(q, k)                rotary_bias_kernel (in place)
//     attn, lse = causal_attention(qkv)       attention_tc.cu (tcgen05 flash, no score matrix)
//     partials[layer] = document_mass(qkv, lse)   mass.cu (tcgen05), probed layers only
//     residual += attn @ Wo^T                 cuBLASLt, fp32 accumulator added into the fp32 residual
//     normed = rms(residual) * post_norm
//     gate|up = normed @ Wgu^T; act = silu(gate) * up
//     residual += act @ Wdown^T
//     normed = rms(residual) * next input_norm
//   finalize(partials) -> per-prompt unit-sum rows, += device accumulator
//
// The order of operations per layer is the reference's LlamaForwardPass
// (attnrank/src/model.cu:324-419): pre-norm, q/k/v (+bias), RoPE, attention, o_proj + residual,
// post-norm, gate/up, SiLU*up, down + residual.
#include "engine.h"

#include <algorithm>
#include <cstring>
#include <numeric>
#include <regex>

#include "layer_kernels.h"
#include "mass_plan.h"
#include "synthetic.h"

namespace arb {

void check_cuda(cudaError_t status, const char* what) {
  if (status != cudaSuccess) {
    throw Error(std::string("CUDA error in ") + what + ": " + cudaGetErrorString(status));
  }
}

namespace {

void check_lt(cublasStatus_t status, const char* what) {
  if (status != CUBLAS_STATUS_SUCCESS) {
    throw Error(std::string("cuBLASLt error ") + std::to_string(static_cast<int>(status)) + " in " + what);
  }
}

constexpr size_t kLtWorkspaceBytes = 64ull << 20;

uint16_t float_to_bf16_bits(float value) {
  uint32_t bits;
  std::memcpy(&bits, &value, sizeof(bits));
  if ((bits & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((bits >> 16) | 0x40u);  // NaN stays NaN
  return static_cast<uint16_t>(synthetic_round_bf16(bits));
}

float half_to_float(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  uint32_t exponent = (h >> 10) & 0x1fu;
  uint32_t mantissa = h & 0x3ffu;
  uint32_t bits;
  if (exponent == 0) {
    if (mantissa == 0) {
      bits = sign;
    } else {  // subnormal half -> normal float
      exponent = 127 - 15 + 1;
      while ((mantissa & 0x400u) == 0) {
        mantissa <<= 1;
        --exponent;
      }
      mantissa &= 0x3ffu;
      bits = sign | (exponent << 23) | (mantissa << 13);
    }
  } else if (exponent == 0x1f) {
    bits = sign | 0x7f800000u | (mantissa << 13);
  } else {
    bits = sign | ((exponent + 127 - 15) << 23) | (mantissa << 13);
  }
  float value;
  std::memcpy(&value, &bits, sizeof(value));
  return value;
}

float element_as_float(const void* data, int dtype, size_t index) {
  switch (dtype) {
    case 0: return static_cast<const float*>(data)[index];
    case 1: return half_to_float(static_cast<const uint16_t*>(data)[index]);
    case 2: {
      const uint32_t bits = static_cast<uint32_t>(static_cast<const uint16_t*>(data)[index]) << 16;
      float value;
      std::memcpy(&value, &bits, sizeof(value));
      return value;
    }
    default: throw Error("unsupported tensor dtype code " + std::to_string(dtype));
  }
}

// Host -> device copy ordered on the engine's stream and complete on return. A plain cudaMemcpy
// from pageable memory may return before its DMA lands, and it is not ordered with the engine's
// non-blocking stream, so a kernel there could read the destination too early.
void copy_to_device(void* dst, const void* host, size_t bytes, cudaStream_t stream, const char* what) {
  check_cuda(cudaMemcpyAsync(dst, host, bytes, cudaMemcpyHostToDevice, stream), what);
  check_cuda(cudaStreamSynchronize(stream), what);
}

// Upload `count` elements of host data as bf16 into dst (host-side conversion).
void upload_bf16(void* dst, const void* host, int dtype, size_t count, cudaStream_t stream) {
  if (dtype == 2) {
    copy_to_device(dst, host, count * 2, stream, "weight upload");
    return;
  }
  std::vector<uint16_t> staged(count);
  for (size_t i = 0; i < count; ++i) staged[i] = float_to_bf16_bits(element_as_float(host, dtype, i));
  copy_to_device(dst, staged.data(), count * 2, stream, "weight upload");
}

void upload_f32(float* dst, const void* host, int dtype, size_t count, cudaStream_t stream) {
  std::vector<float> staged(count);
  for (size_t i = 0; i < count; ++i) staged[i] = element_as_float(host, dtype, i);
  copy_to_device(dst, staged.data(), count * 4, stream, "weight upload");
}

enum LayerTensor : int {
  kQ = 0, kK, kV, kQBias, kKBias, kVBias, kO, kGate, kUp, kDown, kInputNorm, kPostNorm, kLayerTensorCount
};

struct GemmPlan {
  cublasLtMatmulDesc_t op = nullptr;
  cublasLtMatrixLayout_t a = nullptr, b = nullptr, c = nullptr;
  cublasLtMatmulAlgo_t algo;
  bool bias = false;  // the fp32 bias epilogue is part of the plan
};

using GemmKey = std::tuple<int, int, int, int>;  // m, n, k, epilogue (0 none, 1 bias, 2 accumulate fp32)

void destroy_plans(std::map<GemmKey, GemmPlan>& plans) {
  for (auto& entry : plans) {
    cublasLtMatmulDescDestroy(entry.second.op);
    cublasLtMatrixLayoutDestroy(entry.second.a);
    cublasLtMatrixLayoutDestroy(entry.second.b);
    cublasLtMatrixLayoutDestroy(entry.second.c);
  }
  plans.clear();
}

}  // namespace

const char* kernel_class_name(int klass) {
  static const char* names[kKernelClassCount] = {
      "embedding_rms_norm", "gemm_qkv",      "rotary_bias", "causal_attention", "document_mass", "gemm_out",
      "rms_norm_residual",  "gemm_gate_up",  "silu_multiply", "gemm_down",     "positions",     "finalize_mass"};
  return klass >= 0 && klass < kKernelClassCount ? names[klass] : "";
}

bool kernel_class_is_tensor(int klass) {
  return klass == kClassGemmQkv || klass == kClassAttention || klass == kClassMass || klass == kClassGemmOut ||
         klass == kClassGemmGateUp || klass == kClassGemmDown;
}

struct Engine::KernelTimer {
  struct Record {
    int klass;
    double work;
  };
  bool enabled = false;
  std::vector<cudaEvent_t> pool;  // two events per record
  std::vector<Record> records;
  double milliseconds[kKernelClassCount] = {};
  double work[kKernelClassCount] = {};
  int64_t launches[kKernelClassCount] = {};
  ~KernelTimer() {
    for (cudaEvent_t event : pool) cudaEventDestroy(event);
  }
  cudaEvent_t event(size_t index) {
    while (pool.size() <= index) {
      cudaEvent_t created = nullptr;
      check_cuda(cudaEventCreate(&created), "timing event");
      pool.push_back(created);
    }
    return pool[index];
  }
};

template <typename Launch>
void Engine::timed(int klass, double work, Launch&& launch) {
  KernelTimer& timer = *timer_;
  if (!timer.enabled) {
    launch();
    return;
  }
  const size_t first = timer.records.size() * 2;
  check_cuda(cudaEventRecord(timer.event(first), stream_), "timing event");
  launch();
  check_cuda(cudaEventRecord(timer.event(first + 1), stream_), "timing event");
  timer.records.push_back({klass, work});
}

void Engine::set_kernel_timing(bool enabled) { timer_->enabled = enabled; }

void Engine::kernel_timing(double* milliseconds, double* work, int64_t* launches) {
  KernelTimer& timer = *timer_;
  synchronize();
  for (size_t i = 0; i < timer.records.size(); ++i) {
    float elapsed = 0.0f;
    check_cuda(cudaEventElapsedTime(&elapsed, timer.pool[2 * i], timer.pool[2 * i + 1]), "timing read");
    const int klass = timer.records[i].klass;
    timer.milliseconds[klass] += elapsed;
    timer.work[klass] += timer.records[i].work;
    timer.launches[klass] += 1;
  }
  timer.records.clear();
  for (int k = 0; k < kKernelClassCount; ++k) {
    if (milliseconds != nullptr) milliseconds[k] = timer.milliseconds[k];
    if (work != nullptr) work[k] = timer.work[k];
    if (launches != nullptr) launches[k] = timer.launches[k];
    timer.milliseconds[k] = 0;
    timer.work[k] = 0;
    timer.launches[k] = 0;
  }
}

// Upload `count` elements of host data (dtype 0 = fp32, 1 = fp16, 2 = bf16) into dst in the
// engine's activation type. bf16 -> fp16 and fp32 -> 16-bit are converted on the device
// (round to nearest even), so a bf16 checkpoint gives exactly the fp16 weights of the seeded
// synthetic path.
void Engine::upload_matrix(void* dst, const void* host, int dtype, size_t count) {
  const int target = options_.activation_dtype;
  if (dtype == target) {
    copy_to_device(dst, host, count * 2, stream_, "weight upload");
    return;
  }
  if (target == kActBf16 && dtype == 1) {
    upload_bf16(dst, host, dtype, count, stream_);
    return;
  }
  if (dtype != 0 && dtype != 2) throw Error("unsupported tensor dtype code " + std::to_string(dtype));
  const size_t bytes = count * (dtype == 0 ? 4 : 2);
  void* staging = nullptr;
  check_cuda(cudaMalloc(&staging, bytes), "weight staging allocation");
  cudaError_t status = cudaMemcpyAsync(staging, host, bytes, cudaMemcpyHostToDevice, stream_);  // ordered before the conversion
  if (status == cudaSuccess) {
    status = dtype == 0 ? launch_f32_to_activation(static_cast<const float*>(staging), dst, static_cast<long long>(count),
                                                   target, stream_)
                        : launch_bf16_to_fp16(staging, dst, static_cast<long long>(count), stream_);
  }
  if (status == cudaSuccess) status = cudaStreamSynchronize(stream_);
  cudaFree(staging);
  check_cuda(status, "weight conversion");
}

struct Engine::GemmPlans {
  std::map<GemmKey, GemmPlan> by_shape;
};

Engine::Engine(const ModelConfig& config, const RuntimeOptions& options)
    : config_(config), options_(options), plans_(new GemmPlans), timer_(new KernelTimer) {
  const ModelConfig& c = config_;
  if (c.hidden_size <= 0 || c.num_attention_heads <= 0 || c.hidden_size % c.num_attention_heads != 0) {
    throw Error("invalid attention head configuration");
  }
  if (c.num_key_value_heads <= 0 || c.num_attention_heads % c.num_key_value_heads != 0) {
    throw Error("invalid key/value head configuration");
  }
  if (c.head_dim() != 128) throw Error("the B200 attention kernels require head_dim 128 (got " + std::to_string(c.head_dim()) + ")");
  if (c.hidden_size % 8 != 0 || c.intermediate_size % 8 != 0) throw Error("hidden and intermediate sizes must be multiples of 8");
  if (c.num_hidden_layers <= 0 || c.vocab_size <= 0 || c.intermediate_size <= 0) throw Error("invalid model dimensions");
  if (options_.max_sequence_length <= 0) throw Error("max_sequence_length must be positive");
  if (options_.prefill_chunk_tokens <= 0) throw Error("prefill_chunk_tokens must be positive");
  if (options_.max_batch_tokens <= 0) throw Error("max_batch_tokens must be positive");
  if (options_.max_batch_prompts <= 0) throw Error("max_batch_prompts must be positive");
  if (options_.activation_dtype != kActFp16 && options_.activation_dtype != kActBf16) {
    throw Error("activation_dtype must be 1 (fp16) or 2 (bf16)");
  }
  if (options_.attention_kernel != 0 && options_.attention_kernel != 1) {
    throw Error("attention_kernel must be 0 (tcgen05) or 1 (mma.sync)");
  }
  if (options_.max_batch_tokens < options_.max_sequence_length) options_.max_batch_tokens = options_.max_sequence_length;
  capacity_tokens_ = options_.max_batch_tokens;

  int device_count = 0;
  check_cuda(cudaGetDeviceCount(&device_count), "cudaGetDeviceCount");
  if (device_count == 0) throw Error("no CUDA device available");
  if (options_.device_index < 0) options_.device_index = 0;
  if (options_.device_index >= device_count) {
    throw Error("requested CUDA device " + std::to_string(options_.device_index) + " but only " +
                std::to_string(device_count) + " are present");
  }
  check_cuda(cudaSetDevice(options_.device_index), "cudaSetDevice");
  cudaDeviceProp properties{};
  check_cuda(cudaGetDeviceProperties(&properties, options_.device_index), "cudaGetDeviceProperties");
  if (properties.major != 10) {
    throw Error(std::string("this build targets sm_100a (B200); device is ") + properties.name);
  }
  check_cuda(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
  check_lt(cublasLtCreate(&lt_), "cublasLtCreate");
  allocate();
}

Engine::~Engine() {
  if (stream_ != nullptr) cudaStreamSynchronize(stream_);
  generation_.reset();
  timer_.reset();
  destroy_plans(plans_->by_shape);
  for (void* pointer : allocations_) cudaFree(pointer);
  if (partials_ != nullptr) cudaFree(partials_);
  if (rows_device_ != nullptr) cudaFree(rows_device_);
  for (int i = 0; i < 2; ++i) {
    if (meta_host_[i] != nullptr) cudaFreeHost(meta_host_[i]);
    if (meta_free_[i] != nullptr) cudaEventDestroy(meta_free_[i]);
  }
  if (status_host_ != nullptr) cudaFreeHost(status_host_);
  if (lt_ != nullptr) cublasLtDestroy(lt_);
  if (stream_ != nullptr) cudaStreamDestroy(stream_);
}

void* Engine::device_alloc(size_t bytes) {
  void* pointer = nullptr;
  if (bytes == 0) return nullptr;
  const cudaError_t status = cudaMalloc(&pointer, bytes);
  if (status != cudaSuccess) {
    throw Error("device allocation of " + std::to_string(bytes) + " bytes failed: " + cudaGetErrorString(status));
  }
  allocations_.push_back(pointer);
  return pointer;
}

void Engine::allocate() {
  const ModelConfig& c = config_;
  const size_t H = c.hidden_size, I = c.intermediate_size, V = c.vocab_size;
  const size_t Wqkv = c.qkv_width(), Hq = c.num_attention_heads, D = c.head_dim();
  embedding_ = device_alloc(V * H * 2);
  final_norm_ = static_cast<float*>(device_alloc(H * 4));
  layers_.resize(c.num_hidden_layers);
  loaded_.assign(c.num_hidden_layers, std::vector<bool>(kLayerTensorCount, false));
  for (auto& layer : layers_) {
    layer.qkv = device_alloc(Wqkv * H * 2);
    if (c.attention_bias) {
      layer.qkv_bias = static_cast<float*>(device_alloc(Wqkv * 4));
      layer.qkv_bias_half = device_alloc(Wqkv * 2);
    }
    layer.out = device_alloc(H * Hq * D * 2);
    layer.gate_up = device_alloc(2 * I * H * 2);
    layer.down = device_alloc(H * I * 2);
    layer.input_norm = static_cast<float*>(device_alloc(H * 4));
    layer.post_norm = static_cast<float*>(device_alloc(H * 4));
  }
  const size_t T = capacity_tokens_;
  residual_ = static_cast<float*>(device_alloc(T * H * 4));
  normed_ = device_alloc(T * H * 2);
  qkv_ = device_alloc(T * Wqkv * 2);
  attn_ = device_alloc(T * Hq * D * 2);
  delta_ = device_alloc(2 * H * 2);  // the generation step's two 16-bit projection rows
  gate_up_bytes_ = T * 2 * I * 2;
  gate_up_ = device_alloc(gate_up_bytes_);
  act_ = device_alloc(T * I * 2);
  lse_ = static_cast<float*>(device_alloc(T * Hq * 4));
  positions_ = static_cast<int32_t*>(device_alloc(T * 4));
  const size_t table = static_cast<size_t>(options_.max_sequence_length) * (D / 2);
  cos_table_ = static_cast<float*>(device_alloc(table * 4));
  sin_table_ = static_cast<float*>(device_alloc(table * 4));
  status_ = static_cast<int*>(device_alloc(sizeof(int) * 4));
  lt_workspace_bytes_ = kLtWorkspaceBytes;
  lt_workspace_ = device_alloc(lt_workspace_bytes_);

  const size_t P = options_.max_batch_prompts;
  meta_capacity_ = T + (P + 1) + 2 * P + 2 * P * kMassMaxSpans + 2 * (T / kAttentionQueryTile + P) + 2 * (P + 1) + 64;
  for (int i = 0; i < 2; ++i) {
    meta_device_[i] = static_cast<int32_t*>(device_alloc(meta_capacity_ * 4));
    check_cuda(cudaHostAlloc(reinterpret_cast<void**>(&meta_host_[i]), meta_capacity_ * 4, cudaHostAllocDefault),
               "cudaHostAlloc");
    check_cuda(cudaEventCreateWithFlags(&meta_free_[i], cudaEventDisableTiming), "cudaEventCreate");
  }
  check_cuda(cudaHostAlloc(reinterpret_cast<void**>(&status_host_), sizeof(int) * 4, cudaHostAllocDefault),
             "cudaHostAlloc");
  check_cuda(cudaMemsetAsync(status_, 0, sizeof(int) * 4, stream_), "status reset");
  check_cuda(launch_rope_table(cos_table_, sin_table_, options_.max_sequence_length, static_cast<int>(D), c.rope_theta,
                               stream_),
             "rope table");
  check_cuda(cudaStreamSynchronize(stream_), "engine set-up");
}

void Engine::synchronize() { check_cuda(cudaStreamSynchronize(stream_), "cudaStreamSynchronize"); }

void Engine::load_tensor(const std::string& name, int dtype, const std::vector<int64_t>& shape, const void* host) {
  const ModelConfig& c = config_;
  const int64_t H = c.hidden_size, I = c.intermediate_size, V = c.vocab_size;
  const int64_t Hq = c.num_attention_heads, D = c.head_dim(), KV = c.kv_width();
  int64_t count = 1;
  for (int64_t d : shape) count *= d;
  auto expect = [&](int64_t rows, int64_t cols) {
    const bool ok = (shape.size() == 2 && shape[0] == rows && shape[1] == cols) ||
                    (cols == 1 && shape.size() == 1 && shape[0] == rows);
    if (!ok) throw Error("tensor '" + name + "' has an unexpected shape");
  };
  if (name == "model.embed_tokens.weight") {
    expect(V, H);
    upload_matrix(embedding_, host, dtype, static_cast<size_t>(count));
    embedding_loaded_ = true;
    return;
  }
  if (name == "model.norm.weight") {
    expect(H, 1);
    upload_f32(final_norm_, host, dtype, static_cast<size_t>(count), stream_);
    return;
  }
  if (name == "lm_head.weight") {
    // the output head (model.cu:140-146); only generation reads it
    expect(V, H);
    if (lm_head_ == nullptr) {
      lm_head_ = device_alloc(static_cast<size_t>(V) * H * 2);
      release_decode_graphs();  // captured steps hold the head's address
    }
    upload_matrix(lm_head_, host, dtype, static_cast<size_t>(count));
    return;
  }
  static const std::regex layer_pattern(R"(model\.layers\.(\d+)\.(.+))");
  std::smatch match;
  if (!std::regex_match(name, match, layer_pattern)) return;  // rotary buffers and the like: unused
  const int index = std::stoi(match[1].str());
  if (index < 0 || index >= c.num_hidden_layers) throw Error("tensor '" + name + "' names a layer out of range");
  const std::string suffix = match[2].str();
  LayerWeights& layer = layers_[index];
  auto* qkv = static_cast<uint16_t*>(layer.qkv);
  if (suffix == "self_attn.q_proj.weight") {
    expect(Hq * D, H);
    upload_matrix(qkv, host, dtype, count);
    loaded_[index][kQ] = true;
  } else if (suffix == "self_attn.k_proj.weight") {
    expect(KV, H);
    upload_matrix(qkv + Hq * D * H, host, dtype, count);
    loaded_[index][kK] = true;
  } else if (suffix == "self_attn.v_proj.weight") {
    expect(KV, H);
    upload_matrix(qkv + (Hq * D + KV) * H, host, dtype, count);
    loaded_[index][kV] = true;
  } else if (suffix == "self_attn.q_proj.bias" || suffix == "self_attn.k_proj.bias" ||
             suffix == "self_attn.v_proj.bias") {
    if (layer.qkv_bias == nullptr) throw Error("tensor '" + name + "' given but the config has no attention bias");
    const char which = suffix[10];
    const int64_t offset = which == 'q' ? 0 : which == 'k' ? Hq * D : Hq * D + KV;
    expect(which == 'q' ? Hq * D : KV, 1);
    upload_f32(layer.qkv_bias + offset, host, dtype, count, stream_);
    refresh_half_bias(index);
    loaded_[index][which == 'q' ? kQBias : which == 'k' ? kKBias : kVBias] = true;
  } else if (suffix == "self_attn.o_proj.weight") {
    expect(H, Hq * D);
    upload_matrix(layer.out, host, dtype, count);
    loaded_[index][kO] = true;
  } else if (suffix == "mlp.gate_proj.weight") {
    expect(I, H);
    upload_matrix(layer.gate_up, host, dtype, count);
    loaded_[index][kGate] = true;
  } else if (suffix == "mlp.up_proj.weight") {
    expect(I, H);
    upload_matrix(static_cast<uint16_t*>(layer.gate_up) + I * H, host, dtype, count);
    loaded_[index][kUp] = true;
  } else if (suffix == "mlp.down_proj.weight") {
    expect(H, I);
    upload_matrix(layer.down, host, dtype, count);
    loaded_[index][kDown] = true;
  } else if (suffix == "input_layernorm.weight") {
    expect(H, 1);
    upload_f32(layer.input_norm, host, dtype, count, stream_);
    loaded_[index][kInputNorm] = true;
  } else if (suffix == "post_attention_layernorm.weight") {
    expect(H, 1);
    upload_f32(layer.post_norm, host, dtype, count, stream_);
    loaded_[index][kPostNorm] = true;
  }
}

void Engine::init_synthetic(uint64_t seed, float standard_deviation) {
  const ModelConfig& c = config_;
  const long long H = c.hidden_size, I = c.intermediate_size, V = c.vocab_size;
  const long long QD = static_cast<long long>(c.num_attention_heads) * c.head_dim(), KV = c.kv_width();
  const float scale = synthetic_scale(standard_deviation);
  auto fill = [&](void* dst, long long count, int layer, int kind) {
    check_cuda(launch_synthetic_fill(dst, count, synthetic_tensor_key(seed, layer, kind), scale,
                                     options_.activation_dtype, stream_),
               "synthetic fill");
  };
  auto ones = [&](float* dst, long long count, int layer, int kind) {
    check_cuda(launch_synthetic_fill_f32(dst, count, synthetic_tensor_key(seed, layer, kind), 0.0f, 1.0f, stream_),
               "synthetic fill");
  };
  fill(embedding_, V * H, -1, kTensorEmbedding);
  ones(final_norm_, H, -1, kTensorFinalNorm);
  if (!c.tie_word_embeddings) {
    if (lm_head_ == nullptr) {
      lm_head_ = device_alloc(static_cast<size_t>(V) * H * 2);
      release_decode_graphs();
    }
    fill(lm_head_, V * H, -1, kTensorLmHead);
  }
  for (int l = 0; l < c.num_hidden_layers; ++l) {
    LayerWeights& layer = layers_[l];
    auto* qkv = static_cast<uint16_t*>(layer.qkv);
    fill(qkv, QD * H, l, kTensorQuery);
    fill(qkv + QD * H, KV * H, l, kTensorKey);
    fill(qkv + (QD + KV) * H, KV * H, l, kTensorValue);
    if (layer.qkv_bias != nullptr) {
      const uint64_t keys[3] = {synthetic_tensor_key(seed, l, kTensorQueryBias), synthetic_tensor_key(seed, l, kTensorKeyBias),
                                synthetic_tensor_key(seed, l, kTensorValueBias)};
      check_cuda(launch_synthetic_fill_f32(layer.qkv_bias, QD, keys[0], scale, 0.0f, stream_), "synthetic fill");
      check_cuda(launch_synthetic_fill_f32(layer.qkv_bias + QD, KV, keys[1], scale, 0.0f, stream_), "synthetic fill");
      check_cuda(launch_synthetic_fill_f32(layer.qkv_bias + QD + KV, KV, keys[2], scale, 0.0f, stream_), "synthetic fill");
      refresh_half_bias(l);
    }
    fill(layer.out, H * QD, l, kTensorOutput);
    fill(layer.gate_up, I * H, l, kTensorGate);
    fill(static_cast<uint16_t*>(layer.gate_up) + I * H, I * H, l, kTensorUp);
    fill(layer.down, H * I, l, kTensorDown);
    ones(layer.input_norm, H, l, kTensorInputNorm);
    ones(layer.post_norm, H, l, kTensorPostNorm);
    std::fill(loaded_[l].begin(), loaded_[l].end(), true);
  }
  embedding_loaded_ = true;
  synchronize();
}

bool Engine::weights_complete(std::string* missing) const {
  if (!embedding_loaded_) {
    if (missing) *missing = "model.embed_tokens.weight";
    return false;
  }
  static const char* names[kLayerTensorCount] = {
      "self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight", "self_attn.q_proj.bias",
      "self_attn.k_proj.bias", "self_attn.v_proj.bias", "self_attn.o_proj.weight", "mlp.gate_proj.weight",
      "mlp.up_proj.weight", "mlp.down_proj.weight", "input_layernorm.weight", "post_attention_layernorm.weight"};
  for (int l = 0; l < config_.num_hidden_layers; ++l) {
    for (int t = 0; t < kLayerTensorCount; ++t) {
      const bool is_bias = t == kQBias || t == kKBias || t == kVBias;
      if (is_bias && !config_.attention_bias) continue;
      if (!loaded_[l][t]) {
        if (missing) *missing = "model.layers." + std::to_string(l) + "." + names[t];
        return false;
      }
    }
  }
  return true;
}

LayerRange Engine::resolve_layers(int layer_begin, int layer_end) const {
  // AttentionLayerProbeRequest::resolve_layers (attnrank/src/model.cpp:66-68): negatives mean "from 0" / "to the end".
  LayerRange range{layer_begin < 0 ? 0 : layer_begin, layer_end < 0 ? config_.num_hidden_layers : layer_end};
  if (range.begin < 0 || range.end > config_.num_hidden_layers || range.count() <= 0) {
    throw Error("probe layers [" + std::to_string(range.begin) + "," + std::to_string(range.end) + ") are out of range");
  }
  return range;
}

void Engine::refresh_half_bias(int layer) {
  LayerWeights& w = layers_[layer];
  if (w.qkv_bias == nullptr) return;
  check_cuda(launch_f32_to_activation(w.qkv_bias, w.qkv_bias_half, config_.qkv_width(), options_.activation_dtype,
                                      stream_),
             "bias conversion");
  synchronize();
}

bool Engine::gemm(const void* x, const void* w, void* y, int m, int n, int k, const void* bias) {
  return gemm_plan_and_run(x, w, y, m, n, k, bias, false);
}

// residual[m, n] (fp32) += x[m, k] w[n, k]^T: the projection's fp32 accumulator is added to the
// fp32 residual in the GEMM epilogue (beta = 1), as the reference adds its fp32 GEMM output
// (model.cu:360-364 writes CUDA_R_32F; add_in_place at :397 and :418), with no 16-bit rounding of
// the projection in between.
void Engine::gemm_residual(const void* x, const void* w, float* residual, int m, int n, int k) {
  gemm_plan_and_run(x, w, residual, m, n, k, nullptr, true);
}

bool Engine::gemm_plan_and_run(const void* x, const void* w, void* y, int m, int n, int k, const void* bias,
                               bool accumulate) {
  auto& cache = plans_->by_shape;
  const auto key = std::make_tuple(m, n, k, bias != nullptr ? 1 : (accumulate ? 2 : 0));
  auto found = cache.find(key);
  if (found == cache.end()) {
    if (cache.size() > 512) {
      synchronize();  // plans may still be referenced by queued work only through copies; be conservative
      destroy_plans(cache);
    }
    GemmPlan plan;
    auto create_op = [&] {
      check_lt(cublasLtMatmulDescCreate(&plan.op, CUBLAS_COMPUTE_32F, CUDA_R_32F), "matmul desc");
      const cublasOperation_t transa = CUBLAS_OP_T, transb = CUBLAS_OP_N;
      check_lt(cublasLtMatmulDescSetAttribute(plan.op, CUBLASLT_MATMUL_DESC_TRANSA, &transa, sizeof(transa)),
               "transa");
      check_lt(cublasLtMatmulDescSetAttribute(plan.op, CUBLASLT_MATMUL_DESC_TRANSB, &transb, sizeof(transb)),
               "transb");
    };
    create_op();
    // column-major view: D[n, m] = W[k, n]^T * X[k, m]  (row-major Y[m, n] = X[m, k] W[n, k]^T)
    const cudaDataType_t type = options_.activation_dtype == kActFp16 ? CUDA_R_16F : CUDA_R_16BF;
    check_lt(cublasLtMatrixLayoutCreate(&plan.a, type, k, n, k), "layout a");
    check_lt(cublasLtMatrixLayoutCreate(&plan.b, type, k, m, k), "layout b");
    check_lt(cublasLtMatrixLayoutCreate(&plan.c, accumulate ? CUDA_R_32F : type, n, m, n), "layout c");
    cublasLtMatmulPreference_t preference = nullptr;
    check_lt(cublasLtMatmulPreferenceCreate(&preference), "preference");
    check_lt(cublasLtMatmulPreferenceSetAttribute(preference, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES,
                                                  &lt_workspace_bytes_, sizeof(lt_workspace_bytes_)),
             "preference workspace");
    constexpr int kCandidates = 8;
    cublasLtMatmulHeuristicResult_t results[kCandidates] = {};
    int returned = 0;
    cublasStatus_t status = CUBLAS_STATUS_NOT_SUPPORTED;
    if (bias != nullptr) {
      // y = x W^T + b, b in y's 16-bit type, added to the fp32 accumulator before the rounding of y
      const cublasLtEpilogue_t epilogue = CUBLASLT_EPILOGUE_BIAS;
      if (cublasLtMatmulDescSetAttribute(plan.op, CUBLASLT_MATMUL_DESC_EPILOGUE, &epilogue, sizeof(epilogue)) ==
              CUBLAS_STATUS_SUCCESS &&
          cublasLtMatmulDescSetAttribute(plan.op, CUBLASLT_MATMUL_DESC_BIAS_POINTER, &bias, sizeof(bias)) ==
              CUBLAS_STATUS_SUCCESS) {
        status = cublasLtMatmulAlgoGetHeuristic(lt_, plan.op, plan.a, plan.b, plan.c, plan.c, preference, kCandidates,
                                                results, &returned);
      }
      plan.bias = status == CUBLAS_STATUS_SUCCESS && returned > 0;
      if (!plan.bias) {  // no algorithm with this epilogue: a plain GEMM, and the caller adds the bias
        cublasLtMatmulDescDestroy(plan.op);
        create_op();
      }
    }
    if (!plan.bias) {
      returned = 0;
      status = cublasLtMatmulAlgoGetHeuristic(lt_, plan.op, plan.a, plan.b, plan.c, plan.c, preference, kCandidates,
                                              results, &returned);
    }
    cublasLtMatmulPreferenceDestroy(preference);
    if (status != CUBLAS_STATUS_SUCCESS || returned == 0) {
      cublasLtMatmulDescDestroy(plan.op);
      cublasLtMatrixLayoutDestroy(plan.a);
      cublasLtMatrixLayoutDestroy(plan.b);
      cublasLtMatrixLayoutDestroy(plan.c);
      throw Error("cuBLASLt found no algorithm for a " + std::to_string(m) + "x" + std::to_string(n) + "x" +
                  std::to_string(k) + " 16-bit GEMM");
    }
    // From here the cache owns the plan's descriptors, with the heuristic's first choice. Each
    // candidate is then timed once on this call's own buffers (y is overwritten by the real launch
    // below) and the fastest kept; the first call of a shape happens in warm-up, not in a timed scan.
    // An accumulating GEMM must not add into y more than once: its candidates run on the gate|up
    // buffer instead (as fp32 [m, n]; no live data there when the o_proj and down GEMMs run), and
    // with too small a buffer the heuristic's first choice is kept untimed.
    plan.algo = results[0].algo;
    found = cache.emplace(key, plan).first;
    void* trial = y;
    if (accumulate) {
      trial = static_cast<size_t>(m) * n * sizeof(float) <= gate_up_bytes_ ? gate_up_ : nullptr;
    }
    if (returned > 1 && trial != nullptr) {
      struct Events {  // released on every path out, the throwing ones included
        cudaEvent_t start = nullptr, stop = nullptr;
        ~Events() {
          if (start != nullptr) cudaEventDestroy(start);
          if (stop != nullptr) cudaEventDestroy(stop);
        }
      } events;
      cudaEvent_t& start = events.start;
      cudaEvent_t& stop = events.stop;
      check_cuda(cudaEventCreate(&start), "autotune event");
      check_cuda(cudaEventCreate(&stop), "autotune event");
      const float one = 1.0f;
      const float trial_beta = accumulate ? 1.0f : 0.0f;
      float best = 0.0f;
      for (int i = 0; i < returned; ++i) {
        if (results[i].state != CUBLAS_STATUS_SUCCESS) continue;
        bool ok = cublasLtMatmul(lt_, plan.op, &one, w, plan.a, x, plan.b, &trial_beta, trial, plan.c, trial, plan.c,
                                 &results[i].algo, lt_workspace_, lt_workspace_bytes_, stream_) ==
                  CUBLAS_STATUS_SUCCESS;  // warm
        check_cuda(cudaEventRecord(start, stream_), "autotune event");
        for (int r = 0; ok && r < 3; ++r) {
          ok = cublasLtMatmul(lt_, plan.op, &one, w, plan.a, x, plan.b, &trial_beta, trial, plan.c, trial, plan.c,
                              &results[i].algo, lt_workspace_, lt_workspace_bytes_, stream_) == CUBLAS_STATUS_SUCCESS;
        }
        check_cuda(cudaEventRecord(stop, stream_), "autotune event");
        check_cuda(cudaEventSynchronize(stop), "autotune event");
        float ms = 0.0f;
        check_cuda(cudaEventElapsedTime(&ms, start, stop), "autotune event");
        if (ok && (best == 0.0f || ms < best)) {
          best = ms;
          found->second.algo = results[i].algo;
        }
      }
    }
  }
  const float alpha = 1.0f, beta = accumulate ? 1.0f : 0.0f;
  const GemmPlan& plan = found->second;
  if (plan.bias) {
    check_lt(cublasLtMatmulDescSetAttribute(plan.op, CUBLASLT_MATMUL_DESC_BIAS_POINTER, &bias, sizeof(bias)),
             "bias pointer");
  }
  check_lt(cublasLtMatmul(lt_, plan.op, &alpha, w, plan.a, x, plan.b, &beta, y, plan.c, y, plan.c, &plan.algo,
                          lt_workspace_, lt_workspace_bytes_, stream_),
           "cublasLtMatmul");
  return plan.bias;
}

// Consecutive prompts into batches of at most capacity_tokens_ tokens and max_batch_prompts
// prompts. The batch count is the smallest those limits allow (the greedy fill's), and each batch
// closes near an equal share of the tokens, so a scan shard does not end on a sliver of a batch
// that runs its GEMMs at a fraction of their rate.
std::vector<Engine::Batch> Engine::plan_batches(const std::vector<PromptView>& prompts) const {
  auto greedy = [&](double target) {
    std::vector<Batch> batches;
    Batch current;
    for (int i = 0; i < static_cast<int>(prompts.size()); ++i) {
      const int tokens = prompts[i].token_count;
      const bool full = current.tokens + tokens > capacity_tokens_ || current.count + 1 > options_.max_batch_prompts;
      // past the share: close here if that leaves the batch nearer to it than taking the prompt
      const bool past_share = current.tokens + 0.5 * tokens > target;
      if (current.count > 0 && (full || past_share)) {
        batches.push_back(current);
        current = Batch{};
      }
      if (current.count == 0) current.first = i;
      current.count += 1;
      current.tokens += tokens;
    }
    if (current.count > 0) batches.push_back(current);
    return batches;
  };
  std::vector<Batch> batches = greedy(static_cast<double>(capacity_tokens_) + 1.0);
  if (batches.size() < 2) return batches;
  double total = 0.0;
  for (const PromptView& p : prompts) total += p.token_count;
  std::vector<Batch> balanced = greedy(total / static_cast<double>(batches.size()));
  return balanced.size() <= batches.size() ? balanced : batches;
}

void Engine::ensure_partials(size_t items, int span_count, int layers) {
  const size_t needed = items * span_count * layers;
  if (needed <= partials_capacity_) return;
  synchronize();
  if (partials_ != nullptr) cudaFree(partials_);
  partials_ = nullptr;
  const size_t capacity = std::max(needed, partials_capacity_ * 2);
  partials_capacity_ = 0;  // a failed allocation leaves no buffer to be mistaken for a large one
  check_cuda(cudaMalloc(reinterpret_cast<void**>(&partials_), capacity * sizeof(float)), "partials allocation");
  partials_capacity_ = capacity;
}

void Engine::probe(const std::vector<PromptView>& prompts, int span_count, LayerRange range, bool normalize_by_length,
                   double* rows_host, double* raw_rows_host, float* device_accumulator) {
  validate(prompts, span_count, range);
  const int layers = range.count();
  const size_t row_values = prompts.size() * static_cast<size_t>(layers) * span_count;
  const bool want_rows = rows_host != nullptr || raw_rows_host != nullptr;
  if (want_rows && row_values * 2 > rows_capacity_) {
    synchronize();
    if (rows_device_ != nullptr) cudaFree(rows_device_);
    rows_device_ = nullptr;
    rows_capacity_ = 0;  // as for the partials: no stale capacity after a failed allocation
    check_cuda(cudaMalloc(reinterpret_cast<void**>(&rows_device_), row_values * 2 * sizeof(double)), "rows allocation");
    rows_capacity_ = row_values * 2;
  }
  double* rows_device = want_rows ? rows_device_ : nullptr;
  double* raw_rows_device = want_rows ? rows_device_ + row_values : nullptr;
  check_cuda(cudaMemsetAsync(status_, 0, sizeof(int), stream_), "status reset");

  const std::vector<Batch> batches = plan_batches(prompts);
  for (size_t b = 0; b < batches.size(); ++b) {
    const Batch& batch = batches[b];
    const size_t offset = static_cast<size_t>(batch.first) * layers * span_count;
    run_batch(prompts, batch, span_count, range, normalize_by_length, rows_device ? rows_device + offset : nullptr,
              raw_rows_device ? raw_rows_device + offset : nullptr, device_accumulator, static_cast<int>(b & 1));
  }
  if (rows_host != nullptr) {
    check_cuda(cudaMemcpyAsync(rows_host, rows_device, row_values * sizeof(double), cudaMemcpyDeviceToHost, stream_),
               "rows download");
  }
  if (raw_rows_host != nullptr) {
    check_cuda(cudaMemcpyAsync(raw_rows_host, raw_rows_device, row_values * sizeof(double), cudaMemcpyDeviceToHost,
                               stream_),
               "rows download");
  }
  raise_on_status(read_status());
}

void Engine::raise_on_status(int status) {
  if (status != 0) {
    static const char* reasons[] = {"ok", "a token id is outside the vocabulary", "a position exceeds the RoPE table",
                                    "a device wait timed out"};
    const char* reason = status > 0 && status < 4 ? reasons[status] : "unknown device error";
    throw Error(std::string("device reported an error during the probe: ") + reason);
  }
}

void Engine::reset_status() { check_cuda(cudaMemsetAsync(status_, 0, sizeof(int), stream_), "status reset"); }

void Engine::validate(const std::vector<PromptView>& prompts, int span_count, LayerRange range) const {
  if (prompts.empty()) throw Error("attention probe requires at least one prompt");
  if (span_count <= 0) throw Error("attention probe requires document spans");
  if (span_count > kMassMaxSpans) {
    throw Error("at most " + std::to_string(kMassMaxSpans) + " document spans are supported (got " +
                std::to_string(span_count) + ")");
  }
  if (range.begin < 0 || range.end > config_.num_hidden_layers || range.count() <= 0) {
    throw Error("probe layers are out of range");
  }
  std::string missing;
  if (!weights_complete(&missing)) throw Error("checkpoint is missing tensor '" + missing + "'");
  for (size_t i = 0; i < prompts.size(); ++i) {
    const PromptView& p = prompts[i];
    if (p.token_count <= 0) throw Error("probe prompt " + std::to_string(i) + " is empty");
    if (p.token_count > options_.max_sequence_length) {
      throw Error("probe input of " + std::to_string(p.token_count) + " tokens exceeds the context window");
    }
    // Degenerate spans are accepted as the reference accepts them (DocumentAttentionProbe and
    // reduce_document_attention_kernel, attnrank/src/model.cu:248-251, kernels.cu:211-219): the
    // query span is clipped to [0, tokens), so an empty or reversed one gives all-zero rows, and a
    // document span with end <= begin holds no keys (zero mass). A negative document begin is
    // rejected: there the reference reads before the score row.
    for (int s = 0; s < span_count; ++s) {
      if (p.spans[2 * s] < 0) {
        throw Error("probe prompt " + std::to_string(i) + " has a document span that begins before token 0");
      }
    }
  }
}

// Metadata blob of one batch: tokens | prompt offsets | query spans | spans | attention tiles |
// mass item offsets, all int32, written at `host` (capacity in int32 elements).
BatchLayout Engine::build_metadata(const std::vector<PromptView>& prompts, const Batch& batch, int span_count,
                                           int32_t* host, size_t capacity) const {
  const ModelConfig& c = config_;
  const int P = batch.count;
  const int S = span_count;
  const int group = c.num_attention_heads / c.num_key_value_heads;
  size_t needed = static_cast<size_t>(batch.tokens) + (P + 1) + 2 * P + 2 * static_cast<size_t>(P) * S + 2 * (P + 1);
  for (int i = 0; i < P; ++i) {
    needed += 2 * ((prompts[batch.first + i].token_count + kAttentionQueryTile - 1) / kAttentionQueryTile);
  }
  if (needed > capacity) throw Error("batch metadata exceeds its buffer");
  size_t cursor = 0;
  const size_t tokens_at = cursor;
  for (int i = 0; i < P; ++i) {
    const PromptView& p = prompts[batch.first + i];
    std::memcpy(host + cursor, p.tokens, sizeof(int32_t) * p.token_count);
    cursor += p.token_count;
  }
  const size_t offsets_at = cursor;
  host[cursor++] = 0;
  for (int i = 0; i < P; ++i) {
    host[cursor] = host[cursor - 1] + prompts[batch.first + i].token_count;
    ++cursor;
  }
  const size_t queries_at = cursor;
  for (int i = 0; i < P; ++i) {
    host[cursor++] = prompts[batch.first + i].query_begin;
    host[cursor++] = prompts[batch.first + i].query_end;
  }
  const size_t spans_at = cursor;
  for (int i = 0; i < P; ++i) {
    std::memcpy(host + cursor, prompts[batch.first + i].spans, sizeof(int32_t) * 2 * S);
    cursor += 2 * S;
  }
  const size_t tiles_at = cursor;
  int max_tiles = 0;
  for (int i = 0; i < P; ++i) {
    max_tiles = std::max(max_tiles, (prompts[batch.first + i].token_count + kAttentionQueryTile - 1) / kAttentionQueryTile);
  }
  int tile_count = 0;
  for (int t = max_tiles - 1; t >= 0; --t) {  // heaviest (latest) query tiles first
    for (int i = 0; i < P; ++i) {
      if (t * kAttentionQueryTile < prompts[batch.first + i].token_count) {
        host[cursor++] = i;
        host[cursor++] = t;
        ++tile_count;
      }
    }
  }
  const size_t items_at = cursor;
  host[cursor++] = 0;
  for (int i = 0; i < P; ++i) {
    const MassItemShape shape = mass_item_shape(host + queries_at + 2 * i, host + spans_at + 2 * static_cast<size_t>(i) * S,
                                                S, prompts[batch.first + i].token_count, group);
    host[cursor] = host[cursor - 1] + mass_items_for_prompt(shape, c.num_key_value_heads);
    ++cursor;
  }
  const size_t fused_items_at = cursor;
  host[cursor++] = 0;
  for (int i = 0; i < P; ++i) {
    const int tiles = fused_mass_tiles(host + queries_at + 2 * i, prompts[batch.first + i].token_count);
    host[cursor] = host[cursor - 1] + c.num_attention_heads * tiles * kFusedMassSlotsPerTile;
    ++cursor;
  }
  BatchLayout layout;
  const double D = c.head_dim(), Hq = c.num_attention_heads;
  for (int i = 0; i < P; ++i) {
    const PromptView& p = prompts[batch.first + i];
    const double L = p.token_count;
    double pairs = L * (L + 1) / 2;  // causal (query, key) pairs
    if (c.sliding_window > 0 && p.token_count > c.sliding_window) {
      const double W = c.sliding_window;
      pairs = W * (W + 1) / 2 + (L - W) * W;
    }
    layout.attention_flops += 4 * D * Hq * pairs;
    // work of the rows and keys that exist: spans clipped to the prompt as the kernels clip them
    double span_keys = 0;
    for (int s = 0; s < S; ++s) span_keys += std::max(0, std::min(p.spans[2 * s + 1], p.token_count) - p.spans[2 * s]);
    const int query_rows = std::max(0, std::min(p.query_end, p.token_count) - std::max(p.query_begin, 0));
    layout.mass_flops += 2 * D * Hq * static_cast<double>(query_rows) * span_keys;
  }
  layout.tokens_at = tokens_at;
  layout.offsets_at = offsets_at;
  layout.queries_at = queries_at;
  layout.spans_at = spans_at;
  layout.tiles_at = tiles_at;
  layout.items_at = items_at;
  layout.fused_items_at = fused_items_at;
  layout.size = cursor;
  layout.first = batch.first;
  layout.prompts = P;
  layout.tokens = batch.tokens;
  layout.tile_count = tile_count;
  layout.item_count = host[items_at + P];
  layout.fused_item_count = host[cursor - 1];
  return layout;
}

// The probe path: stage the batch metadata in pinned memory (double-buffered), upload, execute.
void Engine::run_batch(const std::vector<PromptView>& prompts, const Batch& batch, int span_count, LayerRange range,
                       bool normalize_by_length, double* rows_device, double* raw_rows_device,
                       float* device_accumulator, int slot) {
  check_cuda(cudaEventSynchronize(meta_free_[slot]), "metadata buffer reuse");
  const BatchLayout layout = build_metadata(prompts, batch, span_count, meta_host_[slot], meta_capacity_);
  check_cuda(cudaMemcpyAsync(meta_device_[slot], meta_host_[slot], layout.size * sizeof(int32_t),
                             cudaMemcpyHostToDevice, stream_),
             "metadata upload");
  check_cuda(cudaEventRecord(meta_free_[slot], stream_), "cudaEventRecord");
  ensure_partials(static_cast<size_t>(std::max(layout.item_count, layout.fused_item_count)), span_count,
                  range.count());
  execute_batch(layout, meta_device_[slot], span_count, range, normalize_by_length, rows_device, raw_rows_device,
                device_accumulator);
}

std::unique_ptr<PreparedScan> Engine::prepare_scan(const std::vector<PromptView>& prompts, int span_count,
                                                   LayerRange range, bool normalize_by_length) {
  validate(prompts, span_count, range);
  auto prepared = std::make_unique<PreparedScan>();
  prepared->span_count = span_count;
  prepared->range = range;
  prepared->normalize_by_length = normalize_by_length;
  prepared->prompt_count = static_cast<int>(prompts.size());
  std::vector<int32_t> host;
  size_t max_items = 0;
  for (const Batch& batch : plan_batches(prompts)) {
    const size_t base = host.size();
    host.resize(base + meta_capacity_);
    BatchLayout layout = build_metadata(prompts, batch, span_count, host.data() + base, meta_capacity_);
    host.resize(base + layout.size);
    layout.tokens_at += base;
    layout.offsets_at += base;
    layout.queries_at += base;
    layout.spans_at += base;
    layout.tiles_at += base;
    layout.items_at += base;
    layout.fused_items_at += base;
    max_items = std::max(max_items, static_cast<size_t>(std::max(layout.item_count, layout.fused_item_count)));
    prepared->batches.push_back(layout);
  }
  ensure_partials(max_items, span_count, range.count());
  check_cuda(cudaMalloc(reinterpret_cast<void**>(&prepared->device), host.size() * sizeof(int32_t)),
             "prepared scan allocation");
  copy_to_device(prepared->device, host.data(), host.size() * sizeof(int32_t), stream_, "prepared scan upload");
  prepared->device_bytes = host.size() * sizeof(int32_t);
  return prepared;
}

void Engine::run_prepared(const PreparedScan& prepared, float* device_accumulator) {
  for (const BatchLayout& layout : prepared.batches) {
    execute_batch(layout, prepared.device, prepared.span_count, prepared.range, prepared.normalize_by_length, nullptr,
                  nullptr, device_accumulator);
  }
}

int Engine::read_status() {
  check_cuda(cudaMemcpyAsync(status_host_, status_, sizeof(int), cudaMemcpyDeviceToHost, stream_), "status download");
  synchronize();
  last_status_ = *status_host_;
  return last_status_;
}

PreparedScan::~PreparedScan() {
  if (device != nullptr) cudaFree(device);
}

void Engine::execute_batch(const BatchLayout& layout, const int32_t* dev, int span_count, LayerRange range,
                           bool normalize_by_length, double* rows_device, double* raw_rows_device,
                           float* device_accumulator) {
  const ModelConfig& c = config_;
  const int P = layout.prompts;
  const int M = layout.tokens;
  const int S = span_count;
  const int tile_count = layout.tile_count;
  const int item_count = layout.item_count;
  const int32_t* d_tokens = dev + layout.tokens_at;
  const int32_t* d_offsets = dev + layout.offsets_at;
  const int32_t* d_queries = dev + layout.queries_at;
  const int32_t* d_spans = dev + layout.spans_at;
  const int32_t* d_tiles = dev + layout.tiles_at;
  const bool fused = options_.attention_kernel == 0;  // tcgen05 attention captures the mass itself
  const int32_t* d_items = dev + (fused ? layout.fused_items_at : layout.items_at);
  const int mass_items = fused ? layout.fused_item_count : item_count;
  const int layers = range.count();

  const int H = c.hidden_size, I = c.intermediate_size, Hq = c.num_attention_heads, Hkv = c.num_key_value_heads;
  const int D = c.head_dim(), Wqkv = c.qkv_width();
  const int dtype = options_.activation_dtype;
  const double m = M;
  timed(kClassPositions, 4.0 * M + 4.0 * (P + 1), [&] {
    check_cuda(launch_positions(d_offsets, P, M, positions_, stream_), "positions");
  });
  timed(kClassEmbedding, m * H * (2 + 4 + 2) + 4.0 * M, [&] {
    check_cuda(launch_embed_rms_norm(d_tokens, M, embedding_, c.vocab_size, H, layers_[0].input_norm, c.rms_norm_eps,
                                     residual_, normed_, status_, dtype, stream_),
               "embedding");
  });

  AttentionArgs attention;
  attention.qkv = qkv_;
  attention.out = attn_;
  attention.lse = lse_;
  attention.prompt_offsets = d_offsets;
  attention.tiles = d_tiles;
  attention.tile_count = tile_count;
  attention.query_heads = Hq;
  attention.kv_heads = Hkv;
  attention.head_dim = D;
  attention.sliding_window = c.sliding_window;
  attention.dtype = dtype;
  attention.rows = M;
  attention.status = status_;
  attention.query_spans = d_queries;
  attention.spans = d_spans;
  attention.mass_items = d_items;
  attention.span_count = S;
  attention.normalize_by_length = normalize_by_length ? 1 : 0;
  attention.reference_chunk = options_.prefill_chunk_tokens;

  MassArgs mass;
  mass.qkv = qkv_;
  mass.qkv_rows_capacity = capacity_tokens_;
  mass.lse = lse_;
  mass.prompt_offsets = d_offsets;
  mass.query_spans = d_queries;
  mass.spans = d_spans;
  mass.item_offsets = dev + layout.items_at;
  mass.prompt_count = P;
  mass.span_count = S;
  mass.item_count = item_count;
  mass.query_heads = Hq;
  mass.kv_heads = Hkv;
  mass.head_dim = D;
  mass.sliding_window = c.sliding_window;
  mass.reference_chunk = options_.prefill_chunk_tokens;
  mass.normalize_by_length = normalize_by_length ? 1 : 0;
  mass.status = status_;
  mass.dtype = dtype;

  // algorithmic work of each launch: FLOPs for GEMMs / attention / mass, HBM bytes otherwise
  const double norm_bytes = m * H * (4 + 2);  // read the fp32 residual, write the 16-bit row
  const double silu_bytes = m * I * 2 * 3;
  const int last_layer = range.end - 1;
  for (int l = 0; l <= last_layer; ++l) {
    const LayerWeights& w = layers_[l];
    // fp16 engine: the q|k|v bias (rounded once to fp16) is added in the GEMM epilogue when
    // cuBLASLt offers it; otherwise, and for bf16 (whose rounding of the bias would be 16x
    // coarser), the RoPE kernel adds the fp32 bias
    bool bias_done = false;
    const void* epilogue_bias = dtype == kActFp16 ? w.qkv_bias_half : nullptr;
    timed(kClassGemmQkv, 2 * m * Wqkv * H, [&] { bias_done = gemm(normed_, w.qkv, qkv_, M, Wqkv, H, epilogue_bias); });
    const float* rotary_bias = bias_done ? nullptr : w.qkv_bias;
    const double rotated = Hq + Hkv + (rotary_bias != nullptr ? Hkv : 0);
    timed(kClassRotary, m * rotated * D * 2 * 2, [&] {
      check_cuda(launch_rotary_bias(qkv_, rotary_bias, positions_, M, Hq, Hkv, D, cos_table_, sin_table_,
                                    options_.max_sequence_length, status_, dtype, stream_),
                 "rotary");
    });
    const bool probed = l >= range.begin;
    float* layer_partials = probed ? partials_ + static_cast<size_t>(l - range.begin) * mass_items * S : nullptr;
    attention.mass_partials = fused ? layer_partials : nullptr;
    timed(kClassAttention, layout.attention_flops, [&] {
      check_cuda(fused ? launch_causal_attention_tc(attention, stream_) : launch_causal_attention(attention, stream_),
                 "attention");
    });
    if (probed && !fused) {
      mass.partials = layer_partials;
      timed(kClassMass, layout.mass_flops, [&] { check_cuda(launch_document_mass(mass, stream_), "document mass"); });
    }
    // The last probed layer's attention output, o_proj and MLP feed only layers that are not run:
    // no probe output depends on them (the reference computes them, model.cu:334-337), so the
    // forward ends at the last mass capture.
    if (l == last_layer) break;
    timed(kClassGemmOut, 2 * m * H * Hq * D, [&] { gemm_residual(attn_, w.out, residual_, M, H, Hq * D); });
    timed(kClassNorm, norm_bytes, [&] {
      check_cuda(launch_rms_norm_residual(residual_, nullptr, w.post_norm, M, H, c.rms_norm_eps, normed_, dtype, stream_),
                 "post-attention norm");
    });
    timed(kClassGemmGateUp, 2 * m * 2 * I * H, [&] { gemm(normed_, w.gate_up, gate_up_, M, 2 * I, H); });
    timed(kClassSilu, silu_bytes, [&] {
      check_cuda(launch_silu_multiply(gate_up_, static_cast<const uint16_t*>(gate_up_) + I, 2LL * I, act_, I, M, I,
                                      dtype, stream_),
                 "swiglu");
    });
    timed(kClassGemmDown, 2 * m * H * I, [&] { gemm_residual(act_, w.down, residual_, M, H, I); });
    const float* next_norm = l + 1 < c.num_hidden_layers ? layers_[l + 1].input_norm : final_norm_;
    timed(kClassNorm, norm_bytes, [&] {
      check_cuda(launch_rms_norm_residual(residual_, nullptr, next_norm, M, H, c.rms_norm_eps, normed_, dtype, stream_),
                 "pre-attention norm");
    });
  }

  FinalizeArgs finalize;
  finalize.partials = partials_;
  finalize.item_offsets = d_items;
  finalize.query_spans = d_queries;
  finalize.prompt_offsets = d_offsets;
  finalize.prompt_count = P;
  finalize.span_count = S;
  finalize.item_count = mass_items;
  finalize.layers = layers;
  finalize.query_heads = Hq;
  finalize.rows = rows_device;
  finalize.raw_rows = raw_rows_device;
  finalize.accumulator = device_accumulator;
  timed(kClassFinalize, 4.0 * layers * mass_items * S, [&] {
    check_cuda(launch_finalize_mass(finalize, stream_), "finalize");
  });
}

}  // namespace arb
