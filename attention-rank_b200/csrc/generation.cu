// Generation on the B200 engine: CudaLlamaModel::generate (include/attnrank/model.hpp:131-136,
// :156; attnrank/src/model.cu:532-565).
//
// The reference prefills the prompt in 512-token chunks against its fp32 KV cache, reads the last
// row's logits (final RMSNorm + lm_head GEMM, model.cu:341-350), then loops: select a token on
// the host, run one forward_chunk of that single token, read logits again. Here:
//   * the prefill is one packed forward of the whole prompt through the probe's batched kernels
//     (cuBLASLt GEMMs, tcgen05 attention), with K and V of every layer copied into a 16-bit
//     cache after RoPE; only the last row goes through lm_head;
//   * a decode step is the chain of single-token kernels of decode.cu: per layer RMSNorm + q|k|v
//     + RoPE + cache append, split attention, o_proj, RMSNorm + gate|up + SwiGLU, down_proj (each
//     norm fused into the projection that consumes it), then final RMSNorm + lm_head. The chain is
//     captured once into a CUDA graph that reads the token and its position from device memory, so
//     every later step is one graph launch (or, opt-in, one persistent kernel per step);
//   * greedy selection (the reference's default, temperature 0) is a device argmax that writes the
//     next step's token, so consecutive steps chain on the device; the host only reads each token
//     back to test for eos, with the next step already queued behind it.
#include <algorithm>
#include <cstdlib>
#include <string>

#include "common.cuh"
#include "decode.h"
#include "engine.h"
#include "layer_kernels.h"
#include "synthetic.h"

namespace arb {

namespace {
constexpr int kStateUpload = 0;  // staging[0..1]: {token, position} host -> device
constexpr int kStateSlots = 2;   // staging[2..5]: two {token, position} downloads
constexpr int kStagingMeta = 8;  // metadata staging starts here
}  // namespace

GenerationState::~GenerationState() {
  for (auto& graph : graphs) {
    if (graph != nullptr) cudaGraphExecDestroy(graph);
  }
  for (auto& event : slot_ready) {
    if (event != nullptr) cudaEventDestroy(event);
  }
  if (staging != nullptr) cudaFreeHost(staging);
  if (logits_host != nullptr) cudaFreeHost(logits_host);
}

const void* Engine::output_head() const {
  if (lm_head_ != nullptr) return lm_head_;
  if (config_.tie_word_embeddings) return embedding_;
  throw Error("generation needs lm_head.weight (the config does not tie it to the embedding)");
}

void Engine::release_decode_graphs() {
  if (!generation_) return;
  for (int i = 0; i < 2; ++i) {
    if (generation_->graphs[i] != nullptr) {
      cudaGraphExecDestroy(generation_->graphs[i]);
      generation_->graphs[i] = nullptr;
    }
    generation_->warmed[i] = false;
  }
}

int Engine::generation_position() const { return generation_ ? generation_->position : -1; }

void Engine::ensure_generation() {
  if (generation_) return;
  const ModelConfig& c = config_;
  if (c.head_dim() != 128) throw Error("generation needs head_dim 128");
  if (c.num_attention_heads / c.num_key_value_heads > kDecodeMaxGroup) {
    throw Error("generation supports at most " + std::to_string(kDecodeMaxGroup) + " query heads per KV head");
  }
  auto g = std::make_unique<GenerationState>();
  const size_t L = c.num_hidden_layers, Hq = c.num_attention_heads, D = c.head_dim(), V = c.vocab_size;
  g->context = options_.max_sequence_length;
  g->layer_elements = static_cast<size_t>(c.num_key_value_heads) * g->context * D;
  g->k_cache = device_alloc(L * g->layer_elements * 2);
  g->v_cache = device_alloc(L * g->layer_elements * 2);
  g->q = device_alloc(Hq * D * 2);
  g->partials = static_cast<float*>(device_alloc(Hq * kDecodeSplits * D * 4));
  g->stats = static_cast<float*>(device_alloc(Hq * kDecodeSplits * 2 * 4));
  g->logits = static_cast<float*>(device_alloc(V * 4));
  g->pick_values = static_cast<float*>(device_alloc(kDecodePickSlots * sizeof(float)));
  g->pick_indices = static_cast<int32_t*>(device_alloc(kDecodePickSlots * sizeof(int32_t)));
  g->tickets = static_cast<unsigned*>(device_alloc((2 + c.num_key_value_heads) * sizeof(unsigned)));
  g->state = static_cast<int32_t*>(device_alloc(4 * sizeof(int32_t)));
  g->meta_capacity = static_cast<size_t>(capacity_tokens_) + 2 + 2 * (capacity_tokens_ / kAttentionQueryTile + 1);
  g->meta = static_cast<int32_t*>(device_alloc(g->meta_capacity * 4));
  check_cuda(cudaHostAlloc(reinterpret_cast<void**>(&g->staging), (kStagingMeta + g->meta_capacity) * 4,
                           cudaHostAllocDefault),
             "cudaHostAlloc");
  for (auto& event : g->slot_ready) {
    check_cuda(cudaEventCreateWithFlags(&event, cudaEventDisableTiming), "cudaEventCreate");
  }
  // the persistent step kernel's table of per-layer weights and cache rows (stable addresses)
  std::vector<DecodeLayerWeights> table(L);
  for (size_t l = 0; l < L; ++l) {
    const LayerWeights& w = layers_[l];
    const bool half_bias = options_.activation_dtype == kActFp16 && w.qkv_bias_half != nullptr;
    table[l].qkv = w.qkv;
    table[l].qkv_bias_half = half_bias ? w.qkv_bias_half : nullptr;
    table[l].qkv_bias = half_bias ? nullptr : w.qkv_bias;
    table[l].out = w.out;
    table[l].gate_up = w.gate_up;
    table[l].down = w.down;
    table[l].input_norm = w.input_norm;
    table[l].post_norm = w.post_norm;
    table[l].k_cache = static_cast<uint16_t*>(g->k_cache) + l * g->layer_elements;
    table[l].v_cache = static_cast<uint16_t*>(g->v_cache) + l * g->layer_elements;
  }
  g->layer_table = device_alloc(L * sizeof(DecodeLayerWeights));
  check_cuda(cudaMemcpyAsync(g->layer_table, table.data(), L * sizeof(DecodeLayerWeights), cudaMemcpyHostToDevice,
                             stream_),
             "decode layer table");
  synchronize();  // the host table goes out of scope
  // ATTNRANK_DECODE_PERSISTENT=1: one persistent kernel per step (measured slower than the
  // per-phase kernels on B200: 3.48 against 3.11 ms per Qwen-7B token); ATTNRANK_DECODE_PDL=0:
  // per-phase kernels without programmatic launch
  const char* persistent = std::getenv("ATTNRANK_DECODE_PERSISTENT");
  g->persistent = persistent != nullptr && persistent[0] == '1';
  const char* pdl = std::getenv("ATTNRANK_DECODE_PDL");
  g->programmatic = !(pdl != nullptr && pdl[0] == '0');
  generation_ = std::move(g);
}

int Engine::decode_mode() const {
  if (!generation_) return -1;
  return generation_->persistent ? 2 : generation_->programmatic ? 1 : 0;
}

void Engine::prefill_generation(int M) {
  const ModelConfig& c = config_;
  GenerationState& g = *generation_;
  const int H = c.hidden_size, I = c.intermediate_size, Hq = c.num_attention_heads, Hkv = c.num_key_value_heads;
  const int D = c.head_dim(), Wqkv = c.qkv_width();
  const int dtype = options_.activation_dtype;
  const int32_t* d_tokens = g.meta;
  const int32_t* d_offsets = g.meta + M;
  const int32_t* d_tiles = g.meta + M + 2;
  const int tiles = (M + kAttentionQueryTile - 1) / kAttentionQueryTile;

  check_cuda(launch_positions(d_offsets, 1, M, positions_, stream_), "positions");
  check_cuda(launch_embed_rms_norm(d_tokens, M, embedding_, c.vocab_size, H, layers_[0].input_norm, c.rms_norm_eps,
                                   residual_, normed_, status_, dtype, stream_),
             "embedding");
  AttentionArgs attention;
  attention.qkv = qkv_;
  attention.out = attn_;
  attention.lse = lse_;
  attention.prompt_offsets = d_offsets;
  attention.tiles = d_tiles;
  attention.tile_count = tiles;
  attention.query_heads = Hq;
  attention.kv_heads = Hkv;
  attention.head_dim = D;
  attention.sliding_window = c.sliding_window;
  attention.dtype = dtype;
  attention.rows = M;
  attention.status = status_;  // no mass capture: mass_partials stays null

  for (int l = 0; l < c.num_hidden_layers; ++l) {
    const LayerWeights& w = layers_[l];
    const void* epilogue_bias = dtype == kActFp16 ? w.qkv_bias_half : nullptr;
    const bool bias_done = gemm(normed_, w.qkv, qkv_, M, Wqkv, H, epilogue_bias);
    check_cuda(launch_rotary_bias(qkv_, bias_done ? nullptr : w.qkv_bias, positions_, M, Hq, Hkv, D, cos_table_,
                                  sin_table_, options_.max_sequence_length, status_, dtype, stream_),
               "rotary");
    auto* k_layer = static_cast<uint16_t*>(g.k_cache) + static_cast<size_t>(l) * g.layer_elements;
    auto* v_layer = static_cast<uint16_t*>(g.v_cache) + static_cast<size_t>(l) * g.layer_elements;
    check_cuda(launch_store_kv(qkv_, M, Hq, Hkv, D, k_layer, v_layer, g.context, dtype, stream_), "KV cache store");
    check_cuda(options_.attention_kernel == 0 ? launch_causal_attention_tc(attention, stream_)
                                              : launch_causal_attention(attention, stream_),
               "attention");
    gemm_residual(attn_, w.out, residual_, M, H, Hq * D);
    check_cuda(launch_rms_norm_residual(residual_, nullptr, w.post_norm, M, H, c.rms_norm_eps, normed_, dtype, stream_),
               "post-attention norm");
    gemm(normed_, w.gate_up, gate_up_, M, 2 * I, H);
    check_cuda(launch_silu_multiply(gate_up_, static_cast<const uint16_t*>(gate_up_) + I, 2LL * I, act_, I, M, I, dtype,
                                    stream_),
               "swiglu");
    gemm_residual(act_, w.down, residual_, M, H, I);
    const float* next_norm = l + 1 < c.num_hidden_layers ? layers_[l + 1].input_norm : final_norm_;
    check_cuda(launch_rms_norm_residual(residual_, nullptr, next_norm, M, H, c.rms_norm_eps, normed_, dtype, stream_),
               "norm");
  }
  // normed_ holds final_norm(hidden); the logits of the last row (read_logits, model.cu:341-350)
  DecodeGemvArgs head;
  head.kind = kDecodeLogits;
  head.w = output_head();
  head.rows = c.vocab_size;
  head.k = H;
  head.x = static_cast<const uint16_t*>(normed_) + static_cast<size_t>(M - 1) * H;
  head.y = g.logits;
  head.dtype = dtype;
  check_cuda(launch_decode_gemv(head, false, stream_), "lm_head");
}

bool Engine::launch_persistent_step(bool greedy) {
  const ModelConfig& c = config_;
  GenerationState& g = *generation_;
  const int H = c.hidden_size, I = c.intermediate_size, Hq = c.num_attention_heads, Hkv = c.num_key_value_heads;
  const int D = c.head_dim();
  const int dtype = options_.activation_dtype;
  DecodeStepArgs s;
  s.layers = static_cast<const DecodeLayerWeights*>(g.layer_table);
  s.layer_count = c.num_hidden_layers;
  s.qkv.kind = kDecodeQkv;
  s.qkv.rows = c.qkv_width();
  s.qkv.k = H;
  s.qkv.eps = c.rms_norm_eps;
  s.qkv.embed_table = embedding_;
  s.qkv.vocab = c.vocab_size;
  s.qkv.query_heads = Hq;
  s.qkv.kv_heads = Hkv;
  s.qkv.head_dim = D;
  s.qkv.cos_table = cos_table_;
  s.qkv.sin_table = sin_table_;
  s.qkv.table_positions = options_.max_sequence_length;
  s.qkv.state = g.state;
  s.qkv.q_out = g.q;
  s.qkv.context = g.context;
  s.qkv.status = status_;
  s.qkv.dtype = dtype;
  void* delta_attention = delta_;
  void* delta_mlp = static_cast<uint16_t*>(delta_) + H;
  s.qkv.delta = delta_mlp;
  s.out_proj.kind = kDecodePlain;
  s.out_proj.rows = H;
  s.out_proj.k = Hq * D;
  s.out_proj.x = attn_;
  s.out_proj.y = delta_attention;
  s.out_proj.dtype = dtype;
  s.gate_up.kind = kDecodeGateUp;
  s.gate_up.rows = I;
  s.gate_up.k = H;
  s.gate_up.eps = c.rms_norm_eps;
  s.gate_up.delta = delta_attention;
  s.gate_up.y = act_;
  s.gate_up.dtype = dtype;
  s.down.kind = kDecodePlain;
  s.down.rows = H;
  s.down.k = I;
  s.down.x = act_;
  s.down.y = delta_mlp;
  s.down.dtype = dtype;
  s.head.kind = kDecodeLogits;
  s.head.w = output_head();
  s.head.rows = c.vocab_size;
  s.head.k = H;
  s.head.delta = delta_mlp;
  s.head.gamma = final_norm_;
  s.head.eps = c.rms_norm_eps;
  s.head.y = g.logits;
  s.head.state = g.state;
  s.head.pick = greedy;
  s.head.pick_values = g.pick_values;
  s.head.pick_indices = g.pick_indices;
  s.head.dtype = dtype;
  s.attention.q = g.q;
  s.attention.context = g.context;
  s.attention.state = g.state;
  s.attention.query_heads = Hq;
  s.attention.kv_heads = Hkv;
  s.attention.head_dim = D;
  s.attention.sliding_window = c.sliding_window;
  s.attention.partials = g.partials;
  s.attention.stats = g.stats;
  s.attention.tickets = g.tickets + 1;
  s.attention.out = attn_;
  s.attention.dtype = dtype;
  s.residual[0] = residual_;
  s.residual[1] = residual_ + H;
  s.barrier = g.tickets + 1 + Hkv;
  s.status = status_;
  s.dtype = dtype;
  s.max_k = std::max(std::max(H, I), Hq * D);
  check_cuda(cudaMemsetAsync(g.tickets, 0, (2 + Hkv) * sizeof(unsigned), stream_), "decode tickets");
  const cudaError_t status = ::arb::launch_decode_step(s, stream_);
  if (status == cudaSuccess) return true;
  cudaGetLastError();  // a refused cooperative launch ran nothing: the per-phase kernels take over
  return false;
}

void Engine::launch_decode_step(bool greedy) {
  const ModelConfig& c = config_;
  GenerationState& g = *generation_;
  if (g.persistent) {
    if (launch_persistent_step(greedy)) return;
    g.persistent = false;
  }
  const int H = c.hidden_size, I = c.intermediate_size, Hq = c.num_attention_heads, Hkv = c.num_key_value_heads;
  const int D = c.head_dim();
  const int dtype = options_.activation_dtype;
  const bool pdl = g.programmatic;
  // residual stream: two fp32 rows used in turn (a fused norm reads one and its CTA 0 writes the
  // sum into the other); the two deltas are the o_proj and down_proj outputs
  float* residual[2] = {residual_, residual_ + H};
  int current = 0;
  void* delta_attention = delta_;
  void* delta_mlp = static_cast<uint16_t*>(delta_) + H;
  check_cuda(launch_embed_rms_norm(g.state, 1, embedding_, c.vocab_size, H, layers_[0].input_norm, c.rms_norm_eps,
                                   residual[0], normed_, status_, dtype, stream_),
             "decode embedding");
  DecodeGemvArgs qkv;
  qkv.kind = kDecodeQkv;
  qkv.rows = c.qkv_width();
  qkv.k = H;
  qkv.eps = c.rms_norm_eps;
  qkv.query_heads = Hq;
  qkv.kv_heads = Hkv;
  qkv.head_dim = D;
  qkv.cos_table = cos_table_;
  qkv.sin_table = sin_table_;
  qkv.table_positions = options_.max_sequence_length;
  qkv.state = g.state;
  qkv.q_out = g.q;
  qkv.context = g.context;
  qkv.status = status_;
  qkv.dtype = dtype;
  DecodeAttentionArgs attention;
  attention.q = g.q;
  attention.context = g.context;
  attention.state = g.state;
  attention.query_heads = Hq;
  attention.kv_heads = Hkv;
  attention.head_dim = D;
  attention.sliding_window = c.sliding_window;
  attention.partials = g.partials;
  attention.stats = g.stats;
  attention.tickets = g.tickets + 1;
  attention.out = attn_;
  attention.dtype = dtype;
  DecodeGemvArgs out_proj;
  out_proj.kind = kDecodePlain;
  out_proj.rows = H;
  out_proj.k = Hq * D;
  out_proj.x = attn_;
  out_proj.y = delta_attention;
  out_proj.dtype = dtype;
  DecodeGemvArgs gate_up;
  gate_up.kind = kDecodeGateUp;
  gate_up.rows = I;
  gate_up.k = H;
  gate_up.eps = c.rms_norm_eps;
  gate_up.delta = delta_attention;
  gate_up.y = act_;
  gate_up.dtype = dtype;
  DecodeGemvArgs down;
  down.kind = kDecodePlain;
  down.rows = H;
  down.k = I;
  down.x = act_;
  down.y = delta_mlp;
  down.dtype = dtype;
  for (int l = 0; l < c.num_hidden_layers; ++l) {
    const LayerWeights& w = layers_[l];
    auto* k_layer = static_cast<uint16_t*>(g.k_cache) + static_cast<size_t>(l) * g.layer_elements;
    auto* v_layer = static_cast<uint16_t*>(g.v_cache) + static_cast<size_t>(l) * g.layer_elements;
    // pre-attention norm fused into q|k|v (layer 0: the embedding row itself, no delta)
    qkv.w = w.qkv;
    qkv.residual_in = residual[current];
    qkv.delta = l == 0 ? nullptr : delta_mlp;
    qkv.residual_out = l == 0 ? nullptr : residual[current ^ 1];
    if (l > 0) current ^= 1;
    qkv.gamma = w.input_norm;
    // the prefill's bias placement: fp16 adds its fp16 copy before rounding (GEMM epilogue),
    // bf16 adds the fp32 bias after rounding (RoPE kernel)
    const bool half_bias = dtype == kActFp16 && w.qkv_bias_half != nullptr;
    qkv.bias_half = half_bias ? w.qkv_bias_half : nullptr;
    qkv.bias = half_bias ? nullptr : w.qkv_bias;
    qkv.k_cache = k_layer;
    qkv.v_cache = v_layer;
    check_cuda(launch_decode_gemv(qkv, pdl, stream_), "decode q|k|v");
    attention.k_cache = k_layer;
    attention.v_cache = v_layer;
    check_cuda(launch_decode_attention(attention, pdl, stream_), "decode attention");
    out_proj.w = w.out;
    check_cuda(launch_decode_gemv(out_proj, pdl, stream_), "decode o_proj");
    // post-attention norm fused into gate|up
    gate_up.w = w.gate_up;
    gate_up.residual_in = residual[current];
    gate_up.residual_out = residual[current ^ 1];
    current ^= 1;
    gate_up.gamma = w.post_norm;
    check_cuda(launch_decode_gemv(gate_up, pdl, stream_), "decode gate|up");
    down.w = w.down;
    check_cuda(launch_decode_gemv(down, pdl, stream_), "decode down_proj");
  }
  // final norm fused into lm_head; greedy: the first maximum becomes the next step's token
  DecodeGemvArgs head;
  head.kind = kDecodeLogits;
  head.w = output_head();
  head.rows = c.vocab_size;
  head.k = H;
  head.residual_in = residual[current];
  head.delta = delta_mlp;
  head.gamma = final_norm_;
  head.eps = c.rms_norm_eps;
  head.y = g.logits;
  head.state = g.state;
  head.pick = greedy;
  head.pick_values = g.pick_values;
  head.pick_indices = g.pick_indices;
  head.ticket = g.tickets;
  head.dtype = dtype;
  check_cuda(launch_decode_gemv(head, pdl, stream_), "decode lm_head");
}

void Engine::run_decode_step(bool greedy) {
  GenerationState& g = *generation_;
  const int kind = greedy ? 1 : 0;
  if (!g.warmed[kind]) {
    // the first step runs eagerly: launch errors surface here, and kernel attributes are set
    // before anything is captured
    launch_decode_step(greedy);
    g.warmed[kind] = true;
  } else {
    if (g.graphs[kind] == nullptr) {
      // a cooperative launch or programmatic edges in a captured graph need driver support:
      // without it the capture is repeated with per-phase kernels, then with ordinary launches
      for (int attempt = 0; attempt < 3 && g.graphs[kind] == nullptr; ++attempt) {
        cudaGraph_t graph = nullptr;
        check_cuda(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeRelaxed), "decode capture");
        try {
          launch_decode_step(greedy);
        } catch (...) {
          cudaStreamEndCapture(stream_, &graph);
          if (graph != nullptr) cudaGraphDestroy(graph);
          throw;
        }
        cudaError_t status = cudaStreamEndCapture(stream_, &graph);
        if (status == cudaSuccess) status = cudaGraphInstantiate(&g.graphs[kind], graph, 0);
        if (graph != nullptr) cudaGraphDestroy(graph);
        if (status != cudaSuccess) {
          cudaGetLastError();
          g.graphs[kind] = nullptr;
          if (attempt == 2 || (!g.persistent && !g.programmatic)) check_cuda(status, "decode graph");
          if (g.persistent) {
            g.persistent = false;
          } else {
            g.programmatic = false;
          }
        }
      }
    }
    check_cuda(cudaGraphLaunch(g.graphs[kind], stream_), "decode graph launch");
  }
  g.position += 1;
}

void Engine::begin_generation(const int32_t* prompt, int count) {
  if (prompt == nullptr || count <= 0) throw Error("generation requires a non-empty prompt");
  if (count >= options_.max_sequence_length) {
    throw Error("prompt of " + std::to_string(count) + " tokens exceeds the " +
                std::to_string(options_.max_sequence_length) + " token window");
  }
  if (count > capacity_tokens_) {
    throw Error("prompt of " + std::to_string(count) + " tokens exceeds max_batch_tokens (" +
                std::to_string(capacity_tokens_) + ")");
  }
  std::string missing;
  if (!weights_complete(&missing)) throw Error("missing tensor: " + missing);
  output_head();  // the head must exist before any work is queued
  ensure_generation();
  GenerationState& g = *generation_;
  synchronize();  // the staging area may still feed an earlier copy
  int32_t* meta = g.staging + kStagingMeta;
  std::copy(prompt, prompt + count, meta);
  meta[count] = 0;
  meta[count + 1] = count;
  const int tiles = (count + kAttentionQueryTile - 1) / kAttentionQueryTile;
  for (int t = 0; t < tiles; ++t) {  // heaviest (last) query tile first
    meta[count + 2 + 2 * t] = 0;
    meta[count + 3 + 2 * t] = tiles - 1 - t;
  }
  g.staging[kStateUpload] = 0;
  g.staging[kStateUpload + 1] = count - 1;  // the last prompt token's position
  check_cuda(cudaMemsetAsync(g.tickets, 0, (2 + config_.num_key_value_heads) * sizeof(unsigned), stream_),
             "ticket reset");
  check_cuda(cudaMemcpyAsync(g.meta, meta, static_cast<size_t>(count + 2 + 2 * tiles) * 4, cudaMemcpyHostToDevice,
                             stream_),
             "prompt upload");
  check_cuda(cudaMemcpyAsync(g.state, g.staging + kStateUpload, 2 * sizeof(int32_t), cudaMemcpyHostToDevice, stream_),
             "state upload");
  g.position = -1;
  prefill_generation(count);
  const int status = read_status();  // synchronises
  if (status != 0) {
    reset_status();
    raise_on_status(status);
  }
  g.position = count;
}

void Engine::decode_token(int32_t token) {
  if (!generation_ || generation_->position < 0) throw Error("decode_token needs a prompt (begin_generation)");
  GenerationState& g = *generation_;
  if (token < 0 || token >= config_.vocab_size) throw Error("token id " + std::to_string(token) + " is out of range");
  if (g.position >= g.context) throw Error("the context window is full");
  synchronize();  // the upload slot may still feed the previous step
  g.staging[kStateUpload] = token;
  g.staging[kStateUpload + 1] = g.position;
  check_cuda(cudaMemcpyAsync(g.state, g.staging + kStateUpload, 2 * sizeof(int32_t), cudaMemcpyHostToDevice, stream_),
             "state upload");
  run_decode_step(false);
}

void Engine::read_logits(float* host) {
  if (!generation_ || generation_->position < 0) throw Error("no logits: generation has not started");
  check_cuda(cudaMemcpyAsync(host, generation_->logits, static_cast<size_t>(config_.vocab_size) * 4,
                             cudaMemcpyDeviceToHost, stream_),
             "logits download");
  const int status = read_status();  // synchronises
  if (status != 0) {
    reset_status();
    raise_on_status(status);
  }
}

std::vector<int32_t> Engine::generate(const int32_t* prompt, int count, int max_new_tokens, int eos_token_id,
                                      const SamplerConfig& sampler_config) {
  std::unique_ptr<TokenSampler> sampler = make_token_sampler(sampler_config);  // validates the config
  begin_generation(prompt, count);
  GenerationState& g = *generation_;
  std::vector<int32_t> out;
  const int limit = std::min(max_new_tokens, g.context - count);
  if (limit <= 0) return out;
  const int V = config_.vocab_size;

  if (sampler->greedy()) {
    int32_t* slots = g.staging + kStateSlots;
    // step j feeds token j (position count + j) and leaves token j + 1 in g.state; its copy of the
    // state lands in slot j % 2
    auto enqueue_copy = [&](int j) {
      check_cuda(cudaMemcpyAsync(slots + 2 * (j % 2), g.state, 2 * sizeof(int32_t), cudaMemcpyDeviceToHost, stream_),
                 "token download");
      check_cuda(cudaEventRecord(g.slot_ready[j % 2], stream_), "cudaEventRecord");
    };
    auto wait_token = [&](int j) {
      check_cuda(cudaEventSynchronize(g.slot_ready[j % 2]), "cudaEventSynchronize");
      return slots[2 * (j % 2)];
    };
    check_cuda(launch_argmax_token(g.logits, V, g.state, stream_), "greedy pick");
    enqueue_copy(1);  // token 0 into slot 1
    if (limit > 1) {
      run_decode_step(true);  // step 0 -> token 1
      enqueue_copy(0);
    }
    int32_t token = wait_token(1);
    for (int s = 0;; ++s) {
      // token s is known here; step s (producing token s + 1) is queued when s + 1 < limit
      if (token == eos_token_id) break;
      out.push_back(token);
      if (s + 1 >= limit) break;
      if (s + 2 < limit) {  // keep one step ahead of the host
        run_decode_step(true);  // step s + 1 -> token s + 2
        enqueue_copy(s + 1);
      }
      token = wait_token(s);
    }
    synchronize();  // a step queued past eos finishes before the buffers are reused
  } else {
    if (g.logits_host == nullptr) {
      check_cuda(cudaHostAlloc(reinterpret_cast<void**>(&g.logits_host), static_cast<size_t>(V) * 4,
                               cudaHostAllocDefault),
                 "cudaHostAlloc");
    }
    read_logits(g.logits_host);
    for (int s = 0; s < limit; ++s) {
      const int32_t token = sampler->select(g.logits_host, V);
      if (token == eos_token_id) break;
      out.push_back(token);
      if (s + 1 >= limit) break;
      decode_token(token);
      read_logits(g.logits_host);
    }
  }
  const int status = read_status();
  if (status != 0) {
    reset_status();
    raise_on_status(status);
  }
  g.position = -1;  // the cache may hold a step past eos: a new prompt starts over
  return out;
}

}  // namespace arb
