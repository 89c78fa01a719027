// Single-token decode kernels: the answering step of CudaLlamaModel::generate
// (attnrank/src/model.cu:532-565) on the B200 engine.
//
// One token runs through every layer per step, so each projection is a matrix-vector product
// that streams its 16-bit weight matrix from HBM exactly once. The reference runs these steps
// through cuBLAS at m = 1 plus its elementwise kernels (model.cu:324-350); here each projection
// is one bandwidth-bound kernel that also does the elementwise work around it:
//   q|k|v   RMSNorm(residual + delta) prologue; bias + RoPE + KV-cache append epilogue
//           (model.cu:367-392, scatter_kv_cache :426-440)
//   o_proj  plain, 16-bit out
//   gate|up RMSNorm(residual + delta) prologue; SiLU * up epilogue (model.cu:398-415)
//   down    plain, 16-bit out
//   lm_head final RMSNorm prologue; fp32 logits (model.cu:341-350), optionally the greedy pick
// Attention of the one query row over the cache is split over key ranges; the last CTA of each
// KV head merges the splits (one CTA per (split, KV head) serves every query head of the group).
// Every launch reads the step's token and position from device memory (`state` = {token,
// position}), so a captured CUDA graph of the whole step replays without host arguments, and
// every kernel waits for its producer with griddepcontrol.wait after issuing the loads that do
// not depend on it (programmatic dependent launch).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace arb {

// Key-range splits of the decode attention per KV head.
constexpr int kDecodeSplits = 32;
// Largest GQA group (query heads per KV head) the decode attention handles.
constexpr int kDecodeMaxGroup = 16;
// Largest hidden size of the fused RMSNorm prologue (256 threads x 4 x 8 values).
constexpr int kDecodeMaxNormHidden = 8192;
// Per-CTA slots of the greedy pick (>= the largest logits grid).
constexpr int kDecodePickSlots = 8192;

enum DecodeGemvKind : int {
  kDecodePlain = 0,   // y[n] = w[n] . x, 16-bit
  kDecodeLogits = 1,  // y[n] = w[n] . x, fp32
  kDecodeGateUp = 2,  // y[j] = silu(w[j] . x) * (w[inter + j] . x), 16-bit; rows = inter
  kDecodeQkv = 3,     // q|k|v with bias, RoPE and the cache append; rows = (Hq + 2 Hkv) D
};

struct DecodeGemvArgs {
  int kind = kDecodePlain;
  const void* w = nullptr;  // 16-bit [rows (2 x inter for gate|up), k] row-major
  int rows = 0;
  int k = 0;                // % 8 == 0
  // input: x (16-bit [k]), or -- when residual_in is set -- x = 16-bit(v * rsqrt(mean(v^2) + eps)
  // * gamma) with v = residual_in + delta (delta nullable), the engine's RMSNorm with residual;
  // CTA 0 then stores v into residual_out (nullable; must not alias residual_in)
  const void* x = nullptr;
  const float* residual_in = nullptr;
  // or v = the embedding row of token state[0] (16-bit [vocab, k]); residual_in then unused
  const void* embed_table = nullptr;
  int vocab = 0;
  const void* delta = nullptr;
  const float* gamma = nullptr;
  float eps = 0.0f;
  float* residual_out = nullptr;
  void* y = nullptr;  // plain / logits / gate|up output
  // kDecodeQkv
  const void* bias_half = nullptr;  // 16-bit bias added before rounding (the fp16 GEMM epilogue), or null
  const float* bias = nullptr;      // fp32 bias added after rounding (the bf16 path), or null
  int query_heads = 0;
  int kv_heads = 0;
  int head_dim = 0;
  const float* cos_table = nullptr;  // [table_positions, D / 2]
  const float* sin_table = nullptr;
  int table_positions = 0;
  void* q_out = nullptr;    // 16-bit [Hq D], rotated
  void* k_cache = nullptr;  // this layer's 16-bit [Hkv, context, D]; row `position` is written
  void* v_cache = nullptr;
  int context = 0;
  int* status = nullptr;
  // state = {token, position}: read by kDecodeQkv; with `pick` (kDecodeLogits), the first maximum
  // of the logits (GreedySampler::select, model.cpp:70-73) is written as {index, position + 1}
  int32_t* state = nullptr;
  bool pick = false;
  float* pick_values = nullptr;   // [kDecodePickSlots] scratch
  int32_t* pick_indices = nullptr;
  unsigned* ticket = nullptr;     // zero between launches
  int dtype = 1;
};
// `programmatic`: launched with programmatic stream serialization (it may start before its
// predecessor on the stream ends; it waits for it before reading its outputs).
cudaError_t launch_decode_gemv(const DecodeGemvArgs& args, bool programmatic, cudaStream_t stream);

struct DecodeAttentionArgs {
  const void* q = nullptr;          // 16-bit [Hq D]
  const void* k_cache = nullptr;    // this layer's 16-bit [Hkv, context, D]
  const void* v_cache = nullptr;
  int context = 0;
  const int32_t* state = nullptr;   // keys 0 .. state[1] are visible
  int query_heads = 0;
  int kv_heads = 0;
  int head_dim = 0;                 // 128
  int sliding_window = 0;
  float* partials = nullptr;        // fp32 [Hq, kDecodeSplits, D]
  float* stats = nullptr;           // fp32 [Hq, kDecodeSplits, 2] (running max in log2 units, sum)
  unsigned* tickets = nullptr;      // [Hkv], zero between launches
  void* out = nullptr;              // 16-bit [Hq D]
  int dtype = 1;
};
cudaError_t launch_decode_attention(const DecodeAttentionArgs& args, bool programmatic, cudaStream_t stream);

// One decode step as ONE persistent kernel (a cooperative launch of as many CTAs as fit): the
// phases q|k|v, attention, o_proj, gate|up, down of every layer and the output head run in turn,
// separated by a grid-wide barrier, so the step pays no launch, ramp-up or drain between phases.
// Before arriving at a barrier every CTA sends its share of the next phase's weights towards L2,
// which keeps HBM busy across the phase boundary. The barrier's wait is bounded: on a timeout it
// reports kStatusWaitTimeout and every CTA returns. Layer 0's q|k|v prologue reads the embedding
// row of the step's token itself. The phase bodies are those of the per-phase kernels.
struct DecodeLayerWeights {
  const void* qkv = nullptr;
  const void* qkv_bias_half = nullptr;
  const float* qkv_bias = nullptr;
  const void* out = nullptr;
  const void* gate_up = nullptr;
  const void* down = nullptr;
  const float* input_norm = nullptr;
  const float* post_norm = nullptr;
  void* k_cache = nullptr;
  void* v_cache = nullptr;
};

struct DecodeStepArgs {
  const DecodeLayerWeights* layers = nullptr;  // device array [layer_count]
  int layer_count = 0;
  // phase templates; the kernel fills in each layer's weights, norms, caches and residual rows
  DecodeGemvArgs qkv;       // embed_table, vocab, state, RoPE tables, q_out, context, status set
  DecodeGemvArgs out_proj;  // x = attention output, y = delta of the attention block
  DecodeGemvArgs gate_up;   // delta = delta of the attention block, y = SwiGLU output
  DecodeGemvArgs down;      // x = SwiGLU output, y = delta of the MLP block
  DecodeGemvArgs head;      // delta = delta of the MLP block, gamma = final norm, y = logits, pick
  DecodeAttentionArgs attention;
  float* residual[2] = {nullptr, nullptr};  // two fp32 rows used in turn
  unsigned* barrier = nullptr;              // zero before every launch
  int* status = nullptr;
  int dtype = 1;
  int max_k = 0;                            // largest row length staged (shared memory: 2 max_k bytes)
};
// Cooperative launch of the step; cudaErrorCooperativeLaunchTooLarge (or another error) when the
// device cannot hold the grid, in which case the per-phase kernels are the way.
cudaError_t launch_decode_step(const DecodeStepArgs& args, cudaStream_t stream);

// The bounded grid barrier of the persistent decode step, made to run out on purpose: `ctas` CTAs
// (at most 1024) wait on a counter value nothing writes, for `spin_limit` polls (at most the
// production limit), then record kStatusWaitTimeout in *status and return. counter and status
// start at zero.
cudaError_t launch_bounded_wait_selftest(unsigned* counter, int* status, int ctas, unsigned spin_limit,
                                         cudaStream_t stream);

// K and V of a prefilled prompt (rows 0 .. tokens-1 of the q|k|v buffer, after RoPE) into the
// cache at positions 0 .. tokens-1.
cudaError_t launch_store_kv(const void* qkv, int tokens, int query_heads, int kv_heads, int head_dim, void* k_cache,
                            void* v_cache, int context, int dtype, cudaStream_t stream);

// Greedy selection over logits[0, count) alone (std::max_element order): state = {index, state[1] + 1}.
cudaError_t launch_argmax_token(const float* logits, int count, int32_t* state, cudaStream_t stream);

}  // namespace arb
