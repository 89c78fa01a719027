// Single-token decode kernels: the answering step of CudaLlamaModel::generate
// (attnrank/src/model.cu:532-565) on the B200 engine.
//
// One token runs through every layer per step, so each projection is a matrix-vector product
// that streams its 16-bit weight matrix from HBM exactly once. The reference runs these steps
// through cuBLAS at m = 1 plus its elementwise kernels (model.cu:324-350); here each projection
// is one bandwidth-bound kernel with its elementwise successor fused into the epilogue:
//   q|k|v   + bias + RoPE + KV-cache append  (model.cu:367-392, scatter_kv_cache :426-440)
//   gate|up + SiLU * up                      (model.cu:410-415)
//   o_proj, down_proj                        plain, 16-bit out (the engine's RMSNorm kernel follows)
//   lm_head                                  fp32 logits (model.cu:341-350)
// Attention of the one query row over the cache is split over key ranges and combined (one CTA
// per (split, KV head) serves every query head of the GQA group from one load of K and V).
// Every launch reads the step's token and position from device memory (`state` = {token,
// position}), so a captured CUDA graph of the whole step replays without host arguments.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace arb {

// Key-range splits of the decode attention per KV head (the combine step merges them).
constexpr int kDecodeSplits = 32;
// Largest GQA group (query heads per KV head) the decode attention handles.
constexpr int kDecodeMaxGroup = 16;

// y[n] = w[n, :] . x for n < rows; w 16-bit [rows, k] row-major, x 16-bit [k], k % 8 == 0.
// y is 16-bit (rounded once) or fp32 when f32_out.
cudaError_t launch_decode_gemv(const void* w, const void* x, int rows, int k, void* y, bool f32_out, int dtype,
                               cudaStream_t stream);

// act[j] = silu(g_j) * u_j, g_j = w[j] . x, u_j = w[inter + j] . x (the fused gate|up matrix
// [2 inter, k]); g and u are rounded to 16 bits first, as the prefill's GEMM output is.
cudaError_t launch_decode_gate_up(const void* w, const void* x, int inter, int k, void* act, int dtype,
                                  cudaStream_t stream);

struct DecodeQkvArgs {
  const void* w = nullptr;          // 16-bit [(Hq + 2 Hkv) D, hidden]
  const void* x = nullptr;          // 16-bit [hidden]
  int hidden = 0;
  const void* bias_half = nullptr;  // 16-bit bias added before rounding (the fp16 GEMM epilogue), or null
  const float* bias = nullptr;      // fp32 bias added after rounding (the bf16 path), or null
  int query_heads = 0;
  int kv_heads = 0;
  int head_dim = 0;
  const float* cos_table = nullptr;  // [table_positions, D / 2]
  const float* sin_table = nullptr;
  int table_positions = 0;
  const int32_t* state = nullptr;   // {token, position}
  void* q_out = nullptr;            // 16-bit [Hq D], rotated
  void* k_cache = nullptr;          // this layer's 16-bit [Hkv, context, D]; row `position` is written
  void* v_cache = nullptr;
  int context = 0;
  int* status = nullptr;
  int dtype = 1;
};
cudaError_t launch_decode_qkv(const DecodeQkvArgs& args, cudaStream_t stream);

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
  void* out = nullptr;              // 16-bit [Hq D]
  int dtype = 1;
};
// Split attention followed by the combine step (two launches).
cudaError_t launch_decode_attention(const DecodeAttentionArgs& args, cudaStream_t stream);

// K and V of a prefilled prompt (rows 0 .. tokens-1 of the q|k|v buffer, after RoPE) into the
// cache at positions 0 .. tokens-1.
cudaError_t launch_store_kv(const void* qkv, int tokens, int query_heads, int kv_heads, int head_dim, void* k_cache,
                            void* v_cache, int context, int dtype, cudaStream_t stream);

// Greedy selection: the index of the first maximum of logits[0, count) (std::max_element
// order, as GreedySampler::select, model.cpp:70-73). Writes state = {index, state[1] + 1}.
cudaError_t launch_argmax_token(const float* logits, int count, int32_t* state, cudaStream_t stream);

}  // namespace arb
