// Host-side launchers of the fused per-layer kernels (layer_kernels.cu, attention.cu, mass.cu,
// synthetic.cu). All pointers are device pointers; all launches are asynchronous on `stream`.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"

namespace arb {

int sm_count();

cudaError_t launch_embed_rms_norm(const int32_t* token_ids, int tokens, const void* table, int vocab,
                                  int hidden, const float* gamma, float eps, float* residual,
                                  void* normed, int* status, int dtype, cudaStream_t stream);

// residual += delta; normed = 16-bit(rms(residual) * gamma). With delta == nullptr the residual
// is only read (it already holds the sum) and is not written.
cudaError_t launch_rms_norm_residual(float* residual, const void* delta, const float* gamma, int tokens,
                                     int hidden, float eps, void* normed, int dtype, cudaStream_t stream);

cudaError_t launch_rotary_bias(void* qkv, const float* bias, const int32_t* positions, int tokens,
                               int query_heads, int kv_heads, int head_dim, const float* cos_table,
                               const float* sin_table, int table_positions, int* status, int dtype,
                               cudaStream_t stream);

cudaError_t launch_rope_table(float* cos_out, float* sin_out, int positions, int head_dim, float theta,
                              cudaStream_t stream);

cudaError_t launch_silu_multiply(const void* gate, const void* up, long long in_stride, void* out,
                                 long long out_stride, int tokens, int width, int dtype, cudaStream_t stream);

cudaError_t launch_positions(const int32_t* prompt_offsets, int prompt_count, int tokens,
                             int32_t* positions, cudaStream_t stream);

// Causal prefill attention over packed prompts: attention_tc.cu (tcgen05, the engine's kernel)
// and attention.cu (mma.sync, kept as the alternative).
struct AttentionArgs {
  const void* qkv = nullptr;        // 16-bit [tokens, (Hq + 2 Hkv) * D], Q | K | V column blocks
  void* out = nullptr;              // 16-bit [tokens, Hq * D]
  float* lse = nullptr;             // fp32 [tokens, Hq], log2-domain log-sum-exp of scaled scores
  const int32_t* prompt_offsets = nullptr;  // [prompts + 1]
  const int32_t* tiles = nullptr;   // [tile_count * 2] (prompt, query tile) pairs, heaviest first
  int tile_count = 0;
  int query_heads = 0;
  int kv_heads = 0;
  int head_dim = 0;
  int sliding_window = 0;           // 0 = unlimited
  int dtype = kActFp16;             // ActivationType of qkv and out
  int rows = 0;                     // rows of qkv (tensor-map extent; tcgen05 kernel)
  int* status = nullptr;            // device status word (tcgen05 kernel: wait timeouts)
  // Fused attention mass (tcgen05 kernel only; mass_partials == nullptr: none). Partial slot of
  // (prompt p, query head h, query tile t): mass_items[p] + h * tiles_p + (t - first_p), where
  // first_p.. are the query tiles that hold rows of p's query span (fused_mass_tiles).
  const int32_t* query_spans = nullptr;   // [prompts * 2], prompt-relative
  const int32_t* spans = nullptr;         // [prompts * span_count * 2], prompt-relative
  const int32_t* mass_items = nullptr;    // [prompts + 1]
  float* mass_partials = nullptr;         // [items * span_count], each the sum over the tile's rows
  int span_count = 0;
  int normalize_by_length = 0;
  int reference_chunk = 0;
};

cudaError_t launch_causal_attention(const AttentionArgs& args, cudaStream_t stream);
cudaError_t launch_causal_attention_tc(const AttentionArgs& args, cudaStream_t stream);
constexpr int kAttentionQueryTile = 128;
// Fused mass partial slots per (query head, query tile): one, the fixed-order sum over the tile's
// rows, summed in a fixed order by the finalize kernel.
constexpr int kFusedMassSlotsPerTile = 1;

// Query tiles (kAttentionQueryTile rows) that hold rows of a prompt's query span: the fused mass
// writes one partial per (query head, such tile).
inline int fused_mass_tiles(const int32_t* query_span, int length) {
  const int begin = query_span[0] < 0 ? 0 : query_span[0];
  const int end = query_span[1] > length ? length : query_span[1];
  if (end <= begin) return 0;
  return (end - 1) / kAttentionQueryTile - begin / kAttentionQueryTile + 1;
}

// Query->document attention mass (mass.cu).
struct MassArgs {
  const void* qkv = nullptr;        // same packed projection buffer as AttentionArgs::qkv
  int qkv_rows_capacity = 0;        // rows addressable through the TMA descriptors
  const float* lse = nullptr;       // fp32 [tokens, Hq] from the attention kernel
  const int32_t* prompt_offsets = nullptr;  // [prompts + 1]
  const int32_t* query_spans = nullptr;     // [prompts * 2], prompt-relative [begin, end)
  const int32_t* spans = nullptr;           // [prompts * span_count * 2], prompt-relative
  const int32_t* item_offsets = nullptr;    // [prompts + 1] work items per prompt (prefix sums)
  int prompt_count = 0;
  int span_count = 0;
  int item_count = 0;
  int query_heads = 0;
  int kv_heads = 0;
  int head_dim = 0;
  int sliding_window = 0;
  int reference_chunk = 0;          // chunk length that bounds normalize_by_length divisors
  int normalize_by_length = 0;
  float* partials = nullptr;        // fp32 [item_count, span_count]
  int* status = nullptr;
  int dtype = kActFp16;             // ActivationType of qkv
};
cudaError_t launch_document_mass(const MassArgs& args, cudaStream_t stream);
constexpr int kMassRowTile = 128;   // GQA-stacked query rows per CTA
constexpr int kMassKeyTile = 128;   // keys per tcgen05.mma N tile
constexpr int kMassKeyTilesPerItem = 4;  // key tiles walked by one CTA
constexpr int kMassMaxSpans = 32;

// Work decomposition shared by the host planner, the mass kernel and the finalizer.
struct MassItemShape {
  int row_tiles;   // ceil(group * padded_query_rows / kMassRowTile)
  int key_splits;  // ceil(key_tiles / kMassKeyTilesPerItem)
  int key_begin;   // first key (multiple of kMassKeyTile) touched by any span
  int key_tiles;   // 128-key tiles in [key_begin, key_end)
};

// Deterministic per-prompt normalisation + cross-prompt accumulation (mass.cu).
struct FinalizeArgs {
  const float* partials = nullptr;  // [layers][item_count][span_count]
  const int32_t* item_offsets = nullptr;
  const int32_t* query_spans = nullptr;
  const int32_t* prompt_offsets = nullptr;
  int prompt_count = 0;
  int span_count = 0;
  int item_count = 0;
  int layers = 0;
  int query_heads = 0;
  double* rows = nullptr;           // optional [prompts][layers][span_count], unit-sum rows
  double* raw_rows = nullptr;       // optional [prompts][layers][span_count], mass / observations
  float* accumulator = nullptr;     // optional [layers][span_count], += sum over prompts of rows
};
cudaError_t launch_finalize_mass(const FinalizeArgs& args, cudaStream_t stream);

// Seeded synthetic weights (synthetic.cu): the bf16 value of every element, stored as bf16 or
// converted (exactly representable or round-to-nearest-even) to fp16.
cudaError_t launch_synthetic_fill(void* dst, long long count, uint64_t key, float scale, int dtype,
                                  cudaStream_t stream);
// In-place-free conversions used when uploading host weights.
cudaError_t launch_bf16_to_fp16(const void* src, void* dst, long long count, cudaStream_t stream);
cudaError_t launch_f32_to_activation(const float* src, void* dst, long long count, int dtype, cudaStream_t stream);
cudaError_t launch_synthetic_fill_f32(float* dst, long long count, uint64_t key, float scale,
                                      float offset, cudaStream_t stream);

}  // namespace arb
