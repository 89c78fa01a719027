// One kernel-level attention-mass call (ar_document_attention_mass and its allocation-free
// variant): argument checks, the int32 metadata blob, the scratch carve-up and the launches.
// The two entry points differ only in where their device scratch comes from.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

#include <cuda_runtime.h>

namespace arb {

// A checked batch: metadata = offsets | query spans | spans | item offsets (int32).
struct MassBatch {
  std::vector<int32_t> meta;
  size_t queries_at = 0;
  size_t spans_at = 0;
  size_t items_at = 0;
  int prompt_count = 0;
  int span_count = 0;
  int item_count = 0;
};

struct MassCallArgs {
  const void* qkv = nullptr;
  int qkv_rows = 0;
  const float* lse = nullptr;
  const int32_t* prompt_offsets = nullptr;  // host, prompt_count + 1
  int prompt_count = 0;
  const int32_t* query_spans = nullptr;     // host, 2 per prompt
  const int32_t* spans = nullptr;           // host, 2 * span_count per prompt
  int span_count = 0;
  int query_heads = 0;
  int kv_heads = 0;
  int head_dim = 0;
  int sliding_window = 0;
  int prefill_chunk_tokens = 0;
  int normalize_by_length = 0;
  double* mass_out = nullptr;               // host, prompt_count * span_count
  int dtype = 0;
};

// Device scratch of one call, carved from one block of `bytes()` bytes.
struct MassScratchLayout {
  size_t status_at = 0;
  size_t meta_at = 0;
  size_t partials_at = 0;
  size_t rows_at = 0;
  size_t total = 0;
};

// Every argument check, on the host, before any CUDA call; throws arb::Error naming `who`.
// Offsets must start at 0 or later, never decrease and end at or before qkv_rows; query spans
// must not be reversed or start before 0; document spans must not start before 0 or be reversed.
MassBatch plan_mass_batch(const char* who, const MassCallArgs& call);

MassScratchLayout mass_scratch_layout(const MassBatch& batch);

// Status reset, metadata upload, mass and finalize kernels, download of the rows and status,
// stream synchronisation; throws on a CUDA failure or a device-reported status. `scratch` holds
// at least layout.total bytes, 256-byte aligned.
void run_mass_batch(const char* who, const MassCallArgs& call, const MassBatch& batch, const MassScratchLayout& layout,
                    void* scratch, cudaStream_t stream);

}  // namespace arb
