// Host side of one kernel-level attention-mass call, shared by ar_document_attention_mass (scratch
// from the stream-ordered allocator) and ar_document_attention_mass_noalloc (scratch from a fixed
// device array). The checks follow the reference's own argument errors for spans and lengths
// (attnrank/src/model.cu:638-647): every one runs on the host before any CUDA call.
#include "mass_call.h"

#include <string>

#include "engine.h"
#include "layer_kernels.h"
#include "mass_plan.h"

namespace arb {
namespace {

constexpr size_t kScratchAlign = 256;

size_t align_up(size_t value) { return (value + kScratchAlign - 1) / kScratchAlign * kScratchAlign; }

[[noreturn]] void reject(const char* who, const std::string& why) { throw Error(std::string(who) + ": " + why); }

}  // namespace

MassBatch plan_mass_batch(const char* who, const MassCallArgs& call) {
  if (call.prompt_count <= 0 || call.span_count <= 0 || call.span_count > kMassMaxSpans) {
    reject(who, "1..32 spans and at least one prompt are required");
  }
  if (call.head_dim != 128 || call.kv_heads <= 0 || call.query_heads <= 0 || call.query_heads % call.kv_heads != 0) {
    reject(who, "head_dim must be 128 and query_heads a multiple of kv_heads");
  }
  if (call.dtype != kActFp16 && call.dtype != kActBf16) reject(who, "dtype must be fp16 or bf16");
  if (call.prompt_offsets == nullptr || call.query_spans == nullptr || call.spans == nullptr ||
      call.mass_out == nullptr || call.qkv == nullptr || call.lse == nullptr) {
    reject(who, "null argument");
  }
  if (call.qkv_rows < 0) reject(who, "qkv_rows must not be negative");
  if (call.prompt_offsets[0] < 0) reject(who, "prompt offsets must start at 0 or later");
  for (int p = 0; p < call.prompt_count; ++p) {
    if (call.prompt_offsets[p + 1] < call.prompt_offsets[p]) reject(who, "prompt offsets must be non-decreasing");
  }
  if (call.prompt_offsets[call.prompt_count] > call.qkv_rows) reject(who, "prompts exceed qkv rows");

  const int group = call.query_heads / call.kv_heads;
  MassBatch batch;
  batch.prompt_count = call.prompt_count;
  batch.span_count = call.span_count;
  const size_t span_values = 2 * static_cast<size_t>(call.prompt_count) * call.span_count;
  batch.meta.reserve(call.prompt_count + 1 + 2 * static_cast<size_t>(call.prompt_count) + span_values +
                     call.prompt_count + 1);
  batch.meta.insert(batch.meta.end(), call.prompt_offsets, call.prompt_offsets + call.prompt_count + 1);
  batch.queries_at = batch.meta.size();
  batch.meta.insert(batch.meta.end(), call.query_spans, call.query_spans + 2 * call.prompt_count);
  batch.spans_at = batch.meta.size();
  batch.meta.insert(batch.meta.end(), call.spans, call.spans + span_values);
  batch.items_at = batch.meta.size();
  batch.meta.push_back(0);
  for (int p = 0; p < call.prompt_count; ++p) {
    const int length = call.prompt_offsets[p + 1] - call.prompt_offsets[p];
    const int32_t* query = call.query_spans + 2 * p;
    if (query[0] < 0 || query[1] < query[0]) reject(who, "invalid query span");
    const int32_t* spans = call.spans + 2 * static_cast<size_t>(p) * call.span_count;
    for (int s = 0; s < call.span_count; ++s) {
      if (spans[2 * s] < 0 || spans[2 * s + 1] < spans[2 * s]) reject(who, "invalid document span");
    }
    const MassItemShape shape = mass_item_shape(query, spans, call.span_count, length, group);
    const long long next = static_cast<long long>(batch.meta.back()) + mass_items_for_prompt(shape, call.kv_heads);
    if (next > (1LL << 30)) reject(who, "too many work items in one call; split the prompts");
    batch.meta.push_back(static_cast<int32_t>(next));
  }
  batch.item_count = batch.meta.back();
  return batch;
}

MassScratchLayout mass_scratch_layout(const MassBatch& batch) {
  MassScratchLayout layout;
  layout.status_at = 0;
  layout.meta_at = align_up(layout.status_at + sizeof(int));
  layout.partials_at = align_up(layout.meta_at + batch.meta.size() * sizeof(int32_t));
  layout.rows_at =
      align_up(layout.partials_at + static_cast<size_t>(batch.item_count) * batch.span_count * sizeof(float));
  layout.total = layout.rows_at + static_cast<size_t>(batch.prompt_count) * batch.span_count * sizeof(double);
  return layout;
}

void run_mass_batch(const char* who, const MassCallArgs& call, const MassBatch& batch, const MassScratchLayout& layout,
                    void* scratch, cudaStream_t stream) {
  auto* base = static_cast<unsigned char*>(scratch);
  auto* status = reinterpret_cast<int*>(base + layout.status_at);
  auto* meta_device = reinterpret_cast<int32_t*>(base + layout.meta_at);
  auto* partials = reinterpret_cast<float*>(base + layout.partials_at);
  auto* rows = reinterpret_cast<double*>(base + layout.rows_at);

  // scratch may hold an earlier call's contents: the status word starts at zero; partials and
  // rows are rewritten in full by the kernels
  check_cuda(cudaMemsetAsync(status, 0, sizeof(int), stream), "status reset");
  check_cuda(cudaMemcpyAsync(meta_device, batch.meta.data(), batch.meta.size() * sizeof(int32_t),
                             cudaMemcpyHostToDevice, stream),
             "metadata upload");
  MassArgs args;
  args.qkv = call.qkv;
  args.dtype = call.dtype;
  args.qkv_rows_capacity = call.qkv_rows;
  args.lse = call.lse;
  args.prompt_offsets = meta_device;
  args.query_spans = meta_device + batch.queries_at;
  args.spans = meta_device + batch.spans_at;
  args.item_offsets = meta_device + batch.items_at;
  args.prompt_count = batch.prompt_count;
  args.span_count = batch.span_count;
  args.item_count = batch.item_count;
  args.query_heads = call.query_heads;
  args.kv_heads = call.kv_heads;
  args.head_dim = call.head_dim;
  args.sliding_window = call.sliding_window;
  args.reference_chunk = call.prefill_chunk_tokens;
  args.normalize_by_length = call.normalize_by_length;
  args.partials = partials;
  args.status = status;
  check_cuda(launch_document_mass(args, stream), who);
  FinalizeArgs finalize;
  finalize.partials = partials;
  finalize.item_offsets = args.item_offsets;
  finalize.query_spans = args.query_spans;
  finalize.prompt_offsets = meta_device;
  finalize.prompt_count = batch.prompt_count;
  finalize.span_count = batch.span_count;
  finalize.item_count = batch.item_count;
  finalize.layers = 1;
  finalize.query_heads = call.query_heads;
  finalize.raw_rows = rows;
  check_cuda(launch_finalize_mass(finalize, stream), "finalize");
  int status_host = 0;
  check_cuda(cudaMemcpyAsync(call.mass_out, rows,
                             static_cast<size_t>(batch.prompt_count) * batch.span_count * sizeof(double),
                             cudaMemcpyDeviceToHost, stream),
             "mass download");
  check_cuda(cudaMemcpyAsync(&status_host, status, sizeof(int), cudaMemcpyDeviceToHost, stream), "status download");
  check_cuda(cudaStreamSynchronize(stream), who);
  if (status_host != 0) {
    throw Error(std::string("device reported an error in ") + who + " (code " + std::to_string(status_host) + ")");
  }
}

}  // namespace arb
