// Allocation-free variant of ar_document_attention_mass.
//
// Some callers cannot let a library allocate device memory while they run: an application that
// has reserved the whole GPU under a fixed memory budget, a serving loop on a latency-critical
// path where an allocator call may block or synchronise, or a host framework that owns every
// device allocation of its process. This entry point does the same work as
// ar_document_attention_mass but takes its scratch (batch metadata, per-CTA partial sums, the
// finished rows and the status word) from one fixed array that the library reserves when it is
// loaded. It calls no cudaMalloc, cudaFree or other allocating routine.
//
// The array is a file-scope __device__ object: every GPU that loads the library holds
// kNoAllocScratchBytes of it until the process exits, and every call shares it. In host code
// its name is only a host-side handle, so its device address is taken with
// cudaGetSymbolAddress, once per device, on the first call made on that device with that device
// current. Make that first call before any stream capture. Calls whose work overlaps on the GPU
// race on the shared array: issue them on one stream, or wait between them.
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/attnrank_b200.h"
#include "engine.h"
#include "layer_kernels.h"
#include "mass_plan.h"

namespace arb {
namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;  // 8 MiB per device
constexpr size_t kAlign = 256;

static __device__ __align__(256) unsigned char g_mass_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_address[kMaxDevices] = {};

size_t align_up(size_t value) { return (value + kAlign - 1) / kAlign * kAlign; }

// Device address of this device's scratch array (the device must be current).
void* scratch_for_current_device() {
  int device = 0;
  check_cuda(cudaGetDevice(&device), "cudaGetDevice");
  if (device < 0 || device >= kMaxDevices) throw Error("document_attention_mass_noalloc: device index out of range");
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_address[device] == nullptr) {
    void* address = nullptr;
    check_cuda(cudaGetSymbolAddress(&address, g_mass_scratch), "cudaGetSymbolAddress(scratch)");
    g_scratch_address[device] = address;
  }
  return g_scratch_address[device];
}

}  // namespace

void set_last_error(const std::string& message);  // capi.cu: the message ar_last_error() returns

}  // namespace arb

extern "C" int ar_document_attention_mass_noalloc(const void* qkv, int qkv_rows, const float* lse,
                                                  const int32_t* prompt_offsets_host, int prompt_count,
                                                  const int32_t* query_spans_host, const int32_t* spans_host,
                                                  int span_count, int query_heads, int kv_heads, int head_dim,
                                                  int sliding_window, int prefill_chunk_tokens,
                                                  int normalize_by_length, double* mass_out, int dtype,
                                                  void* stream) {
  using namespace arb;
  try {
    if (prompt_count <= 0 || span_count <= 0 || span_count > kMassMaxSpans) {
      throw Error("document_attention_mass_noalloc: 1..32 spans and at least one prompt are required");
    }
    if (head_dim != 128 || kv_heads <= 0 || query_heads % kv_heads != 0) {
      throw Error("document_attention_mass_noalloc: head_dim must be 128 and query_heads a multiple of kv_heads");
    }
    if (prompt_offsets_host[prompt_count] > qkv_rows) {
      throw Error("document_attention_mass_noalloc: prompts exceed qkv rows");
    }
    const int group = query_heads / kv_heads;
    std::vector<int32_t> meta;
    meta.insert(meta.end(), prompt_offsets_host, prompt_offsets_host + prompt_count + 1);
    const size_t queries_at = meta.size();
    meta.insert(meta.end(), query_spans_host, query_spans_host + 2 * prompt_count);
    const size_t spans_at = meta.size();
    meta.insert(meta.end(), spans_host, spans_host + 2 * static_cast<size_t>(prompt_count) * span_count);
    const size_t items_at = meta.size();
    meta.push_back(0);
    for (int p = 0; p < prompt_count; ++p) {
      const int length = prompt_offsets_host[p + 1] - prompt_offsets_host[p];
      if (length < 0 || query_spans_host[2 * p] < 0 || query_spans_host[2 * p + 1] < query_spans_host[2 * p]) {
        throw Error("document_attention_mass_noalloc: invalid prompt offsets or query span");
      }
      for (int s = 0; s < span_count; ++s) {
        const int32_t* span = spans_host + 2 * (static_cast<size_t>(p) * span_count + s);
        if (span[0] < 0 || span[1] < span[0]) throw Error("document_attention_mass_noalloc: invalid document span");
      }
      const MassItemShape shape = mass_item_shape(query_spans_host + 2 * p,
                                                  spans_host + 2 * static_cast<size_t>(p) * span_count, span_count,
                                                  length, group);
      meta.push_back(meta.back() + mass_items_for_prompt(shape, kv_heads));
    }
    const int item_count = meta.back();

    // carve the fixed array: status | metadata | partials | rows
    const size_t status_at = 0;
    const size_t meta_at = align_up(status_at + sizeof(int));
    const size_t partials_at = align_up(meta_at + meta.size() * sizeof(int32_t));
    const size_t rows_at = align_up(partials_at + static_cast<size_t>(item_count) * span_count * sizeof(float));
    const size_t needed = rows_at + static_cast<size_t>(prompt_count) * span_count * sizeof(double);
    if (needed > kNoAllocScratchBytes) {
      throw Error("document_attention_mass_noalloc: this batch needs " + std::to_string(needed) +
                  " bytes of scratch but the fixed array holds " + std::to_string(kNoAllocScratchBytes) +
                  "; split the prompts over several calls or use ar_document_attention_mass");
    }
    auto* base = static_cast<unsigned char*>(scratch_for_current_device());
    auto* status = reinterpret_cast<int*>(base + status_at);
    auto* meta_device = reinterpret_cast<int32_t*>(base + meta_at);
    auto* partials = reinterpret_cast<float*>(base + partials_at);
    auto* rows = reinterpret_cast<double*>(base + rows_at);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);

    // the status word keeps the previous call's value: clear it; partials and rows are fully rewritten
    check_cuda(cudaMemsetAsync(status, 0, sizeof(int), s), "status reset");
    check_cuda(cudaMemcpyAsync(meta_device, meta.data(), meta.size() * sizeof(int32_t), cudaMemcpyHostToDevice, s),
               "metadata upload");
    MassArgs args;
    args.qkv = qkv;
    args.dtype = dtype;
    args.qkv_rows_capacity = qkv_rows;
    args.lse = lse;
    args.prompt_offsets = meta_device;
    args.query_spans = meta_device + queries_at;
    args.spans = meta_device + spans_at;
    args.item_offsets = meta_device + items_at;
    args.prompt_count = prompt_count;
    args.span_count = span_count;
    args.item_count = item_count;
    args.query_heads = query_heads;
    args.kv_heads = kv_heads;
    args.head_dim = head_dim;
    args.sliding_window = sliding_window;
    args.reference_chunk = prefill_chunk_tokens;
    args.normalize_by_length = normalize_by_length;
    args.partials = partials;
    args.status = status;
    check_cuda(launch_document_mass(args, s), "document_attention_mass_noalloc");
    FinalizeArgs finalize;
    finalize.partials = partials;
    finalize.item_offsets = args.item_offsets;
    finalize.query_spans = args.query_spans;
    finalize.prompt_offsets = meta_device;
    finalize.prompt_count = prompt_count;
    finalize.span_count = span_count;
    finalize.item_count = item_count;
    finalize.layers = 1;
    finalize.query_heads = query_heads;
    finalize.raw_rows = rows;
    check_cuda(launch_finalize_mass(finalize, s), "finalize");
    int status_host = 0;
    check_cuda(cudaMemcpyAsync(mass_out, rows, static_cast<size_t>(prompt_count) * span_count * sizeof(double),
                               cudaMemcpyDeviceToHost, s),
               "mass download");
    check_cuda(cudaMemcpyAsync(&status_host, status, sizeof(int), cudaMemcpyDeviceToHost, s), "status download");
    check_cuda(cudaStreamSynchronize(s), "document_attention_mass_noalloc");
    if (status_host != 0) {
      throw Error("device reported an error in document_attention_mass_noalloc (code " + std::to_string(status_host) +
                  ")");
    }
    set_last_error("");
    return AR_OK;
  } catch (const std::exception& error) {
    const std::string what = error.what();
    set_last_error(what);
    if (what.find("device reported") != std::string::npos) return AR_ERR_DEVICE;
    if (what.find("CUDA error") != std::string::npos) return AR_ERR_CUDA;
    return AR_ERR_INVALID;
  }
}
