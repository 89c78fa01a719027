// Allocation-free variant of ar_document_attention_mass.
//
// Some callers cannot let a library allocate device memory while they run: an application that
// has reserved the whole GPU under a fixed memory budget, a serving loop on a latency-critical
// path where an allocator call may block or synchronise, or a host framework that owns every
// device allocation of its process. This entry point does the same work as
// ar_document_attention_mass (the same checks, kernels and launches, through mass_call.h) but
// takes its scratch (status word, batch metadata, per-CTA partial sums, finished rows) from one
// fixed array that the library reserves when it is loaded. It calls no cudaMalloc, cudaFree or
// other allocating routine.
//
// The array is a file-scope __device__ object: every GPU that loads the library holds
// kNoAllocScratchBytes of it until the process exits, and every call shares it. In host code
// its name is only a host-side handle, so its device address is taken with
// cudaGetSymbolAddress, once per device, on the first call made on that device with that device
// current, and cached. Make that first call before any stream capture. The cached address is
// not refreshed after cudaDeviceReset; a process that resets a device must not call this entry
// point on it again.
//
// Calls whose GPU work overlapped would race on the shared array. Within a process the library
// prevents that: a per-device lock is held from the status reset until the call's stream has
// drained, so concurrent calls from several host threads run one after another.
#include <mutex>
#include <string>

#include "../../include/attnrank_b200.h"
#include "capi_guard.h"
#include "engine.h"
#include "mass_call.h"

namespace arb {
namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;  // 8 MiB per device

static __device__ __align__(256) unsigned char g_mass_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_address[kMaxDevices] = {};
std::mutex g_call_mutex[kMaxDevices];  // one call at a time per device on the shared array

// Index of the current device, checked against the table size.
int current_device() {
  int device = 0;
  check_cuda(cudaGetDevice(&device), "cudaGetDevice");
  if (device < 0 || device >= kMaxDevices) throw Error("document_attention_mass_noalloc: device index out of range");
  return device;
}

// Device address of this device's scratch array (the device must be current).
void* scratch_for_device(int device) {
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_address[device] == nullptr) {
    void* address = nullptr;
    check_cuda(cudaGetSymbolAddress(&address, g_mass_scratch), "cudaGetSymbolAddress(scratch)");
    g_scratch_address[device] = address;
  }
  return g_scratch_address[device];
}

}  // namespace
}  // namespace arb

extern "C" int ar_document_attention_mass_noalloc(const void* qkv, int qkv_rows, const float* lse,
                                                  const int32_t* prompt_offsets_host, int prompt_count,
                                                  const int32_t* query_spans_host, const int32_t* spans_host,
                                                  int span_count, int query_heads, int kv_heads, int head_dim,
                                                  int sliding_window, int prefill_chunk_tokens,
                                                  int normalize_by_length, double* mass_out, int dtype,
                                                  void* stream) {
  using namespace arb;
  return guarded_call([&] {
    const char* who = "document_attention_mass_noalloc";
    const MassCallArgs call{qkv, qkv_rows, lse, prompt_offsets_host, prompt_count, query_spans_host, spans_host,
                            span_count, query_heads, kv_heads, head_dim, sliding_window, prefill_chunk_tokens,
                            normalize_by_length, mass_out, dtype};
    const MassBatch batch = plan_mass_batch(who, call);
    const MassScratchLayout layout = mass_scratch_layout(batch);
    if (layout.total > kNoAllocScratchBytes) {
      throw Error(std::string(who) + ": this batch needs " + std::to_string(layout.total) +
                  " bytes of scratch but the fixed array holds " + std::to_string(kNoAllocScratchBytes) +
                  "; split the prompts over several calls or use ar_document_attention_mass");
    }
    const int device = current_device();
    void* scratch = scratch_for_device(device);
    std::lock_guard<std::mutex> lock(g_call_mutex[device]);
    run_mass_batch(who, call, batch, layout, scratch, static_cast<cudaStream_t>(stream));
    return AR_OK;
  });
}
