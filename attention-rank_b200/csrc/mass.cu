// Query->document attention mass on tcgen05 / TMEM, fused with the span-masked softmax
// reduction; no attention matrix is ever written to memory.
//
// Reference semantics (attnrank/src/kernels.cu:202-236 over the softmax of :117-162, driven by
// model.cu:468-470 and normalised by model.cu:593-617): for every probed layer and document
// span s,
//     mass[s] = sum_{h < Hq} sum_{q in query span} sum_{k in span s} softmax_k(Q_hq . K_{h/g,k} / sqrt(D))
// with the causal (and optional sliding-window) mask, optionally dividing each (h, q) term by
// the span length clipped at the end of the prefill chunk that holds q.
//
// B200 design. One CTA = (prompt, KV head, 128-row tile of GQA-stacked query rows, a run of
// 128-key tiles). Q and K tiles arrive by TMA (128B swizzle, no multicast) into shared memory,
// one elected thread issues tcgen05.mma (M=128, N=128, K=16 x 8, fp16 or bf16 -> fp32) into a TMEM
// accumulator, double-buffered so the MMA and TMA of tile j+1 overlap the epilogue of tile j.
// The epilogue (4 warps, one TMEM lane = one query row per thread) turns raw scores into
// probabilities with the row's log-sum-exp produced by the attention kernel, p = 2^(s*c - lse2),
// so a single pass gives exact softmax mass, and adds them into per-(span, row) sums in shared
// memory. Each CTA writes one partial per span; a deterministic finaliser reduces them.
//
// Every mbarrier wait is bounded: on expiry the kernel records kStatusWaitTimeout, drains its own
// copies and MMAs (again bounded), frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <mutex>

#include "common.cuh"
#include "layer_kernels.h"
#include "mass_plan.h"

namespace arb {
namespace {

constexpr int kThreads = 128;
constexpr int kHeadDim = 128;
constexpr uint32_t kTmemColumns = 256;          // two 128-column fp32 accumulators
constexpr uint32_t kHalfTileBytes = 128 * 128;  // 128 rows x 64 16-bit values (one 128B-swizzled half)
constexpr uint32_t kTileBytes = 2 * kHalfTileBytes;  // 128 rows x 128 16-bit values
constexpr uint32_t kQBoxRows = 8;
constexpr uint32_t kSpinLimit = 1u << 24;

struct __align__(8) MassShared {
  uint64_t q_bar;
  uint64_t k_bar[2];
  uint64_t mma_bar[2];
  uint32_t tmem_base;
  volatile int abort;
  int span_begin[kMassMaxSpans];
  int span_end[kMassMaxSpans];
  float warp_sums[4][kMassMaxSpans];
};

// dynamic shared memory layout (1024-byte aligned base):
//   [0, 32K)      Q tile: two 128B-swizzled halves of 128 rows x 64 columns
//   [32K, 96K)    K tiles: two stages x two halves
//   [96K, ...)    MassShared
//   then          per-(span, row) running sums, fp32 [span_count][128]
// Sized by the call's span count: up to 24 spans two CTAs share an SM (one CTA's exponentials
// and span sums overlap the other's loads and MMAs).
constexpr uint32_t kQOffset = 0;
constexpr uint32_t kKOffset = kTileBytes;
constexpr uint32_t kControlOffset = 3 * kTileBytes;
constexpr uint32_t kSigmaOffset = kControlOffset + ((sizeof(MassShared) + 15) & ~static_cast<uint32_t>(15));
constexpr size_t smem_bytes(int span_count) {
  return kSigmaOffset + static_cast<size_t>(span_count) * kMassRowTile * 4 + 1024;  // + alignment slack
}

__device__ __forceinline__ uint32_t smem_u32(const void* pointer) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(pointer));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t phase) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(phase)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// K-major operand, 128B swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_descriptor(uint32_t address) {
  uint64_t desc = 0;
  desc |= static_cast<uint64_t>((address >> 4) & 0x3FFFu);  // start address
  desc |= static_cast<uint64_t>(1) << 16;                   // leading byte offset (unused for SW128 K-major)
  desc |= static_cast<uint64_t>(1024 >> 4) << 32;           // stride byte offset: next 8-row group
  desc |= static_cast<uint64_t>(1) << 46;                   // descriptor version (sm_100)
  desc |= static_cast<uint64_t>(2) << 61;                   // layout: SWIZZLE_128B
  return desc;
}

// kind::f16 instruction descriptor: fp32 accumulator, both operands K-major, M=128, N=128, A and B
// of the same 16-bit format (0 = fp16, 1 = bf16).
constexpr uint32_t instr_desc(uint32_t format) {
  return (1u << 4)              // D format fp32
         | (format << 7)        // A format
         | (format << 10)       // B format
         | ((128u >> 3) << 17)  // N
         | ((128u >> 4) << 24);  // M
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate),
        "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_load_32(uint32_t address, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(address));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct KernelArgs {
  const float* lse;
  const int32_t* prompt_offsets;
  const int32_t* query_spans;
  const int32_t* spans;
  const int32_t* item_offsets;
  int prompt_count;
  int span_count;
  int query_heads;
  int kv_heads;
  int sliding_window;
  int reference_chunk;
  int normalize_by_length;
  float* partials;
  int* status;
  uint32_t instr_desc;
};

__global__ void __launch_bounds__(kThreads, 2)
    document_mass_kernel(const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap k_map,
                         const KernelArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* sigma = reinterpret_cast<float*>(smem + kSigmaOffset);
  MassShared& ctl = *reinterpret_cast<MassShared*>(smem + kControlOffset);
  const uint32_t q_smem = smem_u32(smem + kQOffset);
  const uint32_t k_smem = smem_u32(smem + kKOffset);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int item = blockIdx.x;
  const int S = args.span_count;

  // ---- which prompt / KV head / row tile / key run this CTA owns
  int lo = 0, hi = args.prompt_count - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (args.item_offsets[mid] <= item) lo = mid; else hi = mid - 1;
  }
  const int prompt = lo;
  const int prompt_begin = args.prompt_offsets[prompt];
  const int length = args.prompt_offsets[prompt + 1] - prompt_begin;
  const int group = args.query_heads / args.kv_heads;
  const int32_t* query_span = args.query_spans + 2 * prompt;
  const int32_t* prompt_spans = args.spans + 2 * static_cast<size_t>(prompt) * S;
  const ProbeRows rows = probe_rows(query_span, length);
  const MassItemShape shape = mass_item_shape(query_span, prompt_spans, S, length, group);
  const int local = item - args.item_offsets[prompt];
  const int per_head = shape.row_tiles * shape.key_splits;
  const int kv_head = local / per_head;
  const int row_tile = (local % per_head) / shape.key_splits;
  const int key_split = local % shape.key_splits;
  const int first_tile = key_split * kMassKeyTilesPerItem;
  int tiles = shape.key_tiles - first_tile;
  if (tiles > kMassKeyTilesPerItem) tiles = kMassKeyTilesPerItem;
  if (tiles < 0) tiles = 0;
  const int key0 = shape.key_begin + first_tile * kMassKeyTile;

  // ---- set-up: barriers, TMEM, spans, zeroed sums
  if (tid == 0) {
    mbar_init(smem_u32(&ctl.q_bar), 1);
    mbar_init(smem_u32(&ctl.k_bar[0]), 1);
    mbar_init(smem_u32(&ctl.k_bar[1]), 1);
    mbar_init(smem_u32(&ctl.mma_bar[0]), 1);
    mbar_init(smem_u32(&ctl.mma_bar[1]), 1);
    ctl.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&ctl.tmem_base)),
                 "r"(kTmemColumns));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  if (tid < S) {
    ctl.span_begin[tid] = prompt_spans[2 * tid];
    ctl.span_end[tid] = prompt_spans[2 * tid + 1];
  }
  for (int i = tid; i < S * kMassRowTile; i += kThreads) sigma[i] = 0.0f;
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = ctl.tmem_base;

  // ---- this thread's query row (TMEM lane tid)
  const int slot = row_tile * kMassRowTile + tid;
  const int head_local = rows.padded > 0 ? slot / rows.padded : group;
  const int token_local = rows.padded > 0 ? slot % rows.padded : 0;
  const bool row_valid = tiles > 0 && head_local < group && token_local < rows.query_end - rows.query_begin;
  const int query = rows.query_begin + token_local;  // prompt-relative position
  const int head = kv_head * group + head_local;
  const float lse2 = row_valid ? args.lse[static_cast<size_t>(prompt_begin + query) * args.query_heads + head] : 0.0f;
  const int key_min = args.sliding_window > 0 ? query - args.sliding_window + 1 : 0;
  const int key_max = min(query, length - 1);
  const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(kHeadDim));

  const uint32_t q_bar = smem_u32(&ctl.q_bar);
  const uint32_t k_bar[2] = {smem_u32(&ctl.k_bar[0]), smem_u32(&ctl.k_bar[1])};
  const uint32_t mma_bar[2] = {smem_u32(&ctl.mma_bar[0]), smem_u32(&ctl.mma_bar[1])};

  auto load_k = [&](int j) {
    const int stage = j & 1;
    const int y = prompt_begin + key0 + j * kMassKeyTile;
    const int x = (args.query_heads + kv_head) * kHeadDim;
    mbar_expect_tx(k_bar[stage], kTileBytes);
    tma_load_2d(k_smem + stage * kTileBytes, &k_map, x, y, k_bar[stage]);
    tma_load_2d(k_smem + stage * kTileBytes + kHalfTileBytes, &k_map, x + 64, y, k_bar[stage]);
  };
  auto issue_mma = [&](int j) {
    const int stage = j & 1;
    tmem_fence_after();
#pragma unroll
    for (int kk = 0; kk < kHeadDim / 16; ++kk) {
      const uint32_t offset = (kk >> 2) * kHalfTileBytes + (kk & 3) * 32;
      umma_f16(tmem + stage * 128, smem_descriptor(q_smem + offset),
               smem_descriptor(k_smem + stage * kTileBytes + offset), args.instr_desc, kk > 0 ? 1u : 0u);
    }
    umma_commit(mma_bar[stage]);
  };

  // ---- prologue (one thread): Q tile, first two K tiles, first MMA.
  // Thread 0 tracks its in-flight work so that an aborted CTA can drain it before exiting.
  int k_issued = 0;    // K tiles whose TMA was issued
  int k_consumed = 0;  // K tiles whose arrival was waited on
  int mma_issued = 0;  // tiles whose MMA was issued
  int mma_waited = 0;  // tiles whose MMA completion thread 0 waited on
  if (tid == 0 && tiles > 0) {
    mbar_expect_tx(q_bar, kTileBytes);
    for (int group8 = 0; group8 < kMassRowTile / static_cast<int>(kQBoxRows); ++group8) {
      const int first_slot = row_tile * kMassRowTile + group8 * kQBoxRows;
      int h = rows.padded > 0 ? first_slot / rows.padded : 0;
      int t0 = rows.padded > 0 ? first_slot % rows.padded : 0;
      if (h >= group) {  // padding rows past the last head: load any in-range box, results are masked
        h = group - 1;
        t0 = 0;
      }
      const int x = (kv_head * group + h) * kHeadDim;
      const int y = prompt_begin + rows.query_begin + t0;
      const uint32_t dst = q_smem + group8 * kQBoxRows * 128;
      tma_load_2d(dst, &q_map, x, y, q_bar);
      tma_load_2d(dst + kHalfTileBytes, &q_map, x + 64, y, q_bar);
    }
    load_k(0);
    k_issued = 1;
    if (tiles > 1) {
      load_k(1);
      k_issued = 2;
    }
    if (mbar_wait(q_bar, 0) && mbar_wait(k_bar[0], 0)) {
      k_consumed = 1;
      issue_mma(0);
      mma_issued = 1;
    } else {
      report_status(args.status, kStatusWaitTimeout);
      ctl.abort = 1;
    }
  }
  __syncthreads();

  for (int j = 0; j < tiles && !ctl.abort; ++j) {
    if (tid == 0 && j + 1 < tiles && !ctl.abort) {
      if (mbar_wait(k_bar[(j + 1) & 1], ((j + 1) >> 1) & 1)) {
        k_consumed = j + 2;
        issue_mma(j + 1);
        mma_issued = j + 2;
      } else {
        report_status(args.status, kStatusWaitTimeout);
        ctl.abort = 1;
      }
    }
    // warp-uniform: the TMEM loads below are warp-collective (.sync.aligned)
    const bool ready = __all_sync(0xffffffffu, mbar_wait(mma_bar[j & 1], (j >> 1) & 1));
    if (ready) mma_waited = j + 1;
    if (!ready) {
      report_status(args.status, kStatusWaitTimeout);
      ctl.abort = 1;
    } else {
      tmem_fence_after();
      const int tile_key0 = key0 + j * kMassKeyTile;
#pragma unroll 1
      for (int chunk = 0; chunk < kMassKeyTile / 32; ++chunk) {
        uint32_t raw[32];
        tmem_load_32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + (j & 1) * 128 + chunk * 32, raw);
        const int base = tile_key0 + chunk * 32;
        float p[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int key = base + i;
          const bool visible = row_valid && key >= key_min && key <= key_max;
          p[i] = visible ? exp2f(__uint_as_float(raw[i]) * scale_log2 - lse2) : 0.0f;
        }
        for (int s = 0; s < S; ++s) {
          const int b = max(ctl.span_begin[s], base);
          const int e = min(ctl.span_end[s], base + 32);
          if (b >= e) continue;  // uniform across the CTA
          const int lo_i = b - base;
          const int hi_i = e - base;
          float acc = 0.0f;
#pragma unroll
          for (int i = 0; i < 32; ++i) acc += (i >= lo_i && i < hi_i) ? p[i] : 0.0f;
          sigma[s * kMassRowTile + tid] += acc;
        }
      }
    }
    tmem_fence_before();
    __syncthreads();
    if (tid == 0 && j + 2 < tiles && !ctl.abort) {
      load_k(j + 2);
      k_issued = j + 3;
    }
  }

  // ---- drain after an abort: outstanding TMA loads and MMAs of this CTA (bounded waits)
  if (tid == 0 && ctl.abort) {
    if (k_issued > 0 && k_consumed == 0) mbar_wait(q_bar, 0);
    for (int j = k_consumed; j < k_issued; ++j) mbar_wait(k_bar[j & 1], (j >> 1) & 1);
    for (int j = mma_waited; j < mma_issued; ++j) mbar_wait(mma_bar[j & 1], (j >> 1) & 1);
  }

  // ---- per-row divisors (normalize_by_length), then the per-span sum over this CTA's rows
  if (row_valid && args.normalize_by_length) {
    const int chunk = args.reference_chunk > 0 ? args.reference_chunk : length;
    int chunk_end = (query / chunk + 1) * chunk;
    if (chunk_end > length) chunk_end = length;
    for (int s = 0; s < S; ++s) {
      const int e = min(ctl.span_end[s], chunk_end);
      const int divisor = e - ctl.span_begin[s];
      if (divisor > 0) sigma[s * kMassRowTile + tid] /= static_cast<float>(divisor);
    }
  }
  for (int s = 0; s < S; ++s) {
    float v = sigma[s * kMassRowTile + tid];
    v = warp_sum(v);
    if (lane == 0) ctl.warp_sums[warp][s] = v;
  }
  tmem_fence_before();
  __syncthreads();
  if (tid < S) {
    const float total = ctl.warp_sums[0][tid] + ctl.warp_sums[1][tid] + ctl.warp_sums[2][tid] + ctl.warp_sums[3][tid];
    args.partials[static_cast<size_t>(item) * S + tid] = ctl.abort ? 0.0f : total;
  }
  if (warp == 0) {
    tmem_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemColumns));
  }
}

// ---------------------------------------------------------------------------------------------
// Deterministic finaliser: per (prompt, layer) sum the CTA partials in a fixed order, divide by
// the number of (head, query row) observations, normalise the row to unit sum (model.cu:602-615,
// :503-508) in fp64, then add the rows of all prompts into the [layers, spans] accumulator in
// prompt order (the per-prompt sum of attnrank.cpp:350-362, kept on the device).
// ---------------------------------------------------------------------------------------------
__global__ void finalize_mass_kernel(const float* __restrict__ partials, const int32_t* __restrict__ item_offsets,
                                     const int32_t* __restrict__ query_spans, const int32_t* __restrict__ prompt_offsets,
                                     int prompt_count, int span_count, int item_count, int layers, int query_heads,
                                     double* __restrict__ rows_out, double* __restrict__ raw_rows_out,
                                     float* __restrict__ accumulator) {
  // one warp per layer, lane s owns span s; every sum runs in a fixed order
  const int layer = blockIdx.x;
  const int s = threadIdx.x;
  const bool active = s < span_count;
  const float* layer_partials = partials + static_cast<size_t>(layer) * item_count * span_count;
  double total = 0.0;
  for (int p = 0; p < prompt_count; ++p) {
    const int length = prompt_offsets[p + 1] - prompt_offsets[p];
    const ProbeRows rows = probe_rows(query_spans + 2 * p, length);
    const double observations = static_cast<double>(rows.query_end - rows.query_begin) * query_heads;
    double raw = 0.0;
    if (active) {
      for (int item = item_offsets[p]; item < item_offsets[p + 1]; ++item) {
        raw += static_cast<double>(layer_partials[static_cast<size_t>(item) * span_count + s]);
      }
    }
    double row = observations > 0.0 ? raw / observations : 0.0;
    if (active && raw_rows_out != nullptr) raw_rows_out[(static_cast<size_t>(p) * layers + layer) * span_count + s] = row;
    double sum = row;  // inactive lanes hold 0
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, offset);
    if (sum > 0.0) row /= sum;
    if (active && rows_out != nullptr) rows_out[(static_cast<size_t>(p) * layers + layer) * span_count + s] = row;
    total += row;
  }
  if (active && accumulator != nullptr) accumulator[layer * span_count + s] += static_cast<float>(total);
}

// The same per-(prompt, layer) rows without the cross-prompt accumulator (the kernel-level C ABI):
// one warp per (prompt, layer), so the prompts no longer queue behind one another. Every value is
// computed exactly as in finalize_mass_kernel (same order of each sum).
__global__ void finalize_rows_kernel(const float* __restrict__ partials, const int32_t* __restrict__ item_offsets,
                                     const int32_t* __restrict__ query_spans, const int32_t* __restrict__ prompt_offsets,
                                     int span_count, int item_count, int layers, int query_heads,
                                     double* __restrict__ rows_out, double* __restrict__ raw_rows_out) {
  const int p = blockIdx.x;
  const int layer = blockIdx.y;
  const int s = threadIdx.x;
  const bool active = s < span_count;
  const float* layer_partials = partials + static_cast<size_t>(layer) * item_count * span_count;
  const int length = prompt_offsets[p + 1] - prompt_offsets[p];
  const ProbeRows rows = probe_rows(query_spans + 2 * p, length);
  const double observations = static_cast<double>(rows.query_end - rows.query_begin) * query_heads;
  double raw = 0.0;
  if (active) {
    for (int item = item_offsets[p]; item < item_offsets[p + 1]; ++item) {
      raw += static_cast<double>(layer_partials[static_cast<size_t>(item) * span_count + s]);
    }
  }
  double row = observations > 0.0 ? raw / observations : 0.0;
  if (active && raw_rows_out != nullptr) raw_rows_out[(static_cast<size_t>(p) * layers + layer) * span_count + s] = row;
  double sum = row;  // inactive lanes hold 0
#pragma unroll
  for (int offset = 16; offset > 0; offset >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, offset);
  if (sum > 0.0) row /= sum;
  if (active && rows_out != nullptr) rows_out[(static_cast<size_t>(p) * layers + layer) * span_count + s] = row;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* pointer = nullptr;
    cudaDriverEntryPointQueryResult result;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &pointer, cudaEnableDefault, &result) == cudaSuccess &&
        result == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(pointer);
    }
  });
  return fn;
}

bool encode_rows_map(CUtensorMap* map, const void* base, int width, int rows, int box_rows, int dtype) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = encode_fn();
  if (encode == nullptr) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(width) * 2};
  const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t element_strides[2] = {1, 1};
  const CUtensorMapDataType type =
      dtype == kActFp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const CUresult status = encode(map, type, 2, const_cast<void*>(base), dims, strides,
                                 box, element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return status == CUDA_SUCCESS;
}

}  // namespace

cudaError_t launch_document_mass(const MassArgs& args, cudaStream_t stream) {
  if (args.item_count <= 0) return cudaSuccess;
  if (args.head_dim != kHeadDim || args.kv_heads <= 0 || args.query_heads % args.kv_heads != 0 ||
      args.span_count <= 0 || args.span_count > kMassMaxSpans || args.prompt_count <= 0) {
    return cudaErrorInvalidValue;
  }
  const int width = (args.query_heads + 2 * args.kv_heads) * kHeadDim;
  if ((reinterpret_cast<uintptr_t>(args.qkv) & 15) != 0) return cudaErrorInvalidValue;
  if (args.dtype != kActFp16 && args.dtype != kActBf16) return cudaErrorInvalidValue;
  CUtensorMap q_map;
  CUtensorMap k_map;
  if (!encode_rows_map(&q_map, args.qkv, width, args.qkv_rows_capacity, kQBoxRows, args.dtype) ||
      !encode_rows_map(&k_map, args.qkv, width, args.qkv_rows_capacity, kMassKeyTile, args.dtype)) {
    return cudaErrorInvalidValue;
  }
  int device = 0;
  cudaGetDevice(&device);
  static uint64_t configured_devices = 0;
  if (device < 64 && !(configured_devices & (1ull << device))) {
    const cudaError_t status = cudaFuncSetAttribute(document_mass_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                    static_cast<int>(smem_bytes(kMassMaxSpans)));
    if (status != cudaSuccess) return status;
    configured_devices |= 1ull << device;
  }
  KernelArgs kernel_args;
  kernel_args.lse = args.lse;
  kernel_args.prompt_offsets = args.prompt_offsets;
  kernel_args.query_spans = args.query_spans;
  kernel_args.spans = args.spans;
  kernel_args.item_offsets = args.item_offsets;
  kernel_args.prompt_count = args.prompt_count;
  kernel_args.span_count = args.span_count;
  kernel_args.query_heads = args.query_heads;
  kernel_args.kv_heads = args.kv_heads;
  kernel_args.sliding_window = args.sliding_window;
  kernel_args.reference_chunk = args.reference_chunk;
  kernel_args.normalize_by_length = args.normalize_by_length;
  kernel_args.partials = args.partials;
  kernel_args.status = args.status;
  kernel_args.instr_desc = instr_desc(args.dtype == kActFp16 ? 0u : 1u);
  document_mass_kernel<<<args.item_count, kThreads, smem_bytes(args.span_count), stream>>>(q_map, k_map, kernel_args);
  return cudaGetLastError();
}

cudaError_t launch_finalize_mass(const FinalizeArgs& args, cudaStream_t stream) {
  if (args.prompt_count <= 0 || args.layers <= 0) return cudaSuccess;
  if (args.span_count <= 0 || args.span_count > kMassMaxSpans) return cudaErrorInvalidValue;
  if (args.accumulator == nullptr) {
    if (args.layers > 65535) return cudaErrorInvalidValue;  // grid y
    finalize_rows_kernel<<<dim3(args.prompt_count, args.layers), 32, 0, stream>>>(
        args.partials, args.item_offsets, args.query_spans, args.prompt_offsets, args.span_count, args.item_count,
        args.layers, args.query_heads, args.rows, args.raw_rows);
    return cudaGetLastError();
  }
  finalize_mass_kernel<<<args.layers, 32, 0, stream>>>(args.partials, args.item_offsets, args.query_spans, args.prompt_offsets,
                                             args.prompt_count, args.span_count, args.item_count, args.layers,
                                             args.query_heads, args.rows, args.raw_rows, args.accumulator);
  return cudaGetLastError();
}

}  // namespace arb
