// Causal GQA prefill attention on tcgen05 / TMEM (sm_100a), packed variable-length prompts, with
// per-row log-sum-exp for the attention-mass kernel.
//
// Same contract as the mma.sync kernel in attention.cu (which it replaces on the engine path):
// reference semantics of LlamaForwardPass::attend (attnrank/src/model.cu:426-480) and
// softmax_causal_kernel (attnrank/src/kernels.cu:117-162); key k is visible to query q iff
// k <= q, k < prompt length and, with a sliding window, k > q - window.
//
// One CTA = one (prompt, 128-row query tile, query head). 160 threads:
//   warps 0-3 (softmax): thread r owns query row r = TMEM lane r. For every 64-key tile it
//     reads S = Q K^T (fp32) from TMEM, applies the mask, keeps the row's running max / sum,
//     writes P (16-bit) back into the same TMEM columns, and signals the control warp.
//   warp 4 (control): allocates TMEM, lane 0 issues every TMA load (no multicast) and every
//     tcgen05.mma, and commits MMA completion to mbarriers.
// Pipeline per key tile j (K/V double-buffered in shared memory, S double-buffered in TMEM):
//     S_{j+1} = Q K_{j+1}^T  overlaps the softmax of tile j;
//     O += P_j V_j  (A = P from TMEM, B = V from shared memory, MN-major) after the softmax.
// A CTA holds 256 TMEM columns (S0 | S1 | O) and 96 KB of shared memory, so two CTAs share an
// SM: one's softmax, set-up and epilogue overlap the other's MMAs.
//
// Fused attention mass (optional, `mass_partials` non-null): for the query rows of the probe
// (the prompt's query span) the softmax warps also add each tile's probabilities into per-span
// sums, kept relative to the same running reference as O and l (rescaled with them) and divided
// by l at the end, so each row contributes sum_{k in span} softmax(q.k / sqrt(D)) exactly
// (reference: reduce_document_attention over softmax_causal_kernel's output, kernels.cu:202-236,
// :117-162, with the normalize_by_length divisor of kernels.cu:211). Each CTA writes one partial
// per span: the fixed-order sum over its rows.
// Rescaling: exponents use a reference max m_ref that moves only when the row max exceeds it by
// more than 8 (log2 units), so p <= 2^8 and the O accumulator in TMEM is rescaled rarely.
// Every mbarrier wait is bounded (time and polls); on expiry the kernel records
// kStatusWaitTimeout, waits (bounded) for its own MMAs and copies, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "layer_kernels.h"

namespace arb {
namespace {

constexpr int kHeadDim = 128;
constexpr int kTile = 128;                         // query rows per CTA
constexpr int kKeys = 64;                          // keys per tile
constexpr int kSoftmaxThreads = 128;
constexpr int kThreads = kSoftmaxThreads + 32;     // + control warp
constexpr uint32_t kTmemColumns = 256;             // S0 [0,64) S1 [64,128) O [128,256)
constexpr uint32_t kTmemO = 2 * kKeys;
constexpr uint32_t kRowBytes = 128;                // 64 16-bit values: one 128B-swizzled row of a half
constexpr uint32_t kQHalfBytes = kTile * kRowBytes;      // 128 rows x 64 values (16 KB)
constexpr uint32_t kQBytes = 2 * kQHalfBytes;            // 128 rows x 128 values
constexpr uint32_t kKvHalfBytes = kKeys * kRowBytes;     // 64 rows x 64 values (8 KB)
constexpr uint32_t kKvBytes = 2 * kKvHalfBytes;          // 64 rows x 128 values
constexpr uint32_t kSpinLimit = 1u << 26;          // hard backstop on polls per wait
constexpr uint64_t kWaitLimitNs = 500ull * 1000 * 1000;  // a wait gives up after 0.5 s
constexpr float kRescaleThreshold = 8.0f;          // log2 units
constexpr int kChains = 4;                         // independent accumulators per row reduction

// shared memory (1024-byte aligned): Q | K stage 0,1 | V stage 0,1 | control
constexpr uint32_t kQOffset = 0;
constexpr uint32_t kKOffset = kQBytes;
constexpr uint32_t kVOffset = kQBytes + 2 * kKvBytes;
constexpr uint32_t kControlOffset = kQBytes + 4 * kKvBytes;

constexpr int kMaxSpans = kMassMaxSpans;

struct __align__(16) Control {
  uint64_t q_bar;
  uint64_t k_bar[2];  // K and V stages load separately: K_{j+2} as soon as S_j has read K_j
  uint64_t v_bar[2];
  uint64_t s_bar[2];
  uint64_t o_bar;
  uint64_t p_bar[2];
  uint64_t done_bar;  // every MMA of the CTA completed (one commit after the last P.V)
  uint32_t tmem_base;
  volatile int abort;
  int span_lo[kMaxSpans];  // fused mass: the prompt's document spans
  int span_hi[kMaxSpans];
  float warp_sums[4][kMaxSpans];
};
// dynamic shared memory: the fixed part, then (fused mass only) float sigma[span_count][128]
constexpr size_t kSigmaOffset = kControlOffset + ((sizeof(Control) + 15) & ~size_t(15));
constexpr size_t kSmemBytes = kSigmaOffset + 1024;
constexpr size_t smem_bytes(int span_count) { return kSmemBytes + static_cast<size_t>(span_count) * kTile * 4; }

__device__ __forceinline__ uint32_t smem_u32(const void* pointer) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(pointer));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait for the completion of phase `phase` (parity); gives up after kWaitLimitNs (or
// kSpinLimit polls), or earlier once *abort is set by another thread of the CTA. Every caller
// waits on a barrier at most one phase ahead of the last phase it saw complete, so the parity
// is unambiguous.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t phase, const volatile int* abort = nullptr) {
  uint64_t start = 0;
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
    if ((i & 1023) == 1023) {
      if (abort != nullptr && *abort) return false;
      const uint64_t now = global_ns();
      if (start == 0) {
        start = now;
      } else if (now - start > kWaitLimitNs) {
        return false;
      }
    }
  }
  return false;
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// K-major 128B-swizzled operand: 128-byte rows, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t desc_k_major(uint32_t address) {
  return static_cast<uint64_t>((address >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) | (static_cast<uint64_t>(2) << 61);
}
// MN-major 128B-swizzled operand (V as B of P.V): each 128-byte row holds 64 consecutive N (head
// dim) values of one K (key); 8 rows form a 1024-byte atom; the two 64-wide N halves are 8 KB
// apart (leading byte offset), consecutive 8-key groups 1024 bytes apart (stride byte offset).
__device__ __forceinline__ uint64_t desc_mn_major(uint32_t address) {
  return static_cast<uint64_t>((address >> 4) & 0x3FFFu) | (static_cast<uint64_t>(kKvHalfBytes >> 4) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) | (static_cast<uint64_t>(2) << 61);
}

// kind::f16 instruction descriptor, fp32 accumulator, M = 128, N = n; format 0 = fp16, 1 = bf16
// (A and B always of the same format); A K-major, B K-major or MN-major.
constexpr uint32_t idesc(uint32_t format, bool b_mn_major, uint32_t n) {
  return (1u << 4) | (format << 7) | (format << 10) | (b_mn_major ? (1u << 16) : 0u) | ((n >> 3) << 17) |
         ((128u >> 4) << 24);
}

__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(d), "l"(a), "l"(b), "r"(id), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t id, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(d), "r"(a_tmem), "l"(b), "r"(id), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t address, uint32_t (&r)[32]) {
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
}
__device__ __forceinline__ void tmem_st32(uint32_t address, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(address), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void softmax_barrier() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// Packed fp32 pairs (sm_100a f32x2 arithmetic): one instruction does two lanes' worth of FMA or
// add, which frees issue slots in the softmax loop for the exponentials.
__device__ __forceinline__ unsigned long long pack_f32x2(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void unpack_f32x2(unsigned long long v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ unsigned long long fma_f32x2(unsigned long long a, unsigned long long b,
                                                        unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ unsigned long long add_f32x2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// max(a, b, c) in one instruction
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x with the SFU's ex2 instruction, results below 2^-126 flushed to zero: a row's largest
// probability relative to its reference is at least 1, so those vanish in O, l and the span sums
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct Args {
  void* out;
  float* lse;
  const int32_t* prompt_offsets;
  const int32_t* tiles;
  int query_heads;
  int kv_heads;
  int sliding_window;
  uint32_t idesc_s;
  uint32_t idesc_pv;
  int* status;
  // fused mass (mass_partials == nullptr: attention only)
  const int32_t* query_spans;  // [prompts][2], prompt-relative
  const int32_t* spans;        // [prompts][span_count][2]
  const int32_t* mass_items;   // [prompts + 1] partial slots per prompt: Hq x query tiles in the span
  float* mass_partials;        // [items][span_count]
  int span_count;
  int normalize_by_length;
  int reference_chunk;
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 2)
    attention_tc_kernel(const __grid_constant__ CUtensorMap map, const Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Control& ctl = *reinterpret_cast<Control*>(smem + kControlOffset);
  const uint32_t q_smem = smem_u32(smem + kQOffset);
  const uint32_t k_smem = smem_u32(smem + kKOffset);
  const uint32_t v_smem = smem_u32(smem + kVOffset);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int prompt = args.tiles[2 * blockIdx.x];
  const int query_tile = args.tiles[2 * blockIdx.x + 1];
  const int head = blockIdx.y;
  const int group = args.query_heads / args.kv_heads;
  const int kv_head = head / group;
  const int prompt_begin = args.prompt_offsets[prompt];
  const int length = args.prompt_offsets[prompt + 1] - prompt_begin;
  const int q0 = query_tile * kTile;
  const int last_query = min(q0 + kTile, length) - 1;
  const int first_key = args.sliding_window > 0 ? max(0, q0 - args.sliding_window + 1) : 0;
  const int tile_begin = first_key / kKeys;
  const int tile_end = last_query / kKeys + 1;
  const int tiles = tile_end - tile_begin;

  // fused mass: does this query tile hold rows of the probe's query span?
  int query_lo = 0, query_hi = 0;
  if (args.mass_partials != nullptr) {
    query_lo = max(args.query_spans[2 * prompt], 0);
    query_hi = min(args.query_spans[2 * prompt + 1], length);
  }
  const bool capture = args.mass_partials != nullptr && query_hi > query_lo && q0 < query_hi && q0 + kTile > query_lo;
  const int S = capture ? args.span_count : 0;
  float* sigma = reinterpret_cast<float*>(smem + kSigmaOffset);
  if (tid < S) {
    const int32_t* span = args.spans + 2 * (static_cast<size_t>(prompt) * args.span_count + tid);
    ctl.span_lo[tid] = max(span[0], 0);
    ctl.span_hi[tid] = span[1];
  }
  for (int i = tid; i < S * kTile; i += kThreads) sigma[i] = 0.0f;

  // The control lane initialises the barriers and issues the Q, K and V loads of the first two
  // tiles before the TMEM allocation and the CTA barrier, so their latency overlaps the set-up.
  const bool control_lane = warp == 4 && lane == 0;
  const int q_x = head * kHeadDim;
  const int k_x = (args.query_heads + kv_head) * kHeadDim;
  const int v_x = (args.query_heads + args.kv_heads + kv_head) * kHeadDim;
  // last load issued on each K and V stage (tile index, -1 = none): an aborted CTA waits for them
  // before its shared memory is released; MMAs are drained through done_bar
  int last_k[2] = {-1, -1};
  int last_v[2] = {-1, -1};
  auto load_tile = [&](int j, uint32_t smem_base, int x, uint64_t* bars) {
    const int stage = j & 1;
    const int y = prompt_begin + (tile_begin + j) * kKeys;
    const uint32_t bar = smem_u32(&bars[stage]);
    mbar_expect_tx(bar, kKvBytes);
    tma_load_2d(smem_base + stage * kKvBytes, &map, x, y, bar);
    tma_load_2d(smem_base + stage * kKvBytes + kKvHalfBytes, &map, x + 64, y, bar);
  };
  auto load_k = [&](int j) {
    last_k[j & 1] = j;
    load_tile(j, k_smem, k_x, ctl.k_bar);
  };
  auto load_v = [&](int j) {
    last_v[j & 1] = j;
    load_tile(j, v_smem, v_x, ctl.v_bar);
  };
  if (control_lane) {
    mbar_init(smem_u32(&ctl.q_bar), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&ctl.k_bar[i]), 1);
      mbar_init(smem_u32(&ctl.v_bar[i]), 1);
      mbar_init(smem_u32(&ctl.s_bar[i]), 1);
      mbar_init(smem_u32(&ctl.p_bar[i]), kSoftmaxThreads);
    }
    mbar_init(smem_u32(&ctl.o_bar), 1);
    mbar_init(smem_u32(&ctl.done_bar), 1);
    // a CTA of a launch that already reported an error does no work (bounds a failing launch to
    // about one wave of timed-out CTAs); read once here so that the whole CTA agrees
    const int abort = (args.status != nullptr && *reinterpret_cast<volatile int*>(args.status) != 0) ? 1 : 0;
    ctl.abort = abort;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (tiles > 0 && !abort) {
      const uint32_t bar = smem_u32(&ctl.q_bar);
      mbar_expect_tx(bar, kQBytes);
      for (int half = 0; half < 2; ++half) {  // four 64 x 64 boxes: (column half, row half)
        for (int rows = 0; rows < 2; ++rows) {
          tma_load_2d(q_smem + half * kQHalfBytes + rows * kKvHalfBytes, &map, q_x + 64 * half,
                      prompt_begin + q0 + rows * kKeys, bar);
        }
      }
      load_k(0);
      load_v(0);
      if (tiles > 1) {
        load_k(1);
        load_v(1);
      }
    }
  }
  if (warp == 4) {
    __syncwarp();
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&ctl.tmem_base)),
                 "r"(kTmemColumns));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = ctl.tmem_base;
  const uint32_t q_bar = smem_u32(&ctl.q_bar);
  const uint32_t o_bar = smem_u32(&ctl.o_bar);
  const uint32_t done_bar = smem_u32(&ctl.done_bar);
  const bool skip = ctl.abort != 0;

  if (warp == 4) {
    // ------------------------------------------------------------------ control warp (lane 0)
    if (lane == 0 && tiles > 0 && !skip) {
      auto issue_s = [&](int j) {
        const int stage = j & 1;
        fence_after();
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk) {  // 16 head-dim values per MMA (32 bytes of a row)
          const uint32_t q_offset = (kk >> 2) * kQHalfBytes + (kk & 3) * 32;
          const uint32_t k_offset = (kk >> 2) * kKvHalfBytes + (kk & 3) * 32;
          mma_ss(tmem + stage * kKeys, desc_k_major(q_smem + q_offset),
                 desc_k_major(k_smem + stage * kKvBytes + k_offset), args.idesc_s, kk > 0 ? 1u : 0u);
        }
        mma_commit(smem_u32(&ctl.s_bar[stage]));
      };
      auto issue_pv = [&](int j) {
        const int stage = j & 1;
        fence_after();
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk) {  // 16 keys per MMA: 8 packed TMEM columns of P
          mma_ts(tmem + kTmemO, tmem + stage * kKeys + kk * 8,
                 desc_mn_major(v_smem + stage * kKvBytes + kk * 16 * kRowBytes), args.idesc_pv,
                 (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(o_bar);
      };
      // S_0 and S_1 go out at once (both S buffers are free). Afterwards S_{j+2} is issued right
      // behind PV_j: it overwrites the TMEM columns from which PV_j reads P_j, and the tensor pipe
      // executes one thread's tcgen05.mma operations in issue order, so no completion wait sits
      // between them and S_{j+2} is ready when the softmax of tile j+1 ends.
      bool ok = mbar_wait(q_bar, 0) && mbar_wait(smem_u32(&ctl.k_bar[0]), 0);
      if (ok) issue_s(0);
      if (ok && tiles > 1) {
        ok = mbar_wait(smem_u32(&ctl.k_bar[1]), 0);
        if (ok) issue_s(1);
      }
      for (int j = 0; ok && j < tiles; ++j) {
        if (j + 2 < tiles) {
          // S_j has read K_j (its completion is what the softmax of tile j waits for): refill
          ok = mbar_wait(smem_u32(&ctl.s_bar[j & 1]), (j >> 1) & 1);
          if (!ok) break;
          load_k(j + 2);
        }
        ok = mbar_wait(smem_u32(&ctl.p_bar[j & 1]), (j >> 1) & 1, &ctl.abort) &&  // softmax wrote P_j
             mbar_wait(smem_u32(&ctl.v_bar[j & 1]), (j >> 1) & 1);
        if (!ok) break;
        issue_pv(j);
        if (j + 2 < tiles) {
          ok = mbar_wait(smem_u32(&ctl.k_bar[j & 1]), ((j + 2) >> 1) & 1);
          if (!ok) break;
          issue_s(j + 2);
          ok = mbar_wait(o_bar, j & 1);  // PV_j done: V_j's buffer is free
          if (!ok) break;
          load_v(j + 2);
        }
      }
      if (!ok) {
        report_status(args.status, kStatusWaitTimeout);
        ctl.abort = 1;
        __threadfence_block();
      }
      // done_bar tracks every MMA this thread issued; TMEM and shared memory are released only
      // after it completes (and, on abort, after the last load of each stage has landed)
      mma_commit(done_bar);
      mbar_wait(done_bar, 0);
      if (!ok) {
        mbar_wait(q_bar, 0);
        for (int s = 0; s < 2; ++s) {
          if (last_k[s] >= 0) mbar_wait(smem_u32(&ctl.k_bar[s]), (last_k[s] >> 1) & 1);
          if (last_v[s] >= 0) mbar_wait(smem_u32(&ctl.v_bar[s]), (last_v[s] >> 1) & 1);
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax warps
    const int row = tid;                       // TMEM lane
    const int query = q0 + row;                // prompt-relative
    const bool row_in = capture && query >= query_lo && query < query_hi;  // a probe row
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(kHeadDim));
    float m_ref = -INFINITY;
    float l = 0.0f;
    bool ok = tiles > 0 && !skip;
    // tcgen05.ld / tcgen05.st are warp-collective (.sync.aligned): every branch around them is
    // decided uniformly per warp (__all_sync / __any_sync), never per row
    for (int j = 0; ok && j < tiles; ++j) {
      const int stage = j & 1;
      const bool ready = mbar_wait(smem_u32(&ctl.s_bar[stage]), (j >> 1) & 1, &ctl.abort) && !ctl.abort;
      if (!__all_sync(0xffffffffu, ready)) {
        ok = false;
        break;
      }
      fence_after();
      const int k0 = (tile_begin + j) * kKeys;
      float x[kKeys];
      {
        uint32_t raw[2][32];  // both 32-column loads in flight before one wait
        tmem_ld32(tmem + lane_base + stage * kKeys, raw[0]);
        tmem_ld32(tmem + lane_base + stage * kKeys + 32, raw[1]);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {  // raw scores; the log2-domain scale is folded into the exponent
          x[i] = __uint_as_float(raw[0][i]);
          x[32 + i] = __uint_as_float(raw[1][i]);
        }
      }
      const bool diagonal = k0 + kKeys - 1 > q0 || k0 + kKeys > length || args.sliding_window > 0;
      if (diagonal) {
        const int key_min = args.sliding_window > 0 ? query - args.sliding_window + 1 : 0;
        const int key_max = min(query, length - 1);
#pragma unroll
        for (int i = 0; i < kKeys; ++i) {
          const int key = k0 + i;
          if (key < key_min || key > key_max) x[i] = -INFINITY;
        }
      }
      // row max and (below) row sum with kChains independent accumulators: short dependency chains
      float m_part[kChains];
#pragma unroll
      for (int c = 0; c < kChains; ++c) m_part[c] = x[c];
#pragma unroll
      for (int i = kChains; i < kKeys; i += 2) {
        m_part[(i / 2) % kChains] = max3(m_part[(i / 2) % kChains], x[i], x[i + 1]);
      }
#pragma unroll
      for (int c = 1; c < kChains; ++c) m_part[0] = fmaxf(m_part[0], m_part[c]);
      const float m_tile = m_part[0] * scale_log2;  // the tile max in log2 units (the scale is positive)
      // the row's reference max moves when the tile max exceeds it by more than the threshold
      // (or on the row's first unmasked key); O already holds earlier tiles only when j > 0
      const bool move = m_tile > m_ref + kRescaleThreshold || (m_ref == -INFINITY && m_tile != -INFINITY);
      const bool rescale = move && j > 0 && m_ref != -INFINITY;
      if (__any_sync(0xffffffffu, rescale)) {
        // O (accumulated through PV_{j-1}) is rescaled by the whole warp, factor 1 on the rows
        // that keep their reference; S_j was issued behind PV_{j-2} and has completed, so o_bar
        // is at most one phase behind here
        const bool o_ready = mbar_wait(o_bar, (j - 1) & 1, &ctl.abort);
        if (!__all_sync(0xffffffffu, o_ready)) {
          ok = false;
          break;
        }
        fence_after();
        const float factor = rescale ? exp2f(m_ref - m_tile) : 1.0f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t raw[32];
          tmem_ld32(tmem + lane_base + kTmemO + c * 32, raw);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) raw[i] = __float_as_uint(__uint_as_float(raw[i]) * factor);
          tmem_st32(tmem + lane_base + kTmemO + c * 32, raw);
        }
        l *= factor;
        if (row_in && factor != 1.0f) {
          for (int s = 0; s < S; ++s) sigma[s * kTile + row] *= factor;
        }
      }
      if (move) m_ref = m_tile;
      const float neg_reference = m_ref == -INFINITY ? 0.0f : -m_ref;
      float sum = 0.0f;
      {
        uint32_t packed[kKeys / 2];  // 64 probabilities -> 32 TMEM columns of 16-bit pairs
        // p = 2^(s * log2(e) / sqrt(D) - m_ref): one packed FFMA per pair of scores, one ex2 each;
        // the row sum runs in kChains / 2 packed accumulators (kChains partial sums)
        unsigned long long s_pair[kChains / 2];
#pragma unroll
        for (int c = 0; c < kChains / 2; ++c) s_pair[c] = 0ull;
        const unsigned long long scale2 = pack_f32x2(scale_log2, scale_log2);
        const unsigned long long reference2 = pack_f32x2(neg_reference, neg_reference);
#pragma unroll
        for (int i = 0; i < kKeys / 2; ++i) {
          float t0, t1;
          unpack_f32x2(fma_f32x2(pack_f32x2(x[2 * i], x[2 * i + 1]), scale2, reference2), t0, t1);
          const float p0 = ex2_ftz(t0);
          const float p1 = ex2_ftz(t1);
          s_pair[i % (kChains / 2)] = add_f32x2(s_pair[i % (kChains / 2)], pack_f32x2(p0, p1));
          packed[i] = pack2<T>(p0, p1);
          x[2 * i] = p0;
          x[2 * i + 1] = p1;
        }
        tmem_st32(tmem + lane_base + stage * kKeys, packed);
#pragma unroll
        for (int c = 0; c < kChains / 2; ++c) {
          float a, b;
          unpack_f32x2(s_pair[c], a, b);
          sum += a + b;
        }
      }
      // fused mass: span sums of this tile's fp32 probabilities, by the warps that hold probe rows
      // (spans and k0 are CTA-uniform); a span that covers the whole tile takes the tile's sum
      if (S > 0 && __any_sync(0xffffffffu, row_in)) {
        for (int s = 0; s < S; ++s) {
          const int lo = max(ctl.span_lo[s], k0) - k0;
          const int hi = min(ctl.span_hi[s], k0 + kKeys) - k0;
          if (lo >= hi) continue;
          float acc = sum;
          if (lo > 0 || hi < kKeys) {
            float a_part[kChains] = {};
#pragma unroll
            for (int i = 0; i < kKeys; ++i) a_part[i % kChains] += (i >= lo && i < hi) ? x[i] : 0.0f;
            acc = 0.0f;
#pragma unroll
            for (int c = 0; c < kChains; ++c) acc += a_part[c];
          }
          if (row_in) sigma[s * kTile + row] += acc;
        }
      }
      l += sum;
      tmem_wait_st();
      fence_before();
      mbar_arrive(smem_u32(&ctl.p_bar[stage]));
    }
    // ---- epilogue: O / l -> shared (swizzled rows) -> coalesced global stores; LSE.
    // done_bar, not o_bar: PV of tile tiles-2 may still be in flight here, two phases behind.
    const bool done = __all_sync(0xffffffffu, ok && mbar_wait(done_bar, 0, &ctl.abort) && !ctl.abort);
    if (!done && tiles > 0 && !skip) {
      report_status(args.status, kStatusWaitTimeout);
      ctl.abort = 1;
    }
    fence_after();
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
    uint8_t* stage_rows = smem + kQOffset;  // the Q tile is no longer read: every MMA completed
#pragma unroll 1
    for (int c2 = 0; c2 < 2; ++c2) {  // 64 O columns per step: two TMEM loads in flight before one wait
      uint32_t raw[2][32];
      if (done) {
        tmem_ld32(tmem + lane_base + kTmemO + c2 * 64, raw[0]);
        tmem_ld32(tmem + lane_base + kTmemO + c2 * 64 + 32, raw[1]);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) raw[0][i] = raw[1][i] = 0u;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {  // four 16-byte chunks of 8 values
          float y[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) y[i] = __uint_as_float(raw[h][v * 8 + i]) * inv;
          const int chunk = (c2 * 2 + h) * 4 + v;  // 0..15 across the 256-byte row
          *reinterpret_cast<uint4*>(stage_rows + row * 256 + ((chunk ^ (row & 15)) << 4)) = pack8<T>(y);
        }
      }
    }
    if (query < length && done) {
      args.lse[static_cast<size_t>(prompt_begin + query) * args.query_heads + head] = m_ref + log2f(l);
    }
    if (S > 0) {
      // fused mass: row values = span sums / l, with the reference's per-(row, span) length divisor
      int chunk_end = length;
      if (args.normalize_by_length) {
        const int chunk = args.reference_chunk > 0 ? args.reference_chunk : length;
        chunk_end = min((query / chunk + 1) * chunk, length);
      }
      for (int s = 0; s < S; ++s) {
        float v = 0.0f;
        if (row_in && done) {
          v = sigma[s * kTile + row] * inv;
          if (args.normalize_by_length) {
            const int divisor = min(ctl.span_hi[s], chunk_end) - ctl.span_lo[s];
            if (divisor > 0) v /= static_cast<float>(divisor);
          }
        }
        v = warp_sum(v);
        if (lane == 0) ctl.warp_sums[warp][s] = v;
      }
    }
    softmax_barrier();
    if (S > 0 && tid < S) {
      const int first_tile = query_lo / kTile;
      const int query_tiles = (query_hi - 1) / kTile - first_tile + 1;
      const int item = args.mass_items[prompt] + head * query_tiles + (query_tile - first_tile);
      const float total = ctl.warp_sums[0][tid] + ctl.warp_sums[1][tid] + ctl.warp_sums[2][tid] + ctl.warp_sums[3][tid];
      args.mass_partials[static_cast<size_t>(item) * S + tid] = total;
    }
    const int out_width = args.query_heads * kHeadDim;
    T* out = static_cast<T*>(args.out);
#pragma unroll 1
    for (int i = 0; i < 16; ++i) {  // each warp writes its 32 rows, two rows per instruction
      const int r = warp * 32 + i * 2 + (lane >> 4);
      const int chunk = lane & 15;
      if (q0 + r < length) {
        const uint4 value = *reinterpret_cast<const uint4*>(stage_rows + r * 256 + ((chunk ^ (r & 15)) << 4));
        *reinterpret_cast<uint4*>(out + static_cast<size_t>(prompt_begin + q0 + r) * out_width + head * kHeadDim +
                                  chunk * 8) = value;
      }
    }
  }

  fence_before();
  __syncthreads();
  if (warp == 4) {
    __syncwarp();
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemColumns));
  }
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

template <typename T>
cudaError_t launch_typed(const AttentionArgs& a, cudaStream_t stream) {
  int device = 0;
  cudaGetDevice(&device);
  static uint64_t configured = 0;  // the shared-memory opt-in is a per-device attribute
  if (device >= 64 || !(configured & (1ull << device))) {
    const cudaError_t status = cudaFuncSetAttribute(attention_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                    static_cast<int>(smem_bytes(kMaxSpans)));
    if (status != cudaSuccess) return status;
    if (device < 64) configured |= 1ull << device;
  }
  PFN_cuTensorMapEncodeTiled_v12000 encode = encode_fn();
  if (encode == nullptr) return cudaErrorNotSupported;
  // rows beyond the batch read as zeros (the map's extent is the batch's token count)
  const int width = (a.query_heads + 2 * a.kv_heads) * kHeadDim;
  CUtensorMap map;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(a.rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(width) * 2};
  const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(kKeys)};  // 64 x 64 boxes for Q, K and V
  const cuuint32_t element_strides[2] = {1, 1};
  const CUtensorMapDataType type =
      std::is_same_v<T, __half> ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (encode(&map, type, 2, const_cast<void*>(a.qkv), dims, strides, box, element_strides,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
    return cudaErrorInvalidValue;
  }
  Args args;
  args.out = a.out;
  args.lse = a.lse;
  args.prompt_offsets = a.prompt_offsets;
  args.tiles = a.tiles;
  args.query_heads = a.query_heads;
  args.kv_heads = a.kv_heads;
  args.sliding_window = a.sliding_window;
  const uint32_t format = std::is_same_v<T, __half> ? 0u : 1u;
  args.idesc_s = idesc(format, false, kKeys);     // S = Q K^T: 128 x 64 per tile
  args.idesc_pv = idesc(format, true, kHeadDim);  // O += P V: 128 x 128
  args.status = a.status;
  args.query_spans = a.query_spans;
  args.spans = a.spans;
  args.mass_items = a.mass_items;
  args.mass_partials = a.mass_partials;
  args.span_count = a.mass_partials != nullptr ? a.span_count : 0;
  args.normalize_by_length = a.normalize_by_length;
  args.reference_chunk = a.reference_chunk;
  const dim3 grid(a.tile_count, a.query_heads);
  attention_tc_kernel<T><<<grid, kThreads, smem_bytes(args.span_count), stream>>>(map, args);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_causal_attention_tc(const AttentionArgs& args, cudaStream_t stream) {
  if (args.tile_count <= 0) return cudaSuccess;
  if (args.head_dim != kHeadDim || args.kv_heads <= 0 || args.query_heads % args.kv_heads != 0 || args.rows <= 0) {
    return cudaErrorInvalidValue;
  }
  // TMA: 16-byte aligned base; every x coordinate is a multiple of 64 elements (128 bytes)
  if ((reinterpret_cast<uintptr_t>(args.qkv) & 15) != 0) return cudaErrorInvalidValue;
  if (args.mass_partials != nullptr &&
      (args.span_count <= 0 || args.span_count > kMaxSpans || args.query_spans == nullptr || args.spans == nullptr ||
       args.mass_items == nullptr)) {
    return cudaErrorInvalidValue;
  }
  if (args.dtype == kActFp16) return launch_typed<__half>(args, stream);
  if (args.dtype == kActBf16) return launch_typed<__nv_bfloat16>(args, stream);
  return cudaErrorInvalidValue;
}

}  // namespace arb
