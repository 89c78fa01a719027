// Causal GQA prefill attention on tcgen05 / TMEM (sm_100a), packed variable-length prompts, with
// per-row log-sum-exp and the fused span-masked attention mass of the probe.
//
// Same contract as the mma.sync kernel in attention.cu (which it replaces on the engine path):
// reference semantics of LlamaForwardPass::attend (attnrank/src/model.cu:426-480) and
// softmax_causal_kernel (attnrank/src/kernels.cu:117-162); key k is visible to query q iff
// k <= q, k < prompt length and, with a sliding window, k > q - window.
//
// Persistent: one CTA per SM walks a list of work items, an item being one (prompt, 128-row query
// tile, query head), heaviest first. A CTA runs two independent lanes, each with its own item
// sequence (one item of every round of 2 * gridDim.x items, rounds taken alternately forwards and
// backwards: lane_item), its own shared-memory buffers
// and its own 256 TMEM columns; the lanes share the SM's tensor pipe, so one lane's MMAs run
// while the other lane's softmax runs, and one lane's item set-up and epilogue hide behind the
// other lane's work. 384 threads:
//   warps 0-3 / 4-7 (softmax of lane 0 / 1): thread r owns query row r = TMEM lane r. Per
//     128-key tile it reads S = Q K^T (fp32) from TMEM, masks, keeps the row's running max and
//     sum, writes P (16-bit) back into the S columns and arrives on the lane's p barrier; after
//     the item's last tile it writes O / l, the LSE and the fused mass partials.
//   warps 8 / 9 (control of lane 0 / 1): lane 0 of the warp issues every TMA load (no
//     multicast) and every tcgen05.mma of its lane and commits completions to mbarriers.
//   warps 10-11: none (they complete the third warpgroup for the register split below).
// Per lane and key tile j (Q, K, V single-buffered in shared memory, S single-buffered in TMEM):
//     S_j = Q K_j^T;  softmax_j;  O += P_j V_j  (A = P from TMEM, B = V from shared memory,
//     MN-major), then S_{j+1} right behind P_j V_j: one thread's tcgen05.mma operations execute in
//     issue order, so S_{j+1} may overwrite the TMEM columns P_j V_j reads, and the completion of
//     S_{j+1} also means that P_j V_j is done (the softmax may then rescale O without a wait).
//     K_{j+1} loads as soon as S_j completes, V_{j+1} as soon as P_j V_j completes; the next
//     item's Q and first K load during the current item's last tile.
// TMEM per lane: S [0, 128) | O [128, 256); shared memory per lane: Q | K | V, 32 KB each.
//
// Fused attention mass (optional, `mass_partials` non-null): for the query rows of the probe
// (the prompt's query span) the softmax warps also add each tile's probabilities into per-span
// sums, kept relative to the same running reference as O and l (rescaled with them) and divided
// by l at the end, so each row contributes sum_{k in span} softmax(q.k / sqrt(D)) exactly
// (reference: reduce_document_attention over softmax_causal_kernel's output, kernels.cu:202-236,
// :117-162, with the normalize_by_length divisor of kernels.cu:211). Each item writes one partial
// per span: the fixed-order sum over its rows.
// Rescaling: exponents use a reference max m_ref that moves only when the row max exceeds it by
// more than 8 (log2 units), so p <= 2^8 and the O accumulator in TMEM is rescaled rarely.
// Every mbarrier wait is bounded (time and polls); on expiry the lane records kStatusWaitTimeout
// and stops, its control thread waits (bounded) for its own MMAs and copies, and TMEM is freed
// before the CTA returns.
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
constexpr int kTile = 128;                          // query rows per item
constexpr int kKeys = 128;                          // keys per tile
constexpr int kLanes = 2;
constexpr int kLaneThreads = 128;                   // softmax threads of a lane
// + a third warpgroup: its warps 0 and 1 are the control warps of lanes 0 and 1, warps 2 and 3
// only exist so that it is a whole warpgroup for setmaxnreg
constexpr int kThreads = (kLanes + 1) * kLaneThreads;
// Registers: 384 threads start at 168 each (three warps per SM sub-partition of 16K registers);
// the control warpgroup gives registers back and the two softmax warpgroups take them, so the
// split adds up to the launch's total: 2 x 200 + 104 = 3 x 168 (both sides then run without spills).
constexpr uint32_t kSoftmaxRegisters = 200;
constexpr uint32_t kControlRegisters = 104;
static_assert(2 * kSoftmaxRegisters + kControlRegisters == 3 * 168, "register split must match the launch");
constexpr uint32_t kTmemColumns = 512;              // lane l: S [256 l, 256 l + 128) | O [256 l + 128, 256 l + 256)
constexpr uint32_t kTmemLane = 256;
constexpr uint32_t kTmemO = 128;
constexpr uint32_t kRowBytes = 128;                 // 64 16-bit values: one 128B-swizzled row of a half
constexpr uint32_t kHalfBytes = 128 * kRowBytes;    // 128 rows x 64 values (16 KB)
constexpr uint32_t kBlockBytes = 2 * kHalfBytes;    // 128 rows x 128 values: a Q, K or V block
constexpr uint32_t kLaneBytes = 3 * kBlockBytes;    // Q | K | V
constexpr uint32_t kSpinLimit = 1u << 26;           // hard backstop on polls per wait
constexpr uint64_t kWaitLimitNs = 500ull * 1000 * 1000;  // a wait gives up after 0.5 s
constexpr float kRescaleThreshold = 8.0f;           // log2 units
constexpr int kChains = 4;                          // independent accumulators per row reduction
constexpr int kMaxSpans = kMassMaxSpans;

struct __align__(16) LaneControl {
  uint64_t q_bar;
  uint64_t k_bar;
  uint64_t v_bar;
  uint64_t s_bar;     // S_j completed (and with it every earlier MMA of the lane)
  uint64_t o_bar;     // P_j V_j completed
  uint64_t p_bar;     // the lane's 128 softmax threads wrote P_j
  uint64_t done_bar;  // every MMA of the lane completed (one commit when the lane stops)
  volatile int abort;
  int span_lo[kMaxSpans];  // fused mass: the current item's document spans
  int span_hi[kMaxSpans];
  float warp_sums[4][kMaxSpans];
};
struct __align__(16) Control {
  LaneControl lane[kLanes];
  uint32_t tmem_base;
};
// dynamic shared memory: lanes' Q | K | V blocks, the control block, then (fused mass only)
// float sigma[lane][span_count][128]
constexpr size_t kControlOffset = kLanes * kLaneBytes;
constexpr size_t kSigmaOffset = kControlOffset + ((sizeof(Control) + 15) & ~size_t(15));
constexpr size_t smem_bytes(int span_count) {
  return kSigmaOffset + static_cast<size_t>(kLanes) * span_count * kTile * 4 + 1024;  // + alignment slack
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
// dim) values of one K (key); 8 rows form a 1024-byte atom; the two 64-wide N halves are 16 KB
// apart (leading byte offset), consecutive 8-key groups 1024 bytes apart (stride byte offset).
__device__ __forceinline__ uint64_t desc_mn_major(uint32_t address) {
  return static_cast<uint64_t>((address >> 4) & 0x3FFFu) | (static_cast<uint64_t>(kHalfBytes >> 4) << 16) |
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
__device__ __forceinline__ void tmem_st16(uint32_t address, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(address), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
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
  const int32_t* tiles;  // (prompt, query tile) pairs, heaviest first
  int item_count;        // tile pairs x query heads
  int query_heads;
  int kv_heads;
  int sliding_window;
  uint32_t idesc_s;
  uint32_t idesc_pv;
  int* status;
  // fused mass (mass_partials == nullptr: attention only)
  const int32_t* query_spans;  // [prompts][2], prompt-relative
  const int32_t* spans;        // [prompts][span_count][2]
  const int32_t* mass_items;   // [prompts + 1] partial slots per prompt: Hq x query tiles in the span x 4 warps
  float* mass_partials;        // [slots][span_count]
  int span_count;
  int normalize_by_length;
  int reference_chunk;
};

// One work item: a (prompt, query tile) pair of the tile list and a query head. Work index i is
// tile pair i / Hq and head i % Hq, so the heaviest tiles of every head come first.
struct Item {
  int prompt;
  int query_tile;
  int head;
  int kv_head;
  int prompt_begin;
  int length;
  int q0;          // first query row (prompt-relative)
  int tile_begin;  // first 128-key tile
  int tiles;       // 128-key tiles [tile_begin, tile_begin + tiles), at least one
};

// Work index of a lane's round-th item: rounds of 2 * gridDim.x consecutive items of the
// heaviest-first list, taken forwards on even rounds and backwards on odd ones, so that the lanes
// that take the heaviest item of one round take the lightest of the next.
__device__ __forceinline__ int lane_item(int slot, int round, int lanes_total) {
  return round * lanes_total + ((round & 1) ? lanes_total - 1 - slot : slot);
}

__device__ __forceinline__ Item decode_item(const Args& args, int index) {
  Item it;
  const int pair = index / args.query_heads;
  it.head = index - pair * args.query_heads;
  it.prompt = args.tiles[2 * pair];
  it.query_tile = args.tiles[2 * pair + 1];
  it.kv_head = it.head / (args.query_heads / args.kv_heads);
  it.prompt_begin = args.prompt_offsets[it.prompt];
  it.length = args.prompt_offsets[it.prompt + 1] - it.prompt_begin;
  it.q0 = it.query_tile * kTile;
  const int last_query = min(it.q0 + kTile, it.length) - 1;  // the tile list holds tiles with q0 < length
  const int first_key = args.sliding_window > 0 ? max(0, it.q0 - args.sliding_window + 1) : 0;
  it.tile_begin = first_key / kKeys;
  it.tiles = last_query / kKeys + 1 - it.tile_begin;
  return it;
}

// ---------------------------------------------------------------------------------------------
// control thread of one lane: TMA loads and tcgen05.mma issue
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void control_lane(const CUtensorMap* map, const Args& args, LaneControl& lc,
                                             uint32_t q_smem, uint32_t tmem, int slot, int lanes_total) {
  const uint32_t k_smem = q_smem + kBlockBytes;
  const uint32_t v_smem = q_smem + 2 * kBlockBytes;
  const uint32_t q_bar = smem_u32(&lc.q_bar);
  const uint32_t k_bar = smem_u32(&lc.k_bar);
  const uint32_t v_bar = smem_u32(&lc.v_bar);
  const uint32_t s_bar = smem_u32(&lc.s_bar);
  const uint32_t o_bar = smem_u32(&lc.o_bar);
  const uint32_t p_bar = smem_u32(&lc.p_bar);
  const uint32_t done_bar = smem_u32(&lc.done_bar);
  // loads issued and completions waited for per barrier: at most one load per block is in flight
  int q_issued = 0, k_issued = 0, v_issued = 0;
  int q_seen = 0, k_seen = 0, v_seen = 0;
  auto load_block = [&](uint32_t dst, int x, int y, uint32_t bar) {
    mbar_expect_tx(bar, kBlockBytes);
    tma_load_2d(dst, map, x, y, bar);
    tma_load_2d(dst + kHalfBytes, map, x + 64, y, bar);
  };
  auto load_q = [&](const Item& it) {
    load_block(q_smem, it.head * kHeadDim, it.prompt_begin + it.q0, q_bar);
    ++q_issued;
  };
  auto load_k = [&](const Item& it, int j) {
    load_block(k_smem, (args.query_heads + it.kv_head) * kHeadDim, it.prompt_begin + (it.tile_begin + j) * kKeys,
               k_bar);
    ++k_issued;
  };
  auto load_v = [&](const Item& it, int j) {
    load_block(v_smem, (args.query_heads + args.kv_heads + it.kv_head) * kHeadDim,
               it.prompt_begin + (it.tile_begin + j) * kKeys, v_bar);
    ++v_issued;
  };
  auto issue_s = [&]() {  // S = Q K^T, 128 x 128, 16 head-dim values (32 bytes of a row) per MMA
    fence_after();
#pragma unroll
    for (int kk = 0; kk < kHeadDim / 16; ++kk) {
      const uint32_t offset = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
      mma_ss(tmem, desc_k_major(q_smem + offset), desc_k_major(k_smem + offset), args.idesc_s, kk > 0 ? 1u : 0u);
    }
    mma_commit(s_bar);
  };
  auto issue_pv = [&](bool accumulate) {  // O += P V, 16 keys (8 packed TMEM columns of P) per MMA
    fence_after();
#pragma unroll
    for (int kk = 0; kk < kKeys / 16; ++kk) {
      mma_ts(tmem + kTmemO, tmem + kk * 8, desc_mn_major(v_smem + kk * 16 * kRowBytes), args.idesc_pv,
             (accumulate || kk > 0) ? 1u : 0u);
    }
    mma_commit(o_bar);
  };

  bool ok = lc.abort == 0;
  bool issued_mma = false;
  bool prefetched = false;
  int tile_no = 0;  // tiles of this lane so far: the phase counter of the s, p and o barriers
  for (int round = 0; ok; ++round) {
    const int index = lane_item(slot, round, lanes_total);
    if (index >= args.item_count) break;
    const Item it = decode_item(args, index);
    if (!prefetched) {
      load_q(it);
      load_k(it, 0);
    }
    prefetched = false;
    ok = mbar_wait(q_bar, q_seen++ & 1);
    ok = mbar_wait(k_bar, k_seen++ & 1) && ok;
    if (!ok) break;
    issue_s();  // behind the previous item's last P.V, which reads the TMEM columns S_0 overwrites
    issued_mma = true;
    if (tile_no > 0) {  // the V block is free once the previous item's last P.V completed
      ok = mbar_wait(o_bar, (tile_no - 1) & 1);
      if (!ok) break;
    }
    load_v(it, 0);
    for (int j = 0; j < it.tiles; ++j) {
      const int t = tile_no + j;
      ok = mbar_wait(s_bar, t & 1);  // S_j done: the K block is free (on the last tile, the Q block too)
      if (!ok) break;
      if (j + 1 < it.tiles) {
        load_k(it, j + 1);
      } else if (lane_item(slot, round + 1, lanes_total) < args.item_count) {
        const Item next = decode_item(args, lane_item(slot, round + 1, lanes_total));
        load_q(next);
        load_k(next, 0);
        prefetched = true;
      }
      ok = mbar_wait(p_bar, t & 1, &lc.abort);  // the softmax wrote P_j
      ok = ok && mbar_wait(v_bar, v_seen++ & 1);
      if (!ok) break;
      issue_pv(j > 0);
      if (j + 1 < it.tiles) {
        ok = mbar_wait(k_bar, k_seen++ & 1);
        if (!ok) break;
        issue_s();  // behind P_j V_j, which reads the TMEM columns S_{j+1} overwrites
        ok = mbar_wait(o_bar, t & 1);  // P_j V_j done: the V block is free
        if (!ok) break;
        load_v(it, j + 1);
      }
    }
    tile_no += it.tiles;
  }
  if (!ok) {
    report_status(args.status, kStatusWaitTimeout);
    lc.abort = 1;
    __threadfence_block();
  }
  // TMEM and shared memory are released only after every MMA of the lane completed and every
  // load it issued landed
  if (issued_mma) {
    mma_commit(done_bar);
    mbar_wait(done_bar, 0);
  }
  if (q_issued > q_seen) mbar_wait(q_bar, (q_issued - 1) & 1);
  if (k_issued > k_seen) mbar_wait(k_bar, (k_issued - 1) & 1);
  if (v_issued > v_seen) mbar_wait(v_bar, (v_issued - 1) & 1);
}

// ---------------------------------------------------------------------------------------------
// softmax threads of one lane (thread `row` owns TMEM lane `row`)
// ---------------------------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void softmax_lane(const Args& args, LaneControl& lc, float* sigma, uint32_t tmem,
                                             int row, int slot, int lanes_total) {
  const int warp = row >> 5;  // warp of the lane = TMEM lane quadrant
  const int lane_id = row & 31;
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t s_bar = smem_u32(&lc.s_bar);
  const uint32_t o_bar = smem_u32(&lc.o_bar);
  const uint32_t p_bar = smem_u32(&lc.p_bar);
  const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(kHeadDim));
  const int S = args.mass_partials != nullptr ? args.span_count : 0;
  const int out_width = args.query_heads * kHeadDim;
  T* out = static_cast<T*>(args.out);
  bool ok = lc.abort == 0;
  int tile_no = 0;
  // tcgen05.ld / tcgen05.st are warp-collective (.sync.aligned): every branch around them is
  // decided uniformly per warp (__all_sync / __any_sync), never per row. No barrier spans the
  // lane's warps, so a warp that stops early cannot hold the others.
  for (int round = 0; ok; ++round) {
    const int index = lane_item(slot, round, lanes_total);
    if (index >= args.item_count) break;
    const Item it = decode_item(args, index);
    const int query = it.q0 + row;  // prompt-relative
    // fused mass: does this item hold rows of the probe's query span?
    int query_lo = 0, query_hi = 0;
    if (S > 0) {
      query_lo = max(args.query_spans[2 * it.prompt], 0);
      query_hi = min(args.query_spans[2 * it.prompt + 1], it.length);
    }
    const bool capture = S > 0 && query_hi > query_lo && it.q0 < query_hi && it.q0 + kTile > query_lo;
    const bool row_in = capture && query >= query_lo && query < query_hi;
    const int32_t* item_spans = S > 0 ? args.spans + 2 * static_cast<size_t>(it.prompt) * S : nullptr;
    if (row_in) {
      for (int s = 0; s < S; ++s) sigma[s * kTile + row] = 0.0f;
    }
    float m_ref = -INFINITY;
    float l = 0.0f;
    for (int j = 0; j < it.tiles; ++j) {
      const int t = tile_no + j;
      const bool ready = mbar_wait(s_bar, t & 1, &lc.abort) && !lc.abort;
      if (!__all_sync(0xffffffffu, ready)) {
        ok = false;
        break;
      }
      fence_after();
      const int k0 = (it.tile_begin + j) * kKeys;
      float x[kKeys];
      {
        uint32_t raw[4][32];  // all four 32-column loads in flight before one wait
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tmem + lane_base + c * 32, raw[c]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int i = 0; i < 32; ++i) x[c * 32 + i] = __uint_as_float(raw[c][i]);
        }
      }
      const bool diagonal = k0 + kKeys - 1 > it.q0 || k0 + kKeys > it.length || args.sliding_window > 0;
      if (diagonal) {
        const int key_min = args.sliding_window > 0 ? query - args.sliding_window + 1 : 0;
        const int key_max = min(query, it.length - 1);
#pragma unroll
        for (int i = 0; i < kKeys; ++i) {
          const int key = k0 + i;
          if (key < key_min || key > key_max) x[i] = -INFINITY;
        }
      }
      // row max with kChains independent accumulators (short dependency chains)
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
      // (or on the row's first unmasked key); O holds earlier tiles only when j > 0
      const bool move = m_tile > m_ref + kRescaleThreshold || (m_ref == -INFINITY && m_tile != -INFINITY);
      const bool rescale = move && j > 0 && m_ref != -INFINITY;
      if (__any_sync(0xffffffffu, rescale)) {
        // S_j completed, so every earlier P.V of the lane did too: O is stable. The whole warp
        // takes part; rows that keep their reference scale by 1.
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
        // p = 2^(s * log2(e) / sqrt(D) - m_ref): one packed FFMA per pair of scores, one ex2 each;
        // 32 probabilities -> 16 TMEM columns of 16-bit pairs per store
        unsigned long long s_pair[kChains / 2];
#pragma unroll
        for (int c = 0; c < kChains / 2; ++c) s_pair[c] = 0ull;
        const unsigned long long scale2 = pack_f32x2(scale_log2, scale_log2);
        const unsigned long long reference2 = pack_f32x2(neg_reference, neg_reference);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t packed[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int a = c * 32 + 2 * i;
            float t0, t1;
            unpack_f32x2(fma_f32x2(pack_f32x2(x[a], x[a + 1]), scale2, reference2), t0, t1);
            const float p0 = ex2_ftz(t0);
            const float p1 = ex2_ftz(t1);
            s_pair[i % (kChains / 2)] = add_f32x2(s_pair[i % (kChains / 2)], pack_f32x2(p0, p1));
            packed[i] = pack2<T>(p0, p1);
            x[a] = p0;
            x[a + 1] = p1;
          }
          tmem_st16(tmem + lane_base + c * 16, packed);
        }
#pragma unroll
        for (int c = 0; c < kChains / 2; ++c) {
          float a, b;
          unpack_f32x2(s_pair[c], a, b);
          sum += a + b;
        }
      }
      // fused mass: span sums of this tile's fp32 probabilities, by the warps that hold probe rows
      // (spans and k0 are item-uniform); a span that covers the whole tile takes the tile's sum
      if (capture && __any_sync(0xffffffffu, row_in)) {
        for (int s = 0; s < S; ++s) {
          const int lo = max(max(__ldg(item_spans + 2 * s), 0), k0) - k0;
          const int hi = min(__ldg(item_spans + 2 * s + 1), k0 + kKeys) - k0;
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
      mbar_arrive(p_bar);
    }
    if (!ok) break;
    // ---- epilogue: O / l straight from TMEM to global memory (one 256-byte row per thread), LSE,
    // the fused mass partial of each warp. The item's last P.V is the o barrier's next phase: no
    // later P.V can start before this lane's softmax threads write the next item's first P.
    const bool done = mbar_wait(o_bar, (tile_no + it.tiles - 1) & 1, &lc.abort) && !lc.abort;
    if (!__all_sync(0xffffffffu, done)) {
      ok = false;
      break;
    }
    fence_after();
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
    {
      uint32_t raw[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tmem + lane_base + kTmemO + c * 32, raw[c]);
      tmem_wait_ld();
      if (query < it.length) {
        T* out_row = out + static_cast<size_t>(it.prompt_begin + query) * out_width + it.head * kHeadDim;
#pragma unroll
        for (int v = 0; v < 16; ++v) {
          float y[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) y[i] = __uint_as_float(raw[v >> 2][(v & 3) * 8 + i]) * inv;
          *reinterpret_cast<uint4*>(out_row + v * 8) = pack8<T>(y);
        }
        args.lse[static_cast<size_t>(it.prompt_begin + query) * args.query_heads + it.head] = m_ref + log2f(l);
      }
    }
    if (capture) {
      // row values = span sums / l, with the reference's per-(row, span) length divisor; each
      // warp writes the fixed-order sum over its 32 rows into its own partial slot
      int chunk_end = it.length;
      if (args.normalize_by_length) {
        const int chunk = args.reference_chunk > 0 ? args.reference_chunk : it.length;
        chunk_end = min((query / chunk + 1) * chunk, it.length);
      }
      const int first_tile = query_lo / kTile;
      const int query_tiles = (query_hi - 1) / kTile - first_tile + 1;
      const int slot = (args.mass_items[it.prompt] +
                        (it.head * query_tiles + (it.query_tile - first_tile)) * kFusedMassSlotsPerTile) + warp;
      for (int s = 0; s < S; ++s) {
        float v = 0.0f;
        if (row_in) {
          v = sigma[s * kTile + row] * inv;
          if (args.normalize_by_length) {
            const int lo = max(__ldg(item_spans + 2 * s), 0);
            const int divisor = min(__ldg(item_spans + 2 * s + 1), chunk_end) - lo;
            if (divisor > 0) v /= static_cast<float>(divisor);
          }
        }
        v = warp_sum(v);
        if (lane_id == 0) args.mass_partials[static_cast<size_t>(slot) * S + s] = v;
      }
    }
    tile_no += it.tiles;
  }
  if (!ok) {
    report_status(args.status, kStatusWaitTimeout);
    lc.abort = 1;
    __threadfence_block();
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap map, const Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Control& ctl = *reinterpret_cast<Control*>(smem + kControlOffset);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const bool softmax = warp < kLanes * 4;
  const int lane = softmax ? warp / 4 : min(warp - kLanes * 4, kLanes - 1);  // warps 10, 11: no role
  const int slot = blockIdx.x * kLanes + lane;  // the lane's place in every round of items
  const int lanes_total = gridDim.x * kLanes;

  if (tid == 0) {
    // a CTA of a launch that already reported an error does no work (bounds a failing launch to
    // one wave of timed-out lanes); read once here so that the whole CTA agrees
    const int abort = (args.status != nullptr && *reinterpret_cast<volatile int*>(args.status) != 0) ? 1 : 0;
    for (int l = 0; l < kLanes; ++l) {
      LaneControl& c = ctl.lane[l];
      mbar_init(smem_u32(&c.q_bar), 1);
      mbar_init(smem_u32(&c.k_bar), 1);
      mbar_init(smem_u32(&c.v_bar), 1);
      mbar_init(smem_u32(&c.s_bar), 1);
      mbar_init(smem_u32(&c.o_bar), 1);
      mbar_init(smem_u32(&c.p_bar), kLaneThreads);
      mbar_init(smem_u32(&c.done_bar), 1);
      c.abort = abort;
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kLanes * 4) {
    __syncwarp();
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&ctl.tmem_base)),
                 "r"(kTmemColumns));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = ctl.tmem_base + lane * kTmemLane;  // the lane's first column (TMEM lane 0)
  LaneControl& lc = ctl.lane[lane];
  const uint32_t q_smem = smem_u32(smem + lane * kLaneBytes);
  const int S = args.mass_partials != nullptr ? args.span_count : 0;
  float* sigma = reinterpret_cast<float*>(smem + kSigmaOffset) + static_cast<size_t>(lane) * S * kTile;

  if (!softmax) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kControlRegisters));
    if (warp < kLanes * 4 + kLanes && (tid & 31) == 0) {
      control_lane(&map, args, lc, q_smem, tmem, slot, lanes_total);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegisters));
    softmax_lane<T>(args, lc, sigma, tmem, tid - lane * kLaneThreads, slot, lanes_total);
  }

  fence_before();
  __syncthreads();
  if (warp == kLanes * 4) {
    __syncwarp();
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(ctl.tmem_base), "r"(kTmemColumns));
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
  const size_t smem = smem_bytes(a.mass_partials != nullptr ? a.span_count : 0);
  static uint64_t configured = 0;  // the shared-memory opt-in is a per-device attribute
  if (device >= 64 || !(configured & (1ull << device))) {
    int limit = 0;
    cudaDeviceGetAttribute(&limit, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    if (static_cast<size_t>(limit) < smem_bytes(kMaxSpans)) return cudaErrorInvalidConfiguration;
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
  const cuuint32_t box[2] = {64, 128};  // 64 columns (128 bytes, one swizzle row) x 128 rows: half a block
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
  args.item_count = a.tile_count * a.query_heads;
  args.query_heads = a.query_heads;
  args.kv_heads = a.kv_heads;
  args.sliding_window = a.sliding_window;
  const uint32_t format = std::is_same_v<T, __half> ? 0u : 1u;
  args.idesc_s = idesc(format, false, kKeys);     // S = Q K^T: 128 x 128 per tile
  args.idesc_pv = idesc(format, true, kHeadDim);  // O += P V: 128 x 128
  args.status = a.status;
  args.query_spans = a.query_spans;
  args.spans = a.spans;
  args.mass_items = a.mass_items;
  args.mass_partials = a.mass_partials;
  args.span_count = a.mass_partials != nullptr ? a.span_count : 0;
  args.normalize_by_length = a.normalize_by_length;
  args.reference_chunk = a.reference_chunk;
  // persistent: one CTA per SM (its shared memory admits no second), two lanes of items each
  const int grid = std::max(1, std::min(sm_count(), (args.item_count + kLanes - 1) / kLanes));
  attention_tc_kernel<T><<<grid, kThreads, smem, stream>>>(map, args);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_causal_attention_tc(const AttentionArgs& args, cudaStream_t stream) {
  if (args.tile_count <= 0) return cudaSuccess;
  if (args.head_dim != kHeadDim || args.kv_heads <= 0 || args.query_heads % args.kv_heads != 0 || args.rows <= 0) {
    return cudaErrorInvalidValue;
  }
  if (static_cast<long long>(args.tile_count) * args.query_heads >= (1LL << 31)) return cudaErrorInvalidValue;
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
