// Single-token decode kernels (declarations and the reference mapping in decode.h).
//
// Matrix-vector products (decode_gemv_kernel): a CTA of 8 warps works on kItems = 8 / kSplit
// items (2 or 4 weight rows each); the kSplit warps of an item take equal slices of the K range,
// so a warp's chain of dependent loads is short, and their partial sums meet in shared memory in
// a fixed order. A lane keeps 8 or 16 16-byte streaming loads (ld.global.nc.L1::no_allocate)
// outstanding before its first FMA (kInFlight). Before waiting for its producer a CTA sends its first
// slice of weights towards L2 (cp.async.bulk.prefetch.L2), since weights never depend on the
// previous kernel; x is then staged in shared memory once per CTA (or built there by the fused
// RMSNorm prologue). Accumulation is fp32; 16-bit outputs are rounded once.
#include <cfloat>
#include <climits>
#include <cstdlib>

#include "common.cuh"
#include "decode.h"
#include "layer_kernels.h"

namespace arb {

int sm_count();

namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kNormVpt = kDecodeMaxNormHidden / (kGemvThreads * 8);  // 8-value chunks per thread
constexpr int kDecodeThreads = 256;
constexpr int kDecodeKeys = 64;    // keys staged in shared memory per pass
constexpr int kDecodeDim = 128;    // head_dim the decode attention is written for
constexpr int kKeyStride = kDecodeDim + 8;  // padded K row (halves): 16-byte reads of 8 rows hit 32 banks

template <typename T>
struct Scalar;
template <>
struct Scalar<__half> {
  static __device__ __forceinline__ __half from(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float to(__half v) { return __half2float(v); }
};
template <>
struct Scalar<__nv_bfloat16> {
  static __device__ __forceinline__ __nv_bfloat16 from(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float to(__nv_bfloat16 v) { return __bfloat162float(v); }
};

// v rounded to the 16-bit type and back
template <typename T>
__device__ __forceinline__ float round16(float v) {
  return Scalar<T>::to(Scalar<T>::from(v));
}

// Programmatic dependent launch: wait until the preceding kernel on the stream has completed and
// its writes are visible (a no-op for kernels launched without the attribute) ...
__device__ __forceinline__ void wait_for_producer() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// ... and let the next kernel on the stream be scheduled while this one runs.
__device__ __forceinline__ void release_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void prefetch_l2(const void* address, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(__cvta_generic_to_global(address)), "r"(bytes)
               : "memory");
}

// larger value first; equal values: the smaller index (the first maximum)
__device__ __forceinline__ bool better(float value, int index, float than_value, int than_index) {
  return value > than_value || (value == than_value && index < than_index);
}

template <int kKind>
struct GemvShape {
  static constexpr int kRows = (kKind == kDecodeGateUp || kKind == kDecodeQkv) ? 4 : 2;
};

template <int kKind>
__device__ __forceinline__ int item_count(const DecodeGemvArgs& a) {
  if constexpr (kKind == kDecodeQkv) return a.rows / 4;
  return (a.rows + 1) / 2;
}

// Weight rows of work item `item`.
//   plain / logits: 2i, 2i + 1;  gate|up: gate rows 2i, 2i + 1 and their up rows inter + 2i, +1;
//   q|k|v: for query and key heads the rotation pairs (2j, 2j + D/2), (2j + 1, 2j + 1 + D/2) of
//   head h, for value heads rows 4j .. 4j + 3 (item = h * D/4 + j).
// A row past the end repeats the last row; its result is not stored.
template <int kKind>
__device__ __forceinline__ void item_rows(const DecodeGemvArgs& a, int item, int (&row)[GemvShape<kKind>::kRows]) {
  if constexpr (kKind == kDecodePlain || kKind == kDecodeLogits) {
    row[0] = 2 * item;
    row[1] = min(2 * item + 1, a.rows - 1);
  } else if constexpr (kKind == kDecodeGateUp) {
    const int j0 = 2 * item;
    const int j1 = min(j0 + 1, a.rows - 1);
    row[0] = j0;
    row[1] = j1;
    row[2] = a.rows + j0;
    row[3] = a.rows + j1;
  } else {
    const int per_head = a.head_dim >> 2;
    const int head = item / per_head;
    const int j = item - head * per_head;
    if (head < a.query_heads + a.kv_heads) {
      row[0] = head * a.head_dim + 2 * j;
      row[1] = row[0] + 1;
      row[2] = row[0] + (a.head_dim >> 1);
      row[3] = row[2] + 1;
    } else {
#pragma unroll
      for (int r = 0; r < 4; ++r) row[r] = head * a.head_dim + 4 * j + r;
    }
  }
}

// x into shared memory: copied, or built by the RMSNorm prologue (the formula of the engine's
// rms_norm_residual_kernel: v = residual + delta, y = v * rsqrt(sum(v^2) / k + eps) * gamma), where
// v may also be the embedding row of the step's token (embed_rms_norm_kernel's formula; an id out
// of range gives a zero row and a status, as there). Block 0 keeps v in residual_out.
template <typename T>
__device__ __forceinline__ void stage_x(const DecodeGemvArgs& a, uint4* xs, float* scratch, int block) {
  const int chunks = a.k >> 3;
  if (a.residual_in == nullptr && a.embed_table == nullptr) {
    const T* x = static_cast<const T*>(a.x);
    for (int i = threadIdx.x; i < chunks; i += kGemvThreads) {
      xs[i] = __ldcg(reinterpret_cast<const uint4*>(x + 8 * static_cast<size_t>(i)));
    }
    __syncthreads();
    return;
  }
  const T* delta = static_cast<const T*>(a.delta);
  const T* embedded = nullptr;
  if (a.embed_table != nullptr) {
    const int token = __ldcg(a.state);
    if (token >= 0 && token < a.vocab) {
      embedded = static_cast<const T*>(a.embed_table) + static_cast<size_t>(token) * a.k;
    } else if (block == 0 && threadIdx.x == 0) {
      report_status(a.status, kStatusTokenOutOfRange);
    }
  }
  float values[kNormVpt][8];
  float squares = 0.0f;
#pragma unroll
  for (int v = 0; v < kNormVpt; ++v) {
    const int chunk = threadIdx.x + v * kGemvThreads;
    if (chunk < chunks && a.embed_table != nullptr) {
      if (embedded != nullptr) {
        unpack8<T>(load_nc(embedded + 8 * chunk), values[v]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) values[v][i] = 0.0f;
      }
    } else if (chunk < chunks) {
      const float4 r0 = __ldcg(reinterpret_cast<const float4*>(a.residual_in + 8 * chunk));
      const float4 r1 = __ldcg(reinterpret_cast<const float4*>(a.residual_in + 8 * chunk + 4));
      float d[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
      if (delta != nullptr) unpack8<T>(__ldcg(reinterpret_cast<const uint4*>(delta + 8 * chunk)), d);
      values[v][0] = r0.x + d[0];
      values[v][1] = r0.y + d[1];
      values[v][2] = r0.z + d[2];
      values[v][3] = r0.w + d[3];
      values[v][4] = r1.x + d[4];
      values[v][5] = r1.y + d[5];
      values[v][6] = r1.z + d[6];
      values[v][7] = r1.w + d[7];
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) values[v][i] = 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) squares += values[v][i] * values[v][i];
  }
  const float total = block_sum(squares, scratch);
  const float scale = rsqrtf(total / static_cast<float>(a.k) + a.eps);
  const bool keep = a.residual_out != nullptr && block == 0;
#pragma unroll
  for (int v = 0; v < kNormVpt; ++v) {
    const int chunk = threadIdx.x + v * kGemvThreads;
    if (chunk >= chunks) continue;
    const float4 g0 = __ldg(reinterpret_cast<const float4*>(a.gamma + 8 * chunk));
    const float4 g1 = __ldg(reinterpret_cast<const float4*>(a.gamma + 8 * chunk + 4));
    const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    if (keep) {
      float4* out = reinterpret_cast<float4*>(a.residual_out + 8 * chunk);
      out[0] = make_float4(values[v][0], values[v][1], values[v][2], values[v][3]);
      out[1] = make_float4(values[v][4], values[v][5], values[v][6], values[v][7]);
    }
    float y[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = values[v][i] * scale * g[i];
    xs[chunk] = pack8<T>(y);
  }
  __syncthreads();
}

// acc[r] = rows[r][8 c] . x over chunks c in [begin, end), summed over the warp (all lanes);
// kInFlight 16-byte weight loads per lane are issued before the first FMA of a batch
template <typename T, int kRows, int kInFlight>
__device__ __forceinline__ void warp_dot_range(const T* (&rows)[kRows], const uint4* __restrict__ xs, int begin,
                                               int end, float (&acc)[kRows]) {
  constexpr int kUnroll = kInFlight / kRows;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int r = 0; r < kRows; ++r) acc[r] = 0.0f;
  int c = begin + lane;
  for (; c + 32 * (kUnroll - 1) < end; c += 32 * kUnroll) {
    uint4 w[kRows][kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
#pragma unroll
      for (int r = 0; r < kRows; ++r) w[r][u] = load_stream(rows[r] + 8 * static_cast<size_t>(c + 32 * u));
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      float xv[8];
      unpack8<T>(xs[c + 32 * u], xv);
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        float wv[8];
        unpack8<T>(w[r][u], wv);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[r] = fmaf(wv[i], xv[i], acc[r]);
      }
    }
  }
  for (; c < end; c += 32) {
    float xv[8];
    unpack8<T>(xs[c], xv);
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      float wv[8];
      unpack8<T>(load_stream(rows[r] + 8 * static_cast<size_t>(c)), wv);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[r] = fmaf(wv[i], xv[i], acc[r]);
    }
  }
#pragma unroll
  for (int r = 0; r < kRows; ++r) acc[r] = warp_sum(acc[r]);
}

// Epilogue of one item (lane 0 of the item's first warp); `best` tracks the greedy pick.
template <typename T, int kKind>
__device__ __forceinline__ void finish_item(const DecodeGemvArgs& a, int item, const float (&sum)[GemvShape<kKind>::kRows],
                                            float& best, int& best_at) {
  if constexpr (kKind == kDecodePlain || kKind == kDecodeLogits) {
    const int r0 = 2 * item;
    const bool pair = r0 + 1 < a.rows;
    if constexpr (kKind == kDecodeLogits) {
      float* out = static_cast<float*>(a.y);
      out[r0] = sum[0];
      if (pair) out[r0 + 1] = sum[1];
      if (sum[0] > best) {
        best = sum[0];
        best_at = r0;
      }
      if (pair && sum[1] > best) {
        best = sum[1];
        best_at = r0 + 1;
      }
    } else {
      T* out = static_cast<T*>(a.y);
      if (pair) {
        *reinterpret_cast<uint32_t*>(out + r0) = pack2<T>(sum[0], sum[1]);
      } else {
        out[r0] = Scalar<T>::from(sum[0]);
      }
    }
  } else if constexpr (kKind == kDecodeGateUp) {
    // silu(g) * u = g / (1 + e^-g) * u on the 16-bit projections, as the prefill's SwiGLU kernel
    const int j0 = 2 * item;
    const bool pair = j0 + 1 < a.rows;
    float value[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float g = round16<T>(sum[i]);
      const float u = round16<T>(sum[2 + i]);
      value[i] = __fdividef(g, 1.0f + __expf(-g)) * u;
    }
    T* out = static_cast<T*>(a.y);
    if (pair) {
      *reinterpret_cast<uint32_t*>(out + j0) = pack2<T>(value[0], value[1]);
    } else {
      out[j0] = Scalar<T>::from(value[0]);
    }
  }
}

// Operands of a q|k|v item's epilogue (bias, rotation), loaded before its dot products so that
// their latency hides behind the weight stream.
struct QkvOperands {
  float bias_half[4];
  float bias[4];
  float c0, c1, s0, s1;
};

template <typename T>
__device__ __forceinline__ void load_qkv_operands(const DecodeGemvArgs& a, int item, int position, QkvOperands& o) {
  int row[4];
  item_rows<kDecodeQkv>(a, item, row);
  const T* bias_half = static_cast<const T*>(a.bias_half);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    o.bias_half[r] = bias_half != nullptr ? Scalar<T>::to(bias_half[row[r]]) : 0.0f;
    o.bias[r] = a.bias != nullptr ? a.bias[row[r]] : 0.0f;
  }
  o.c0 = o.c1 = 1.0f;
  o.s0 = o.s1 = 0.0f;
  const int per_head = a.head_dim >> 2;
  const int head = item / per_head;
  const int j = item - head * per_head;
  if (head < a.query_heads + a.kv_heads && position >= 0 && position < a.table_positions) {
    const size_t at = static_cast<size_t>(position) * (a.head_dim >> 1) + 2 * j;
    o.c0 = a.cos_table[at];
    o.c1 = a.cos_table[at + 1];
    o.s0 = a.sin_table[at];
    o.s1 = a.sin_table[at + 1];
  }
}

// q|k|v epilogue: bias where the prefill adds it, RoPE on query and key heads (the prefill's
// rotary expression), the query to q_out, key and value rows to the cache at `position`.
template <typename T>
__device__ __forceinline__ void finish_qkv(const DecodeGemvArgs& a, int item, int position, const float (&sum)[4],
                                           const QkvOperands& o) {
  const int D = a.head_dim;
  const int half = D >> 1;
  const int per_head = D >> 2;
  const int head = item / per_head;
  const int j = item - head * per_head;
  const int rotated = a.query_heads + a.kv_heads;
  if (position < 0 || position >= a.table_positions || position >= a.context) return;  // reported once per launch
  float v[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    float value = sum[r];
    if (a.bias_half != nullptr) value += o.bias_half[r];
    value = round16<T>(value);
    if (a.bias != nullptr) value += o.bias[r];
    v[r] = value;
  }
  if (head < rotated) {
    const float lo0 = v[0] * o.c0 - v[2] * o.s0;
    const float hi0 = v[2] * o.c0 + v[0] * o.s0;
    const float lo1 = v[1] * o.c1 - v[3] * o.s1;
    const float hi1 = v[3] * o.c1 + v[1] * o.s1;
    T* dst = head < a.query_heads
                 ? static_cast<T*>(a.q_out) + static_cast<size_t>(head) * D
                 : static_cast<T*>(a.k_cache) + (static_cast<size_t>(head - a.query_heads) * a.context + position) * D;
    *reinterpret_cast<uint32_t*>(dst + 2 * j) = pack2<T>(lo0, lo1);
    *reinterpret_cast<uint32_t*>(dst + half + 2 * j) = pack2<T>(hi0, hi1);
  } else {
    T* dst = static_cast<T*>(a.v_cache) + (static_cast<size_t>(head - rotated) * a.context + position) * D + 4 * j;
    uint2 packed;
    packed.x = pack2<T>(v[0], v[1]);
    packed.y = pack2<T>(v[2], v[3]);
    *reinterpret_cast<uint2*>(dst) = packed;
  }
}

// The CTA's first maximum (lane 0 of every warp holds a candidate) into pick slot `block`.
__device__ void pick_slot(const DecodeGemvArgs& a, float best, int best_at, int block) {
  __shared__ float values[kGemvWarps];
  __shared__ int indices[kGemvWarps];
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    values[warp] = best;
    indices[warp] = best_at;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = values[0];
    int at = indices[0];
    for (int w = 1; w < kGemvWarps; ++w) {
      if (better(values[w], indices[w], v, at)) {
        v = values[w];
        at = indices[w];
      }
    }
    a.pick_values[block] = v;
    a.pick_indices[block] = at;
  }
  __syncthreads();
}

// One CTA reduces pick slots [0, slots) into state = {first maximum, position + 1}.
__device__ void reduce_pick(const DecodeGemvArgs& a, int slots) {
  __shared__ float values[kGemvWarps];
  __shared__ int indices[kGemvWarps];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  float v = -INFINITY;
  int at = INT_MAX;
  for (int s = threadIdx.x; s < slots; s += kGemvThreads) {
    const float sv = __ldcg(a.pick_values + s);
    const int si = __ldcg(a.pick_indices + s);
    if (better(sv, si, v, at)) {
      v = sv;
      at = si;
    }
  }
#pragma unroll
  for (int offset = 16; offset > 0; offset >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, offset);
    const int oi = __shfl_xor_sync(0xffffffffu, at, offset);
    if (better(ov, oi, v, at)) {
      v = ov;
      at = oi;
    }
  }
  if (lane == 0) {
    values[warp] = v;
    indices[warp] = at;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kGemvWarps; ++w) {
      if (better(values[w], indices[w], values[0], indices[0])) {
        values[0] = values[w];
        indices[0] = indices[w];
      }
    }
    a.state[0] = indices[0] == INT_MAX ? 0 : indices[0];
    a.state[1] = a.state[1] + 1;
  }
  __syncthreads();
}

// Standalone kernels: the last CTA to finish (an atomic ticket; no CTA waits for another) reduces.
__device__ void finish_pick(const DecodeGemvArgs& a, float best, int best_at, int block, int blocks) {
  __shared__ bool last;
  pick_slot(a, best, best_at, block);
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(a.ticket, 1u) == static_cast<unsigned>(blocks) - 1u;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  reduce_pick(a, blocks);
  if (threadIdx.x == 0) *a.ticket = 0u;
}

// First slice of this block's first work item towards L2 (weights never depend on the producer).
template <int kKind, int kSplit>
__device__ __forceinline__ void gemv_prefetch(const DecodeGemvArgs& a, int block) {
  constexpr int kRows = GemvShape<kKind>::kRows;
  constexpr int kItems = kGemvWarps / kSplit;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int local = warp / kSplit;
  const int slice = warp - local * kSplit;
  const int chunks = a.k >> 3;
  const int begin = slice * chunks / kSplit;
  const int end = (slice + 1) * chunks / kSplit;
  const int item = block * kItems + local;
  if (item < item_count<kKind>(a) && lane < kRows && end > begin) {
    int row[kRows];
    item_rows<kKind>(a, item, row);
    const uint16_t* w = static_cast<const uint16_t*>(a.w);
    prefetch_l2(w + static_cast<size_t>(row[lane]) * a.k + 8 * static_cast<size_t>(begin),
                static_cast<uint32_t>(end - begin) * 16u);
  }
}

// One projection over the work items of blocks block, block + blocks, ... (a grid-stride loop);
// `slot_pick`: the greedy pick leaves this block's candidate in its slot (the caller reduces),
// else the last block reduces by ticket.
template <typename T, int kKind, int kSplit, int kInFlight>
__device__ void gemv_body(const DecodeGemvArgs& a, int block, int blocks, bool slot_pick) {
  constexpr int kRows = GemvShape<kKind>::kRows;
  constexpr int kItems = kGemvWarps / kSplit;
  extern __shared__ uint4 xs[];
  __shared__ float partial[kGemvWarps][kRows];
  __shared__ float scratch[32];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int local = warp / kSplit;
  const int slice = warp - local * kSplit;
  const int chunks = a.k >> 3;
  const int begin = slice * chunks / kSplit;
  const int end = (slice + 1) * chunks / kSplit;
  const int items = item_count<kKind>(a);
  const T* w = static_cast<const T*>(a.w);
  const int position = kKind == kDecodeQkv ? __ldcg(a.state + 1) : 0;
  if constexpr (kKind == kDecodeQkv) {
    if ((position < 0 || position >= a.table_positions || position >= a.context) && block == 0 &&
        threadIdx.x == 0) {
      report_status(a.status, kStatusPositionOutOfRange);
    }
  }
  stage_x<T>(a, xs, scratch, block);

  float best = -INFINITY;
  int best_at = INT_MAX;
  if constexpr (kSplit == 1) {
    // every warp walks its own items: no block-wide step between them, loads stay in flight
    for (int item = block * kGemvWarps + warp; item < items; item += blocks * kGemvWarps) {
      int row[kRows];
      item_rows<kKind>(a, item, row);
      const T* row_ptr[kRows];
#pragma unroll
      for (int r = 0; r < kRows; ++r) row_ptr[r] = w + static_cast<size_t>(row[r]) * a.k;
      float acc[kRows];
      warp_dot_range<T, kRows, kInFlight>(row_ptr, xs, 0, chunks, acc);
      if (lane == 0) finish_item<T, kKind>(a, item, acc, best, best_at);
    }
  } else {
    for (int group = block; group * kItems < items; group += blocks) {
      const int item = group * kItems + local;
      float acc[kRows];
      [[maybe_unused]] QkvOperands operands;
      if constexpr (kKind == kDecodeQkv) {
        if (slice == 0 && lane == 0 && item < items) load_qkv_operands<T>(a, item, position, operands);
      }
      if (item < items) {
        int row[kRows];
        item_rows<kKind>(a, item, row);
        const T* row_ptr[kRows];
#pragma unroll
        for (int r = 0; r < kRows; ++r) row_ptr[r] = w + static_cast<size_t>(row[r]) * a.k;
        warp_dot_range<T, kRows, kInFlight>(row_ptr, xs, begin, end, acc);
      } else {
#pragma unroll
        for (int r = 0; r < kRows; ++r) acc[r] = 0.0f;
      }
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < kRows; ++r) partial[warp][r] = acc[r];
      }
      __syncthreads();
      if (slice == 0 && lane == 0 && item < items) {
        float sum[kRows];
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
          float s = 0.0f;
#pragma unroll
          for (int q = 0; q < kSplit; ++q) s += partial[warp + q][r];
          sum[r] = s;
        }
        if constexpr (kKind == kDecodeQkv) {
          finish_qkv<T>(a, item, position, sum, operands);
        } else {
          finish_item<T, kKind>(a, item, sum, best, best_at);
        }
      }
      __syncthreads();
    }
  }
  if constexpr (kKind == kDecodeLogits) {
    if (a.pick) {
      if (slot_pick) {
        pick_slot(a, best, best_at, block);
      } else {
        finish_pick(a, best, best_at, block, blocks);
      }
    }
  }
  __syncthreads();  // shared memory is reused by the caller's next body
}

template <typename T, int kKind, int kSplit, int kInFlight>
__global__ void __launch_bounds__(kGemvThreads) decode_gemv_kernel(const DecodeGemvArgs a) {
  gemv_prefetch<kKind, kSplit>(a, blockIdx.x);
  wait_for_producer();
  release_dependents();
  gemv_body<T, kKind, kSplit, kInFlight>(a, blockIdx.x, gridDim.x, false);
}

__device__ __forceinline__ float warp_max(float value) {
#pragma unroll
  for (int offset = 16; offset > 0; offset >>= 1) value = fmaxf(value, __shfl_xor_sync(0xffffffffu, value, offset));
  return value;
}

// One CTA per (key-range split, KV head). Warp w owns query heads w, w + 8 of the group:
// lane l scores keys l and l + 32 of each 64-key pass (scores scaled into log2 units), keeps the
// online-softmax max and sum, and accumulates output dims 4l .. 4l + 3 in fp32. The last CTA of
// a KV head (ticket) merges the splits of the group's heads:
//   out[h, d] = sum_s 2^(m_s - M) O_s[d] / sum_s 2^(m_s - M) l_s.
template <typename T>
__device__ void attention_body(const DecodeAttentionArgs& a, int split, int kv_head, int splits, float scale_log2) {
  __shared__ __align__(16) float q_s[kDecodeMaxGroup][kDecodeDim];  // read as float4
  __shared__ __align__(16) T k_s[kDecodeKeys][kKeyStride];
  __shared__ __align__(16) T v_s[kDecodeKeys][kDecodeDim];
  __shared__ float p_s[kDecodeMaxGroup][kDecodeKeys];
  __shared__ bool last;
  constexpr int kWarps = kDecodeThreads / 32;
  constexpr int kHeadsPerWarp = kDecodeMaxGroup / kWarps;
  const int group = a.query_heads / a.kv_heads;
  __syncthreads();  // shared memory may still hold the caller's previous body
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // The step's position was fixed before this step's first kernel ran, and cache rows below it
  // come from earlier steps: both are read before waiting for the q|k|v kernel, whose output
  // (q and the cache row at `position`) is read after.
  const int position = __ldcg(a.state + 1);
  const bool valid = position >= 0 && position < a.context;
  const int length = valid ? position + 1 : 0;
  const int first = a.sliding_window > 0 && length > a.sliding_window ? length - a.sliding_window : 0;
  const int span = length - first;
  const int per_split = (span + kDecodeSplits - 1) / kDecodeSplits;
  const int begin = first + split * per_split;
  const int end = min(begin + per_split, length);
  const T* k_head = static_cast<const T*>(a.k_cache) + static_cast<size_t>(kv_head) * a.context * kDecodeDim;
  const T* v_head = static_cast<const T*>(a.v_cache) + static_cast<size_t>(kv_head) * a.context * kDecodeDim;
  // K and V rows [base, base + keys) into shared memory, except row `skip`
  auto stage_keys = [&](int base, int keys, int skip) {
    for (int i = threadIdx.x; i < keys * (kDecodeDim / 8); i += kDecodeThreads) {
      const int key = i / (kDecodeDim / 8);
      if (base + key == skip) continue;
      const int c = i - key * (kDecodeDim / 8);
      const size_t at = static_cast<size_t>(base + key) * kDecodeDim + 8 * c;
      *reinterpret_cast<uint4*>(&k_s[key][8 * c]) = __ldcg(reinterpret_cast<const uint4*>(k_head + at));
      *reinterpret_cast<uint4*>(&v_s[key][8 * c]) = __ldcg(reinterpret_cast<const uint4*>(v_head + at));
    }
  };
  if (begin < end) stage_keys(begin, min(kDecodeKeys, end - begin), position);  // the first pass's history rows
  wait_for_producer();
  release_dependents();
  if (position >= begin && position < end && position < begin + kDecodeKeys) {
    // the newest row, written by the q|k|v kernel of this step
    for (int i = threadIdx.x; i < kDecodeDim / 8; i += kDecodeThreads) {
      const size_t at = static_cast<size_t>(position) * kDecodeDim + 8 * i;
      *reinterpret_cast<uint4*>(&k_s[position - begin][8 * i]) = __ldcg(reinterpret_cast<const uint4*>(k_head + at));
      *reinterpret_cast<uint4*>(&v_s[position - begin][8 * i]) = __ldcg(reinterpret_cast<const uint4*>(v_head + at));
    }
  }
  for (int i = threadIdx.x; i < group * (kDecodeDim / 8); i += kDecodeThreads) {
    const int g = i / (kDecodeDim / 8);
    const int c = i - g * (kDecodeDim / 8);
    float qv[8];
    unpack8<T>(__ldcg(reinterpret_cast<const uint4*>(static_cast<const T*>(a.q) +
                                                      static_cast<size_t>(kv_head * group + g) * kDecodeDim + 8 * c)),
               qv);
#pragma unroll
    for (int e = 0; e < 8; ++e) q_s[g][8 * c + e] = qv[e] * scale_log2;
  }
  float m[kHeadsPerWarp];
  float l[kHeadsPerWarp];
  float o[kHeadsPerWarp][4];
#pragma unroll
  for (int h = 0; h < kHeadsPerWarp; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) o[h][i] = 0.0f;
  }
  for (int base = begin; base < end; base += kDecodeKeys) {
    const int keys = min(kDecodeKeys, end - base);
    if (base != begin) {
      __syncthreads();  // the previous pass's K, V and P are consumed
      stage_keys(base, keys, -1);
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < kHeadsPerWarp; ++h) {
      const int g = warp + kWarps * h;
      if (g >= group) break;
      float s[2];
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const int key = lane + 32 * which;
        s[which] = -INFINITY;
        if (key < keys) {
          float dot = 0.0f;
#pragma unroll 4
          for (int c = 0; c < kDecodeDim / 8; ++c) {
            float kv[8];
            unpack8<T>(*reinterpret_cast<const uint4*>(&k_s[key][8 * c]), kv);
            const float4 q0 = *reinterpret_cast<const float4*>(&q_s[g][8 * c]);
            const float4 q1 = *reinterpret_cast<const float4*>(&q_s[g][8 * c + 4]);
            dot = fmaf(q0.x, kv[0], dot);
            dot = fmaf(q0.y, kv[1], dot);
            dot = fmaf(q0.z, kv[2], dot);
            dot = fmaf(q0.w, kv[3], dot);
            dot = fmaf(q1.x, kv[4], dot);
            dot = fmaf(q1.y, kv[5], dot);
            dot = fmaf(q1.z, kv[6], dot);
            dot = fmaf(q1.w, kv[7], dot);
          }
          s[which] = dot;
        }
      }
      const float m_new = fmaxf(m[h], warp_max(fmaxf(s[0], s[1])));  // finite: keys >= 1
      const float alpha = exp2f(m[h] - m_new);
      const float p0 = exp2f(s[0] - m_new);
      const float p1 = exp2f(s[1] - m_new);
      l[h] = l[h] * alpha + warp_sum(p0 + p1);
      m[h] = m_new;
      p_s[g][lane] = p0;
      p_s[g][lane + 32] = p1;
      __syncwarp();
#pragma unroll
      for (int i = 0; i < 4; ++i) o[h][i] *= alpha;
      for (int key = 0; key < keys; ++key) {
        const float p = p_s[g][key];
        const uint2 raw = *reinterpret_cast<const uint2*>(&v_s[key][4 * lane]);
        const float2 v01 = Pair<T>::to_float2(*reinterpret_cast<const typename Pair<T>::type*>(&raw.x));
        const float2 v23 = Pair<T>::to_float2(*reinterpret_cast<const typename Pair<T>::type*>(&raw.y));
        o[h][0] = fmaf(p, v01.x, o[h][0]);
        o[h][1] = fmaf(p, v01.y, o[h][1]);
        o[h][2] = fmaf(p, v23.x, o[h][2]);
        o[h][3] = fmaf(p, v23.y, o[h][3]);
      }
      __syncwarp();
    }
  }
#pragma unroll
  for (int h = 0; h < kHeadsPerWarp; ++h) {
    const int g = warp + kWarps * h;
    if (g >= group) break;
    const int head = kv_head * group + g;
    const size_t slot = static_cast<size_t>(head) * kDecodeSplits + split;
    *reinterpret_cast<float4*>(a.partials + slot * kDecodeDim + 4 * lane) = make_float4(o[h][0], o[h][1], o[h][2], o[h][3]);
    if (lane == 0) {
      a.stats[2 * slot] = m[h];  // -inf for an empty split
      a.stats[2 * slot + 1] = l[h];
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(a.tickets + kv_head, 1u) == static_cast<unsigned>(splits) - 1u;
  __syncthreads();
  if (!last) return;
  __threadfence();
  // warp w merges heads w, w + 8: lane s holds split s's (m, l); lane l combines dims 4l..4l+3
  static_assert(kDecodeSplits == 32, "one split per lane");
  for (int g = warp; g < group; g += kWarps) {
    const int head = kv_head * group + g;
    const float* st = a.stats + static_cast<size_t>(head) * kDecodeSplits * 2;
    const float* part = a.partials + static_cast<size_t>(head) * kDecodeSplits * kDecodeDim;
    const float ms = __ldcg(st + 2 * lane);
    const float ls = __ldcg(st + 2 * lane + 1);
    const float top = warp_max(ms);
    const float weight = ms == -INFINITY ? 0.0f : exp2f(ms - top);
    const float total = warp_sum(weight * ls);
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 8
    for (int split = 0; split < kDecodeSplits; ++split) {
      const float ws = __shfl_sync(0xffffffffu, weight, split);
      if (ws == 0.0f) continue;  // an empty split (uniform over the warp)
      const float4 p = __ldcg(reinterpret_cast<const float4*>(part + static_cast<size_t>(split) * kDecodeDim + 4 * lane));
      acc[0] = fmaf(ws, p.x, acc[0]);
      acc[1] = fmaf(ws, p.y, acc[1]);
      acc[2] = fmaf(ws, p.z, acc[2]);
      acc[3] = fmaf(ws, p.w, acc[3]);
    }
    const float inverse = total > 0.0f ? 1.0f / total : 0.0f;
    uint2 packed;
    packed.x = pack2<T>(acc[0] * inverse, acc[1] * inverse);
    packed.y = pack2<T>(acc[2] * inverse, acc[3] * inverse);
    *reinterpret_cast<uint2*>(static_cast<T*>(a.out) + static_cast<size_t>(head) * kDecodeDim + 4 * lane) = packed;
  }
  if (threadIdx.x == 0) a.tickets[kv_head] = 0u;
}

template <typename T>
__global__ void __launch_bounds__(kDecodeThreads) decode_attention_kernel(const DecodeAttentionArgs a,
                                                                          float scale_log2) {
  attention_body<T>(a, blockIdx.x, blockIdx.y, gridDim.x, scale_log2);
}

// ---- the persistent decode step --------------------------------------------------------------
constexpr unsigned kBarrierSpinLimit = 1u << 22;  // polls of 64 ns or more: over 0.25 s

// Grid-wide barrier of a cooperative launch. Thread 0 of each CTA publishes the CTA's writes
// (fence), arrives on the counter and polls it until every CTA of this generation has arrived.
// The poll is bounded; false after a timeout or when the status word already reports an error,
// and then every CTA returns.
__device__ bool grid_barrier(unsigned* counter, unsigned& target, int* status,
                             unsigned spin_limit = kBarrierSpinLimit) {
  __shared__ int proceed;
  __syncthreads();
  if (threadIdx.x == 0) {
    target += gridDim.x;
    __threadfence();
    atomicAdd(counter, 1u);
    int ok = 1;
    for (unsigned spins = 0;; ++spins) {
      unsigned arrived;
      asm volatile("ld.acquire.gpu.u32 %0, [%1];" : "=r"(arrived) : "l"(counter) : "memory");
      if (arrived >= target) break;
      if (*reinterpret_cast<volatile int*>(status) != 0) {
        ok = 0;
        break;
      }
      if (spins >= spin_limit) {
        report_status(status, kStatusWaitTimeout);
        ok = 0;
        break;
      }
      __nanosleep(64);
    }
    __threadfence();
    proceed = ok;
  }
  __syncthreads();
  return proceed != 0;
}

template <typename T>
__global__ void __launch_bounds__(kGemvThreads, 2) decode_step_kernel(const DecodeStepArgs s) {
  unsigned target = 0;
  int current = 0;
  const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(s.attention.head_dim));
  const int attention_blocks = kDecodeSplits * s.attention.kv_heads;
  for (int l = 0; l < s.layer_count; ++l) {
    const DecodeLayerWeights p = s.layers[l];
    // pre-attention RMSNorm + q|k|v + bias + RoPE + cache append (layer 0: the embedding row)
    DecodeGemvArgs qkv = s.qkv;
    qkv.w = p.qkv;
    qkv.bias_half = p.qkv_bias_half;
    qkv.bias = p.qkv_bias;
    qkv.gamma = p.input_norm;
    qkv.k_cache = p.k_cache;
    qkv.v_cache = p.v_cache;
    if (l == 0) {
      qkv.residual_in = nullptr;
      qkv.delta = nullptr;
      qkv.residual_out = s.residual[0];
    } else {
      qkv.embed_table = nullptr;
      qkv.residual_in = s.residual[current];
      qkv.residual_out = s.residual[current ^ 1];
      current ^= 1;
    }
    if (l == 0) gemv_prefetch<kDecodeQkv, 4>(qkv, blockIdx.x);
    gemv_body<T, kDecodeQkv, 4, 8>(qkv, blockIdx.x, gridDim.x, true);
    DecodeAttentionArgs attention = s.attention;
    attention.k_cache = p.k_cache;
    attention.v_cache = p.v_cache;
    if (!grid_barrier(s.barrier, target, s.status)) return;
    // split attention over the cache; the last CTA of each KV head merges its splits
    for (int b = blockIdx.x; b < attention_blocks; b += gridDim.x) {
      attention_body<T>(attention, b % kDecodeSplits, b / kDecodeSplits, kDecodeSplits, scale_log2);
    }
    DecodeGemvArgs out_proj = s.out_proj;
    out_proj.w = p.out;
    gemv_prefetch<kDecodePlain, 4>(out_proj, blockIdx.x);
    if (!grid_barrier(s.barrier, target, s.status)) return;
    gemv_body<T, kDecodePlain, 4, 8>(out_proj, blockIdx.x, gridDim.x, true);
    // post-attention RMSNorm + gate|up + SwiGLU
    DecodeGemvArgs gate_up = s.gate_up;
    gate_up.w = p.gate_up;
    gate_up.gamma = p.post_norm;
    gate_up.residual_in = s.residual[current];
    gate_up.residual_out = s.residual[current ^ 1];
    current ^= 1;
    gemv_prefetch<kDecodeGateUp, 1>(gate_up, blockIdx.x);
    if (!grid_barrier(s.barrier, target, s.status)) return;
    gemv_body<T, kDecodeGateUp, 1, 16>(gate_up, blockIdx.x, gridDim.x, true);
    DecodeGemvArgs down = s.down;
    down.w = p.down;
    gemv_prefetch<kDecodePlain, 8>(down, blockIdx.x);
    if (!grid_barrier(s.barrier, target, s.status)) return;
    gemv_body<T, kDecodePlain, 8, 16>(down, blockIdx.x, gridDim.x, true);
    if (l + 1 < s.layer_count) {
      DecodeGemvArgs next = s.qkv;
      next.w = s.layers[l + 1].qkv;
      gemv_prefetch<kDecodeQkv, 4>(next, blockIdx.x);
    } else {
      gemv_prefetch<kDecodeLogits, 1>(s.head, blockIdx.x);
    }
    if (!grid_barrier(s.barrier, target, s.status)) return;
  }
  // final RMSNorm + output head; greedy: every CTA's candidate, then block 0 picks
  DecodeGemvArgs head = s.head;
  head.residual_in = s.residual[current];
  gemv_body<T, kDecodeLogits, 1, 16>(head, blockIdx.x, gridDim.x, true);
  if (head.pick) {
    if (!grid_barrier(s.barrier, target, s.status)) return;
    if (blockIdx.x == 0) reduce_pick(head, gridDim.x);
  }
}

// Self-test of the bounded grid barrier: every CTA waits for one arrival more than the grid makes,
// a counter value nothing will ever write, so the wait must run out after `spin_limit` polls,
// record kStatusWaitTimeout and let every CTA return (the others see the status word and stop).
__global__ void bounded_wait_selftest_kernel(unsigned* counter, int* status, unsigned spin_limit) {
  unsigned target = 1;  // grid_barrier adds gridDim.x: one more than the CTAs that arrive
  grid_barrier(counter, target, status, spin_limit);
}

template <typename T>
__global__ void store_kv_kernel(const T* __restrict__ qkv, int tokens, int query_heads, int kv_heads, int head_dim,
                                T* __restrict__ k_cache, T* __restrict__ v_cache, int context) {
  const int chunks_per_head = head_dim >> 3;
  const int chunks = kv_heads * chunks_per_head;  // per row, per K or V
  const int width = (query_heads + 2 * kv_heads) * head_dim;
  const long long total = static_cast<long long>(tokens) * 2 * chunks;
  for (long long item = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; item < total;
       item += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int token = static_cast<int>(item / (2 * chunks));
    const int rest = static_cast<int>(item - static_cast<long long>(token) * 2 * chunks);
    const int which = rest / chunks;  // 0 = K, 1 = V
    const int c = rest - which * chunks;
    const int head = c / chunks_per_head;
    const int part = c - head * chunks_per_head;
    const T* src = qkv + static_cast<size_t>(token) * width + (query_heads + which * kv_heads) * head_dim +
                   head * head_dim + 8 * part;
    T* dst = (which == 0 ? k_cache : v_cache) + (static_cast<size_t>(head) * context + token) * head_dim + 8 * part;
    *reinterpret_cast<uint4*>(dst) = load_nc(src);
  }
}

constexpr int kArgmaxThreads = 1024;

__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(const float* __restrict__ logits, int count,
                                                                int32_t* __restrict__ state) {
  __shared__ float best_value[kArgmaxThreads / 32];
  __shared__ int best_index[kArgmaxThreads / 32];
  // each thread: the first maximum of its strided subsequence (ascending indices)
  float best = -INFINITY;
  int index = INT_MAX;
  if (static_cast<int>(threadIdx.x) < count) {
    best = logits[threadIdx.x];
    index = threadIdx.x;
  }
  for (int i = threadIdx.x + kArgmaxThreads; i < count; i += kArgmaxThreads) {
    const float v = logits[i];
    if (v > best) {
      best = v;
      index = i;
    }
  }
#pragma unroll
  for (int offset = 16; offset > 0; offset >>= 1) {
    const float other = __shfl_xor_sync(0xffffffffu, best, offset);
    const int other_index = __shfl_xor_sync(0xffffffffu, index, offset);
    if (better(other, other_index, best, index)) {
      best = other;
      index = other_index;
    }
  }
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    best_value[warp] = best;
    best_index[warp] = index;
  }
  __syncthreads();
  if (warp == 0) {
    best = best_value[threadIdx.x];
    index = best_index[threadIdx.x];
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) {
      const float other = __shfl_xor_sync(0xffffffffu, best, offset);
      const int other_index = __shfl_xor_sync(0xffffffffu, index, offset);
      if (better(other, other_index, best, index)) {
        best = other;
        index = other_index;
      }
    }
    if (threadIdx.x == 0) {
      state[0] = index == INT_MAX ? 0 : index;
      state[1] = state[1] + 1;
    }
  }
}

template <typename Kernel, typename... Args>
cudaError_t launch(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool programmatic,
                   Args... args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attribute[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = programmatic ? attribute : nullptr;
  config.numAttrs = programmatic ? 1 : 0;
  return cudaLaunchKernelEx(&config, kernel, args...);
}

// CTAs per SM a decode GEMV may fill; ATTNRANK_DECODE_CTAS_PER_SM caps it (0 or unset: as many
// as fit), leaving room for the next kernel's CTAs to start early under programmatic launch.
int decode_ctas_per_sm_cap() {
  static const int cap = [] {
    const char* text = std::getenv("ATTNRANK_DECODE_CTAS_PER_SM");
    return text != nullptr ? std::atoi(text) : 0;
  }();
  return cap;
}

template <typename T, int kKind, int kSplit, int kInFlight>
cudaError_t gemv_typed(const DecodeGemvArgs& args, bool programmatic, cudaStream_t stream) {
  auto kernel = decode_gemv_kernel<T, kKind, kSplit, kInFlight>;
  const size_t smem = static_cast<size_t>(args.k) * 2;
  if (smem > 48 * 1024) {
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    const cudaError_t status =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (status != cudaSuccess) return status;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kGemvThreads, smem) != cudaSuccess || per_sm <= 0) {
    per_sm = 1;
  }
  const int cap_per_sm = decode_ctas_per_sm_cap();
  if (cap_per_sm > 0 && per_sm > cap_per_sm) per_sm = cap_per_sm;
  constexpr int kItems = kGemvWarps / kSplit;
  const int items = kKind == kDecodeQkv ? args.rows / 4 : (args.rows + 1) / 2;
  long long grid = (items + kItems - 1) / kItems;
  const long long cap = static_cast<long long>(sm_count()) * per_sm;
  if (grid > cap) grid = cap;
  if (kKind == kDecodeLogits && grid > kDecodePickSlots) grid = kDecodePickSlots;
  if (grid < 1) grid = 1;
  return launch(kernel, dim3(static_cast<unsigned>(grid)), dim3(kGemvThreads), smem, stream, programmatic, args);
}

template <typename T>
cudaError_t gemv_dispatch(const DecodeGemvArgs& args, bool programmatic, cudaStream_t stream) {
  switch (args.kind) {
    case kDecodePlain:
      return args.k >= 8192 ? gemv_typed<T, kDecodePlain, 8, 16>(args, programmatic, stream)
                            : gemv_typed<T, kDecodePlain, 4, 8>(args, programmatic, stream);
    case kDecodeLogits:
      return gemv_typed<T, kDecodeLogits, 1, 16>(args, programmatic, stream);
    case kDecodeGateUp:
      return gemv_typed<T, kDecodeGateUp, 1, 16>(args, programmatic, stream);
    case kDecodeQkv:
      return gemv_typed<T, kDecodeQkv, 4, 8>(args, programmatic, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

bool valid_dtype(int dtype) { return dtype == kActFp16 || dtype == kActBf16; }

template <typename T>
cudaError_t step_typed(const DecodeStepArgs& args, cudaStream_t stream) {
  auto kernel = decode_step_kernel<T>;
  const size_t smem = static_cast<size_t>(args.max_k) * 2;
  cudaError_t status = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (status != cudaSuccess) return status;
  int per_sm = 0;
  status = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kGemvThreads, smem);
  if (status != cudaSuccess) return status;
  if (per_sm <= 0) return cudaErrorCooperativeLaunchTooLarge;
  const int grid = per_sm * sm_count();
  if (grid > kDecodePickSlots) return cudaErrorCooperativeLaunchTooLarge;
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(grid);
  config.blockDim = dim3(kGemvThreads);
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeCooperative;
  attribute[0].val.cooperative = 1;
  config.attrs = attribute;
  config.numAttrs = 1;
  return cudaLaunchKernelEx(&config, kernel, args);
}

}  // namespace

cudaError_t launch_decode_step(const DecodeStepArgs& args, cudaStream_t stream) {
  if (args.layers == nullptr || args.layer_count <= 0 || args.barrier == nullptr || args.status == nullptr ||
      !valid_dtype(args.dtype) || args.max_k <= 0 || args.max_k % 8 != 0 ||
      args.qkv.k > kDecodeMaxNormHidden || args.attention.head_dim != kDecodeDim ||
      args.attention.query_heads / args.attention.kv_heads > kDecodeMaxGroup) {
    return cudaErrorInvalidValue;
  }
  return args.dtype == kActFp16 ? step_typed<__half>(args, stream) : step_typed<__nv_bfloat16>(args, stream);
}

cudaError_t launch_decode_gemv(const DecodeGemvArgs& args, bool programmatic, cudaStream_t stream) {
  if (args.rows <= 0 || args.k <= 0 || args.k % 8 != 0 || !valid_dtype(args.dtype) || args.w == nullptr ||
      (args.x == nullptr && args.residual_in == nullptr)) {
    return cudaErrorInvalidValue;
  }
  if (args.residual_in != nullptr && (args.k > kDecodeMaxNormHidden || args.gamma == nullptr)) {
    return cudaErrorInvalidValue;
  }
  if (args.kind == kDecodeQkv &&
      (args.head_dim % 4 != 0 || args.query_heads <= 0 || args.kv_heads <= 0 || args.context <= 0 ||
       args.state == nullptr || args.rows != (args.query_heads + 2 * args.kv_heads) * args.head_dim)) {
    return cudaErrorInvalidValue;
  }
  if (args.pick && (args.kind != kDecodeLogits || args.state == nullptr || args.ticket == nullptr ||
                    args.pick_values == nullptr || args.pick_indices == nullptr)) {
    return cudaErrorInvalidValue;
  }
  return args.dtype == kActFp16 ? gemv_dispatch<__half>(args, programmatic, stream)
                                : gemv_dispatch<__nv_bfloat16>(args, programmatic, stream);
}

cudaError_t launch_decode_attention(const DecodeAttentionArgs& args, bool programmatic, cudaStream_t stream) {
  if (args.head_dim != kDecodeDim || args.kv_heads <= 0 || args.query_heads % args.kv_heads != 0 ||
      args.query_heads / args.kv_heads > kDecodeMaxGroup || args.context <= 0 || !valid_dtype(args.dtype) ||
      args.tickets == nullptr) {
    return cudaErrorInvalidValue;
  }
  const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(args.head_dim));
  const dim3 grid(kDecodeSplits, args.kv_heads);
  return args.dtype == kActFp16
             ? launch(decode_attention_kernel<__half>, grid, dim3(kDecodeThreads), 0, stream, programmatic, args,
                      scale_log2)
             : launch(decode_attention_kernel<__nv_bfloat16>, grid, dim3(kDecodeThreads), 0, stream, programmatic,
                      args, scale_log2);
}

cudaError_t launch_bounded_wait_selftest(unsigned* counter, int* status, int ctas, unsigned spin_limit,
                                         cudaStream_t stream) {
  if (ctas <= 0 || ctas > 1024 || spin_limit == 0 || spin_limit > kBarrierSpinLimit) return cudaErrorInvalidValue;
  bounded_wait_selftest_kernel<<<ctas, 32, 0, stream>>>(counter, status, spin_limit);
  return cudaGetLastError();
}

cudaError_t launch_store_kv(const void* qkv, int tokens, int query_heads, int kv_heads, int head_dim, void* k_cache,
                            void* v_cache, int context, int dtype, cudaStream_t stream) {
  if (tokens < 0 || tokens > context || head_dim % 8 != 0 || !valid_dtype(dtype)) return cudaErrorInvalidValue;
  if (tokens == 0) return cudaSuccess;
  const long long total = static_cast<long long>(tokens) * 2 * kv_heads * (head_dim / 8);
  const long long needed = (total + 255) / 256;
  const int grid = static_cast<int>(needed < 8LL * sm_count() ? needed : 8LL * sm_count());
  if (dtype == kActFp16) {
    store_kv_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<const __half*>(qkv), tokens, query_heads, kv_heads,
                                                      head_dim, static_cast<__half*>(k_cache),
                                                      static_cast<__half*>(v_cache), context);
  } else {
    store_kv_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(qkv), tokens, query_heads, kv_heads, head_dim,
        static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), context);
  }
  return cudaGetLastError();
}

cudaError_t launch_argmax_token(const float* logits, int count, int32_t* state, cudaStream_t stream) {
  if (count <= 0) return cudaErrorInvalidValue;
  argmax_kernel<<<1, kArgmaxThreads, 0, stream>>>(logits, count, state);
  return cudaGetLastError();
}

}  // namespace arb
