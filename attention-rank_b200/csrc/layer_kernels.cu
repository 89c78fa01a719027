// Fused per-layer kernels of the attention-profiling prefill, hand-written for sm_100a.
//
// All four are HBM-bound: each moves its operands through HBM exactly once with 128-bit
// coalesced accesses, and grids are sized from the SM count. They replace these reference
// kernels (attnrank/src/kernels.cu):
//   embedding_lookup_kernel  (:50-58)   -> embed_rms_norm_kernel (gather + the first pre-norm)
//   rms_norm_kernel (:60-83) + add_in_place_kernel (:172-175) -> rms_norm_residual_kernel
//   rotary_embedding_kernel (:85-115) + add_row_bias_kernel (:177-184) -> rotary_bias_kernel
//   silu_multiply_kernel (:164-170)     -> silu_multiply_kernel
// The arithmetic of each op follows the reference formula line for line (fp32 math, the same
// order of multiplies), only the storage type of activations changes from fp32 to 16 bits (T =
// __half, the default, or __nv_bfloat16).
#include <algorithm>

#include "common.cuh"
#include "layer_kernels.h"

namespace arb {
namespace {

constexpr int kRowThreadsCap = 256;
constexpr int kRopeUnroll = 4;       // heads loaded per rotary step (loads in flight per thread)
constexpr int kRopeGroupHeads = 8;   // heads of one rotary work item
constexpr int kSiluUnroll = 2;   // 8-value chunks in flight per SwiGLU thread

// ---------------------------------------------------------------------------------------------
// Row kernels: each thread holds VPT vectors of 8 channels of a row in registers, so the row is
// read once, reduced, and written once.
//   * RMSNorm + residual: one CTA per token row. With the grid as large as the batch, the CTAs of
//     every SM issue their rows' loads together and the block scheduler refills a slot as soon
//     as a row is done: 108.7 us at 16384 x 3584 fp16 timed alone (0.99 of copy bandwidth)
//     against 115.9 us for a resident grid walking the rows and 124.7 us for the same with the
//     next row's loads in flight (one process); inside the scan, at power-capped clocks,
//     129.0 us against 138.4 us for the latter.
//   * Embedding + RMSNorm: a resident grid walks the rows and a CTA's next row's loads are
//     issued before the current row's block-wide reduction. Timed alone it equals one CTA per
//     row (86.9 / 85.6 us at 16K x 3584); inside the scan it measured 93.1 us against 112.9 us.
// ---------------------------------------------------------------------------------------------
template <typename T, int VPT>
__device__ __forceinline__ void store_normed_row(const float (&values)[VPT][8], float scale, const float* gamma,
                                                 T* normed_row, int chunks) {
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int chunk = threadIdx.x + k * blockDim.x;
    if (chunk >= chunks) continue;
    const float4 g0 = __ldg(reinterpret_cast<const float4*>(gamma + chunk * 8));
    const float4 g1 = __ldg(reinterpret_cast<const float4*>(gamma + chunk * 8 + 4));
    const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    float y[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = values[k][i] * scale * g[i];
    __stcs(reinterpret_cast<uint4*>(normed_row + chunk * 8), pack8<T>(y));
  }
}

// Sum over the whole block through one of two scratch buffers (alternate them between calls:
// one barrier per call then suffices, since a warp can only reuse a buffer after every warp has
// passed the barrier of the call in between).
__device__ __forceinline__ float block_sum_buffered(float value, float* scratch) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int warps = (blockDim.x + 31) >> 5;
  value = warp_sum(value);
  if (lane == 0) scratch[warp] = value;
  __syncthreads();
  float total = lane < warps ? scratch[lane] : 0.0f;
  return warp_sum(total);
}

template <typename T, int VPT>
__global__ void __launch_bounds__(kRowThreadsCap) embed_rms_norm_kernel(
    const int32_t* __restrict__ token_ids, const T* __restrict__ table, int tokens, int vocab, int hidden,
    const float* __restrict__ gamma, float eps, float* __restrict__ residual, T* __restrict__ normed,
    int* status) {
  __shared__ float scratch[2][32];
  const int chunks = hidden >> 3;
  // the table row of a token id outside [0, vocab) is never read: that row becomes zeros
  auto checked_token = [&](int row) {
    const int token = __ldg(token_ids + row);
    if (token < 0 || token >= vocab) {
      if (threadIdx.x == 0) report_status(status, kStatusTokenOutOfRange);
      return -1;
    }
    return token;
  };
  auto load_row = [&](uint4 (&raw)[VPT], int token) {
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int chunk = threadIdx.x + k * blockDim.x;
      raw[k] = make_uint4(0u, 0u, 0u, 0u);
      if (chunk < chunks && token >= 0) raw[k] = load_nc(table + static_cast<size_t>(token) * hidden + chunk * 8);
    }
  };
  int row = blockIdx.x;
  uint4 next[VPT];
  if (row < tokens) load_row(next, checked_token(row));
  for (int parity = 0; row < tokens; row += gridDim.x, parity ^= 1) {
    uint4 current[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) current[k] = next[k];
    if (row + static_cast<int>(gridDim.x) < tokens) load_row(next, checked_token(row + gridDim.x));
    float values[VPT][8];
    float squares = 0.0f;
    float* residual_row = residual + static_cast<size_t>(row) * hidden;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      unpack8<T>(current[k], values[k]);
      const int chunk = threadIdx.x + k * blockDim.x;
      if (chunk < chunks) {
        float4* out = reinterpret_cast<float4*>(residual_row + chunk * 8);
        __stcs(out, make_float4(values[k][0], values[k][1], values[k][2], values[k][3]));
        __stcs(out + 1, make_float4(values[k][4], values[k][5], values[k][6], values[k][7]));
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) squares += values[k][i] * values[k][i];
    }
    const float total = block_sum_buffered(squares, scratch[parity]);
    const float scale = rsqrtf(total / static_cast<float>(hidden) + eps);
    store_normed_row<T, VPT>(values, scale, gamma, normed + static_cast<size_t>(row) * hidden, chunks);
  }
}

// kDelta false: the residual already holds the sum (the projection GEMM accumulated into it), so
// the row is only read and normalised (6 bytes per element instead of 12).
template <typename T, int VPT, bool kDelta>
__global__ void __launch_bounds__(kRowThreadsCap) rms_norm_residual_kernel(
    float* __restrict__ residual, const T* __restrict__ delta, const float* __restrict__ gamma, int tokens,
    int hidden, float eps, T* __restrict__ normed) {
  __shared__ float scratch[32];
  const int row = blockIdx.x;
  const int chunks = hidden >> 3;
  float* residual_row = residual + static_cast<size_t>(row) * hidden;
  const T* delta_row = kDelta ? delta + static_cast<size_t>(row) * hidden : nullptr;
  float values[VPT][8];
  float squares = 0.0f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int chunk = threadIdx.x + k * blockDim.x;
    if (chunk < chunks) {
      const float4 r0 = load_stream_f4(residual_row + chunk * 8);
      const float4 r1 = load_stream_f4(residual_row + chunk * 8 + 4);
      float d[8] = {};
      if (kDelta) unpack8<T>(load_stream(delta_row + chunk * 8), d);
      values[k][0] = r0.x + d[0];
      values[k][1] = r0.y + d[1];
      values[k][2] = r0.z + d[2];
      values[k][3] = r0.w + d[3];
      values[k][4] = r1.x + d[4];
      values[k][5] = r1.y + d[5];
      values[k][6] = r1.z + d[6];
      values[k][7] = r1.w + d[7];
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) values[k][i] = 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) squares += values[k][i] * values[k][i];
  }
  const float total = block_sum(squares, scratch);
  const float scale = rsqrtf(total / static_cast<float>(hidden) + eps);
  if (kDelta) {
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int chunk = threadIdx.x + k * blockDim.x;
      if (chunk >= chunks) continue;
      float4* out = reinterpret_cast<float4*>(residual_row + chunk * 8);
      __stcs(out, make_float4(values[k][0], values[k][1], values[k][2], values[k][3]));
      __stcs(out + 1, make_float4(values[k][4], values[k][5], values[k][6], values[k][7]));
    }
  }
  store_normed_row<T, VPT>(values, scale, gamma, normed + static_cast<size_t>(row) * hidden, chunks);
}

// ---------------------------------------------------------------------------------------------
// Bias + rotary embedding, in place on the fused [tokens, (Hq + 2 Hkv) * D] projection output.
// A work item is 8 rotation pairs (x_i, x_{i + D/2}) at one offset of one token over a group of
// kRopeGroupHeads heads, so its cos/sin values are loaded once per group (not once per head, which
// made the kernel L1-bound), and there are enough items for one resident wave of threads to share
// them evenly (all heads in one item left most threads with one item and some with two);
// kRopeUnroll heads are loaded before any is stored. Query and key heads get
// bias + rotation; value heads get the bias only (and are skipped without bias). The engine
// applies the bias in the q|k|v GEMM epilogue and passes none. Two 256-thread CTAs per SM leave
// 128 registers a thread: with three (85 registers) the kernel spilled and ran 4% slower.
// ---------------------------------------------------------------------------------------------
template <typename T, bool kBias>
__global__ void __launch_bounds__(256, 2) rotary_bias_kernel(T* __restrict__ qkv, const float* __restrict__ bias,
                                   const int32_t* __restrict__ positions, int tokens, int query_heads,
                                   int kv_heads, int head_dim, const float* __restrict__ cos_table,
                                   const float* __restrict__ sin_table, int table_positions,
                                   int* status) {
  const int half = head_dim >> 1;
  const int chunks_per_head = half >> 3;
  const int rotated_heads = query_heads + kv_heads;
  const int heads = kBias ? rotated_heads + kv_heads : rotated_heads;
  const int row_width = (query_heads + 2 * kv_heads) * head_dim;
  const int groups = (heads + kRopeGroupHeads - 1) / kRopeGroupHeads;
  const int total = tokens * groups * chunks_per_head;  // < 2^31: the launcher bounds tokens
  for (int item = blockIdx.x * blockDim.x + threadIdx.x; item < total; item += gridDim.x * blockDim.x) {
    const int chunk = item % chunks_per_head;
    const int rest = item / chunks_per_head;
    const int group = rest % groups;
    const int token = rest / groups;
    const int group_first = group * kRopeGroupHeads;
    const int group_end = min(group_first + kRopeGroupHeads, heads);
    const int position = positions[token];
    const bool in_table = position >= 0 && position < table_positions;
    if (!in_table) report_status(status, kStatusPositionOutOfRange);
    float c[8];
    float s[8];
    if (in_table && group_first < rotated_heads) {
      const float* cos_row = cos_table + static_cast<size_t>(position) * half + chunk * 8;
      const float* sin_row = sin_table + static_cast<size_t>(position) * half + chunk * 8;
      const float4 c0 = __ldg(reinterpret_cast<const float4*>(cos_row));
      const float4 c1 = __ldg(reinterpret_cast<const float4*>(cos_row + 4));
      const float4 s0 = __ldg(reinterpret_cast<const float4*>(sin_row));
      const float4 s1 = __ldg(reinterpret_cast<const float4*>(sin_row + 4));
      c[0] = c0.x; c[1] = c0.y; c[2] = c0.z; c[3] = c0.w; c[4] = c1.x; c[5] = c1.y; c[6] = c1.z; c[7] = c1.w;
      s[0] = s0.x; s[1] = s0.y; s[2] = s0.z; s[3] = s0.w; s[4] = s1.x; s[5] = s1.y; s[6] = s1.z; s[7] = s1.w;
    }
    // without a valid position only the bias-only value heads are written
    const int first_head = in_table ? group_first : max(group_first, rotated_heads);
    T* row = qkv + static_cast<size_t>(token) * row_width + chunk * 8;
    for (int h0 = first_head; h0 < group_end; h0 += kRopeUnroll) {
      uint4 low_raw[kRopeUnroll];
      uint4 high_raw[kRopeUnroll];
#pragma unroll
      for (int u = 0; u < kRopeUnroll; ++u) {
        if (h0 + u < group_end) {
          low_raw[u] = *reinterpret_cast<const uint4*>(row + (h0 + u) * head_dim);
          high_raw[u] = *reinterpret_cast<const uint4*>(row + (h0 + u) * head_dim + half);
        }
      }
#pragma unroll
      for (int u = 0; u < kRopeUnroll; ++u) {
        const int head = h0 + u;
        if (head >= group_end) break;
        float low[8];
        float high[8];
        unpack8<T>(low_raw[u], low);
        unpack8<T>(high_raw[u], high);
        if constexpr (kBias) {
          const float* b = bias + head * head_dim + chunk * 8;
          const float4 b0 = __ldg(reinterpret_cast<const float4*>(b));
          const float4 b1 = __ldg(reinterpret_cast<const float4*>(b + 4));
          const float4 b2 = __ldg(reinterpret_cast<const float4*>(b + half));
          const float4 b3 = __ldg(reinterpret_cast<const float4*>(b + half + 4));
          const float bl[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
          const float bh[8] = {b2.x, b2.y, b2.z, b2.w, b3.x, b3.y, b3.z, b3.w};
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            low[i] += bl[i];
            high[i] += bh[i];
          }
        }
        if (head < rotated_heads) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float l = low[i];
            const float h = high[i];
            low[i] = l * c[i] - h * s[i];
            high[i] = h * c[i] + l * s[i];
          }
        }
        *reinterpret_cast<uint4*>(row + head * head_dim) = pack8<T>(low);
        *reinterpret_cast<uint4*>(row + head * head_dim + half) = pack8<T>(high);
      }
    }
  }
}

// cos/sin of pos * theta^(-2i/D), written with the same fp32 expression as the reference's
// per-element computation (kernels.cu:95-98), so the table holds identical values.
__global__ void rope_table_kernel(float* __restrict__ cos_out, float* __restrict__ sin_out,
                                  int positions, int head_dim, float theta) {
  const int half = head_dim >> 1;
  const long long total = static_cast<long long>(positions) * half;
  for (long long item = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; item < total;
       item += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int position = static_cast<int>(item / half);
    const int index = static_cast<int>(item - static_cast<long long>(position) * half);
    const float inverse_frequency = powf(theta, -2.0f * index / static_cast<float>(head_dim));
    const float angle = position * inverse_frequency;
    cos_out[item] = cosf(angle);
    sin_out[item] = sinf(angle);
  }
}

// ---------------------------------------------------------------------------------------------
// SwiGLU: a = silu(g) * u with g, u read through arbitrary row strides (the fused gate|up GEMM
// output has g in columns [0, I) and u in [I, 2I) of each row).
// ---------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) silu_multiply_kernel(const T* __restrict__ gate, const T* __restrict__ up,
                                                            long long in_stride, T* __restrict__ out,
                                                            long long out_stride, int tokens, int width) {
  // The (row, 8-value chunk) pairs of the whole batch form one index space; a thread loads
  // kSiluUnroll chunks (grid-stride apart) before it computes any, and no row leaves a partial tail.
  const unsigned chunks = static_cast<unsigned>(width) >> 3;
  const unsigned total = static_cast<unsigned>(tokens) * chunks;  // < 2^31: the launcher checks
  const unsigned stride = gridDim.x * blockDim.x;
  // (token, chunk) of the current item, advanced by the grid stride without a division per item
  const unsigned stride_rows = stride / chunks;
  const unsigned stride_chunks = stride - stride_rows * chunks;
  unsigned first = blockIdx.x * blockDim.x + threadIdx.x;
  unsigned token = first / chunks;
  unsigned chunk = first - token * chunks;
  auto advance = [&]() {
    token += stride_rows;
    chunk += stride_chunks;
    if (chunk >= chunks) {
      chunk -= chunks;
      ++token;
    }
  };
  for (; first < total; first += stride * kSiluUnroll) {
    uint4 g_raw[kSiluUnroll];
    uint4 u_raw[kSiluUnroll];
    long long out_at[kSiluUnroll];
#pragma unroll
    for (int k = 0; k < kSiluUnroll; ++k) {
      const unsigned item = first + k * stride;
      out_at[k] = -1;
      if (item < total) {
        const long long in_at = static_cast<long long>(token) * in_stride + chunk * 8;
        g_raw[k] = load_stream(gate + in_at);
        u_raw[k] = load_stream(up + in_at);
        out_at[k] = static_cast<long long>(token) * out_stride + chunk * 8;
      }
      advance();
    }
#pragma unroll
    for (int k = 0; k < kSiluUnroll; ++k) {
      if (out_at[k] < 0) break;
      float g[8];
      float u[8];
      unpack8<T>(g_raw[k], g);
      unpack8<T>(u_raw[k], u);
      // silu(g) * u = g / (1 + e^-g) * u, the reference formula (kernels.cu:169) with a fast
      // fp32 divide: its few-ulp fp32 error vanishes in the 16-bit rounding of the result
      // (for e^-g = inf the quotient is 0, the limit of silu)
      float a[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = __fdividef(g[i], 1.0f + __expf(-g[i])) * u[i];
      __stcs(reinterpret_cast<uint4*>(out + out_at[k]), pack8<T>(a));
    }
  }
}

// position of every packed token inside its own prompt: t - prompt_offsets[p].
__global__ void positions_kernel(const int32_t* __restrict__ prompt_offsets, int prompt_count,
                                 int tokens, int32_t* __restrict__ positions) {
  for (int token = blockIdx.x * blockDim.x + threadIdx.x; token < tokens;
       token += gridDim.x * blockDim.x) {
    int lo = 0;
    int hi = prompt_count - 1;
    while (lo < hi) {  // last prompt whose offset <= token
      const int mid = (lo + hi + 1) >> 1;
      if (prompt_offsets[mid] <= token) lo = mid; else hi = mid - 1;
    }
    positions[token] = token - prompt_offsets[lo];
  }
}

int row_threads(int hidden, int* vpt) {
  const int chunks = hidden >> 3;
  int per_thread = (chunks + kRowThreadsCap - 1) / kRowThreadsCap;
  if (per_thread < 1) per_thread = 1;
  *vpt = per_thread;
  int threads = (chunks + per_thread - 1) / per_thread;
  threads = (threads + 31) & ~31;
  return threads;
}

}  // namespace

int sm_count() {
  static int cached = 0;
  if (cached == 0) {
    int device = 0;
    cudaGetDevice(&device);
    cudaDeviceGetAttribute(&cached, cudaDevAttrMultiProcessorCount, device);
    if (cached <= 0) cached = 148;
  }
  return cached;
}

// CTAs of `kernel` that fit on one SM at `threads` threads (registers and shared memory decide).
template <typename Kernel>
static int resident_per_sm(Kernel kernel, int threads) {
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, threads, 0) != cudaSuccess || blocks <= 0) {
    blocks = 1;
  }
  return blocks;
}

static int stride_grid(long long items, int threads, int ctas_per_sm) {
  const long long needed = (items + threads - 1) / threads;
  const long long cap = static_cast<long long>(sm_count()) * ctas_per_sm;
  return static_cast<int>(needed < cap ? (needed > 0 ? needed : 1) : cap);
}

template <typename T>
cudaError_t embed_typed(const int32_t* token_ids, int tokens, const void* table, int vocab, int hidden,
                        const float* gamma, float eps, float* residual, void* normed, int* status,
                        cudaStream_t stream) {
  int vpt = 1;
  const int threads = row_threads(hidden, &vpt);
  const auto* t = static_cast<const T*>(table);
  auto* n = static_cast<T*>(normed);
  auto launch = [&](auto kernel) {  // a resident grid walks the rows
    const int grid = std::max(1, std::min(tokens, sm_count() * resident_per_sm(kernel, threads)));
    kernel<<<grid, threads, 0, stream>>>(token_ids, t, tokens, vocab, hidden, gamma, eps, residual, n, status);
  };
  switch (vpt) {
    case 1: launch(embed_rms_norm_kernel<T, 1>); break;
    case 2: launch(embed_rms_norm_kernel<T, 2>); break;
    case 3: launch(embed_rms_norm_kernel<T, 3>); break;
    case 4: launch(embed_rms_norm_kernel<T, 4>); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t norm_typed(float* residual, const void* delta, const float* gamma, int tokens, int hidden, float eps,
                       void* normed, cudaStream_t stream) {
  int vpt = 1;
  const int threads = row_threads(hidden, &vpt);
  const auto* d = static_cast<const T*>(delta);
  auto* n = static_cast<T*>(normed);
  auto launch = [&](auto kernel) {  // one CTA per row
    kernel<<<tokens, threads, 0, stream>>>(residual, d, gamma, tokens, hidden, eps, n);
  };
  const bool add = delta != nullptr;
  switch (vpt) {
    case 1: add ? launch(rms_norm_residual_kernel<T, 1, true>) : launch(rms_norm_residual_kernel<T, 1, false>); break;
    case 2: add ? launch(rms_norm_residual_kernel<T, 2, true>) : launch(rms_norm_residual_kernel<T, 2, false>); break;
    case 3: add ? launch(rms_norm_residual_kernel<T, 3, true>) : launch(rms_norm_residual_kernel<T, 3, false>); break;
    case 4: add ? launch(rms_norm_residual_kernel<T, 4, true>) : launch(rms_norm_residual_kernel<T, 4, false>); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_embed_rms_norm(const int32_t* token_ids, int tokens, const void* table, int vocab,
                                  int hidden, const float* gamma, float eps, float* residual,
                                  void* normed, int* status, int dtype, cudaStream_t stream) {
  if (tokens <= 0) return cudaSuccess;
  if (hidden % 8 != 0 || hidden > 8 * 4 * kRowThreadsCap) return cudaErrorInvalidValue;
  if (dtype == kActFp16)
    return embed_typed<__half>(token_ids, tokens, table, vocab, hidden, gamma, eps, residual, normed, status, stream);
  if (dtype == kActBf16)
    return embed_typed<__nv_bfloat16>(token_ids, tokens, table, vocab, hidden, gamma, eps, residual, normed, status,
                                      stream);
  return cudaErrorInvalidValue;
}

cudaError_t launch_rms_norm_residual(float* residual, const void* delta, const float* gamma, int tokens,
                                     int hidden, float eps, void* normed, int dtype, cudaStream_t stream) {
  if (tokens <= 0) return cudaSuccess;
  if (hidden % 8 != 0 || hidden > 8 * 4 * kRowThreadsCap) return cudaErrorInvalidValue;
  if (dtype == kActFp16) return norm_typed<__half>(residual, delta, gamma, tokens, hidden, eps, normed, stream);
  if (dtype == kActBf16) return norm_typed<__nv_bfloat16>(residual, delta, gamma, tokens, hidden, eps, normed, stream);
  return cudaErrorInvalidValue;
}

cudaError_t launch_rotary_bias(void* qkv, const float* bias, const int32_t* positions, int tokens,
                               int query_heads, int kv_heads, int head_dim, const float* cos_table,
                               const float* sin_table, int table_positions, int* status, int dtype,
                               cudaStream_t stream) {
  if (tokens <= 0) return cudaSuccess;
  if (head_dim % 16 != 0 || head_dim > 1024 || tokens > (1 << 24)) return cudaErrorInvalidValue;
  const int heads = query_heads + kv_heads + (bias != nullptr ? kv_heads : 0);
  const int items = tokens * ((heads + kRopeGroupHeads - 1) / kRopeGroupHeads) * (head_dim / 16);
  const int threads = 256;
  if (dtype != kActFp16 && dtype != kActBf16) return cudaErrorInvalidValue;
  auto launch = [&](auto kernel, auto* data) {
    // one wave of resident CTAs walks all (token, head group, chunk) items (no tail wave)
    const int per_sm = resident_per_sm(kernel, threads);
    const int grid = std::max(1, std::min((items + threads - 1) / threads, sm_count() * per_sm));
    kernel<<<grid, threads, 0, stream>>>(data, bias, positions, tokens, query_heads, kv_heads, head_dim, cos_table,
                                         sin_table, table_positions, status);
  };
  if (dtype == kActFp16) {
    auto* data = static_cast<__half*>(qkv);
    if (bias != nullptr) launch(rotary_bias_kernel<__half, true>, data); else launch(rotary_bias_kernel<__half, false>, data);
  } else {
    auto* data = static_cast<__nv_bfloat16*>(qkv);
    if (bias != nullptr) launch(rotary_bias_kernel<__nv_bfloat16, true>, data);
    else launch(rotary_bias_kernel<__nv_bfloat16, false>, data);
  }
  return cudaGetLastError();
}

cudaError_t launch_rope_table(float* cos_out, float* sin_out, int positions, int head_dim, float theta,
                              cudaStream_t stream) {
  const long long items = static_cast<long long>(positions) * (head_dim / 2);
  if (items <= 0) return cudaSuccess;
  rope_table_kernel<<<stride_grid(items, 256, 8), 256, 0, stream>>>(cos_out, sin_out, positions,
                                                                     head_dim, theta);
  return cudaGetLastError();
}

cudaError_t launch_silu_multiply(const void* gate, const void* up, long long in_stride, void* out,
                                 long long out_stride, int tokens, int width, int dtype, cudaStream_t stream) {
  if (tokens <= 0 || width <= 0) return cudaSuccess;
  const long long items = static_cast<long long>(tokens) * (width / 8);
  if (items >= (1LL << 31)) return cudaErrorInvalidValue;
  const int threads = 256;
  // kSiluUnroll chunks per thread, the grid covering them all: the block scheduler keeps the SMs
  // full (274.5 us against 322.3 us for one resident wave walking the rows, 16K x 18944 fp16)
  const int grid = static_cast<int>(std::max(1LL, (items + threads * kSiluUnroll - 1) / (threads * kSiluUnroll)));
  if (dtype == kActFp16) {
    silu_multiply_kernel<__half><<<grid, threads, 0, stream>>>(static_cast<const __half*>(gate),
                                                               static_cast<const __half*>(up), in_stride,
                                                               static_cast<__half*>(out), out_stride, tokens, width);
  } else if (dtype == kActBf16) {
    silu_multiply_kernel<__nv_bfloat16><<<grid, threads, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(gate), static_cast<const __nv_bfloat16*>(up), in_stride,
        static_cast<__nv_bfloat16*>(out), out_stride, tokens, width);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_positions(const int32_t* prompt_offsets, int prompt_count, int tokens,
                             int32_t* positions, cudaStream_t stream) {
  if (tokens <= 0) return cudaSuccess;
  positions_kernel<<<stride_grid(tokens, 256, 4), 256, 0, stream>>>(prompt_offsets, prompt_count,
                                                                    tokens, positions);
  return cudaGetLastError();
}

}  // namespace arb
