// Single-token decode kernels (declarations and the reference mapping in decode.h).
//
// Matrix-vector products: a CTA of 8 warps stages x in shared memory once, then every warp
// walks work items (2 or 4 weight rows) with a grid stride. A lane keeps kLoadsInFlight
// 16-byte streaming loads (ld.global.nc.L1::no_allocate) outstanding before its first FMA, so an
// SM holds 32 KB per resident CTA in flight -- the weights are read once per step and never
// cached. Accumulation is fp32; each row ends with a warp butterfly sum.
#include <cfloat>
#include <climits>

#include "common.cuh"
#include "decode.h"
#include "layer_kernels.h"

namespace arb {

int sm_count();

namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kLoadsInFlight = 8;  // 16-byte weight loads per lane before the first FMA
constexpr int kDecodeThreads = 128;
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

template <typename T>
__device__ __forceinline__ void stage_vector(const T* __restrict__ x, int chunks, uint4* xs) {
  for (int i = threadIdx.x; i < chunks; i += blockDim.x) xs[i] = load_nc(x + 8 * static_cast<size_t>(i));
  __syncthreads();
}

// acc[r] = rows[r][0, 8 chunks) . x for the whole warp (every lane receives the sums)
template <typename T, int kRows>
__device__ __forceinline__ void warp_dot(const T* (&rows)[kRows], const uint4* __restrict__ xs, int chunks,
                                         float (&acc)[kRows]) {
  constexpr int kUnroll = kLoadsInFlight / kRows;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int r = 0; r < kRows; ++r) acc[r] = 0.0f;
  int c = lane;
  for (; c + 32 * (kUnroll - 1) < chunks; c += 32 * kUnroll) {
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
  for (; c < chunks; c += 32) {
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

template <typename T, bool kF32Out>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const T* __restrict__ w, const T* __restrict__ x,
                                                            int rows, int k, void* __restrict__ y) {
  extern __shared__ uint4 xs[];
  const int chunks = k >> 3;
  stage_vector<T>(x, chunks, xs);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int items = (rows + 1) >> 1;
  for (int item = blockIdx.x * kGemvWarps + warp; item < items; item += gridDim.x * kGemvWarps) {
    const int r0 = 2 * item;
    const bool pair = r0 + 1 < rows;
    const T* row_ptr[2] = {w + static_cast<size_t>(r0) * k, w + static_cast<size_t>(pair ? r0 + 1 : r0) * k};
    float acc[2];
    warp_dot<T, 2>(row_ptr, xs, chunks, acc);
    if (lane == 0) {
      if constexpr (kF32Out) {
        float* out = static_cast<float*>(y);
        out[r0] = acc[0];
        if (pair) out[r0 + 1] = acc[1];
      } else {
        T* out = static_cast<T*>(y);
        if (pair) {
          *reinterpret_cast<uint32_t*>(out + r0) = pack2<T>(acc[0], acc[1]);
        } else {
          out[r0] = Scalar<T>::from(acc[0]);
        }
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kGemvThreads) gate_up_kernel(const T* __restrict__ w, const T* __restrict__ x,
                                                               int inter, int k, T* __restrict__ act) {
  extern __shared__ uint4 xs[];
  const int chunks = k >> 3;
  stage_vector<T>(x, chunks, xs);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int items = (inter + 1) >> 1;
  for (int item = blockIdx.x * kGemvWarps + warp; item < items; item += gridDim.x * kGemvWarps) {
    const int j0 = 2 * item;
    const bool pair = j0 + 1 < inter;
    const int j1 = pair ? j0 + 1 : j0;
    const T* row_ptr[4] = {w + static_cast<size_t>(j0) * k, w + static_cast<size_t>(j1) * k,
                           w + static_cast<size_t>(inter + j0) * k, w + static_cast<size_t>(inter + j1) * k};
    float acc[4];
    warp_dot<T, 4>(row_ptr, xs, chunks, acc);
    if (lane == 0) {
      // silu(g) * u = g / (1 + e^-g) * u on the 16-bit projections, as the prefill's SwiGLU kernel
      float a[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float g = round16<T>(acc[i]);
        const float u = round16<T>(acc[2 + i]);
        a[i] = __fdividef(g, 1.0f + __expf(-g)) * u;
      }
      if (pair) {
        *reinterpret_cast<uint32_t*>(act + j0) = pack2<T>(a[0], a[1]);
      } else {
        act[j0] = Scalar<T>::from(a[0]);
      }
    }
  }
}

// q|k|v projection of the step's token. Work item = 4 rows of one head: for query and key heads
// the rotation pairs (2j, 2j + D/2) and (2j + 1, 2j + 1 + D/2), for value heads rows 4j .. 4j + 3.
template <typename T>
__global__ void __launch_bounds__(kGemvThreads) qkv_rope_kernel(DecodeQkvArgs a) {
  extern __shared__ uint4 xs[];
  const int chunks = a.hidden >> 3;
  stage_vector<T>(static_cast<const T*>(a.x), chunks, xs);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int D = a.head_dim;
  const int half = D >> 1;
  const int per_head = D >> 2;
  const int rotated = a.query_heads + a.kv_heads;
  const int heads = rotated + a.kv_heads;
  const int items = heads * per_head;
  const int position = a.state[1];
  const bool valid = position >= 0 && position < a.table_positions && position < a.context;
  if (!valid && blockIdx.x == 0 && threadIdx.x == 0) report_status(a.status, kStatusPositionOutOfRange);
  const T* w = static_cast<const T*>(a.w);
  const T* bias_half = static_cast<const T*>(a.bias_half);
  for (int item = blockIdx.x * kGemvWarps + warp; item < items; item += gridDim.x * kGemvWarps) {
    const int head = item / per_head;
    const int j = item - head * per_head;
    const bool rotate = head < rotated;
    int row[4];
    if (rotate) {
      row[0] = head * D + 2 * j;
      row[1] = row[0] + 1;
      row[2] = row[0] + half;
      row[3] = row[2] + 1;
    } else {
#pragma unroll
      for (int r = 0; r < 4; ++r) row[r] = head * D + 4 * j + r;
    }
    const T* row_ptr[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) row_ptr[r] = w + static_cast<size_t>(row[r]) * a.hidden;
    float acc[4];
    warp_dot<T, 4>(row_ptr, xs, chunks, acc);
    if (lane != 0 || !valid) continue;
    float v[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      float value = acc[r];
      if (bias_half != nullptr) value += Scalar<T>::to(bias_half[row[r]]);
      value = round16<T>(value);
      if (a.bias != nullptr) value += a.bias[row[r]];
      v[r] = value;
    }
    if (rotate) {
      const size_t at = static_cast<size_t>(position) * half + 2 * j;
      const float c0 = a.cos_table[at], c1 = a.cos_table[at + 1];
      const float s0 = a.sin_table[at], s1 = a.sin_table[at + 1];
      const float lo0 = v[0] * c0 - v[2] * s0;
      const float hi0 = v[2] * c0 + v[0] * s0;
      const float lo1 = v[1] * c1 - v[3] * s1;
      const float hi1 = v[3] * c1 + v[1] * s1;
      T* dst = head < a.query_heads
                   ? static_cast<T*>(a.q_out) + static_cast<size_t>(head) * D
                   : static_cast<T*>(a.k_cache) +
                         (static_cast<size_t>(head - a.query_heads) * a.context + position) * D;
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
}

__device__ __forceinline__ float warp_max(float value) {
#pragma unroll
  for (int offset = 16; offset > 0; offset >>= 1) value = fmaxf(value, __shfl_xor_sync(0xffffffffu, value, offset));
  return value;
}

// One CTA per (key-range split, KV head). Warp w owns query heads w, w + 4, ... of the group:
// lane l scores keys l and l + 32 of each 64-key pass (scores scaled into log2 units), keeps the
// online-softmax max and sum, and accumulates output dims 4l .. 4l + 3 in fp32.
template <typename T>
__global__ void __launch_bounds__(kDecodeThreads) decode_attention_kernel(DecodeAttentionArgs a, float scale_log2) {
  __shared__ float q_s[kDecodeMaxGroup][kDecodeDim];
  __shared__ __align__(16) T k_s[kDecodeKeys][kKeyStride];
  __shared__ __align__(16) T v_s[kDecodeKeys][kDecodeDim];
  __shared__ float p_s[kDecodeMaxGroup][kDecodeKeys];
  constexpr int kHeadsPerWarp = kDecodeMaxGroup / (kDecodeThreads / 32);
  const int split = blockIdx.x;
  const int kv_head = blockIdx.y;
  const int group = a.query_heads / a.kv_heads;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int position = a.state[1];
  const bool valid = position >= 0 && position < a.context;
  const int length = valid ? position + 1 : 0;
  const int first = a.sliding_window > 0 && length > a.sliding_window ? length - a.sliding_window : 0;
  const int span = length - first;
  const int per_split = (span + kDecodeSplits - 1) / kDecodeSplits;
  const int begin = first + split * per_split;
  const int end = min(begin + per_split, length);

  for (int i = threadIdx.x; i < group * kDecodeDim; i += kDecodeThreads) {
    const int g = i / kDecodeDim;
    const int d = i - g * kDecodeDim;
    q_s[g][d] = Scalar<T>::to(static_cast<const T*>(a.q)[static_cast<size_t>(kv_head * group + g) * kDecodeDim + d]) *
                scale_log2;
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
  const T* k_head = static_cast<const T*>(a.k_cache) + static_cast<size_t>(kv_head) * a.context * kDecodeDim;
  const T* v_head = static_cast<const T*>(a.v_cache) + static_cast<size_t>(kv_head) * a.context * kDecodeDim;
  for (int base = begin; base < end; base += kDecodeKeys) {
    const int keys = min(kDecodeKeys, end - base);
    __syncthreads();  // q_s written / the previous pass's K, V and P consumed
    for (int i = threadIdx.x; i < keys * (kDecodeDim / 8); i += kDecodeThreads) {
      const int key = i / (kDecodeDim / 8);
      const int c = i - key * (kDecodeDim / 8);
      const size_t at = static_cast<size_t>(base + key) * kDecodeDim + 8 * c;
      *reinterpret_cast<uint4*>(&k_s[key][8 * c]) = load_nc(k_head + at);
      *reinterpret_cast<uint4*>(&v_s[key][8 * c]) = load_nc(v_head + at);
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < kHeadsPerWarp; ++h) {
      const int g = warp + 4 * h;
      if (g >= group) break;
      float s[2];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int key = lane + 32 * half;
        s[half] = -INFINITY;
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
          s[half] = dot;
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
    const int g = warp + 4 * h;
    if (g >= group) break;
    const int head = kv_head * group + g;
    const size_t slot = static_cast<size_t>(head) * kDecodeSplits + split;
    *reinterpret_cast<float4*>(a.partials + slot * kDecodeDim + 4 * lane) = make_float4(o[h][0], o[h][1], o[h][2], o[h][3]);
    if (lane == 0) {
      a.stats[2 * slot] = m[h];  // -inf for an empty split
      a.stats[2 * slot + 1] = l[h];
    }
  }
}

// out[h, d] = sum_s 2^(m_s - M) O_s[d] / sum_s 2^(m_s - M) l_s over the splits of head h.
template <typename T>
__global__ void __launch_bounds__(kDecodeDim) decode_combine_kernel(const float* __restrict__ partials,
                                                                    const float* __restrict__ stats, T* __restrict__ out) {
  const int head = blockIdx.x;
  const int d = threadIdx.x;
  const float* st = stats + static_cast<size_t>(head) * kDecodeSplits * 2;
  float top = -INFINITY;
  for (int s = 0; s < kDecodeSplits; ++s) top = fmaxf(top, st[2 * s]);
  float sum = 0.0f;
  float acc = 0.0f;
  for (int s = 0; s < kDecodeSplits; ++s) {
    const float m = st[2 * s];
    if (m == -INFINITY) continue;
    const float weight = exp2f(m - top);
    sum = fmaf(weight, st[2 * s + 1], sum);
    acc = fmaf(weight, partials[(static_cast<size_t>(head) * kDecodeSplits + s) * kDecodeDim + d], acc);
  }
  out[static_cast<size_t>(head) * kDecodeDim + d] = Scalar<T>::from(sum > 0.0f ? acc / sum : 0.0f);
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
  // larger value wins; equal values: the smaller index (the first maximum overall)
#pragma unroll
  for (int offset = 16; offset > 0; offset >>= 1) {
    const float other = __shfl_xor_sync(0xffffffffu, best, offset);
    const int other_index = __shfl_xor_sync(0xffffffffu, index, offset);
    if (other > best || (other == best && other_index < index)) {
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
      if (other > best || (other == best && other_index < index)) {
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

template <typename Kernel>
int gemv_grid(Kernel kernel, long long items, size_t smem) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kGemvThreads, smem) != cudaSuccess || per_sm <= 0) {
    per_sm = 1;
  }
  const long long needed = (items + kGemvWarps - 1) / kGemvWarps;
  const long long cap = static_cast<long long>(sm_count()) * per_sm;
  return static_cast<int>(needed < cap ? (needed > 0 ? needed : 1) : cap);
}

// x staged in dynamic shared memory: opt in above the 48 KB default once per kernel
template <typename Kernel>
cudaError_t prepare_smem(Kernel kernel, size_t smem) {
  if (smem <= 48 * 1024) return cudaSuccess;
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
}

template <typename T>
cudaError_t gemv_typed(const void* w, const void* x, int rows, int k, void* y, bool f32_out, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(k) * 2;
  const long long items = (rows + 1) / 2;
  if (f32_out) {
    auto kernel = gemv_kernel<T, true>;
    cudaError_t status = prepare_smem(kernel, smem);
    if (status != cudaSuccess) return status;
    kernel<<<gemv_grid(kernel, items, smem), kGemvThreads, smem, stream>>>(static_cast<const T*>(w),
                                                                          static_cast<const T*>(x), rows, k, y);
  } else {
    auto kernel = gemv_kernel<T, false>;
    cudaError_t status = prepare_smem(kernel, smem);
    if (status != cudaSuccess) return status;
    kernel<<<gemv_grid(kernel, items, smem), kGemvThreads, smem, stream>>>(static_cast<const T*>(w),
                                                                          static_cast<const T*>(x), rows, k, y);
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t gate_up_typed(const void* w, const void* x, int inter, int k, void* act, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(k) * 2;
  auto kernel = gate_up_kernel<T>;
  cudaError_t status = prepare_smem(kernel, smem);
  if (status != cudaSuccess) return status;
  kernel<<<gemv_grid(kernel, (inter + 1) / 2, smem), kGemvThreads, smem, stream>>>(
      static_cast<const T*>(w), static_cast<const T*>(x), inter, k, static_cast<T*>(act));
  return cudaGetLastError();
}

template <typename T>
cudaError_t qkv_typed(const DecodeQkvArgs& args, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(args.hidden) * 2;
  auto kernel = qkv_rope_kernel<T>;
  cudaError_t status = prepare_smem(kernel, smem);
  if (status != cudaSuccess) return status;
  const long long items = static_cast<long long>(args.query_heads + 2 * args.kv_heads) * (args.head_dim / 4);
  kernel<<<gemv_grid(kernel, items, smem), kGemvThreads, smem, stream>>>(args);
  return cudaGetLastError();
}

template <typename T>
cudaError_t attention_typed(const DecodeAttentionArgs& args, cudaStream_t stream) {
  const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(args.head_dim));
  decode_attention_kernel<T><<<dim3(kDecodeSplits, args.kv_heads), kDecodeThreads, 0, stream>>>(args, scale_log2);
  cudaError_t status = cudaGetLastError();
  if (status != cudaSuccess) return status;
  decode_combine_kernel<T><<<args.query_heads, kDecodeDim, 0, stream>>>(args.partials, args.stats,
                                                                        static_cast<T*>(args.out));
  return cudaGetLastError();
}

bool valid_dtype(int dtype) { return dtype == kActFp16 || dtype == kActBf16; }

}  // namespace

cudaError_t launch_decode_gemv(const void* w, const void* x, int rows, int k, void* y, bool f32_out, int dtype,
                               cudaStream_t stream) {
  if (rows <= 0 || k <= 0 || k % 8 != 0 || !valid_dtype(dtype)) return cudaErrorInvalidValue;
  return dtype == kActFp16 ? gemv_typed<__half>(w, x, rows, k, y, f32_out, stream)
                           : gemv_typed<__nv_bfloat16>(w, x, rows, k, y, f32_out, stream);
}

cudaError_t launch_decode_gate_up(const void* w, const void* x, int inter, int k, void* act, int dtype,
                                  cudaStream_t stream) {
  if (inter <= 0 || k <= 0 || k % 8 != 0 || !valid_dtype(dtype)) return cudaErrorInvalidValue;
  return dtype == kActFp16 ? gate_up_typed<__half>(w, x, inter, k, act, stream)
                           : gate_up_typed<__nv_bfloat16>(w, x, inter, k, act, stream);
}

cudaError_t launch_decode_qkv(const DecodeQkvArgs& args, cudaStream_t stream) {
  if (args.hidden <= 0 || args.hidden % 8 != 0 || args.head_dim % 4 != 0 || args.query_heads <= 0 ||
      args.kv_heads <= 0 || args.context <= 0 || !valid_dtype(args.dtype)) {
    return cudaErrorInvalidValue;
  }
  return args.dtype == kActFp16 ? qkv_typed<__half>(args, stream) : qkv_typed<__nv_bfloat16>(args, stream);
}

cudaError_t launch_decode_attention(const DecodeAttentionArgs& args, cudaStream_t stream) {
  if (args.head_dim != kDecodeDim || args.kv_heads <= 0 || args.query_heads % args.kv_heads != 0 ||
      args.query_heads / args.kv_heads > kDecodeMaxGroup || args.context <= 0 || !valid_dtype(args.dtype)) {
    return cudaErrorInvalidValue;
  }
  return args.dtype == kActFp16 ? attention_typed<__half>(args, stream)
                                : attention_typed<__nv_bfloat16>(args, stream);
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
