// Causal GQA prefill attention over packed variable-length prompts, with per-row log-sum-exp.
//
// Replaces the reference's materialised path (attnrank/src/model.cu:426-480: scatter into an
// fp32 KV cache, `group` x cublasSgemmStridedBatched for Q K^T, softmax_causal_kernel over a
// [Hq, T, K] fp32 score buffer, `group` x SGEMM for P V). Here scores never leave the SM: a
// flash-style online softmax keeps the running max/sum per row in registers.
//
// Besides O, the kernel writes the log2-domain log-sum-exp of every (token, head) row. The
// attention-mass kernel (mass.cu) uses it to turn raw scores into exact softmax probabilities
// in a single pass, so mass capture needs no second softmax.
//
// Tensor-core path: mma.sync m16n8k16 (fp16 or bf16 operands) with fp32 accumulation (8 warps x 16 query rows,
// 64-key tiles double-buffered with cp.async, XOR-swizzled shared memory for conflict-free
// ldmatrix). Masking follows softmax_causal_kernel (kernels.cu:117-162): key k is visible to
// query q iff k <= q, k < prompt length, and k > q - sliding_window when a window is set.
#include <cmath>
#include <type_traits>

#include "common.cuh"
#include "layer_kernels.h"

namespace arb {
namespace {

constexpr int kHeadDim = 128;
constexpr int kBlockM = kAttentionQueryTile;  // 128 query rows per CTA
constexpr int kBlockN = 64;                   // keys per tile
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kChunksPerRow = kHeadDim / 8;   // 16-byte chunks per row
constexpr int kQElems = kBlockM * kHeadDim;
constexpr int kKvElems = kBlockN * kHeadDim;
constexpr size_t kSmemBytes = (kQElems + 4 * kKvElems) * 2;  // 96 KB of 16-bit values

__device__ __forceinline__ uint32_t smem_u32(const void* pointer) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(pointer));
}

// element offset of (row, col) in a [rows][128] 16-bit tile with 16-byte chunks XOR-swizzled by row
__device__ __forceinline__ int swizzle(int row, int col) {
  return row * kHeadDim + ((((col >> 3) ^ (row & 7))) << 3) + (col & 7);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t address, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                            uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(address));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t address, uint32_t& r0, uint32_t& r1,
                                                  uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(address));
}

template <typename T>
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same_v<T, __half>) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    causal_attention_kernel(const T* __restrict__ qkv, T* __restrict__ out,
                            float* __restrict__ lse, const int32_t* __restrict__ prompt_offsets,
                            const int32_t* __restrict__ tiles, int query_heads, int kv_heads,
                            int sliding_window) {
  extern __shared__ __align__(128) uint8_t smem_bytes[];
  T* smem = reinterpret_cast<T*>(smem_bytes);
  T* q_smem = smem;
  T* k_smem = smem + kQElems;                 // [2][64][128]
  T* v_smem = smem + kQElems + 2 * kKvElems;  // [2][64][128]

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int prompt = tiles[2 * blockIdx.x];
  const int query_tile = tiles[2 * blockIdx.x + 1];
  const int head = blockIdx.y;
  const int group = query_heads / kv_heads;
  const int kv_head = head / group;
  const int row_width = (query_heads + 2 * kv_heads) * kHeadDim;
  const int out_width = query_heads * kHeadDim;
  const int prompt_begin = prompt_offsets[prompt];
  const int length = prompt_offsets[prompt + 1] - prompt_begin;
  const int q0 = query_tile * kBlockM;
  const T* base = qkv + static_cast<size_t>(prompt_begin) * row_width;
  const T* q_base = base + head * kHeadDim;
  const T* k_base = base + (query_heads + kv_head) * kHeadDim;
  const T* v_base = base + (query_heads + kv_heads + kv_head) * kHeadDim;

  // ---- query tile -> shared (rows past the prompt are zero-filled)
#pragma unroll
  for (int i = 0; i < (kBlockM * kChunksPerRow) / kThreads; ++i) {
    const int id = tid + i * kThreads;
    const int row = id / kChunksPerRow;
    const int chunk = id % kChunksPerRow;
    const bool valid = q0 + row < length;
    const T* src = valid ? q_base + static_cast<size_t>(q0 + row) * row_width + chunk * 8 : qkv;
    cp_async16(smem_u32(q_smem + swizzle(row, chunk * 8)), src, valid ? 16 : 0);
  }
  cp_async_commit();

  const int last_query = min(q0 + kBlockM, length) - 1;
  const int first_key = sliding_window > 0 ? max(0, q0 - sliding_window + 1) : 0;
  const int tile_begin = first_key / kBlockN;
  const int tile_end = last_query / kBlockN + 1;

  auto load_kv = [&](int tile, int stage) {
    const int k0 = tile * kBlockN;
#pragma unroll
    for (int i = 0; i < (kBlockN * kChunksPerRow) / kThreads; ++i) {
      const int id = tid + i * kThreads;
      const int row = id / kChunksPerRow;
      const int chunk = id % kChunksPerRow;
      const bool valid = k0 + row < length;
      const size_t offset = static_cast<size_t>(k0 + row) * row_width + chunk * 8;
      const int dst = stage * kKvElems + swizzle(row, chunk * 8);
      cp_async16(smem_u32(k_smem + dst), valid ? k_base + offset : qkv, valid ? 16 : 0);
      cp_async16(smem_u32(v_smem + dst), valid ? v_base + offset : qkv, valid ? 16 : 0);
    }
    cp_async_commit();
  };

  if (tile_begin < tile_end) load_kv(tile_begin, 0);

  cp_async_wait<1>();  // query tile landed (the first K/V tile may still be in flight)
  __syncthreads();

  uint32_t qa[8][4];
  {
    const int row = warp * 16 + (lane & 15);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int col = kk * 16 + (lane >> 4) * 8;
      ldmatrix_x4(smem_u32(q_smem + swizzle(row, col)), qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
    }
  }

  const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(kHeadDim));
  const int g = lane >> 2;
  const int t = lane & 3;
  const int row_lo = q0 + warp * 16 + g;  // prompt-relative query index of accumulator rows c0/c1
  const int row_hi = row_lo + 8;          // ... and of c2/c3
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.0f, l_hi = 0.0f;

  for (int tile = tile_begin; tile < tile_end; ++tile) {
    const int stage = (tile - tile_begin) & 1;
    if (tile + 1 < tile_end) {
      load_kv(tile + 1, stage ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();

    const T* kt = k_smem + stage * kKvElems;
    const T* vt = v_smem + stage * kKvElems;
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.0f;
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      const int key_row = np * 16 + (lane >> 4) * 8 + (lane & 7);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int col = kk * 16 + ((lane >> 3) & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(smem_u32(kt + swizzle(key_row, col)), b0, b1, b2, b3);
        mma_16816<T>(s[2 * np], qa[kk], b0, b1);
        mma_16816<T>(s[2 * np + 1], qa[kk], b2, b3);
      }
    }

    const int k0 = tile * kBlockN;
    float tile_max_lo = -INFINITY, tile_max_hi = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = k0 + nt * 8 + 2 * t + e;
        const bool ok_lo = key <= row_lo && key < length && (sliding_window <= 0 || key > row_lo - sliding_window);
        const bool ok_hi = key <= row_hi && key < length && (sliding_window <= 0 || key > row_hi - sliding_window);
        s[nt][e] = ok_lo ? s[nt][e] * scale_log2 : -INFINITY;
        s[nt][2 + e] = ok_hi ? s[nt][2 + e] * scale_log2 : -INFINITY;
        tile_max_lo = fmaxf(tile_max_lo, s[nt][e]);
        tile_max_hi = fmaxf(tile_max_hi, s[nt][2 + e]);
      }
    }
    tile_max_lo = fmaxf(tile_max_lo, __shfl_xor_sync(0xffffffffu, tile_max_lo, 1));
    tile_max_lo = fmaxf(tile_max_lo, __shfl_xor_sync(0xffffffffu, tile_max_lo, 2));
    tile_max_hi = fmaxf(tile_max_hi, __shfl_xor_sync(0xffffffffu, tile_max_hi, 1));
    tile_max_hi = fmaxf(tile_max_hi, __shfl_xor_sync(0xffffffffu, tile_max_hi, 2));
    const float new_lo = fmaxf(m_lo, tile_max_lo);
    const float new_hi = fmaxf(m_hi, tile_max_hi);
    const float ref_lo = new_lo == -INFINITY ? 0.0f : new_lo;
    const float ref_hi = new_hi == -INFINITY ? 0.0f : new_hi;
    const float alpha_lo = exp2f(m_lo - ref_lo);
    const float alpha_hi = exp2f(m_hi - ref_hi);
    m_lo = new_lo;
    m_hi = new_hi;

    float sum_lo = 0.0f, sum_hi = 0.0f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = exp2f(s[nt][0] - ref_lo);
      s[nt][1] = exp2f(s[nt][1] - ref_lo);
      s[nt][2] = exp2f(s[nt][2] - ref_hi);
      s[nt][3] = exp2f(s[nt][3] - ref_hi);
      sum_lo += s[nt][0] + s[nt][1];
      sum_hi += s[nt][2] + s[nt][3];
    }
    l_lo = l_lo * alpha_lo + sum_lo;
    l_hi = l_hi * alpha_hi + sum_hi;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      o[dt][0] *= alpha_lo;
      o[dt][1] *= alpha_lo;
      o[dt][2] *= alpha_hi;
      o[dt][3] *= alpha_hi;
    }

#pragma unroll
    for (int kk2 = 0; kk2 < 4; ++kk2) {
      uint32_t pa[4];
      pa[0] = pack2<T>(s[2 * kk2][0], s[2 * kk2][1]);
      pa[1] = pack2<T>(s[2 * kk2][2], s[2 * kk2][3]);
      pa[2] = pack2<T>(s[2 * kk2 + 1][0], s[2 * kk2 + 1][1]);
      pa[3] = pack2<T>(s[2 * kk2 + 1][2], s[2 * kk2 + 1][3]);
      const int key_row = kk2 * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        const int col = dp * 16 + (lane >> 4) * 8;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(smem_u32(vt + swizzle(key_row, col)), b0, b1, b2, b3);
        mma_16816<T>(o[2 * dp], pa, b0, b1);
        mma_16816<T>(o[2 * dp + 1], pa, b2, b3);
      }
    }
    __syncthreads();  // the stage is refilled by the next iteration's prefetch
  }

  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
  const float inv_lo = l_lo > 0.0f ? 1.0f / l_lo : 0.0f;
  const float inv_hi = l_hi > 0.0f ? 1.0f / l_hi : 0.0f;

  if (row_lo < length) {
    T* dst = out + static_cast<size_t>(prompt_begin + row_lo) * out_width + head * kHeadDim;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      *reinterpret_cast<uint32_t*>(dst + dt * 8 + 2 * t) = pack2<T>(o[dt][0] * inv_lo, o[dt][1] * inv_lo);
    }
    if (t == 0) {
      lse[static_cast<size_t>(prompt_begin + row_lo) * query_heads + head] =
          l_lo > 0.0f ? m_lo + log2f(l_lo) : -INFINITY;
    }
  }
  if (row_hi < length) {
    T* dst = out + static_cast<size_t>(prompt_begin + row_hi) * out_width + head * kHeadDim;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      *reinterpret_cast<uint32_t*>(dst + dt * 8 + 2 * t) = pack2<T>(o[dt][2] * inv_hi, o[dt][3] * inv_hi);
    }
    if (t == 0) {
      lse[static_cast<size_t>(prompt_begin + row_hi) * query_heads + head] =
          l_hi > 0.0f ? m_hi + log2f(l_hi) : -INFINITY;
    }
  }
}

// internal linkage: its per-device flag belongs to this copy of the library (a template with
// external linkage would share one flag with any other copy loaded into the same process)
template <typename T>
cudaError_t launch_typed(const AttentionArgs& args, cudaStream_t stream) {
  int device = 0;
  cudaGetDevice(&device);
  static uint64_t configured_devices = 0;  // the shared-memory opt-in is a per-device attribute
  if (device >= 64 || !(configured_devices & (1ull << device))) {
    const cudaError_t status = cudaFuncSetAttribute(
        causal_attention_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes));
    if (status != cudaSuccess) return status;
    if (device < 64) configured_devices |= 1ull << device;
  }
  const dim3 grid(args.tile_count, args.query_heads);
  causal_attention_kernel<T><<<grid, kThreads, kSmemBytes, stream>>>(
      static_cast<const T*>(args.qkv), static_cast<T*>(args.out), args.lse, args.prompt_offsets, args.tiles,
      args.query_heads, args.kv_heads, args.sliding_window);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_causal_attention(const AttentionArgs& args, cudaStream_t stream) {
  if (args.tile_count <= 0) return cudaSuccess;
  if (args.head_dim != kHeadDim || args.kv_heads <= 0 || args.query_heads % args.kv_heads != 0) {
    return cudaErrorInvalidValue;
  }
  if (args.dtype == kActFp16) return launch_typed<__half>(args, stream);
  if (args.dtype == kActBf16) return launch_typed<__nv_bfloat16>(args, stream);
  return cudaErrorInvalidValue;
}

}  // namespace arb
