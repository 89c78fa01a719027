// Seeded synthetic checkpoint generator (device side).
//
// The build's benchmarks and parity tests use random-init weights of the 7B architecture. A
// 15 GB checkpoint is too slow to write and read on every fresh GPU box, so every element is a
// pure function of (seed, tensor tag, element index) and is produced where it is needed: here
// on the device, and by the CPU checker (a separate C implementation) for the oracle and for the
// reference build. The distribution is Irwin-Hall with four 16-bit terms (mean 0, variance
// matched to the requested standard deviation, support +-3.46 sigma), rounded to bf16 with
// round-to-nearest-even. All arithmetic is integer or a single fp32 multiply, so both sides
// produce identical bits. An fp16 engine stores each bf16 value converted to fp16 with
// round-to-nearest-even (__float2half_rn), which the CPU checker reproduces with numpy's
// float32 -> float16 cast.
#include <type_traits>

#include "common.cuh"
#include "layer_kernels.h"
#include "synthetic.h"

namespace arb {
namespace {

__device__ __forceinline__ uint32_t element_bf16_bits(uint64_t key, long long index, float scale,
                                                      float offset) {
  const uint64_t bits = synthetic_mix(key ^ (kSyntheticIndexStride * static_cast<uint64_t>(index + 1)));
  const int sum = static_cast<int>((bits & 0xffffu) + ((bits >> 16) & 0xffffu) +
                                   ((bits >> 32) & 0xffffu) + (bits >> 48));
  const float value = static_cast<float>(sum - kSyntheticCentre) * scale + offset;
  return synthetic_round_bf16(__float_as_uint(value));
}

template <bool kToHalf>
__global__ void synthetic_fill_kernel(uint16_t* __restrict__ dst, long long count, uint64_t key,
                                      float scale) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const uint32_t bits = element_bf16_bits(key, i, scale, 0.0f);
    if constexpr (kToHalf) {
      dst[i] = __half_as_ushort(__float2half_rn(__uint_as_float(bits << 16)));
    } else {
      dst[i] = static_cast<uint16_t>(bits);
    }
  }
}

__global__ void bf16_to_fp16_kernel(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst, long long count) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    dst[i] = __half_as_ushort(__float2half_rn(__uint_as_float(static_cast<uint32_t>(src[i]) << 16)));
  }
}

template <typename T>
__global__ void f32_to_activation_kernel(const float* __restrict__ src, T* __restrict__ dst, long long count) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    if constexpr (std::is_same_v<T, __half>) {
      dst[i] = __float2half_rn(src[i]);
    } else {
      dst[i] = __float2bfloat16_rn(src[i]);
    }
  }
}

__global__ void synthetic_fill_f32_kernel(float* __restrict__ dst, long long count, uint64_t key,
                                          float scale, float offset) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    dst[i] = __uint_as_float(element_bf16_bits(key, i, scale, offset) << 16);
  }
}

}  // namespace

cudaError_t launch_synthetic_fill(void* dst, long long count, uint64_t key, float scale, int dtype,
                                  cudaStream_t stream) {
  if (count <= 0) return cudaSuccess;
  const int grid = sm_count() * 8;
  auto* out = static_cast<uint16_t*>(dst);
  if (dtype == kActFp16) {
    synthetic_fill_kernel<true><<<grid, 256, 0, stream>>>(out, count, key, scale);
  } else if (dtype == kActBf16) {
    synthetic_fill_kernel<false><<<grid, 256, 0, stream>>>(out, count, key, scale);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_bf16_to_fp16(const void* src, void* dst, long long count, cudaStream_t stream) {
  if (count <= 0) return cudaSuccess;
  bf16_to_fp16_kernel<<<sm_count() * 8, 256, 0, stream>>>(static_cast<const uint16_t*>(src),
                                                          static_cast<uint16_t*>(dst), count);
  return cudaGetLastError();
}

cudaError_t launch_f32_to_activation(const float* src, void* dst, long long count, int dtype, cudaStream_t stream) {
  if (count <= 0) return cudaSuccess;
  const int grid = sm_count() * 8;
  if (dtype == kActFp16) {
    f32_to_activation_kernel<__half><<<grid, 256, 0, stream>>>(src, static_cast<__half*>(dst), count);
  } else if (dtype == kActBf16) {
    f32_to_activation_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(src, static_cast<__nv_bfloat16*>(dst), count);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_synthetic_fill_f32(float* dst, long long count, uint64_t key, float scale,
                                      float offset, cudaStream_t stream) {
  if (count <= 0) return cudaSuccess;
  const int grid = sm_count() * 4;
  synthetic_fill_f32_kernel<<<grid, 256, 0, stream>>>(dst, count, key, scale, offset);
  return cudaGetLastError();
}

}  // namespace arb
