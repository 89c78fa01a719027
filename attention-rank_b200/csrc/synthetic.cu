// Seeded synthetic checkpoint generator (device side).
//
// The build's benchmarks and parity tests use random-init weights of the 7B architecture. A
// 15 GB checkpoint is too slow to write and read on every fresh GPU box, so every element is a
// pure function of (seed, tensor tag, element index) and is produced where it is needed: here
// on the device, and by the CPU checker (a separate C implementation) for the oracle and for the
// reference build. The distribution is Irwin-Hall with four 16-bit terms (mean 0, variance
// matched to the requested standard deviation, support +-3.46 sigma), rounded to bf16 with
// round-to-nearest-even. All arithmetic is integer or a single fp32 multiply, so both sides
// produce identical bits.
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

__global__ void synthetic_fill_kernel(uint16_t* __restrict__ dst, long long count, uint64_t key,
                                      float scale) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    dst[i] = static_cast<uint16_t>(element_bf16_bits(key, i, scale, 0.0f));
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

cudaError_t launch_synthetic_fill(void* dst_bf16, long long count, uint64_t key, float scale,
                                  cudaStream_t stream) {
  if (count <= 0) return cudaSuccess;
  const int grid = sm_count() * 8;
  synthetic_fill_kernel<<<grid, 256, 0, stream>>>(static_cast<uint16_t*>(dst_bf16), count, key, scale);
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
