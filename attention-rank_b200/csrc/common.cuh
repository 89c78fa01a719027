// Shared device helpers for the attention-profiling kernels (sm_100a only).
//
// Every kernel in this library works on bf16 activations with fp32 arithmetic and
// 128-bit global accesses. Host-visible error reporting goes through a device status
// word (`int* status`): kernels never trap; they record a code and skip the access.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace arb {

// Device status codes written by kernels into the caller's status word (first writer wins).
enum DeviceStatus : int {
  kStatusOk = 0,
  kStatusTokenOutOfRange = 1,   // a token id outside [0, vocab)
  kStatusPositionOutOfRange = 2,  // a RoPE position beyond the cos/sin table
  kStatusWaitTimeout = 3,       // an mbarrier wait exceeded its iteration limit
};

__device__ __forceinline__ void report_status(int* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

struct alignas(16) Bf16x8 {
  __nv_bfloat162 h[4];
};

__device__ __forceinline__ void unpack8(const uint4& raw, float (&out)[8]) {
  const __nv_bfloat162* pairs = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(pairs[i]);
    out[2 * i] = f.x;
    out[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&in)[8]) {
  uint4 raw;
  __nv_bfloat162* pairs = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) pairs[i] = __floats2bfloat162_rn(in[2 * i], in[2 * i + 1]);
  return raw;
}

__device__ __forceinline__ float warp_sum(float value) {
#pragma unroll
  for (int offset = 16; offset > 0; offset >>= 1) value += __shfl_xor_sync(0xffffffffu, value, offset);
  return value;
}

// Sum over the whole block; every thread receives the total. `scratch` needs one float per warp.
__device__ __forceinline__ float block_sum(float value, float* scratch) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int warps = (blockDim.x + 31) >> 5;
  value = warp_sum(value);
  if (lane == 0) scratch[warp] = value;
  __syncthreads();
  float total = lane < warps ? scratch[lane] : 0.0f;
  total = warp_sum(total);
  return total;
}

__device__ __forceinline__ uint4 load_nc(const void* pointer) {
  return __ldg(reinterpret_cast<const uint4*>(pointer));
}

// Streaming load: the data is read exactly once by this kernel.
__device__ __forceinline__ uint4 load_stream(const void* pointer) {
  uint4 value;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(value.x), "=r"(value.y), "=r"(value.z), "=r"(value.w)
               : "l"(pointer));
  return value;
}

__device__ __forceinline__ float4 load_stream_f4(const float* pointer) {
  float4 value;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(value.x), "=f"(value.y), "=f"(value.z), "=f"(value.w)
               : "l"(pointer));
  return value;
}

}  // namespace arb
