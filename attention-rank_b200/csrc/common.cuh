// Shared device helpers for the attention-profiling kernels (sm_100a only).
//
// Every kernel in this library works on 16-bit activations (fp16 by default, bf16 optional)
// with fp32 arithmetic and 128-bit global accesses. Host-visible error reporting goes through a device status
// word (`int* status`): kernels never trap; they record a code and skip the access.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
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

// Activation element types. The engine computes its GEMM operands and activations in fp16 (the
// reference's GEMM operand type, model.cu:353-365) by default; bf16 is the alternative.
enum ActivationType : int { kActFp16 = 1, kActBf16 = 2 };  // values of AR_DTYPE_F16 / AR_DTYPE_BF16

template <typename T>
struct Pair;
template <>
struct Pair<__half> {
  using type = __half2;
  static __device__ __forceinline__ float2 to_float2(type v) { return __half22float2(v); }
  static __device__ __forceinline__ type from_floats(float lo, float hi) { return __floats2half2_rn(lo, hi); }
};
template <>
struct Pair<__nv_bfloat16> {
  using type = __nv_bfloat162;
  static __device__ __forceinline__ float2 to_float2(type v) { return __bfloat1622float2(v); }
  static __device__ __forceinline__ type from_floats(float lo, float hi) { return __floats2bfloat162_rn(lo, hi); }
};

// eight 16-bit values (one 128-bit access) <-> eight floats
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& raw, float (&out)[8]) {
  const auto* pairs = reinterpret_cast<const typename Pair<T>::type*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = Pair<T>::to_float2(pairs[i]);
    out[2 * i] = f.x;
    out[2 * i + 1] = f.y;
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&in)[8]) {
  uint4 raw;
  auto* pairs = reinterpret_cast<typename Pair<T>::type*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) pairs[i] = Pair<T>::from_floats(in[2 * i], in[2 * i + 1]);
  return raw;
}

// two floats -> two 16-bit values in one 32-bit word, `lo` in the low half
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const typename Pair<T>::type v = Pair<T>::from_floats(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
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
