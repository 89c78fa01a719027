// Definition of the seeded synthetic checkpoint (shared by host and device code of the library).
//
// element(seed, tag, i) = bf16_rne( (u0 + u1 + u2 + u3 - 131070) * std / sd4 )
//   where u0..u3 are the four 16-bit lanes of mix(key ^ (kSyntheticIndexStride * (i + 1))),
//   key = mix(seed + kSyntheticTagStride * (tag + 1)), mix = the 64-bit MurmurHash3 finaliser,
//   sd4 = sqrt(4 * (65536^2 - 1) / 12) (standard deviation of the four-term sum).
// Tensor tags: (layer + 1) * 32 + kind, with layer = -1 for tensors outside the decoder stack.
#pragma once

#include <cmath>
#include <cstdint>

#if defined(__CUDACC__)
#define ARB_HOST_DEVICE __host__ __device__ __forceinline__
#else
#define ARB_HOST_DEVICE inline
#endif

namespace arb {

constexpr uint64_t kSyntheticTagStride = 0x9E3779B97F4A7C15ull;
constexpr uint64_t kSyntheticIndexStride = 0xD6E8FEB86659FD93ull;
constexpr int kSyntheticCentre = 131070;

enum SyntheticKind : int {
  kTensorEmbedding = 0,
  kTensorQuery = 1,
  kTensorKey = 2,
  kTensorValue = 3,
  kTensorOutput = 4,
  kTensorQueryBias = 5,
  kTensorKeyBias = 6,
  kTensorValueBias = 7,
  kTensorGate = 8,
  kTensorUp = 9,
  kTensorDown = 10,
  kTensorInputNorm = 11,
  kTensorPostNorm = 12,
  kTensorFinalNorm = 13,
  kTensorLmHead = 14,
};

ARB_HOST_DEVICE uint64_t synthetic_mix(uint64_t k) {
  k ^= k >> 33;
  k *= 0xff51afd7ed558ccdull;
  k ^= k >> 33;
  k *= 0xc4ceb9fe1a85ec53ull;
  k ^= k >> 33;
  return k;
}

ARB_HOST_DEVICE uint64_t synthetic_tensor_key(uint64_t seed, int layer, int kind) {
  const uint64_t tag = static_cast<uint64_t>((layer + 1) * 32 + kind);
  return synthetic_mix(seed + kSyntheticTagStride * (tag + 1));
}

// fp32 bit pattern -> bf16 bit pattern, round to nearest even (inputs are finite).
ARB_HOST_DEVICE uint32_t synthetic_round_bf16(uint32_t bits) {
  return (bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16;
}

inline float synthetic_scale(double standard_deviation) {
  const double sd4 = std::sqrt(4.0 * (65536.0 * 65536.0 - 1.0) / 12.0);
  return static_cast<float>(standard_deviation / sd4);
}

}  // namespace arb
