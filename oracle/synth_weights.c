/*
 * CPU checker, test infrastructure only: the seeded synthetic checkpoint, restated in plain C.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs use this file
 * (through liboracle.so); the product generates the same weights on the GPU
 * (attention-rank_b200/csrc/synthetic.cu). The two are written separately and a test checks
 * that they agree bit for bit.
 *
 * element(seed, layer, kind, i):
 *   key  = mix(seed + 0x9E3779B97F4A7C15 * (tag + 1)),  tag = (layer + 1) * 32 + kind
 *   bits = mix(key ^ (0xD6E8FEB86659FD93 * (i + 1)))
 *   sum  = bits[0:16) + bits[16:32) + bits[32:48) + bits[48:64)   (Irwin-Hall, 4 terms)
 *   value = bf16_rne((float)(sum - 131070) * scale + offset),  scale = std / sqrt(4 (65536^2 - 1) / 12)
 * mix is the MurmurHash3 64-bit finaliser.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static uint64_t mix64(uint64_t k) {
  k ^= k >> 33;
  k *= 0xff51afd7ed558ccdULL;
  k ^= k >> 33;
  k *= 0xc4ceb9fe1a85ec53ULL;
  k ^= k >> 33;
  return k;
}

uint64_t oracle_tensor_key(uint64_t seed, int layer, int kind) {
  const uint64_t tag = (uint64_t)((layer + 1) * 32 + kind);
  return mix64(seed + 0x9E3779B97F4A7C15ULL * (tag + 1));
}

float oracle_scale(double standard_deviation) {
  return (float)(standard_deviation / sqrt(4.0 * (65536.0 * 65536.0 - 1.0) / 12.0));
}

static uint16_t element_bits(uint64_t key, int64_t index, float scale, float offset) {
  const uint64_t h = mix64(key ^ (0xD6E8FEB86659FD93ULL * (uint64_t)(index + 1)));
  const int sum = (int)((h & 0xffffu) + ((h >> 16) & 0xffffu) + ((h >> 32) & 0xffffu) + (h >> 48));
  const float product = (float)(sum - 131070) * scale;
  const float value = product + offset;
  uint32_t bits;
  memcpy(&bits, &value, sizeof(bits));
  return (uint16_t)((bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16);
}

/* bf16 bit patterns of elements [first, first + count) of one tensor. */
void oracle_fill_bf16(uint16_t* out, int64_t first, int64_t count, uint64_t seed, int layer, int kind,
                      double standard_deviation) {
  const uint64_t key = oracle_tensor_key(seed, layer, kind);
  const float scale = oracle_scale(standard_deviation);
#pragma omp parallel for schedule(static) if (count > (1 << 20))
  for (int64_t i = 0; i < count; ++i) out[i] = element_bits(key, first + i, scale, 0.0f);
}

/* The same elements widened to fp32. */
void oracle_fill_f32(float* out, int64_t first, int64_t count, uint64_t seed, int layer, int kind,
                     double standard_deviation, float offset) {
  const uint64_t key = oracle_tensor_key(seed, layer, kind);
  const float scale = standard_deviation == 0.0 ? 0.0f : oracle_scale(standard_deviation);
#pragma omp parallel for schedule(static) if (count > (1 << 20))
  for (int64_t i = 0; i < count; ++i) {
    const uint32_t bits = (uint32_t)element_bits(key, first + i, scale, offset) << 16;
    memcpy(&out[i], &bits, sizeof(float));
  }
}

/* Rows of a [rows, cols] tensor selected by index (embedding gather), as fp32. */
void oracle_gather_rows_f32(float* out, const int32_t* rows, int64_t row_count, int64_t cols, uint64_t seed,
                            int layer, int kind, double standard_deviation) {
  for (int64_t r = 0; r < row_count; ++r) {
    oracle_fill_f32(out + r * cols, (int64_t)rows[r] * cols, cols, seed, layer, kind, standard_deviation, 0.0f);
  }
}
