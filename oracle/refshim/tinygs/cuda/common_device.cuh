// Stand-in for tinygs/include/tinygs/cuda/common_device.cuh (the parts the
// reference's hot-path kernels use).  Test infrastructure (oracle/_ref build).
#pragma once
#include "tinygs/common.hpp"
#include "tinygs/cuda/common_host.hpp"

namespace tinygs {

// common_device.cuh:156-163: clamp to [0, 1] and its (masked) derivative.
__device__ __forceinline__ float saturate(float x) { return __saturatef(x); }
__device__ __forceinline__ float saturate_deriv(float x) { return (x > 0.0f && x < 1.0f) ? 1.0f : 0.0f; }

// common_device.cuh:166-192: 30-bit Morton code of three 10-bit integers
// (bit i of x goes to bit 3i, of y to 3i+1, of z to 3i+2) and the inverse
// that gathers every third bit.
__host__ __device__ inline uint32_t expand_bits(uint32_t v) {
  uint32_t out = 0;
  for (int i = 0; i < 10; ++i) out |= ((v >> i) & 1u) << (3 * i);
  return out;
}
__host__ __device__ inline uint32_t morton3D(uint32_t x, uint32_t y, uint32_t z) {
  return expand_bits(x) | (expand_bits(y) << 1) | (expand_bits(z) << 2);
}
__host__ __device__ inline uint32_t morton3D_invert(uint32_t code) {
  uint32_t out = 0;
  for (int i = 0; i < 10; ++i) out |= ((code >> (3 * i)) & 1u) << i;
  return out;
}

}  // namespace tinygs
