// Stand-in for tinygs/include/tinygs/common.hpp: only the names the
// reference's hot-path kernels use.  Test infrastructure (oracle/_ref build).
#pragma once
#include <cfloat>
#include <cstddef>
#include <cstdint>
#include <cmath>
#include <memory>
#include <string>
#include <stdexcept>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#define STRINGIFY(x) #x
#define STR(x) STRINGIFY(x)
#define FILE_LINE __FILE__ ":" STR(__LINE__)

#if defined(__CUDACC__)
#define TINYGS_HOST_DEVICE __host__ __device__
#define TINYGS_DEVICE __device__
#define TINYGS_HOST __host__
#else
#define TINYGS_HOST_DEVICE
#define TINYGS_DEVICE
#define TINYGS_HOST
#endif

#if defined(__CUDA_ARCH__)
#define TINYGS_PRAGMA_UNROLL _Pragma("unroll")
#define TINYGS_PRAGMA_NO_UNROLL _Pragma("unroll 1")
#else
#define TINYGS_PRAGMA_UNROLL
#define TINYGS_PRAGMA_NO_UNROLL
#endif

#if __has_include(<nlohmann/json.hpp>)
#include <nlohmann/json.hpp>
namespace tinygs {
using json = nlohmann::json;
}
#endif

namespace tinygs {

using float16_t = __half;
// core/gaussian.hpp: SH storage is always 16 coefficients (degree 3).
constexpr int kMaxSphericalHarmonicsDegree = 3;
constexpr int kMaxSphericalHarmonicsCoefficients = 16;
constexpr uint32_t WARP_SIZE = 32;

// common.hpp:358-364: sigmoid and its inverse (input clamped to [1e-9, 1-1e-9]).
TINYGS_HOST_DEVICE inline float logistic(const float x) { return 1.0f / (1.0f + expf(-x)); }
TINYGS_HOST_DEVICE inline float logit(const float x) {
  const float c = fminf(fmaxf(x, 1e-9f), 1.0f - 1e-9f);
  return -logf(1.0f / c - 1.0f);
}

// common.hpp:367-408: images are stored as 8x8 pixel tiles, row-major over
// tiles, row-major inside a tile.
constexpr uint32_t kImageTile = 8;
constexpr uint32_t kImageTileLog2 = 3;
constexpr uint32_t kImageTileMask = 7;

TINYGS_HOST_DEVICE inline uint32_t get_linear_index_tiled(uint32_t row, uint32_t col, uint32_t tiles_per_row) {
  const uint32_t tile = (row >> kImageTileLog2) * tiles_per_row + (col >> kImageTileLog2);
  const uint32_t inner = ((row & kImageTileMask) << kImageTileLog2) | (col & kImageTileMask);
  return (tile << (2 * kImageTileLog2)) + inner;
}
TINYGS_HOST_DEVICE inline uint32_t get_linear_index(uint32_t row, uint32_t col, uint32_t width) {
  return get_linear_index_tiled(row, col, width >> kImageTileLog2);
}

// vec.hpp:64-88: scalar wrappers the kernels call with a tinygs:: prefix.
template <typename T> TINYGS_HOST_DEVICE T sqrt(T a) { return ::sqrt(a); }
template <typename T> TINYGS_HOST_DEVICE T min(T a, T b) { return a < b ? a : b; }
template <typename T> TINYGS_HOST_DEVICE T max(T a, T b) { return a < b ? b : a; }
template <typename T> TINYGS_HOST_DEVICE T clamp(T a, T lo, T hi) { return a < lo ? lo : (hi < a ? hi : a); }

template <typename T> TINYGS_HOST_DEVICE T div_round_up(T val, T divisor) { return (val + divisor - 1) / divisor; }

}  // namespace tinygs
