// common.cuh -- device-side definitions shared by every kernel of the library.
#pragma once

#include <cstdint>
#include <cstring>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace tgs {

// Programmatic dependent launch.  A kernel launched with pdl_launch may be
// scheduled while the kernel before it on the stream is finishing; its
// pdl_entry() (first statement of the kernel) waits until that kernel has
// completed and its memory is visible, then allows the next kernel to be
// scheduled once every block of this one has got that far.  Results are the
// same as with plain launches; the launch latency and the ramp of the next
// grid overlap the tail of the current one.  A kernel without the launch
// attribute passes the wait at once.
__device__ __forceinline__ void pdl_entry() {
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline void pdl_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Rendering constants of the reference rasterizer
// (tinygs/src/rasterizer/fastgs_ours/rasterization_config.h:18-40 and
//  tinygs/src/rasterizer/fastgs_ours_fp16/rasterization_config.h:21-45).
constexpr int kTile = 16;                 // 16x16 pixel render tile
constexpr int kTilePixels = kTile * kTile; // 256
constexpr int kBucket = 32;               // primitives per backward bucket
constexpr float kDilation = 0.3f;
constexpr float kMinAlpha = 1.0f / 255.0f;
constexpr float kMaxAlphaF32 = 0.999f;
constexpr float kMaxAlphaF16 = 0.99f;
constexpr float kMinTransmittance = 1e-4f;
constexpr int kSortTileItems = 2048;  // items per radix-sort block
// binning works on super-tiles of 8x4 tiles (one bit per tile in a 32-bit
// mask) and cuts each super-tile's depth-ordered list into chunks
constexpr uint32_t kSuperW = 8;
constexpr uint32_t kSuperH = 4;
constexpr int kSuperTiles = 32;
constexpr uint32_t kChunk = 1024;
constexpr uint32_t kSubChunk = 256;  // emission work unit (one warp)
constexpr uint32_t kSubChunks = kChunk / kSubChunk;

// Device-side camera passed by value as a kernel parameter.
struct DevCamera {
  float4 r1, r2, r3;  // rows of w2c
  float3 pos;         // camera centre in world space
  float fx, fy, cx, cy;
  float near_plane, far_plane;
  float w, h;         // image size as float
  uint32_t width, height;
  uint32_t grid_w, grid_h;  // 16x16 render tiles
  uint32_t tiled_w, tiled_h;  // 8x8 storage tiles
  uint32_t plane;     // channel stride of the tiled image
};

// Physical index of pixel (y, x) in the reference's 8x8-tiled image plane
// (tinygs/include/tinygs/common.hpp:389-408).
__host__ __device__ __forceinline__ uint32_t tiled_index(uint32_t y, uint32_t x, uint32_t tiled_w) {
  return (((y >> 3) * tiled_w + (x >> 3)) << 6) + ((y & 7u) << 3) + (x & 7u);
}

// Pixel (dx, dy) of the i-th entry of the 16x16 tile walked as four 8x8
// sub-tiles, row-major inside each; the same order is used for the bucket
// checkpoints so that entry i of a checkpoint is pixel i of the walk.
__device__ __forceinline__ void walk_pixel(uint32_t i, uint32_t& dx, uint32_t& dy) {
  const uint32_t sub = i >> 6, in = i & 63u;
  dx = (in & 7u) + (sub & 1u) * 8u;
  dy = (in >> 3) + (sub >> 1) * 8u;
}

__device__ __forceinline__ float sat(float x) { return __saturatef(x); }

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }

// Per-Gaussian scratch the blend backward accumulates into and the
// preprocess backward consumes: 12 floats, 48 B, three float4.
//   [0..1] dL/dmean2d  [2..3] sum |dL/dmean2d|  [4..6] dL/dconic
//   [7]    dL/dopacity (already times 1-opacity)  [8..10] dL/dcolor  [11] pad
constexpr int kHelperFloats = 12;

// Packed fp16-path primitive record (16 B), the reference's PrimitiveInfo
// layout (fastgs_ours_fp16/rasterization_config.h:54-58).
struct alignas(16) PrimInfo16 {
  __half2 conic_xy;
  __half2 conic_z_opacity;
  uchar4 rgb_pad;
  uint32_t pad;
};

// Error word written by device code when a capacity bound is exceeded.
constexpr uint32_t kOverflowInstances = 1u;
constexpr uint32_t kOverflowBuckets = 2u;
constexpr uint32_t kOverflowEntries = 4u;  // (Gaussian, super-tile) entries

// Device counters of one forward, kept in one 32-byte record.
struct DevCounts {
  uint32_t n_visible;
  uint32_t n_instances;
  uint32_t n_buckets;
  uint32_t overflow;
  uint32_t n_live_buckets;  // buckets the backward runs (forward appends them)
  uint32_t n_entries;       // (Gaussian, super-tile) entries
  uint32_t n_chunks;        // chunks of the super-tile entry lists
  uint32_t pad;
};

// ------------------------------------------------------------------ PCG32
// The random stream of the reference (include/tinygs/random/pcg32.hpp):
// M. E. O'Neill 2014, 64-bit LCG state, XSH-RR output; jump-ahead by the
// LCG's affine map composed by repeated squaring (F. B. Brown 1994).
constexpr uint64_t kPcgMult = 0x5851f42d4c957f2dULL;

struct Pcg {
  uint64_t state, inc;
  // pcg32(initstate, initseq)
  __host__ __device__ static Pcg seeded(uint64_t initstate, uint64_t initseq) {
    Pcg g{0u, (initseq << 1u) | 1u};
    g.next_uint();
    g.state += initstate;
    g.next_uint();
    return g;
  }
  __host__ __device__ uint32_t next_uint() {
    const uint64_t old = state;
    state = old * kPcgMult + inc;
    const uint32_t xorshifted = static_cast<uint32_t>(((old >> 18u) ^ old) >> 27u);
    const uint32_t rot = static_cast<uint32_t>(old >> 59u);
    return (xorshifted >> rot) | (xorshifted << ((~rot + 1u) & 31u));
  }
  __host__ __device__ float next_float() {
    const uint32_t u = (next_uint() >> 9) | 0x3f800000u;
    float f;
    memcpy(&f, &u, 4);
    return f - 1.0f;
  }
  __host__ __device__ void advance(uint64_t delta) {
    uint64_t cur_mult = kPcgMult, cur_plus = inc, acc_mult = 1u, acc_plus = 0u;
    while (delta > 0) {
      if (delta & 1u) {
        acc_mult *= cur_mult;
        acc_plus = acc_plus * cur_mult + cur_plus;
      }
      cur_plus = (cur_mult + 1u) * cur_plus;
      cur_mult *= cur_mult;
      delta >>= 1u;
    }
    state = acc_mult * state + acc_plus;
  }
};

}  // namespace tgs
