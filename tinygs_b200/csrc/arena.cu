// arena.cu -- row operations on a set of Gaussian arrays (parameters,
// gradients or an Adam moment) and the Morton reordering of the Gaussians.
//
// Reference: GPUGaussian3d::remove / append / reorder
// (tinygs/src/core/gpu_gaussian.cu:117-171, 273-311), SimpleAdam::remove /
// duplicate / reset / reset_opacity / reorder
// (tinygs/src/optim/simple_adam.cu:841-1099) and Orchestrator's Morton
// reorder (tinygs/src/orchestrator.cu:26-100, 1038-1060).  The reference
// allocates new thrust vectors for every such operation; here every entry
// point works between caller-owned sets (or in place), and the Morton order
// takes a caller-provided workspace, so nothing allocates.
//
// Every row operation is HBM-bound: a gather moves 2 x 236 B per Gaussian.
// Rows of a segment of width w are read as w consecutive floats (one or two
// 32-byte sectors per row) and written fully coalesced.
#include <algorithm>

#include "../../include/tgs_abi.h"
#include "kernels.h"

namespace tgs {
namespace {

constexpr int kRowThreads = 256;
constexpr int kKeepBlock = 1024;
constexpr int kBBoxBlocks = 256;

struct SegTable {
  const float* src[6];
  float* dst[6];
};

SegTable seg_table(const TgsGaussians& src, const TgsGaussians& dst) {
  return SegTable{{src.means, src.opacities, src.rotations, src.scales, src.sh0, src.sh_rest},
                  {dst.means, dst.opacities, dst.rotations, dst.scales, dst.sh0, dst.sh_rest}};
}

__device__ __forceinline__ int seg_width(int k) {
  return k == 1 ? 1 : (k == 2 ? 4 : (k == 5 ? 45 : 3));
}

// dst row i <- src row idx[i] (or row i when idx is null) of segment
// blockIdx.y, for i < *n_ptr (or n when n_ptr is null).
__global__ void __launch_bounds__(kRowThreads)
    k_gather_rows(SegTable t, const uint32_t* __restrict__ idx, const uint32_t* __restrict__ n_ptr, uint32_t n) {
  const int k = blockIdx.y;
  const uint32_t w = static_cast<uint32_t>(seg_width(k));
  const uint32_t rows = n_ptr != nullptr ? *n_ptr : n;
  const size_t total = static_cast<size_t>(rows) * w;
  const float* __restrict__ src = t.src[k];
  float* __restrict__ dst = t.dst[k];
  for (size_t e = static_cast<size_t>(blockIdx.x) * kRowThreads + threadIdx.x; e < total;
       e += static_cast<size_t>(gridDim.x) * kRowThreads) {
    const uint32_t row = static_cast<uint32_t>(e / w), col = static_cast<uint32_t>(e - static_cast<size_t>(row) * w);
    const uint32_t from = idx != nullptr ? idx[row] : row;
    dst[e] = src[static_cast<size_t>(from) * w + col];
  }
}

// Rows rows[0..count) of segment blockIdx.y (all six, or only segment
// `only` when only >= 0) set to `value`.
__global__ void __launch_bounds__(kRowThreads)
    k_fill_rows(SegTable t, const int32_t* __restrict__ rows, uint32_t count, float value, int only) {
  const int k = only >= 0 ? only : static_cast<int>(blockIdx.y);
  const uint32_t w = static_cast<uint32_t>(seg_width(k));
  float* __restrict__ dst = t.dst[k];
  const size_t total = static_cast<size_t>(count) * w;
  for (size_t e = static_cast<size_t>(blockIdx.x) * kRowThreads + threadIdx.x; e < total;
       e += static_cast<size_t>(gridDim.x) * kRowThreads) {
    const uint32_t r = static_cast<uint32_t>(e / w), col = static_cast<uint32_t>(e - static_cast<size_t>(r) * w);
    dst[static_cast<size_t>(rows[r]) * w + col] = value;
  }
}

__global__ void __launch_bounds__(kRowThreads)
    k_gather_dens(const float4* __restrict__ src, float4* __restrict__ dst, const uint32_t* __restrict__ idx,
                  const uint32_t* __restrict__ n_ptr, uint32_t n) {
  const uint32_t rows = n_ptr != nullptr ? *n_ptr : n;
  for (uint32_t i = blockIdx.x * kRowThreads + threadIdx.x; i < rows; i += gridDim.x * kRowThreads)
    dst[i] = src[idx[i]];
}

__device__ __forceinline__ uint32_t block_scan_excl(uint32_t v, uint32_t& total) {
  __shared__ uint32_t warp_sums[32];
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= static_cast<uint32_t>(o)) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const uint32_t nw = blockDim.x >> 5;
    uint32_t s = lane < nw ? warp_sums[lane] : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= static_cast<uint32_t>(o)) s += y;
    }
    warp_sums[lane] = s;
  }
  __syncthreads();
  total = warp_sums[(blockDim.x >> 5) - 1];
  const uint32_t r = (warp == 0 ? 0u : warp_sums[warp - 1]) + x - v;
  __syncthreads();
  return r;
}

// Kept rows per block of kKeepBlock flags.
__global__ void __launch_bounds__(kKeepBlock)
    k_keep_counts(const uint8_t* __restrict__ keep, uint32_t n, uint32_t* __restrict__ block_counts) {
  const uint32_t i = blockIdx.x * kKeepBlock + threadIdx.x;
  const uint32_t v = (i < n && keep[i] != 0) ? 1u : 0u;
  const uint32_t c = __syncthreads_count(v);
  if (threadIdx.x == 0) block_counts[blockIdx.x] = c;
}

// Exclusive scan of the block counts in place (one block); the total to
// *n_kept.
__global__ void __launch_bounds__(kKeepBlock)
    k_keep_scan(uint32_t* __restrict__ block_counts, uint32_t blocks, uint32_t* __restrict__ n_kept) {
  const uint32_t per = (blocks + kKeepBlock - 1) / kKeepBlock;
  const uint32_t b0 = min(blocks, threadIdx.x * per), b1 = min(blocks, b0 + per);
  uint32_t local = 0;
  for (uint32_t b = b0; b < b1; ++b) local += block_counts[b];
  uint32_t total;
  uint32_t run = block_scan_excl(local, total);
  for (uint32_t b = b0; b < b1; ++b) {
    const uint32_t c = block_counts[b];
    block_counts[b] = run;
    run += c;
  }
  if (threadIdx.x == 0) *n_kept = total;
}

// Stable list of the kept row indices (copy_if over a counting iterator).
__global__ void __launch_bounds__(kKeepBlock)
    k_keep_index(const uint8_t* __restrict__ keep, uint32_t n, const uint32_t* __restrict__ block_offsets,
                 uint32_t* __restrict__ idx) {
  const uint32_t i = blockIdx.x * kKeepBlock + threadIdx.x;
  const uint32_t v = (i < n && keep[i] != 0) ? 1u : 0u;
  uint32_t total;
  const uint32_t r = block_scan_excl(v, total);
  if (v) idx[block_offsets[blockIdx.x] + r] = i;
}

// Morton reorder, orchestrator.cu:26-100.  Per-block bounding box partials.
__global__ void __launch_bounds__(256)
    k_bbox_partial(const float* __restrict__ means, uint32_t n, float* __restrict__ partial) {
  float lo[3] = {INFINITY, INFINITY, INFINITY}, hi[3] = {-INFINITY, -INFINITY, -INFINITY};
  for (uint32_t i = blockIdx.x * 256 + threadIdx.x; i < n; i += gridDim.x * 256) {
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const float v = means[3 * static_cast<size_t>(i) + c];
      lo[c] = fminf(lo[c], v);
      hi[c] = fmaxf(hi[c], v);
    }
  }
  __shared__ float s_lo[3][8], s_hi[3][8];
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
#pragma unroll
  for (int c = 0; c < 3; ++c) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      lo[c] = fminf(lo[c], __shfl_xor_sync(0xffffffffu, lo[c], o));
      hi[c] = fmaxf(hi[c], __shfl_xor_sync(0xffffffffu, hi[c], o));
    }
    if (lane == 0) {
      s_lo[c][warp] = lo[c];
      s_hi[c][warp] = hi[c];
    }
  }
  __syncthreads();
  if (threadIdx.x < 3) {
    const int c = threadIdx.x;
    float a = s_lo[c][0], b = s_hi[c][0];
    for (int w = 1; w < 8; ++w) {
      a = fminf(a, s_lo[c][w]);
      b = fmaxf(b, s_hi[c][w]);
    }
    partial[6 * blockIdx.x + c] = a;
    partial[6 * blockIdx.x + 3 + c] = b;
  }
}

// Bounding box and the inverse extents: the reference evaluates
// 1 / max(max - min, 1e-8) on the host in IEEE float; here the same with
// round-to-nearest intrinsics (no fast-math reciprocal).  bbox: min[3],
// inv[3].
__global__ void k_bbox_final(const float* __restrict__ partial, int blocks, float* __restrict__ bbox) {
  const int c = threadIdx.x;
  if (c >= 3) return;
  float a = INFINITY, b = -INFINITY;
  for (int k = 0; k < blocks; ++k) {
    a = fminf(a, partial[6 * k + c]);
    b = fmaxf(b, partial[6 * k + 3 + c]);
  }
  const float d = __fsub_rn(b, a);
  const float ext = d < 1e-8f ? 1e-8f : d;  // std::max(d, 1e-8f)
  bbox[c] = a;
  bbox[3 + c] = __fdiv_rn(1.0f, ext);
}

// Spreads the 10 low bits of v to every third bit (bit i -> bit 3i).
__device__ __forceinline__ uint32_t spread3(uint32_t v) {
  v &= 0x3ffu;
  v = (v | (v << 16)) & 0x030000ffu;
  v = (v | (v << 8)) & 0x0300f00fu;
  v = (v | (v << 4)) & 0x030c30c3u;
  v = (v | (v << 2)) & 0x09249249u;
  return v;
}

// 30-bit Morton code of each Gaussian's mean within the bounding box, and
// the identity permutation as the sort's values.
__global__ void __launch_bounds__(256)
    k_morton_codes(const float* __restrict__ means, uint32_t n, const float* __restrict__ bbox,
                   uint32_t* __restrict__ code, uint32_t* __restrict__ idx, uint32_t* __restrict__ count) {
  const uint32_t i = blockIdx.x * 256 + threadIdx.x;
  if (i == 0) *count = n;
  if (i >= n) return;
  uint32_t q[3];
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    const float v = __fmul_rn(__fsub_rn(means[3 * static_cast<size_t>(i) + c], bbox[c]), bbox[3 + c]);
    const float u = fminf(fmaxf(v, 0.0f), 1.0f);
    q[c] = __float2uint_rz(__fmul_rn(u, 1023.0f));
  }
  code[i] = spread3(q[0]) | (spread3(q[1]) << 1) | (spread3(q[2]) << 2);
  idx[i] = i;
}

int grid_for(size_t work, int num_sms) {
  const size_t blocks = (work + kRowThreads - 1) / kRowThreads;
  const size_t cap = static_cast<size_t>(num_sms) * 8;
  return static_cast<int>(std::max<size_t>(1, std::min(blocks, cap)));
}

int sms_of_current_device() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

bool set_ok(const TgsGaussians* g) {
  return g != nullptr && g->means && g->opacities && g->rotations && g->scales && g->sh0 && g->sh_rest;
}

// Morton workspace layout: codes[2][n], idx[2][n], hist[256][max_blocks],
// digit totals[256], bbox partials[6][kBBoxBlocks], bbox[8], count.
struct MortonLayout {
  size_t codes0, codes1, idx0, idx1, hist, digit, partial, bbox, count, total;
  int64_t max_blocks;
};

MortonLayout morton_layout(int64_t n) {
  MortonLayout l{};
  auto up = [](size_t b) { return (b + 255) / 256 * 256; };
  const size_t nn = static_cast<size_t>(std::max<int64_t>(n, 1));
  l.max_blocks = (static_cast<int64_t>(nn) + kSortTileItems - 1) / kSortTileItems;
  size_t off = 0;
  l.codes0 = off; off += up(4 * nn);
  l.codes1 = off; off += up(4 * nn);
  l.idx0 = off; off += up(4 * nn);
  l.idx1 = off; off += up(4 * nn);
  l.hist = off; off += up(4 * 256 * static_cast<size_t>(l.max_blocks));
  l.digit = off; off += up(4 * 256);
  l.partial = off; off += up(4 * 6 * kBBoxBlocks);
  l.bbox = off; off += up(4 * 8);
  l.count = off; off += up(4);
  l.total = off;
  return l;
}

}  // namespace
}  // namespace tgs

using namespace tgs;

extern "C" {

int tgs_arena_gather(const TgsGaussians* src, TgsGaussians* dst, const uint32_t* idx, int64_t n,
                     tgs_stream_t stream) {
  if (!set_ok(src) || !set_ok(dst) || n < 0 || n > 0xffffffffLL) return TGS_ERR_INVALID_ARGUMENT;
  if (n == 0) return TGS_OK;
  const dim3 grid(grid_for(static_cast<size_t>(n) * 45, sms_of_current_device()), 6);
  k_gather_rows<<<grid, kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      seg_table(*src, *dst), idx, nullptr, static_cast<uint32_t>(n));
  return cudaGetLastError() == cudaSuccess ? TGS_OK : TGS_ERR_CUDA;
}

int tgs_arena_compact_workspace_bytes(int64_t n, size_t* bytes) {
  if (bytes == nullptr || n < 0) return TGS_ERR_INVALID_ARGUMENT;
  const size_t blocks = static_cast<size_t>((n + kKeepBlock - 1) / kKeepBlock);
  *bytes = (4 * blocks + 255) / 256 * 256 + (4 * static_cast<size_t>(std::max<int64_t>(n, 1)) + 255) / 256 * 256;
  return TGS_OK;
}

int tgs_arena_keep_index(const uint8_t* keep, int64_t n, void* workspace, size_t workspace_bytes,
                         uint32_t* idx_out, uint32_t* n_kept, tgs_stream_t stream) {
  size_t need = 0;
  if (keep == nullptr || idx_out == nullptr || n_kept == nullptr || n < 0 || n > 0xffffffffLL ||
      tgs_arena_compact_workspace_bytes(n, &need) != TGS_OK)
    return TGS_ERR_INVALID_ARGUMENT;
  if (workspace == nullptr || workspace_bytes < need) return TGS_ERR_CAPACITY;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint32_t blocks = static_cast<uint32_t>((n + kKeepBlock - 1) / kKeepBlock);
  uint32_t* block_counts = static_cast<uint32_t*>(workspace);
  if (blocks == 0) {
    cudaMemsetAsync(n_kept, 0, sizeof(uint32_t), s);
    return cudaGetLastError() == cudaSuccess ? TGS_OK : TGS_ERR_CUDA;
  }
  k_keep_counts<<<blocks, kKeepBlock, 0, s>>>(keep, static_cast<uint32_t>(n), block_counts);
  k_keep_scan<<<1, kKeepBlock, 0, s>>>(block_counts, blocks, n_kept);
  k_keep_index<<<blocks, kKeepBlock, 0, s>>>(keep, static_cast<uint32_t>(n), block_counts, idx_out);
  return cudaGetLastError() == cudaSuccess ? TGS_OK : TGS_ERR_CUDA;
}

int tgs_arena_compact(const TgsGaussians* src, TgsGaussians* dst, const uint8_t* keep, int64_t n, void* workspace,
                      size_t workspace_bytes, uint32_t* n_kept, tgs_stream_t stream) {
  if (!set_ok(src) || !set_ok(dst)) return TGS_ERR_INVALID_ARGUMENT;
  size_t need = 0;
  if (tgs_arena_compact_workspace_bytes(n, &need) != TGS_OK) return TGS_ERR_INVALID_ARGUMENT;
  if (workspace == nullptr || workspace_bytes < need) return TGS_ERR_CAPACITY;
  const size_t blocks = static_cast<size_t>((n + kKeepBlock - 1) / kKeepBlock);
  uint32_t* idx = reinterpret_cast<uint32_t*>(static_cast<char*>(workspace) + (4 * blocks + 255) / 256 * 256);
  const int st = tgs_arena_keep_index(keep, n, workspace, workspace_bytes, idx, n_kept, stream);
  if (st != TGS_OK || n == 0) return st;
  const dim3 grid(grid_for(static_cast<size_t>(n) * 45, sms_of_current_device()), 6);
  k_gather_rows<<<grid, kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(seg_table(*src, *dst), idx, n_kept,
                                                                              0u);
  return cudaGetLastError() == cudaSuccess ? TGS_OK : TGS_ERR_CUDA;
}

int tgs_arena_fill_rows(TgsGaussians* set, const int32_t* rows, int64_t count, float value, int32_t segment,
                        tgs_stream_t stream) {
  if (!set_ok(set) || count < 0 || count > 0xffffffffLL || segment < -1 || segment > 5 ||
      (count > 0 && rows == nullptr))
    return TGS_ERR_INVALID_ARGUMENT;
  if (count == 0) return TGS_OK;
  const dim3 grid(grid_for(static_cast<size_t>(count) * 45, sms_of_current_device()), segment < 0 ? 6 : 1);
  k_fill_rows<<<grid, kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(seg_table(*set, *set), rows,
                                                                            static_cast<uint32_t>(count), value,
                                                                            segment);
  return cudaGetLastError() == cudaSuccess ? TGS_OK : TGS_ERR_CUDA;
}

int tgs_dens_gather(const TgsDensificationInfo* src, TgsDensificationInfo* dst, const uint32_t* idx, int64_t n,
                    tgs_stream_t stream) {
  if (src == nullptr || dst == nullptr || idx == nullptr || n < 0 || n > 0xffffffffLL)
    return TGS_ERR_INVALID_ARGUMENT;
  if (n == 0) return TGS_OK;
  k_gather_dens<<<grid_for(static_cast<size_t>(n), sms_of_current_device()), kRowThreads, 0,
                  static_cast<cudaStream_t>(stream)>>>(reinterpret_cast<const float4*>(src),
                                                       reinterpret_cast<float4*>(dst), idx, nullptr,
                                                       static_cast<uint32_t>(n));
  return cudaGetLastError() == cudaSuccess ? TGS_OK : TGS_ERR_CUDA;
}

int tgs_morton_workspace_bytes(int64_t n, size_t* bytes) {
  if (bytes == nullptr || n < 0 || n > 0xffffffffLL) return TGS_ERR_INVALID_ARGUMENT;
  *bytes = morton_layout(n).total;
  return TGS_OK;
}

int tgs_morton_order(const float* means, int64_t n, void* workspace, size_t workspace_bytes, uint32_t* perm,
                     tgs_stream_t stream) {
  if (means == nullptr || perm == nullptr || n < 0 || n > 0xffffffffLL) return TGS_ERR_INVALID_ARGUMENT;
  const MortonLayout l = morton_layout(n);
  if (workspace == nullptr || workspace_bytes < l.total) return TGS_ERR_CAPACITY;
  if (n == 0) return TGS_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* w = static_cast<char*>(workspace);
  uint32_t* keys[2] = {reinterpret_cast<uint32_t*>(w + l.codes0), reinterpret_cast<uint32_t*>(w + l.codes1)};
  uint32_t* vals[2] = {reinterpret_cast<uint32_t*>(w + l.idx0), reinterpret_cast<uint32_t*>(w + l.idx1)};
  float* partial = reinterpret_cast<float*>(w + l.partial);
  float* bbox = reinterpret_cast<float*>(w + l.bbox);
  uint32_t* count = reinterpret_cast<uint32_t*>(w + l.count);
  const int sms = sms_of_current_device();
  const uint32_t un = static_cast<uint32_t>(n);
  const int bb = static_cast<int>(std::min<int64_t>(kBBoxBlocks, (n + 255) / 256));
  k_bbox_partial<<<bb, 256, 0, s>>>(means, un, partial);
  k_bbox_final<<<1, 32, 0, s>>>(partial, bb, bbox);
  k_morton_codes<<<(un + 255) / 256, 256, 0, s>>>(means, un, bbox, keys[0], vals[0], count);
  const SortScratch ss{reinterpret_cast<uint32_t*>(w + l.hist), reinterpret_cast<uint32_t*>(w + l.digit),
                       l.max_blocks, sms};
  int result = 0;
  sort_pairs_u32(keys, vals, count, n, 30, result, ss, s);
  cudaMemcpyAsync(perm, vals[result], sizeof(uint32_t) * static_cast<size_t>(n), cudaMemcpyDeviceToDevice, s);
  return cudaGetLastError() == cudaSuccess ? TGS_OK : TGS_ERR_CUDA;
}

}  // extern "C"
