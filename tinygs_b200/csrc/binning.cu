// binning.cu -- from per-Gaussian screen footprints to per-tile, depth-ordered
// primitive lists.
//
// Stages (reference: tinygs/src/rasterizer/fastgs_ours/forward.cu:133-260,
// kernels_forward.cuh:414-567, and the fp16 twins):
//   1. compaction of visible Gaussians in index order (scan of the per-block
//      counts the preprocess kernel published),
//   2. stable LSD radix sort of the visible list by the depth key (float bits),
//   3. per-Gaussian instance offsets (scan of touched-tile counts in depth
//      order) and instance emission (tile id, Gaussian id),
//   4. stable LSD radix sort of the instances by tile id (only the bits the
//      tile count needs),
//   5. per-tile [start, end) ranges and bucket offsets.
// Stable sorts over an index-ordered input give (tile, depth, index) order,
// a deterministic member of the reference's order set (its ties among equal
// depths follow atomic arrival order).  All counts stay on the device: the
// launches are sized from capacities and each kernel reads the live count.
#include "kernels.h"
#include "tiles.cuh"

namespace tgs {
namespace {

constexpr int kScanBlock = 256;
constexpr int kSortThreads = 256;
constexpr int kSortItems = 16;
constexpr int kSortTile = kSortThreads * kSortItems;  // items per sort block
constexpr int kRadixBits = 8;
constexpr int kRadix = 1 << kRadixBits;

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Exclusive block scan of one value per thread (blockDim.x == 256).
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t& total) {
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
    uint32_t w = lane < nw ? warp_sums[lane] : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= static_cast<uint32_t>(o)) w += y;
    }
    if (lane < nw) warp_sums[lane] = w;
  }
  __syncthreads();
  total = warp_sums[(blockDim.x >> 5) - 1];
  const uint32_t before = warp == 0 ? 0u : warp_sums[warp - 1];
  __syncthreads();
  return before + x - v;
}

// Exclusive scan of `count` block sums in place (one block of 1024 threads);
// the grand total goes to *total_out.  Optional capacity check raises
// `overflow_bit` in counts->overflow.
__global__ void __launch_bounds__(1024)
    k_scan_sums(uint32_t* __restrict__ sums, uint32_t count, uint32_t* __restrict__ total_out,
                DevCounts* __restrict__ counts, uint32_t cap, uint32_t overflow_bit) {
  __shared__ uint32_t warp_sums[32];
  const uint32_t t = threadIdx.x;
  const uint32_t per = (count + 1023u) / 1024u;
  const uint32_t begin = min(count, t * per), end = min(count, begin + per);
  uint32_t local = 0;
  for (uint32_t k = begin; k < end; ++k) local += sums[k];
  // block scan of `local`
  const uint32_t lane = t & 31u, warp = t >> 5;
  uint32_t x = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= static_cast<uint32_t>(o)) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= static_cast<uint32_t>(o)) w += y;
    }
    warp_sums[lane] = w;
  }
  __syncthreads();
  uint32_t run = (warp == 0 ? 0u : warp_sums[warp - 1]) + x - local;
  for (uint32_t k = begin; k < end; ++k) {
    const uint32_t v = sums[k];
    sums[k] = run;
    run += v;
  }
  if (t == 1023) {
    const uint32_t total = warp_sums[31];
    *total_out = total;
    if (counts != nullptr && total > cap) atomicOr(&counts->overflow, overflow_bit);
  }
}

// 1. visible list in index order
__global__ void __launch_bounds__(kScanBlock)
    k_compact_visible(const uint32_t* __restrict__ n_touched, const uint32_t* __restrict__ depth_key,
                      const uint32_t* __restrict__ block_offsets, uint32_t n, uint32_t* __restrict__ out_key,
                      uint32_t* __restrict__ out_idx) {
  const uint32_t i = blockIdx.x * kScanBlock + threadIdx.x;
  const bool vis = i < n && n_touched[i] > 0;
  uint32_t total;
  const uint32_t pos = block_exclusive_scan(vis ? 1u : 0u, total) + block_offsets[blockIdx.x];
  if (vis) {
    out_key[pos] = depth_key[i];
    out_idx[pos] = i;
  }
}

// 2./4. stable LSD radix sort over a device-resident count.
template <typename K>
__global__ void __launch_bounds__(kSortThreads)
    k_radix_hist(const K* __restrict__ keys, const uint32_t* __restrict__ count_ptr,
                 const DevCounts* __restrict__ counts, int shift, int bits, uint32_t* __restrict__ hist,
                 uint32_t max_blocks, uint32_t* __restrict__ digit_total) {
  __shared__ uint32_t h[kRadix];
  const uint32_t mask = (1u << bits) - 1u;
  const uint32_t n = (counts != nullptr && counts->overflow) ? 0u : *count_ptr;
  const uint32_t base = blockIdx.x * kSortTile;
  h[threadIdx.x] = 0;
  __syncthreads();
  if (base < n) {
#pragma unroll 4
    for (int r = 0; r < kSortItems; ++r) {
      const uint32_t idx = base + r * kSortThreads + threadIdx.x;
      if (idx < n) atomicAdd(&h[(static_cast<uint32_t>(keys[idx]) >> shift) & mask], 1u);
    }
  }
  __syncthreads();
  const uint32_t active_blocks = (n + kSortTile - 1) / kSortTile;
  if (blockIdx.x < active_blocks) {
    const uint32_t c = h[threadIdx.x];
    hist[threadIdx.x * max_blocks + blockIdx.x] = c;
    if (c) atomicAdd(&digit_total[threadIdx.x], c);
  }
}

// One block per digit: offsets[d][b] = sum of all smaller digits +
// sum over earlier blocks of digit d.
__global__ void __launch_bounds__(kSortThreads)
    k_radix_scan(uint32_t* __restrict__ hist, const uint32_t* __restrict__ count_ptr,
                 const DevCounts* __restrict__ counts, uint32_t max_blocks,
                 const uint32_t* __restrict__ digit_total) {
  const uint32_t d = blockIdx.x;
  const uint32_t n = (counts != nullptr && counts->overflow) ? 0u : *count_ptr;
  const uint32_t nb = (n + kSortTile - 1) / kSortTile;
  if (nb == 0) return;
  uint32_t total;
  const uint32_t smaller = threadIdx.x < d ? digit_total[threadIdx.x] : 0u;
  // sum of smaller digits via the block scan's total
  uint32_t base_total;
  block_exclusive_scan(smaller, base_total);
  uint32_t* row = hist + static_cast<size_t>(d) * max_blocks;
  uint32_t carry = base_total;
  for (uint32_t start = 0; start < nb; start += kSortThreads) {
    const uint32_t b = start + threadIdx.x;
    const uint32_t v = b < nb ? row[b] : 0u;
    const uint32_t ex = block_exclusive_scan(v, total);
    if (b < nb) row[b] = carry + ex;
    carry += total;
  }
}

template <typename K>
__global__ void __launch_bounds__(kSortThreads)
    k_radix_scatter(const K* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
                    K* __restrict__ keys_out, uint32_t* __restrict__ vals_out,
                    const uint32_t* __restrict__ count_ptr, const DevCounts* __restrict__ counts, int shift,
                    int bits, const uint32_t* __restrict__ hist, uint32_t max_blocks) {
  __shared__ uint32_t s_off[kRadix];
  __shared__ uint32_t s_cnt[kSortThreads / 32][kRadix];
  __shared__ uint32_t s_pre[kSortThreads / 32][kRadix];
  const uint32_t n = (counts != nullptr && counts->overflow) ? 0u : *count_ptr;
  const uint32_t base = blockIdx.x * kSortTile;
  if (base >= n) return;
  const uint32_t t = threadIdx.x, warp = t >> 5;
  s_off[t] = hist[t * max_blocks + blockIdx.x];
#pragma unroll
  for (int w = 0; w < kSortThreads / 32; ++w) s_cnt[w][t] = 0;
  __syncthreads();
  const uint32_t lt = lanemask_lt();
  for (int r = 0; r < kSortItems; ++r) {
    const uint32_t idx = base + r * kSortThreads + t;
    const bool valid = idx < n;
    K key = 0;
    uint32_t val = 0;
    if (valid) {
      key = keys_in[idx];
      val = vals_in[idx];
    }
    const uint32_t digit = (static_cast<uint32_t>(key) >> shift) & ((1u << bits) - 1u);
    // lanes holding the same digit: intersect one ballot per digit bit
    uint32_t peers = __ballot_sync(0xffffffffu, valid);
#pragma unroll
    for (int b = 0; b < kRadixBits; ++b) {
      if (b < bits) {
        const uint32_t m = __ballot_sync(0xffffffffu, (digit >> b) & 1u);
        peers &= ((digit >> b) & 1u) ? m : ~m;
      }
    }
    const uint32_t rank = __popc(peers & lt);
    if (valid && rank == 0) s_cnt[warp][digit] = __popc(peers);
    __syncthreads();
    {
      uint32_t run = s_off[t];
#pragma unroll
      for (int w = 0; w < kSortThreads / 32; ++w) {
        const uint32_t c = s_cnt[w][t];
        s_pre[w][t] = run;
        run += c;
        s_cnt[w][t] = 0;
      }
      s_off[t] = run;
    }
    __syncthreads();
    if (valid) {
      const uint32_t pos = s_pre[warp][digit] + rank;
      keys_out[pos] = key;
      vals_out[pos] = val;
    }
  }
}

// 3a. per-block sums of touched-tile counts over the depth-sorted list
__global__ void __launch_bounds__(kScanBlock)
    k_instance_block_sums(const uint32_t* __restrict__ sorted_idx, const uint32_t* __restrict__ n_touched,
                          const DevCounts* __restrict__ counts, uint32_t* __restrict__ sums) {
  const uint32_t k = blockIdx.x * kScanBlock + threadIdx.x;
  const uint32_t v = k < counts->n_visible ? n_touched[sorted_idx[k]] : 0u;
  const uint32_t s = __reduce_add_sync(0xffffffffu, v);
  __shared__ uint32_t ws[kScanBlock / 32];
  if ((threadIdx.x & 31u) == 0) ws[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t tot = 0;
    for (int w = 0; w < kScanBlock / 32; ++w) tot += ws[w];
    sums[blockIdx.x] = tot;
  }
}

// 3b. instance emission in depth order; also clears the backward scratch of
// every visible Gaussian.  Big footprints are processed by the whole warp.
template <int kFp16>
__global__ void __launch_bounds__(kScanBlock)
    k_create_instances(const uint32_t* __restrict__ sorted_idx, const uint32_t* __restrict__ n_touched,
                       const uint32_t* __restrict__ block_offsets, const ushort4* __restrict__ bounds,
                       const float2* __restrict__ mean2d, const float4* __restrict__ conic_opacity,
                       const PrimInfo16* __restrict__ prim_info, const DevCounts* __restrict__ counts,
                       uint32_t cap, uint32_t grid_w, uint16_t* __restrict__ inst_key,
                       uint32_t* __restrict__ inst_prim, float4* __restrict__ helpers) {
  const uint32_t k = blockIdx.x * kScanBlock + threadIdx.x;
  const bool overflow = counts->overflow != 0u;
  const bool active = k < counts->n_visible && !overflow;
  uint32_t prim = 0, cnt = 0;
  if (active) {
    prim = sorted_idx[k];
    cnt = n_touched[prim];
  }
  uint32_t total;
  uint32_t off = block_exclusive_scan(cnt, total) + block_offsets[blockIdx.x];
  if (!active) cnt = 0;
  if (active && off + cnt > cap) cnt = 0;  // cannot happen without overflow
  // writes stay inside [off, end) even if the emission ever disagreed with
  // the count of the preprocess pass
  const uint32_t end = off + cnt;
  TileTest tt{};
  ushort4 b = make_ushort4(0, 0, 0, 0);
  uint32_t width = 0, n_tiles = 0;
  if (cnt > 0) {
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    helpers[3 * prim] = z;
    helpers[3 * prim + 1] = z;
    helpers[3 * prim + 2] = z;
    b = bounds[prim];
    width = b.y - b.x;
    n_tiles = width * static_cast<uint32_t>(b.w - b.z);
    const float2 m = mean2d[prim];
    tt.mx = m.x - 0.5f;
    tt.my = m.y - 0.5f;
    if constexpr (kFp16) {
      const PrimInfo16 rec = prim_info[prim];
      tt.h_xy = rec.conic_xy;
      tt.h_zw = rec.conic_z_opacity;
      tt.thr = __logf(__high2float(rec.conic_z_opacity) * 255.0f);
    } else {
      const float4 co = conic_opacity[prim];
      tt.ca = co.x;
      tt.cb = co.y;
      tt.cc = co.z;
      tt.thr = __logf(co.w * 255.0f);
    }
    const uint32_t seq = min(n_tiles, kSequentialTiles);
    for (uint32_t q = 0; q < seq; ++q) {
      const uint32_t ty = b.z + q / width, tx = b.x + q % width;
      if (overlaps<kFp16>(tt, tx, ty) && off < end) {
        inst_key[off] = static_cast<uint16_t>(ty * grid_w + tx);
        inst_prim[off] = prim;
        ++off;
      }
    }
  }
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t lt = lanemask_lt();
  uint32_t big = __ballot_sync(0xffffffffu, cnt > 0 && n_tiles > kSequentialTiles);
  while (big) {
    const int src = __ffs(big) - 1;
    big &= big - 1;
    TileTest q;
    q.mx = __shfl_sync(0xffffffffu, tt.mx, src);
    q.my = __shfl_sync(0xffffffffu, tt.my, src);
    q.ca = __shfl_sync(0xffffffffu, tt.ca, src);
    q.cb = __shfl_sync(0xffffffffu, tt.cb, src);
    q.cc = __shfl_sync(0xffffffffu, tt.cc, src);
    q.h_xy = __shfl_sync(0xffffffffu, tt.h_xy, src);
    q.h_zw = __shfl_sync(0xffffffffu, tt.h_zw, src);
    q.thr = __shfl_sync(0xffffffffu, tt.thr, src);
    const uint32_t x0 = __shfl_sync(0xffffffffu, static_cast<uint32_t>(b.x), src);
    const uint32_t y0 = __shfl_sync(0xffffffffu, static_cast<uint32_t>(b.z), src);
    const uint32_t w = __shfl_sync(0xffffffffu, width, src);
    const uint32_t nt = __shfl_sync(0xffffffffu, n_tiles, src);
    const uint32_t p = __shfl_sync(0xffffffffu, prim, src);
    uint32_t wo = __shfl_sync(0xffffffffu, off, src);
    const uint32_t wend = __shfl_sync(0xffffffffu, end, src);
    const uint32_t rounds = (nt - kSequentialTiles + 31u) / 32u;
    for (uint32_t r = 0; r < rounds; ++r) {
      const uint32_t t = kSequentialTiles + r * 32u + lane;
      const uint32_t tx = x0 + t % w, ty = y0 + t / w;
      const bool hit = t < nt && overlaps<kFp16>(q, tx, ty);
      const uint32_t m = __ballot_sync(0xffffffffu, hit);
      const uint32_t pos = wo + __popc(m & lt);
      if (hit && pos < wend) {
        inst_key[pos] = static_cast<uint16_t>(ty * grid_w + tx);
        inst_prim[pos] = p;
      }
      wo += __popc(m);
    }
    if (lane == static_cast<uint32_t>(src)) off = min(wo, wend);
  }
  // a shortfall (never expected) is padded with a tile id past the grid,
  // which the range pass ignores, and reported
  if (cnt > 0 && off < end) {
    atomicOr(const_cast<uint32_t*>(&counts->overflow), kInconsistentTiles);
    for (; off < end; ++off) {
      inst_key[off] = 0xffffu;
      inst_prim[off] = prim;
    }
  }
}

// 5a. tile ranges from the sorted tile ids
__global__ void k_tile_ranges(const uint16_t* __restrict__ keys, const DevCounts* __restrict__ counts,
                              uint32_t n_tiles, uint2* __restrict__ ranges) {
  const uint32_t n = counts->overflow ? 0u : counts->n_instances;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const uint16_t k = keys[i];
    if (k >= n_tiles) continue;
    if (i == 0 || keys[i - 1] != k) ranges[k].x = i;
    if (i + 1 == n || keys[i + 1] != k) ranges[k].y = i + 1;
  }
}

// 5b. bucket offsets (inclusive scan of ceil(count/32) over tiles)
__global__ void __launch_bounds__(1024)
    k_bucket_offsets(const uint2* __restrict__ ranges, uint32_t n_tiles, uint32_t* __restrict__ offsets,
                     DevCounts* __restrict__ counts, uint32_t cap_buckets) {
  __shared__ uint32_t warp_sums[32];
  const uint32_t t = threadIdx.x;
  const uint32_t per = (n_tiles + 1023u) / 1024u;
  const uint32_t begin = min(n_tiles, t * per), end = min(n_tiles, begin + per);
  uint32_t local = 0;
  for (uint32_t k = begin; k < end; ++k) {
    const uint2 r = ranges[k];
    local += (r.y - r.x + 31u) / 32u;
  }
  const uint32_t lane = t & 31u, warp = t >> 5;
  uint32_t x = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= static_cast<uint32_t>(o)) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= static_cast<uint32_t>(o)) w += y;
    }
    warp_sums[lane] = w;
  }
  __syncthreads();
  uint32_t run = (warp == 0 ? 0u : warp_sums[warp - 1]) + x - local;
  for (uint32_t k = begin; k < end; ++k) {
    const uint2 r = ranges[k];
    run += (r.y - r.x + 31u) / 32u;
    offsets[k] = run;
  }
  if (t == 1023) {
    const uint32_t total = warp_sums[31];
    counts->n_buckets = total;
    if (total > cap_buckets) atomicOr(&counts->overflow, kOverflowBuckets);
  }
}

template <typename K>
void radix_sort(K* keys[2], uint32_t* vals[2], const uint32_t* count_ptr, const DevCounts* counts,
                int64_t capacity, int total_bits, int& result, const RasterState& s, cudaStream_t stream) {
  const uint32_t blocks = static_cast<uint32_t>((capacity + kSortTile - 1) / kSortTile);
  const uint32_t max_blocks = static_cast<uint32_t>(s.sort_max_blocks);
  int cur = 0;
  for (int shift = 0; shift < total_bits; shift += kRadixBits) {
    const int bits = min(kRadixBits, total_bits - shift);
    cudaMemsetAsync(s.sort_digit_total, 0, sizeof(uint32_t) * kRadix, stream);
    if (blocks > 0) {
      k_radix_hist<K><<<blocks, kSortThreads, 0, stream>>>(keys[cur], count_ptr, counts, shift, bits, s.sort_hist,
                                                             max_blocks, s.sort_digit_total);
      k_radix_scan<<<kRadix, kSortThreads, 0, stream>>>(s.sort_hist, count_ptr, counts, max_blocks,
                                                         s.sort_digit_total);
      k_radix_scatter<K><<<blocks, kSortThreads, 0, stream>>>(keys[cur], vals[cur], keys[1 - cur], vals[1 - cur],
                                                                count_ptr, counts, shift, bits, s.sort_hist,
                                                                max_blocks);
    }
    cur = 1 - cur;
  }
  result = cur;
}

}  // namespace

void launch_binning(RasterState& s, int64_t n64, const DevCamera& cam, int fp16, cudaStream_t stream) {
  const uint32_t n = static_cast<uint32_t>(n64);
  const uint32_t n_blocks = (n + kScanBlock - 1) / kScanBlock;
  const uint32_t n_tiles = cam.grid_w * cam.grid_h;
  DevCounts* counts = s.counts;
  // 1. compaction (block sums were written by the preprocess kernel)
  k_scan_sums<<<1, 1024, 0, stream>>>(s.block_sums, n_blocks, &counts->n_visible, nullptr, 0, 0);
  if (n_blocks > 0)
    k_compact_visible<<<n_blocks, kScanBlock, 0, stream>>>(s.n_touched, s.depth_key, s.block_sums, n,
                                                            s.vis_key[0], s.vis_idx[0]);
  // 2. depth sort (32-bit keys)
  radix_sort<uint32_t>(s.vis_key, s.vis_idx, &counts->n_visible, nullptr, n64, 32, s.depth_result, s, stream);
  const uint32_t* sorted = s.vis_idx[s.depth_result];
  // 3. instance offsets and emission
  if (n_blocks > 0) {
    k_instance_block_sums<<<n_blocks, kScanBlock, 0, stream>>>(sorted, s.n_touched, counts, s.block_sums);
    k_scan_sums<<<1, 1024, 0, stream>>>(s.block_sums, n_blocks, &counts->n_instances, counts,
                                         static_cast<uint32_t>(s.cap_inst), kOverflowInstances);
    if (fp16)
      k_create_instances<1><<<n_blocks, kScanBlock, 0, stream>>>(
          sorted, s.n_touched, s.block_sums, s.bounds, s.mean2d, s.conic_opacity, s.prim_info, counts,
          static_cast<uint32_t>(s.cap_inst), cam.grid_w, s.inst_key[0], s.inst_prim[0],
          reinterpret_cast<float4*>(s.helpers));
    else
      k_create_instances<0><<<n_blocks, kScanBlock, 0, stream>>>(
          sorted, s.n_touched, s.block_sums, s.bounds, s.mean2d, s.conic_opacity, s.prim_info, counts,
          static_cast<uint32_t>(s.cap_inst), cam.grid_w, s.inst_key[0], s.inst_prim[0],
          reinterpret_cast<float4*>(s.helpers));
  }
  // 4. tile sort on the bits the tile ids need
  int tile_bits = 1;
  while ((1u << tile_bits) < n_tiles) ++tile_bits;
  radix_sort<uint16_t>(s.inst_key, s.inst_prim, &counts->n_instances, counts, s.cap_inst, tile_bits,
                       s.tile_result, s, stream);
  // 5. ranges and buckets
  cudaMemsetAsync(s.ranges, 0, sizeof(uint2) * n_tiles, stream);
  k_tile_ranges<<<s.num_sms * 4, 256, 0, stream>>>(s.inst_key[s.tile_result], counts, n_tiles, s.ranges);
  k_bucket_offsets<<<1, 1024, 0, stream>>>(s.ranges, n_tiles, s.bucket_offsets, counts,
                                            static_cast<uint32_t>(s.cap_buckets));
}

}  // namespace tgs
