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
#include <cstring>

#include "kernels.h"
#include "tiles.cuh"

namespace tgs {
namespace {

constexpr int kScanBlock = 256;
constexpr int kSortThreads = 256;
constexpr int kSortItems = 8;
constexpr int kSortTile = kSortThreads * kSortItems;  // items per sort block
static_assert(kSortTile == kSortTileItems, "scratch sizing in abi.cu uses kSortTileItems");
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
// Per-block digit counts; thread t counts the 8 consecutive items t*8.. of
// the block's tile (one or two 16-byte loads) into its warp's histogram.
template <typename K>
__global__ void __launch_bounds__(kSortThreads)
    k_radix_hist(const K* __restrict__ keys, const uint32_t* __restrict__ count_ptr,
                 const DevCounts* __restrict__ counts, int shift, int bits, uint32_t* __restrict__ hist,
                 uint32_t max_blocks) {
  constexpr int kWarps = kSortThreads / 32;
  __shared__ uint32_t h[kWarps][kRadix];
  const uint32_t mask = (1u << bits) - 1u;
  const uint32_t n = (counts != nullptr && counts->overflow) ? 0u : *count_ptr;
  const uint32_t base = blockIdx.x * kSortTile;
  if (base >= n) return;
  const uint32_t t = threadIdx.x, warp = t >> 5;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) h[w][t] = 0;
  __syncthreads();
  const uint32_t first = base + t * kSortItems;
  K k[kSortItems];
  if (base + kSortTile <= n) {
    constexpr int kVec = kSortItems * sizeof(K) / 16;
    const uint4* src = reinterpret_cast<const uint4*>(keys + first);
#pragma unroll
    for (int v = 0; v < kVec; ++v) {
      const uint4 q = src[v];
      memcpy(&k[v * (16 / sizeof(K))], &q, 16);
    }
#pragma unroll
    for (int j = 0; j < kSortItems; ++j) atomicAdd(&h[warp][(static_cast<uint32_t>(k[j]) >> shift) & mask], 1u);
  } else {
#pragma unroll
    for (int j = 0; j < kSortItems; ++j)
      if (first + j < n) atomicAdd(&h[warp][(static_cast<uint32_t>(keys[first + j]) >> shift) & mask], 1u);
  }
  __syncthreads();
  uint32_t c = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) c += h[w][t];
  hist[t * max_blocks + blockIdx.x] = c;
}

// One block per digit: exclusive scan of the digit's per-block counts in
// place, and the digit's total (the scatter adds the totals of the smaller
// digits).  Thread t owns a contiguous run of blocks.
__global__ void __launch_bounds__(kSortThreads)
    k_radix_scan(uint32_t* __restrict__ hist, const uint32_t* __restrict__ count_ptr,
                 const DevCounts* __restrict__ counts, uint32_t max_blocks, uint32_t* __restrict__ digit_total) {
  const uint32_t d = blockIdx.x;
  const uint32_t n = (counts != nullptr && counts->overflow) ? 0u : *count_ptr;
  const uint32_t nb = (n + kSortTile - 1) / kSortTile;
  uint32_t* row = hist + static_cast<size_t>(d) * max_blocks;
  const uint32_t per = (nb + kSortThreads - 1) / kSortThreads;
  const uint32_t begin = min(nb, threadIdx.x * per), end = min(nb, begin + per);
  uint32_t local = 0;
  for (uint32_t b = begin; b < end; ++b) local += row[b];
  uint32_t total;
  uint32_t run = block_exclusive_scan(local, total);
  for (uint32_t b = begin; b < end; ++b) {
    const uint32_t v = row[b];
    row[b] = run;
    run += v;
  }
  if (threadIdx.x == 0) digit_total[d] = total;
}

// Scatter of one LSD pass.  Each warp ranks its 256 items (8 rounds of 32,
// item order preserved) against warp-private running digit counters in
// shared memory -- no block barrier per round.  The block then turns the
// per-warp counts into block-local digit offsets, reorders its 2048 items by
// digit in shared memory and writes them out as contiguous runs per digit.
template <typename K>
__global__ void __launch_bounds__(kSortThreads)
    k_radix_scatter(const K* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
                    K* __restrict__ keys_out, uint32_t* __restrict__ vals_out,
                    const uint32_t* __restrict__ count_ptr, const DevCounts* __restrict__ counts, int shift,
                    int bits, const uint32_t* __restrict__ hist, uint32_t max_blocks,
                    const uint32_t* __restrict__ digit_total) {
  constexpr int kWarps = kSortThreads / 32;
  constexpr int kPerWarp = kSortTile / kWarps;  // 256
  __shared__ uint32_t s_cnt[kWarps][kRadix];    // running counts, then per-warp offsets
  __shared__ uint32_t s_start[kRadix];          // block-local start of each digit
  __shared__ uint32_t s_global[kRadix];         // global start of this block's digit run
  __shared__ K s_keys[kSortTile];
  __shared__ uint32_t s_vals[kSortTile];
  const uint32_t n = (counts != nullptr && counts->overflow) ? 0u : *count_ptr;
  const uint32_t base = blockIdx.x * kSortTile;
  if (base >= n) return;
  const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5;
  const uint32_t mask_bits = (1u << bits) - 1u;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) s_cnt[w][t] = 0;
  uint32_t all_digits;
  const uint32_t smaller = block_exclusive_scan(digit_total[t], all_digits);
  s_global[t] = smaller + hist[t * max_blocks + blockIdx.x];
  __syncthreads();
  const uint32_t lt = lanemask_lt();
  K key[kSortItems];
  uint32_t val[kSortItems];
  uint32_t rank[kSortItems];
  const uint32_t wbase = base + warp * kPerWarp;
#pragma unroll
  for (int r = 0; r < kSortItems; ++r) {
    const uint32_t idx = wbase + r * 32 + lane;
    const bool valid = idx < n;
    key[r] = valid ? keys_in[idx] : K(0);
    val[r] = valid ? vals_in[idx] : 0u;
    const uint32_t digit = (static_cast<uint32_t>(key[r]) >> shift) & mask_bits;
    uint32_t peers = __ballot_sync(0xffffffffu, valid);
#pragma unroll
    for (int bt = 0; bt < kRadixBits; ++bt) {
      if (bt < bits) {
        const uint32_t m = __ballot_sync(0xffffffffu, (digit >> bt) & 1u);
        peers &= ((digit >> bt) & 1u) ? m : ~m;
      }
    }
    // the lowest lane of each digit group advances the warp's counter
    const int leader = __ffs(peers) - 1;
    uint32_t before = 0;
    if (valid && static_cast<int>(lane) == leader) {
      before = s_cnt[warp][digit];
      s_cnt[warp][digit] = before + __popc(peers);
    }
    before = __shfl_sync(0xffffffffu, before, leader < 0 ? 0 : leader);
    rank[r] = valid ? before + __popc(peers & lt) : 0xffffffffu;
    __syncwarp();
  }
  __syncthreads();
  // per-digit offsets of each warp and block-local digit starts
  uint32_t run = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const uint32_t c = s_cnt[w][t];
    s_cnt[w][t] = run;
    run += c;
  }
  uint32_t block_total;
  const uint32_t start = block_exclusive_scan(run, block_total);
  s_start[t] = start;
  __syncthreads();
#pragma unroll
  for (int r = 0; r < kSortItems; ++r) {
    if (rank[r] != 0xffffffffu) {
      const uint32_t digit = (static_cast<uint32_t>(key[r]) >> shift) & mask_bits;
      const uint32_t pos = s_start[digit] + s_cnt[warp][digit] + rank[r];
      s_keys[pos] = key[r];
      s_vals[pos] = val[r];
    }
  }
  __syncthreads();
  // consecutive items of the same digit go to consecutive global addresses
  for (uint32_t i = t; i < block_total; i += kSortThreads) {
    const K k = s_keys[i];
    const uint32_t digit = (static_cast<uint32_t>(k) >> shift) & mask_bits;
    const uint32_t g = s_global[digit] + (i - s_start[digit]);
    keys_out[g] = k;
    vals_out[g] = s_vals[i];
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

// 3b. instance emission in depth order.  The preprocess pass recorded the
// hit bits of the first kMaskTiles tiles of every rectangle (row-major), which
// are all of them for the small rectangles that make up most of a scene.  A
// warp emits those instances together: it walks its contiguous output range
// 32 slots at a time, each lane finding the Gaussian that owns its slot and
// the matching set bit, so the stores are coalesced.  Tiles past the first
// kMaskTiles of a larger rectangle are queued for k_emit_big: the depth
// order puts the largest (nearest) Gaussians next to each other, so testing
// them here would leave a few warps working long after the rest.
__device__ __forceinline__ uint32_t select_bit(uint64_t m, uint32_t r) {
  // index of the r-th (0-based) set bit of m; r < popc(m)
  const uint32_t lo = static_cast<uint32_t>(m);
  const uint32_t c = __popc(lo);
  uint32_t word = r < c ? lo : static_cast<uint32_t>(m >> 32);
  uint32_t rr = r < c ? r : r - c;
  uint32_t pos = 0;
#pragma unroll
  for (uint32_t step = 16; step >= 1; step >>= 1) {
    const uint32_t below = __popc((word >> pos) & ((1u << step) - 1u));
    if (rr >= below) {
      rr -= below;
      pos += step;
    }
  }
  return (r < c ? 0u : 32u) + pos;
}

template <int kFp16>
__global__ void __launch_bounds__(kScanBlock)
    k_create_instances(const uint32_t* __restrict__ sorted_idx, const uint32_t* __restrict__ n_touched,
                       const uint64_t* __restrict__ tile_mask, const uint32_t* __restrict__ block_offsets,
                       const ushort4* __restrict__ bounds, const float2* __restrict__ mean2d,
                       const float4* __restrict__ conic_opacity, const PrimInfo16* __restrict__ prim_info,
                       const DevCounts* __restrict__ counts, uint32_t cap, uint32_t grid_w,
                       uint16_t* __restrict__ inst_key, uint32_t* __restrict__ inst_prim,
                       uint4* __restrict__ big_list) {
  const uint32_t k = blockIdx.x * kScanBlock + threadIdx.x;
  const bool overflow = counts->overflow != 0u;
  const bool active = k < counts->n_visible && !overflow;
  uint32_t prim = 0, cnt = 0;
  if (active) {
    prim = sorted_idx[k];
    cnt = n_touched[prim];
  }
  uint32_t total;
  const uint32_t off = block_exclusive_scan(cnt, total) + block_offsets[blockIdx.x];
  if (!active) cnt = 0;
  if (active && off + cnt > cap) cnt = 0;  // cannot happen without overflow
  // writes stay inside [off, end) whatever happens below
  const uint32_t end = off + cnt;
  ushort4 b = make_ushort4(0, 0, 0, 0);
  uint32_t width = 0, n_tiles = 0, n_mask = 0;
  uint64_t mask = 0;
  if (cnt > 0) {
    b = bounds[prim];
    width = b.y - b.x;
    n_tiles = width * static_cast<uint32_t>(b.w - b.z);
    mask = tile_mask[prim];
    n_mask = min(static_cast<uint32_t>(__popcll(mask)), cnt);
  }
  const float inv_w = width > 0 ? 1.0f / static_cast<float>(width) : 0.f;
  const uint32_t lane = threadIdx.x & 31u;
  const unsigned full = 0xffffffffu;
  // (1) instances from the hit bits; offsets are non-decreasing over lanes
  const uint32_t w0 = __shfl_sync(full, off, 0), w1 = __shfl_sync(full, end, 31);
  for (uint32_t base = w0; base < w1; base += 32u) {
    const uint32_t slot = base + lane;
    uint32_t owner = 0;
#pragma unroll
    for (uint32_t step = 16; step >= 1; step >>= 1) {
      const uint32_t o = __shfl_sync(full, off, owner + step);
      if (o <= slot) owner += step;
    }
    const uint32_t o_off = __shfl_sync(full, off, owner);
    const uint32_t o_n = __shfl_sync(full, n_mask, owner);
    const uint32_t o_lo = __shfl_sync(full, static_cast<uint32_t>(mask), owner);
    const uint32_t o_hi = __shfl_sync(full, static_cast<uint32_t>(mask >> 32), owner);
    const uint32_t o_x = __shfl_sync(full, static_cast<uint32_t>(b.x), owner);
    const uint32_t o_y = __shfl_sync(full, static_cast<uint32_t>(b.z), owner);
    const uint32_t o_w = __shfl_sync(full, width, owner);
    const float o_inv = __shfl_sync(full, inv_w, owner);
    const uint32_t o_p = __shfl_sync(full, prim, owner);
    const uint32_t r = slot - o_off;
    if (slot < w1 && r < o_n) {
      const uint32_t q = select_bit((static_cast<uint64_t>(o_hi) << 32) | o_lo, r);
      // row = floor(q / w), exact with the half-step offset (q < 64)
      const uint32_t row = __float2uint_rz((static_cast<float>(q) + 0.5f) * o_inv);
      inst_key[slot] = static_cast<uint16_t>((o_y + row) * grid_w + o_x + (q - row * o_w));
      inst_prim[slot] = o_p;
    }
  }
  // (2) tiles past the recorded bits: queue (Gaussian, first slot, end)
  const bool queue = cnt > 0 && n_tiles > kMaskTiles && off + n_mask < end;
  const uint32_t qm = __ballot_sync(full, queue);
  uint32_t qbase = 0;
  if (lane == 0 && qm != 0u) qbase = atomicAdd(const_cast<uint32_t*>(&counts->n_big), __popc(qm));
  qbase = __shfl_sync(full, qbase, 0);
  if (queue) big_list[qbase + __popc(qm & lanemask_lt())] = make_uint4(prim, off + n_mask, end, 0u);
  // a small rectangle with fewer recorded hits than counted (never
  // expected): pad with a tile id past the grid and report
  if (cnt > 0 && n_tiles <= kMaskTiles && n_mask < cnt) {
    atomicOr(const_cast<uint32_t*>(&counts->overflow), kInconsistentTiles);
    for (uint32_t j = off + n_mask; j < end; ++j) {
      inst_key[j] = 0xffffu;
      inst_prim[j] = prim;
    }
  }
}

// 3c. the tiles past kMaskTiles of the queued Gaussians, one block per
// Gaussian: each round the block tests 256 consecutive tiles of the
// rectangle and writes the hits in row-major order at the running slot.
template <int kFp16>
__global__ void __launch_bounds__(kScanBlock)
    k_emit_big(const uint4* __restrict__ big_list, const ushort4* __restrict__ bounds,
               const float2* __restrict__ mean2d, const float4* __restrict__ conic_opacity,
               const PrimInfo16* __restrict__ prim_info, DevCounts* __restrict__ counts, uint32_t grid_w,
               uint16_t* __restrict__ inst_key, uint32_t* __restrict__ inst_prim) {
  __shared__ uint32_t s_warp[kScanBlock / 32];
  const uint32_t n_big = counts->overflow ? 0u : counts->n_big;
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  for (uint32_t item = blockIdx.x; item < n_big; item += gridDim.x) {
    const uint4 it = big_list[item];
    const uint32_t prim = it.x, end = it.z;
    const ushort4 b = bounds[prim];
    const uint32_t w = b.y - b.x, nt = w * static_cast<uint32_t>(b.w - b.z);
    TileTest q{};
    const float2 mm = mean2d[prim];
    q.mx = mm.x - 0.5f;
    q.my = mm.y - 0.5f;
    if constexpr (kFp16) {
      const PrimInfo16 rec = prim_info[prim];
      q.h_xy = rec.conic_xy;
      q.h_zw = rec.conic_z_opacity;
      q.thr = __logf(__high2float(rec.conic_z_opacity) * 255.0f);
    } else {
      const float4 co = conic_opacity[prim];
      q.ca = co.x;
      q.cb = co.y;
      q.cc = co.z;
      q.thr = __logf(co.w * 255.0f);
    }
    uint32_t cursor = it.y;
    for (uint32_t t0 = kMaskTiles; t0 < nt; t0 += kScanBlock) {
      const uint32_t t = t0 + threadIdx.x;
      const uint32_t ty = b.z + t / w, tx = b.x + t % w;
      const bool hit = t < nt && overlaps<kFp16>(q, tx, ty);
      const uint32_t m = __ballot_sync(0xffffffffu, hit);
      if (lane == 0) s_warp[warp] = __popc(m);
      __syncthreads();
      uint32_t before = 0, total = 0;
#pragma unroll
      for (int k = 0; k < kScanBlock / 32; ++k) {
        const uint32_t c = s_warp[k];
        before += static_cast<uint32_t>(k) < warp ? c : 0u;
        total += c;
      }
      const uint32_t pos = cursor + before + __popc(m & lanemask_lt());
      if (hit && pos < end) {
        inst_key[pos] = static_cast<uint16_t>(ty * grid_w + tx);
        inst_prim[pos] = prim;
      }
      cursor += total;
      __syncthreads();
    }
    // a shortfall (never expected) is padded with a tile id past the grid,
    // which the range pass ignores, and reported
    if (cursor < end) {
      if (threadIdx.x == 0) atomicOr(&counts->overflow, kInconsistentTiles);
      for (uint32_t j = cursor + threadIdx.x; j < end; j += kScanBlock) {
        inst_key[j] = 0xffffu;
        inst_prim[j] = prim;
      }
    }
  }
}

// 5a. tile ranges from the sorted tile ids, 8 keys (16 bytes) per thread
__global__ void k_tile_ranges(const uint16_t* __restrict__ keys, const DevCounts* __restrict__ counts,
                              uint32_t n_tiles, uint2* __restrict__ ranges) {
  const uint32_t n = counts->overflow ? 0u : counts->n_instances;
  const uint32_t groups = (n + 7u) / 8u;
  for (uint32_t gi = blockIdx.x * blockDim.x + threadIdx.x; gi < groups; gi += gridDim.x * blockDim.x) {
    const uint32_t i0 = gi * 8u;
    uint16_t k[8];
    if (i0 + 8u <= n) {
      const uint4 v = *reinterpret_cast<const uint4*>(keys + i0);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        k[2 * j] = static_cast<uint16_t>(w[j] & 0xffffu);
        k[2 * j + 1] = static_cast<uint16_t>(w[j] >> 16);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) k[j] = i0 + j < n ? keys[i0 + j] : static_cast<uint16_t>(0xffffu);
    }
    // 0xffff is never a tile id in range (the range check below drops it)
    const uint16_t prev = i0 == 0 ? static_cast<uint16_t>(0xffffu) : keys[i0 - 1];
    const uint16_t next = i0 + 8u < n ? keys[i0 + 8] : static_cast<uint16_t>(0xffffu);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint16_t kk = k[j];
      if (kk >= n_tiles) continue;
      const uint16_t before = j == 0 ? prev : k[j - 1];
      const uint16_t after = j == 7 ? next : k[j + 1];
      if (before != kk) ranges[kk].x = i0 + j;
      if (after != kk) ranges[kk].y = i0 + j + 1;
    }
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
    if (blocks > 0) {
      k_radix_hist<K><<<blocks, kSortThreads, 0, stream>>>(keys[cur], count_ptr, counts, shift, bits, s.sort_hist,
                                                             max_blocks);
      k_radix_scan<<<kRadix, kSortThreads, 0, stream>>>(s.sort_hist, count_ptr, counts, max_blocks,
                                                         s.sort_digit_total);
      k_radix_scatter<K><<<blocks, kSortThreads, 0, stream>>>(keys[cur], vals[cur], keys[1 - cur], vals[1 - cur],
                                                                count_ptr, counts, shift, bits, s.sort_hist,
                                                                max_blocks, s.sort_digit_total);
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
    if (fp16) {
      k_create_instances<1><<<n_blocks, kScanBlock, 0, stream>>>(
          sorted, s.n_touched, s.tile_mask, s.block_sums, s.bounds, s.mean2d, s.conic_opacity, s.prim_info, counts,
          static_cast<uint32_t>(s.cap_inst), cam.grid_w, s.inst_key[0], s.inst_prim[0], s.big_list);
      k_emit_big<1><<<s.num_sms * 8, kScanBlock, 0, stream>>>(s.big_list, s.bounds, s.mean2d, s.conic_opacity,
                                                               s.prim_info, counts, cam.grid_w, s.inst_key[0],
                                                               s.inst_prim[0]);
    } else {
      k_create_instances<0><<<n_blocks, kScanBlock, 0, stream>>>(
          sorted, s.n_touched, s.tile_mask, s.block_sums, s.bounds, s.mean2d, s.conic_opacity, s.prim_info, counts,
          static_cast<uint32_t>(s.cap_inst), cam.grid_w, s.inst_key[0], s.inst_prim[0], s.big_list);
      k_emit_big<0><<<s.num_sms * 8, kScanBlock, 0, stream>>>(s.big_list, s.bounds, s.mean2d, s.conic_opacity,
                                                               s.prim_info, counts, cam.grid_w, s.inst_key[0],
                                                               s.inst_prim[0]);
    }
  }
  // 4. tile sort on the bits the tile ids need
  int tile_bits = 1;
  while ((1u << tile_bits) < n_tiles) ++tile_bits;
  radix_sort<uint16_t>(s.inst_key, s.inst_prim, &counts->n_instances, counts, s.cap_inst, tile_bits,
                       s.tile_result, s, stream);
  // 5. ranges and buckets
  cudaMemsetAsync(s.ranges, 0, sizeof(uint2) * n_tiles, stream);
  k_tile_ranges<<<s.num_sms * 32, 256, 0, stream>>>(s.inst_key[s.tile_result], counts, n_tiles, s.ranges);
  k_bucket_offsets<<<1, 1024, 0, stream>>>(s.ranges, n_tiles, s.bucket_offsets, counts,
                                            static_cast<uint32_t>(s.cap_buckets));
}

}  // namespace tgs
