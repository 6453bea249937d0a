// binning.cu -- from per-Gaussian screen footprints to per-tile, depth-ordered
// primitive lists.
//
// Reference: tinygs/src/rasterizer/fastgs_ours/forward.cu:133-260 and
// kernels_forward.cuh:414-567 (and the fp16 twins): per-Gaussian tile counts,
// a depth sort, instance emission and a sort of all instances by tile.  The
// lists produced here are the same -- every tile holds the Gaussians that pass
// the exact tile test, in (depth, index) order -- built in two levels so that
// no sort runs over the ~10 instances per Gaussian:
//   1. compaction of the candidate Gaussians (culling passed, non-empty tile
//      rectangle) in index order,
//   2. stable LSD radix sort of the candidates by the depth key (float bits),
//   3. one entry per (Gaussian, super-tile of 8x4 tiles) its rectangle
//      overlaps, emitted in depth order, and a stable sort of the entries by
//      super-tile (one 8-bit pass for up to 256 super-tiles),
//   4. the entry list of each super-tile is cut into chunks of 1024 entries;
//      per chunk, the exact tile tests of each entry give a 32-bit hit mask
//      and per-tile counts of each 256-entry sub-chunk (and each Gaussian's
//      touched-tile total),
//   5. scans give every (chunk, tile) its first slot: tiles in index order,
//      chunks in depth order inside a tile; the per-tile [start, end) ranges
//      and bucket offsets fall out of the same scan,
//   6. per 256-entry sub-chunk (one warp), stable ranks of the entries in
//      each tile (ballots over the hit masks) place every instance at its
//      final slot.
// Ties among equal depths follow the index order, a deterministic member of
// the reference's order set (its ties follow atomic arrival order).  All
// counts stay on the device: the launches are sized from capacities (or the
// resident blocks, for grid-stride kernels) and each kernel reads the live
// count.  The kernels are chained with programmatic dependent launch
// (pdl_launch / pdl_entry).
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

// Loads of a thread's contiguous run [begin, end) in batches of 8 whose
// loads are in flight together (a plain loop waits on every load in turn):
// f(k, value) is called for every k in order.
template <typename F>
__device__ __forceinline__ void for_run(const uint32_t* src, uint32_t begin, uint32_t end, F&& f) {
  for (uint32_t k0 = begin; k0 < end; k0 += 8u) {
    uint32_t v[8];
#pragma unroll
    for (uint32_t j = 0; j < 8u; ++j) v[j] = k0 + j < end ? src[k0 + j] : 0u;
#pragma unroll
    for (uint32_t j = 0; j < 8u; ++j)
      if (k0 + j < end) f(k0 + j, v[j]);
  }
}

// Exclusive scan of `count` block sums in place (one block of 1024 threads);
// the grand total goes to *total_out.  Optional capacity check raises
// `overflow_bit` in counts->overflow.
__global__ void __launch_bounds__(1024)
    k_scan_sums(uint32_t* __restrict__ sums, uint32_t count, uint32_t* __restrict__ total_out,
                DevCounts* __restrict__ counts, uint32_t cap, uint32_t overflow_bit) {
  pdl_entry();
  __shared__ uint32_t warp_sums[32];
  const uint32_t t = threadIdx.x;
  const uint32_t per = (count + 1023u) / 1024u;
  const uint32_t begin = min(count, t * per), end = min(count, begin + per);
  uint32_t local = 0;
  for_run(sums, begin, end, [&](uint32_t, uint32_t v) { local += v; });
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
  for_run(sums, begin, end, [&](uint32_t k, uint32_t v) {
    sums[k] = run;
    run += v;
  });
  if (t == 1023) {
    const uint32_t total = warp_sums[31];
    *total_out = total;
    if (counts != nullptr && total > cap) atomicOr(&counts->overflow, overflow_bit);
  }
}

// 1. candidate list in index order
__global__ void __launch_bounds__(kScanBlock)
    k_compact_visible(const ushort4* __restrict__ bounds, const uint32_t* __restrict__ depth_key,
                      const uint32_t* __restrict__ block_offsets, uint32_t n, uint32_t* __restrict__ out_key,
                      uint32_t* __restrict__ out_idx) {
  pdl_entry();
  const uint32_t i = blockIdx.x * kScanBlock + threadIdx.x;
  bool vis = false;
  if (i < n) {
    const ushort4 b = bounds[i];
    vis = b.x < b.y && b.z < b.w;
  }
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
  pdl_entry();
  constexpr int kWarps = kSortThreads / 32;
  __shared__ uint32_t h[kWarps][kRadix];
  const uint32_t mask = (1u << bits) - 1u;
  const uint32_t n = (counts != nullptr && counts->overflow) ? 0u : *count_ptr;
  const uint32_t t = threadIdx.x, warp = t >> 5;
  // grid-stride over the 2048-item tiles (the grid is sized by the resident
  // blocks, not by the capacity)
  for (uint32_t tb = blockIdx.x; tb * kSortTile < n; tb += gridDim.x) {
    const uint32_t base = tb * kSortTile;
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
    hist[t * max_blocks + tb] = c;
    __syncthreads();  // h is cleared again for the next tile
  }
}

// One block per digit: exclusive scan of the digit's per-block counts in
// place, and the digit's total (the scatter adds the totals of the smaller
// digits).  Thread t owns a contiguous run of blocks.
__global__ void __launch_bounds__(kSortThreads)
    k_radix_scan(uint32_t* __restrict__ hist, const uint32_t* __restrict__ count_ptr,
                 const DevCounts* __restrict__ counts, uint32_t max_blocks, uint32_t* __restrict__ digit_total) {
  pdl_entry();
  const uint32_t d = blockIdx.x;
  const uint32_t n = (counts != nullptr && counts->overflow) ? 0u : *count_ptr;
  const uint32_t nb = (n + kSortTile - 1) / kSortTile;
  uint32_t* row = hist + static_cast<size_t>(d) * max_blocks;
  const uint32_t per = (nb + kSortThreads - 1) / kSortThreads;
  const uint32_t begin = min(nb, threadIdx.x * per), end = min(nb, begin + per);
  uint32_t local = 0;
  for_run(row, begin, end, [&](uint32_t, uint32_t v) { local += v; });
  uint32_t total;
  uint32_t run = block_exclusive_scan(local, total);
  for_run(row, begin, end, [&](uint32_t b, uint32_t v) {
    row[b] = run;
    run += v;
  });
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
  pdl_entry();
  constexpr int kWarps = kSortThreads / 32;
  constexpr int kPerWarp = kSortTile / kWarps;  // 256
  __shared__ uint32_t s_cnt[kWarps][kRadix];    // running counts, then per-warp offsets
  __shared__ uint32_t s_start[kRadix];          // block-local start of each digit
  __shared__ uint32_t s_global[kRadix];         // global start of this block's digit run
  __shared__ K s_keys[kSortTile];
  __shared__ uint32_t s_vals[kSortTile];
  const uint32_t n = (counts != nullptr && counts->overflow) ? 0u : *count_ptr;
  if (blockIdx.x * kSortTile >= n) return;
  const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5;
  const uint32_t mask_bits = (1u << bits) - 1u;
  uint32_t all_digits;
  const uint32_t smaller = block_exclusive_scan(digit_total[t], all_digits);
  // grid-stride over the 2048-item tiles (the grid is sized by the resident
  // blocks, not by the capacity)
  for (uint32_t tb = blockIdx.x; tb * kSortTile < n; tb += gridDim.x) {
    const uint32_t base = tb * kSortTile;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s_cnt[w][t] = 0;
    s_global[t] = smaller + hist[t * max_blocks + tb];
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
    __syncthreads();  // shared state is rebuilt for the next tile
  }
}

// Super-tile geometry: 8x4 tiles (128x64 pixels), one bit per tile in a
// 32-bit hit mask (bit = row * 8 + column inside the super-tile).
struct SuperRect {
  uint32_t sx0, sy0, nsx, nsy;
};
__device__ __forceinline__ SuperRect super_rect(ushort4 b) {
  SuperRect r{0, 0, 0, 0};
  if (b.x < b.y && b.z < b.w) {
    r.sx0 = b.x / kSuperW;
    r.sy0 = b.z / kSuperH;
    r.nsx = (b.y - 1u) / kSuperW - r.sx0 + 1u;
    r.nsy = (b.w - 1u) / kSuperH - r.sy0 + 1u;
  }
  return r;
}

// 3a. per-block sums of super-tile entry counts over the depth-sorted list
__global__ void __launch_bounds__(kScanBlock)
    k_entry_block_sums(const uint32_t* __restrict__ sorted_idx, const ushort4* __restrict__ bounds,
                       const DevCounts* __restrict__ counts, uint32_t* __restrict__ sums) {
  pdl_entry();
  const uint32_t k = blockIdx.x * kScanBlock + threadIdx.x;
  uint32_t v = 0;
  if (k < counts->n_visible) {
    const SuperRect r = super_rect(bounds[sorted_idx[k]]);
    v = r.nsx * r.nsy;
  }
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

// 3b. entry emission in depth order: (super-tile id, Gaussian id)
__global__ void __launch_bounds__(kScanBlock)
    k_create_entries(const uint32_t* __restrict__ sorted_idx, const ushort4* __restrict__ bounds,
                     const uint32_t* __restrict__ block_offsets, const DevCounts* __restrict__ counts,
                     uint32_t super_w, uint16_t* __restrict__ ent_key, uint32_t* __restrict__ ent_prim) {
  pdl_entry();
  const uint32_t k = blockIdx.x * kScanBlock + threadIdx.x;
  const bool active = k < counts->n_visible && counts->overflow == 0u;
  uint32_t prim = 0;
  SuperRect r{0, 0, 0, 0};
  if (active) {
    prim = sorted_idx[k];
    r = super_rect(bounds[prim]);
  }
  uint32_t total;
  const uint32_t cnt = r.nsx * r.nsy;
  const uint32_t off = block_exclusive_scan(cnt, total) + block_offsets[blockIdx.x];
  // the warp's entries laid end to end (they are contiguous in the output):
  // lane j writes entry base + j of each round of 32, so every store is
  // coalesced; the owner of an entry is the number of Gaussian starts up to
  // it minus one (Gaussians with no entry start nowhere)
  const unsigned full = 0xffffffffu;
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t w_off = __shfl_sync(full, off, 0);
  const uint32_t start = off - w_off;
  const uint32_t w_total = __shfl_sync(full, start + cnt, 31);
  const uint32_t lt = lanemask_lt();
  uint32_t starts_before = 0;
  for (uint32_t base = 0; base < w_total; base += 32u) {
    const uint32_t sbit = cnt > 0u && start >= base && start < base + 32u ? 1u << (start - base) : 0u;
    const uint32_t starts = __reduce_or_sync(full, sbit);
    const uint32_t owner = (starts_before + __popc(starts & (lt | (1u << lane))) - 1u) & 31u;
    starts_before += __popc(starts);
    const uint32_t o_prim = __shfl_sync(full, prim, owner), o_start = __shfl_sync(full, start, owner);
    const uint32_t o_x0 = __shfl_sync(full, r.sx0, owner), o_y0 = __shfl_sync(full, r.sy0, owner);
    const uint32_t o_w = __shfl_sync(full, r.nsx, owner);
    const uint32_t e = base + lane;
    if (e < w_total) {
      const uint32_t t = e - o_start, ty = t / o_w, tx = t - ty * o_w;
      ent_key[w_off + e] = static_cast<uint16_t>((o_y0 + ty) * super_w + o_x0 + tx);
      ent_prim[w_off + e] = o_prim;
    }
  }
}

// 4a. [start, end) of each super-tile in the sorted entry list
__global__ void k_super_ranges(const uint16_t* __restrict__ keys, const DevCounts* __restrict__ counts,
                               uint2* __restrict__ ranges) {
  pdl_entry();
  const uint32_t n = counts->overflow ? 0u : counts->n_entries;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const uint16_t k = keys[i];
    if (i == 0 || keys[i - 1] != k) ranges[k].x = i;
    if (i + 1 == n || keys[i + 1] != k) ranges[k].y = i + 1;
  }
}

// 4b. chunk table: each super-tile's entries cut into chunks of kChunk
// (one block of 1024 threads; thread t owns a contiguous run of super-tiles).
// With `totals` (the per-digit counts of a single-pass entry sort, i.e. the
// entries of each super-tile), the super-tile ranges are first derived from
// them by an exclusive scan and written to `super_ranges`.
__global__ void __launch_bounds__(1024)
    k_chunk_table(uint2* __restrict__ super_ranges, const uint32_t* __restrict__ totals, uint32_t n_super,
                  uint4* __restrict__ chunks, uint32_t* __restrict__ super_chunk, DevCounts* __restrict__ counts) {
  pdl_entry();
  __shared__ uint32_t warp_sums[32];
  const uint32_t t = threadIdx.x;
  const uint32_t per = (n_super + 1023u) / 1024u;
  const uint32_t begin = min(n_super, t * per), end = min(n_super, begin + per);
  if (totals != nullptr) {
    uint32_t mine = 0;
    for (uint32_t k = begin; k < end; ++k) mine += totals[k];
    uint32_t all;
    uint32_t start = block_exclusive_scan(mine, all);
    for (uint32_t k = begin; k < end; ++k) {
      super_ranges[k] = make_uint2(start, start + totals[k]);
      start += totals[k];
    }
    __syncthreads();
  }
  uint32_t local = 0;
  for (uint32_t k = begin; k < end; ++k) {
    const uint2 r = super_ranges[k];
    local += (r.y - r.x + kChunk - 1u) / kChunk;
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
  uint32_t c = (warp == 0 ? 0u : warp_sums[warp - 1]) + x - local;
  for (uint32_t k = begin; k < end; ++k) {
    const uint2 r = super_ranges[k];
    super_chunk[k] = c;
    for (uint32_t st = r.x; st < r.y; st += kChunk, ++c) chunks[c] = make_uint4(k, st, min(r.y, st + kChunk), 0u);
  }
  if (t == 1023) counts->n_chunks = warp_sums[31];
}

// Tile-test inputs of Gaussian p, as the preprocess pass derived them.
template <int kFp16>
__device__ __forceinline__ TileTest tile_test_of(uint32_t p, const float2* __restrict__ mean2d,
                                                 const float4* __restrict__ conic_opacity,
                                                 const PrimInfo16* __restrict__ prim_info) {
  TileTest q{};
  const float2 m = mean2d[p];
  q.mx = m.x - 0.5f;
  q.my = m.y - 0.5f;
  if constexpr (kFp16) {
    const PrimInfo16 rec = prim_info[p];
    tile_test_f16(q, q.mx, q.my, rec.conic_xy, rec.conic_z_opacity);
  } else {
    const float4 co = conic_opacity[p];
    q.ca = co.x;
    q.cb = co.y;
    q.cc = co.z;
    q.thr = __logf(co.w * 255.0f);
  }
  return q;
}

// 32 x 32 bit-matrix transpose across a warp: lane i holds row i on entry
// (bit j = column j); on exit lane j holds column j (bit i = row i).
__device__ __forceinline__ uint32_t warp_transpose_bits(uint32_t row, uint32_t lane) {
  uint32_t col = row;
#pragma unroll
  for (uint32_t sh = 16, m0 = 0x0000ffffu; sh > 0; sh >>= 1, m0 ^= m0 << sh) {
    const uint32_t other = __shfl_xor_sync(0xffffffffu, col, sh);
    col = (lane & sh) == 0u ? (col & m0) | ((other & m0) << sh) : (col & ~m0) | ((other & ~m0) >> sh);
  }
  return col;
}

// 5a. per chunk: hit mask of every entry (exact tile tests of its rectangle
// inside the super-tile, the warp's (entry, tile) pairs tested 32 at a time),
// per-tile hit counts of the chunk, and each Gaussian's touched-tile total.
template <int kFp16>
__global__ void __launch_bounds__(kScanBlock)
    k_chunk_hits(const uint4* __restrict__ chunks, const uint32_t* __restrict__ ent_prim,
                 const ushort4* __restrict__ bounds, const float2* __restrict__ mean2d,
                 const float4* __restrict__ conic_opacity, const PrimInfo16* __restrict__ prim_info,
                 const DevCounts* __restrict__ counts, uint32_t super_w, uint32_t* __restrict__ masks,
                 uint32_t* __restrict__ chunk_counts, uint32_t* __restrict__ sub_offsets,
                 uint32_t* __restrict__ n_touched) {
  pdl_entry();
  static_assert(kSubChunk == kScanBlock, "one block pass per emission sub-chunk");
  __shared__ uint32_t s_cnt[kSubChunks * kSuperTiles];
  // each entry's test inputs and rectangle, read by the lanes that test its
  // tiles (48 bytes used of 64-byte records)
  __shared__ float4 s_rec[kScanBlock / 32][32][4];
  const unsigned full = 0xffffffffu;
  const uint32_t n_chunks = counts->overflow ? 0u : counts->n_chunks;
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t lt = lanemask_lt();
  for (uint32_t c = blockIdx.x; c < n_chunks; c += gridDim.x) {
    const uint4 ch = chunks[c];
    const uint32_t tx0 = (ch.x % super_w) * kSuperW, ty0 = (ch.x / super_w) * kSuperH;
    if (threadIdx.x < kSubChunks * kSuperTiles) s_cnt[threadIdx.x] = 0;
    __syncthreads();
    for (uint32_t e0 = ch.y; e0 < ch.z; e0 += kScanBlock) {
      uint32_t* sub_cnt = s_cnt + (e0 - ch.y) / kScanBlock * kSuperTiles;
      const uint32_t e = e0 + threadIdx.x;
      const bool valid = e < ch.z;
      uint32_t prim = 0, x0 = 0, y0 = 0, w = 0, h = 0, magic = 0;
      TileTest tt{};
      if (valid) {
        prim = ent_prim[e];
        const ushort4 b = bounds[prim];
        x0 = max(static_cast<uint32_t>(b.x), tx0);
        y0 = max(static_cast<uint32_t>(b.z), ty0);
        w = min(static_cast<uint32_t>(b.y), tx0 + kSuperW) - x0;
        h = min(static_cast<uint32_t>(b.w), ty0 + kSuperH) - y0;
        magic = 255u / w + 1u;  // t / w == (t * magic) >> 8 for t < 33, w <= 8
        tt = tile_test_of<kFp16>(prim, mean2d, conic_opacity, prim_info);
      }
      const uint32_t total = w * h;  // <= 32
      // lay the lanes' rectangles end to end; lane j tests pair base + j
      uint32_t incl = total;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(full, incl, o);
        if (lane >= static_cast<uint32_t>(o)) incl += y;
      }
      const uint32_t start = incl - total;
      const uint32_t pairs = __shfl_sync(full, incl, 31);
      {
        float4* rec = s_rec[threadIdx.x >> 5][lane];
        rec[0] = make_float4(tt.ca, tt.cb, tt.cc, tt.thr);
        rec[1] = make_float4(kFp16 ? tt.xs : tt.mx, kFp16 ? tt.ys : tt.my,
                             __uint_as_float(*reinterpret_cast<const uint32_t*>(&tt.c_xy)),
                             __uint_as_float(*reinterpret_cast<const uint32_t*>(&tt.c_yz)));
        rec[2] = make_float4(__uint_as_float(*reinterpret_cast<const uint32_t*>(&tt.den)),
                             __uint_as_float(start), __uint_as_float(x0 | (y0 << 16)),
                             __uint_as_float(w | (magic << 8)));
      }
      __syncwarp();
      uint32_t local = 0;  // hits in rectangle order (bit t = row t / w, column t % w)
      // owners are lanes 0 .. (valid entries - 1), every one with total >= 1,
      // so the owner of a slot is the number of rectangle starts up to it - 1
      uint32_t starts_before = 0;
      for (uint32_t base = 0; base < pairs; base += 32u) {
        const uint32_t slot = base + lane;
        const uint32_t sbit = total > 0u && start >= base && start < base + 32u ? 1u << (start - base) : 0u;
        const uint32_t starts = __reduce_or_sync(full, sbit);
        const uint32_t owner = (starts_before + __popc(starts & (lt | (1u << lane))) - 1u) & 31u;
        starts_before += __popc(starts);
        const float4* orec = s_rec[threadIdx.x >> 5][owner];
        const float4 r0 = orec[0], r1 = orec[1], r2 = orec[2];
        TileTest q;
        q.ca = r0.x;
        q.cb = r0.y;
        q.cc = r0.z;
        q.thr = r0.w;
        if constexpr (kFp16) {
          q.xs = r1.x;
          q.ys = r1.y;
          const uint32_t cxy = __float_as_uint(r1.z), cyz = __float_as_uint(r1.w), den = __float_as_uint(r2.x);
          q.c_xy = *reinterpret_cast<const __half2*>(&cxy);
          q.c_yz = *reinterpret_cast<const __half2*>(&cyz);
          q.den = *reinterpret_cast<const __half2*>(&den);
        } else {
          q.mx = r1.x;
          q.my = r1.y;
        }
        const uint32_t o_start = __float_as_uint(r2.y), o_xy = __float_as_uint(r2.z), o_wm = __float_as_uint(r2.w);
        const uint32_t o_x = o_xy & 0xffffu, o_y = o_xy >> 16, o_w = o_wm & 0xffu, o_magic = o_wm >> 8;
        const uint32_t t = slot - o_start;
        const uint32_t row = (t * o_magic) >> 8;
        const bool hit = slot < pairs && overlaps<kFp16>(q, o_x + (t - row * o_w), o_y + row);
        const uint32_t m = __ballot_sync(full, hit);
        // this lane's pairs within the round are one run of ballot bits
        const uint32_t lo = max(start, base), hi = min(start + total, base + 32u);
        if (lo < hi) {
          const uint32_t len = hi - lo;
          const uint32_t bits = (m >> (lo - base)) & (len == 32u ? full : ((1u << len) - 1u));
          local |= bits << (lo - start);
        }
      }
      __syncwarp();  // the records are rewritten by the next pass
      // rectangle order -> super-tile bits (row * 8 + column)
      uint32_t mask = 0;
      const uint32_t row_bits = w == 32u ? full : ((1u << w) - 1u);
#pragma unroll
      for (uint32_t r = 0; r < kSuperH; ++r)
        if (r < h) mask |= ((local >> (r * w)) & row_bits) << ((y0 - ty0 + r) * kSuperW + (x0 - tx0));
      if (valid) {
        masks[e] = mask;
        if (mask != 0u) atomicAdd(&n_touched[prim], static_cast<uint32_t>(__popc(mask)));
      }
      // per-tile counts: transpose the warp's 32 x 32 bit matrix of masks
      // (rows = entries, columns = tiles) across the lanes, so that lane j
      // holds column j, and count its bits
      const uint32_t mine = __popc(warp_transpose_bits(mask, lane));
      if (mine) atomicAdd(&sub_cnt[lane], mine);
    }
    __syncthreads();
    if (threadIdx.x < kSuperTiles) {
      // each sub-chunk's first slot within the chunk's run of every tile
      uint32_t run = 0;
#pragma unroll
      for (uint32_t q = 0; q < kSubChunks; ++q) {
        sub_offsets[(c * kSubChunks + q) * kSuperTiles + threadIdx.x] = run;
        run += s_cnt[q * kSuperTiles + threadIdx.x];
      }
      chunk_counts[c * kSuperTiles + threadIdx.x] = run;
    }
    __syncthreads();
  }
}

// 5b. per (super-tile, tile-in-super-tile): exclusive prefix of the chunk
// counts in chunk (depth) order, in place, and the tile's total.
__global__ void k_chunk_prefix(const uint2* __restrict__ super_ranges, const uint32_t* __restrict__ super_chunk,
                               uint32_t n_super, uint32_t super_w, uint32_t grid_w, uint32_t grid_h,
                               const DevCounts* __restrict__ counts, uint32_t* __restrict__ chunk_counts,
                               uint32_t* __restrict__ tile_total) {
  pdl_entry();
  const uint32_t id = blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= n_super * kSuperTiles) return;
  const uint32_t sp = id / kSuperTiles, j = id % kSuperTiles;
  const uint32_t tx = (sp % super_w) * kSuperW + j % kSuperW, ty = (sp / super_w) * kSuperH + j / kSuperW;
  if (tx >= grid_w || ty >= grid_h) return;
  uint32_t run = 0;
  if (counts->overflow == 0u) {
    const uint2 r = super_ranges[sp];
    const uint32_t first = super_chunk[sp], n_ch = (r.y - r.x + kChunk - 1u) / kChunk;
    // the counts of eight chunks are loaded together, then replaced by
    // their prefixes (one thread per tile: a plain loop would wait on every
    // load in turn)
    for (uint32_t c0 = first; c0 < first + n_ch; c0 += 8u) {
      uint32_t v[8];
#pragma unroll
      for (uint32_t q = 0; q < 8u; ++q) v[q] = c0 + q < first + n_ch ? chunk_counts[(c0 + q) * kSuperTiles + j] : 0u;
#pragma unroll
      for (uint32_t q = 0; q < 8u; ++q)
        if (c0 + q < first + n_ch) {
          chunk_counts[(c0 + q) * kSuperTiles + j] = run;
          run += v[q];
        }
    }
  }
  tile_total[ty * grid_w + tx] = run;
}

// 5c. tile ranges (exclusive scan of the tile totals in tile order), the
// instance count, and bucket offsets (inclusive scan of ceil(total / 32));
// one block of 1024 threads, thread t owns a contiguous run of tiles.
__global__ void __launch_bounds__(1024)
    k_tile_offsets(const uint32_t* __restrict__ tile_total, uint32_t n_tiles, uint2* __restrict__ ranges,
                   uint32_t* __restrict__ bucket_offsets, DevCounts* __restrict__ counts, uint32_t cap_inst,
                   uint32_t cap_buckets) {
  pdl_entry();
  __shared__ uint32_t s_inst[32], s_buck[32];
  const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5;
  const uint32_t per = (n_tiles + 1023u) / 1024u;
  const uint32_t begin = min(n_tiles, t * per), end = min(n_tiles, begin + per);
  uint32_t li = 0, lb = 0;
  for_run(tile_total, begin, end, [&](uint32_t, uint32_t v) {
    li += v;
    lb += (v + kBucket - 1u) / kBucket;
  });
  uint32_t xi = li, xb = lb;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t yi = __shfl_up_sync(0xffffffffu, xi, o), yb = __shfl_up_sync(0xffffffffu, xb, o);
    if (lane >= static_cast<uint32_t>(o)) {
      xi += yi;
      xb += yb;
    }
  }
  if (lane == 31) {
    s_inst[warp] = xi;
    s_buck[warp] = xb;
  }
  __syncthreads();
  if (warp == 0) {
    uint32_t wi = s_inst[lane], wb = s_buck[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t yi = __shfl_up_sync(0xffffffffu, wi, o), yb = __shfl_up_sync(0xffffffffu, wb, o);
      if (lane >= static_cast<uint32_t>(o)) {
        wi += yi;
        wb += yb;
      }
    }
    s_inst[lane] = wi;
    s_buck[lane] = wb;
  }
  __syncthreads();
  uint32_t ri = (warp == 0 ? 0u : s_inst[warp - 1]) + xi - li;
  uint32_t rb = (warp == 0 ? 0u : s_buck[warp - 1]) + xb - lb;
  for_run(tile_total, begin, end, [&](uint32_t k, uint32_t v) {
    ranges[k] = make_uint2(ri, ri + v);
    ri += v;
    rb += (v + kBucket - 1u) / kBucket;
    bucket_offsets[k] = rb;
  });
  if (t == 1023) {
    const uint32_t ni = s_inst[31], nb = s_buck[31];
    counts->n_instances = ni;
    counts->n_buckets = nb;
    if (ni > cap_inst) atomicOr(&counts->overflow, kOverflowInstances);
    if (nb > cap_buckets) atomicOr(&counts->overflow, kOverflowBuckets);
  }
}

// 6. per chunk (one warp each): every hit of every entry to its slot.  The
// warp walks the chunk's entries 32 at a time in order; lane j holds the
// next slot of tile j of the super-tile (the tile's start + the chunk's
// prefix for it).  For each tile hit in the window, the ballot of the
// entries that hit it gives each of them its rank, and those entries store
// their Gaussian ids as one contiguous run.  The tiles of the instances are
// implied by the tile ranges and are not stored.
constexpr int kEmitWarps = 4;

__global__ void __launch_bounds__(32 * kEmitWarps)
    k_emit_instances(const uint4* __restrict__ chunks, const uint32_t* __restrict__ ent_prim,
                     const uint32_t* __restrict__ masks, const uint32_t* __restrict__ chunk_prefix,
                     const uint32_t* __restrict__ sub_offsets, const uint2* __restrict__ ranges,
                     const DevCounts* __restrict__ counts, uint32_t super_w, uint32_t grid_w, uint32_t grid_h,
                     uint32_t* __restrict__ inst_prim) {
  pdl_entry();
  const unsigned full = 0xffffffffu;
  const uint32_t n_units = counts->overflow ? 0u : counts->n_chunks * kSubChunks;
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  const uint32_t lt = lanemask_lt();
  for (uint32_t u = blockIdx.x * kEmitWarps + warp; u < n_units; u += gridDim.x * kEmitWarps) {
    const uint32_t c = u / kSubChunks;
    const uint4 ch = chunks[c];
    const uint32_t b = ch.y + (u % kSubChunks) * kSubChunk;
    if (b >= ch.z) continue;  // warp-uniform: the chunk is shorter
    const uint32_t end = min(ch.z, b + kSubChunk);
    const uint32_t tx = (ch.x % super_w) * kSuperW + lane % kSuperW;
    const uint32_t ty = (ch.x / super_w) * kSuperH + lane / kSuperW;
    uint32_t pos = 0;  // next slot of tile `lane`
    if (tx < grid_w && ty < grid_h)
      pos = ranges[ty * grid_w + tx].x + chunk_prefix[c * kSuperTiles + lane] + sub_offsets[u * kSuperTiles + lane];
    // masks and primitives of the next 32 entries are loaded one round ahead
    uint32_t mask_n = 0, prim_n = 0;
    if (b + lane < end) {
      mask_n = masks[b + lane];
      prim_n = ent_prim[b + lane];
    }
    for (uint32_t e0 = b; e0 < end; e0 += 32u) {
      const uint32_t mask = mask_n, prim = prim_n;
      const uint32_t en = e0 + 32u + lane;
      mask_n = 0;
      prim_n = 0;
      if (en < end) {
        mask_n = masks[en];
        prim_n = ent_prim[en];
      }
      // all 32 tiles unconditionally: the ballots and shuffles of different
      // tiles are independent, so the unrolled steps overlap; the slots of
      // tile `lane` advance by its hit count in these 32 entries, one
      // popcount of the transposed masks
#pragma unroll
      for (int j = 0; j < kSuperTiles; ++j) {
        const uint32_t bj = __ballot_sync(full, (mask >> j) & 1u);
        const uint32_t p = __shfl_sync(full, pos, j);
        if ((bj >> lane) & 1u) inst_prim[p + __popc(bj & lt)] = prim;
      }
      pos += __popc(warp_transpose_bits(mask, lane));
    }
  }
}

template <typename K>
void radix_sort(K* keys[2], uint32_t* vals[2], const uint32_t* count_ptr, const DevCounts* counts,
                int64_t capacity, int total_bits, int& result, const SortScratch& ss, cudaStream_t stream) {
  const uint32_t tiles = static_cast<uint32_t>((capacity + kSortTile - 1) / kSortTile);
  const uint32_t resident = static_cast<uint32_t>(ss.num_sms) * 8u;
  const uint32_t blocks = tiles < resident ? tiles : resident;
  const uint32_t max_blocks = static_cast<uint32_t>(ss.max_blocks);
  int cur = 0;
  for (int shift = 0; shift < total_bits; shift += kRadixBits) {
    const int bits = min(kRadixBits, total_bits - shift);
    if (blocks > 0) {
      pdl_launch(k_radix_hist<K>, blocks, kSortThreads, 0, stream, keys[cur], count_ptr, counts, shift, bits,
                 ss.hist, max_blocks);
      pdl_launch(k_radix_scan, kRadix, kSortThreads, 0, stream, ss.hist, count_ptr, counts, max_blocks,
                 ss.digit_total);
      pdl_launch(k_radix_scatter<K>, blocks, kSortThreads, 0, stream, keys[cur], vals[cur], keys[1 - cur],
                 vals[1 - cur], count_ptr, counts, shift, bits, ss.hist, max_blocks, ss.digit_total);
    }
    cur = 1 - cur;
  }
  result = cur;
}

SortScratch sort_scratch(const RasterState& s) {
  return SortScratch{s.sort_hist, s.sort_digit_total, s.sort_max_blocks, s.num_sms};
}

}  // namespace

void sort_pairs_u32(uint32_t* keys[2], uint32_t* vals[2], const uint32_t* count_ptr, int64_t capacity,
                    int total_bits, int& result, const SortScratch& ss, cudaStream_t stream) {
  radix_sort<uint32_t>(keys, vals, count_ptr, nullptr, capacity, total_bits, result, ss, stream);
}

void launch_binning(RasterState& s, int64_t n64, const DevCamera& cam, int fp16, cudaStream_t stream) {
  const uint32_t n = static_cast<uint32_t>(n64);
  const uint32_t n_blocks = (n + kScanBlock - 1) / kScanBlock;
  const uint32_t n_tiles = cam.grid_w * cam.grid_h;
  const uint32_t super_w = (cam.grid_w + kSuperW - 1) / kSuperW, super_h = (cam.grid_h + kSuperH - 1) / kSuperH;
  const uint32_t n_super = super_w * super_h;
  DevCounts* counts = s.counts;
  // 1. compaction (block sums were written by the preprocess kernel)
  pdl_launch(k_scan_sums, 1, 1024, 0, stream, s.block_sums, n_blocks, &counts->n_visible, nullptr, 0, 0);
  if (n_blocks > 0)
    pdl_launch(k_compact_visible, n_blocks, kScanBlock, 0, stream, s.bounds, s.depth_key, s.block_sums, n,
               s.vis_key[0], s.vis_idx[0]);
  // 2. depth sort (32-bit keys)
  radix_sort<uint32_t>(s.vis_key, s.vis_idx, &counts->n_visible, nullptr, n64, 32, s.depth_result,
                       sort_scratch(s), stream);
  const uint32_t* sorted = s.vis_idx[s.depth_result];
  // 3. super-tile entries in depth order, sorted by super-tile
  if (n_blocks > 0) {
    pdl_launch(k_entry_block_sums, n_blocks, kScanBlock, 0, stream, sorted, s.bounds, counts, s.block_sums);
    pdl_launch(k_scan_sums, 1, 1024, 0, stream, s.block_sums, n_blocks, &counts->n_entries, counts,
               static_cast<uint32_t>(s.cap_entries), kOverflowEntries);
    pdl_launch(k_create_entries, n_blocks, kScanBlock, 0, stream, sorted, s.bounds, s.block_sums, counts, super_w,
               s.ent_key[0], s.ent_prim[0]);
  }
  int super_bits = 1;
  while ((1u << super_bits) < n_super) ++super_bits;
  radix_sort<uint16_t>(s.ent_key, s.ent_prim, &counts->n_entries, counts, s.cap_entries, super_bits, s.ent_result,
                       sort_scratch(s), stream);
  const uint16_t* ent_key = s.ent_key[s.ent_result];
  const uint32_t* ent_prim = s.ent_prim[s.ent_result];
  // 4. chunks of each super-tile's entry list
  if (super_bits <= kRadixBits) {
    // one pass: its digit totals are the super-tiles' entry counts
    pdl_launch(k_chunk_table, 1, 1024, 0, stream, s.super_ranges, s.sort_digit_total, n_super, s.chunks,
               s.super_chunk, counts);
  } else {
    cudaMemsetAsync(s.super_ranges, 0, sizeof(uint2) * n_super, stream);
    pdl_launch(k_super_ranges, s.num_sms * 8, 256, 0, stream, ent_key, counts, s.super_ranges);
    pdl_launch(k_chunk_table, 1, 1024, 0, stream, s.super_ranges, nullptr, n_super, s.chunks, s.super_chunk, counts);
  }
  // 5. hit masks and counts, then every (chunk, tile)'s first slot
  // tile tests: one block per chunk (capacity-sized grid; blocks past the
  // live chunk count exit at once): the hardware hands chunks of uneven
  // length to SMs as they free up, where a grid-stride loop over resident
  // blocks left a tail of blocks with one chunk more than the others (cfg2:
  // 212 against 236 us)
  const int chunk_grid = static_cast<int>(s.cap_chunks > 0 ? s.cap_chunks : 1);
  if (fp16)
    pdl_launch(k_chunk_hits<1>, chunk_grid, kScanBlock, 0, stream, s.chunks, ent_prim, s.bounds, s.mean2d,
               s.conic_opacity, s.prim_info, counts, super_w, s.masks, s.chunk_counts, s.sub_offsets, s.n_touched);
  else
    pdl_launch(k_chunk_hits<0>, chunk_grid, kScanBlock, 0, stream, s.chunks, ent_prim, s.bounds, s.mean2d,
               s.conic_opacity, s.prim_info, counts, super_w, s.masks, s.chunk_counts, s.sub_offsets, s.n_touched);
  pdl_launch(k_chunk_prefix, (n_super * kSuperTiles + 255) / 256, 256, 0, stream, s.super_ranges, s.super_chunk,
             n_super, super_w, cam.grid_w, cam.grid_h, counts, s.chunk_counts, s.tile_total);
  pdl_launch(k_tile_offsets, 1, 1024, 0, stream, s.tile_total, n_tiles, s.ranges, s.bucket_offsets, counts,
             static_cast<uint32_t>(s.cap_inst), static_cast<uint32_t>(s.cap_buckets));
  // 6. instances at their final slots
  // (the emission keeps a grid-stride loop over resident blocks: one block
  // per chunk measured 104 against 90 us at cfg2)
  pdl_launch(k_emit_instances, s.num_sms * 16, 32 * kEmitWarps, 0, stream, s.chunks, ent_prim, s.masks,
             s.chunk_counts, s.sub_offsets, s.ranges, counts, super_w, cam.grid_w, cam.grid_h, s.inst_prim[0]);
  s.tile_result = 0;
}

}  // namespace tgs
