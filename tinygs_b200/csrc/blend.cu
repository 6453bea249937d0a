// blend.cu -- per-tile front-to-back alpha blending, forward and backward.
//
// Forward (one CTA per 16x16 tile): primitives are staged through shared
// memory in batches (fp16: one 36-byte record per primitive, read with
// broadcast vector loads), each pixel composites front to back until its
// transmittance would drop below 1e-4, and every 32 primitives the running
// (colour, transmittance) of every pixel is checkpointed so that the
// backward can restart any 32-primitive bucket independently.
//   fp32 reference: fastgs_ours/kernels_forward.cuh:569-715
//   fp16 reference: fastgs_ours_fp16/kernels_forward.cuh:917-1171 (half2
//   arithmetic, two horizontally adjacent pixels per thread, colour and
//   transmittance carried scaled by 255)
// Backward (one warp per bucket, one lane per primitive): the 256 pixels of
// the tile stream through the warp as two diagonal wavefronts (pixels 0-127
// and 128-255, evaluated together with packed fp32x2 instructions; lane l
// sees pixel i - l of each stream at step i), so each pixel's evolving state
// (transmittance, colour still to come) passes from primitive to primitive in
// depth order by a one-lane shuffle while its constant part (centre,
// dL/dpixel) is read from a per-warp ring in shared memory.  Per-primitive
// sums are reduced in registers and added to the per-Gaussian scratch with one
// set of atomics per bucket.
//   fp32 reference: fastgs_ours/kernels_backward.cuh:675-927
//   fp16 reference: fastgs_ours_fp16/kernels_backward.cuh:861-1389; its
//   semantics (no per-pixel contributor mask, alpha capped at fp16(0.99),
//   255-scaled checkpoints) are evaluated here in fp32 arithmetic.
#include "kernels.h"

namespace tgs {
namespace {

// The buckets of a tile that start before its deepest contributor are the
// ones the backward runs; the forward appends them to a list (in no
// particular order) so that the backward's warps only see live work.
__device__ __forceinline__ void publish_live_buckets(uint32_t tile, uint32_t deepest, DevCounts* counts,
                                                     uint32_t* s_live) {
  const uint32_t nl = (deepest + kBucket - 1) / kBucket;
  s_live[0] = nl > 0 ? atomicAdd(&counts->n_live_buckets, nl) : 0u;
  s_live[1] = nl;
}

// ------------------------------------------------------------ forward fp32

__global__ void __launch_bounds__(kTilePixels)
    k_blend_forward_f32(const uint2* __restrict__ ranges, const uint32_t* __restrict__ bucket_offsets,
                        const uint32_t* __restrict__ inst_prim, const float2* __restrict__ mean2d,
                        const float4* __restrict__ conic_opacity, const float* __restrict__ color,
                        const DevCounts* __restrict__ counts, DevCamera cam, float* __restrict__ image,
                        float* __restrict__ alpha, uint32_t* __restrict__ n_contrib,
                        uint32_t* __restrict__ tile_max, uint2* __restrict__ live_buckets,
                        DevCounts* __restrict__ live_count, float4* __restrict__ ckpt) {
  __shared__ float2 s_mean[kTilePixels];
  __shared__ float4 s_co[kTilePixels];
  __shared__ float4 s_col[kTilePixels];
  __shared__ uint32_t s_max[kTilePixels / 32];
  __shared__ uint32_t s_live[2];
  const uint32_t tid = threadIdx.x;
  const uint32_t lx = tid & 15u, ly = tid >> 4;
  const uint32_t tile = blockIdx.y * cam.grid_w + blockIdx.x;
  const uint32_t px = blockIdx.x * kTile + lx, py = blockIdx.y * kTile + ly;
  const bool inside = px < cam.width && py < cam.height;
  const float2 pix = make_float2(static_cast<float>(px) + 0.5f, static_cast<float>(py) + 0.5f);
  const bool ok = counts->overflow == 0u;
  const uint2 r = ok ? ranges[tile] : make_uint2(0, 0);
  const uint32_t count = r.y - r.x;
  const uint32_t first_bucket = tile == 0 ? 0u : bucket_offsets[tile - 1];
  const uint32_t slot = tiled_index(ly, lx, 2);
  float4* my_ckpt = ckpt + static_cast<size_t>(first_bucket) * kTilePixels + slot;

  float cr = 0.f, cg = 0.f, cb = 0.f, T = 1.f;
  uint32_t n_seen = 0, n_used = 0;
  bool done = !inside;
  for (uint32_t start = 0; start < count; start += kTilePixels) {
    if (__syncthreads_count(done) == kTilePixels) break;
    const uint32_t k = start + tid;
    if (k < count) {
      const uint32_t p = inst_prim[r.x + k];
      s_mean[tid] = mean2d[p];
      s_co[tid] = conic_opacity[p];
      s_col[tid] = make_float4(fmaxf(color[3 * p], 0.f), fmaxf(color[3 * p + 1], 0.f),
                               fmaxf(color[3 * p + 2], 0.f), 0.f);
    }
    __syncthreads();
    const uint32_t batch = min(static_cast<uint32_t>(kTilePixels), count - start);
    uint32_t j = 0;
    for (; !done && j < batch; ++j) {
      if ((j & 31u) == 0) my_ckpt[static_cast<size_t>((start + j) >> 5) * kTilePixels] = make_float4(cr, cg, cb, T);
      ++n_seen;
      const float4 co = s_co[j];
      const float2 m = s_mean[j];
      const float dx = m.x - pix.x, dy = m.y - pix.y;
      const float power = 0.5f * (co.x * dx * dx + co.z * dy * dy) + co.y * dx * dy;
      if (power < 0.0f) continue;
      const float a = fminf(co.w * __expf(-power), kMaxAlphaF32);
      if (a < kMinAlpha) continue;
      const float Tn = T * (1.0f - a);
      if (Tn < kMinTransmittance) {
        done = true;
        continue;
      }
      const float4 c = s_col[j];
      const float w = T * a;
      cr += w * c.x;
      cg += w * c.y;
      cb += w * c.z;
      T = Tn;
      n_used = n_seen;
    }
    // checkpoints of the rest of this batch hold the frozen state
    for (j = (j + 31u) & ~31u; j < batch; j += 32u)
      my_ckpt[static_cast<size_t>((start + j) >> 5) * kTilePixels] = make_float4(cr, cg, cb, T);
  }
  if (inside) {
    const uint32_t pi = tiled_index(py, px, cam.tiled_w);
    image[pi] = cr;
    image[pi + cam.plane] = cg;
    image[pi + 2 * cam.plane] = cb;
    if (alpha != nullptr) alpha[pi] = 1.0f - T;
    n_contrib[pi] = n_used;
  }
  const uint32_t wmax = __reduce_max_sync(0xffffffffu, n_used);
  if ((tid & 31u) == 0) s_max[tid >> 5] = wmax;
  __syncthreads();
  if (tid == 0) {
    uint32_t mx = 0;
    for (int w = 0; w < kTilePixels / 32; ++w) mx = max(mx, s_max[w]);
    tile_max[tile] = mx;
    publish_live_buckets(tile, mx, live_count, s_live);
  }
  __syncthreads();
  for (uint32_t j = tid; j < s_live[1]; j += kTilePixels) live_buckets[s_live[0] + j] = make_uint2(tile, j);
}

// ------------------------------------------------------------ forward fp16

__device__ __forceinline__ __half2 h2exp2_approx(__half2 x) {
  __half2 y;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(*reinterpret_cast<uint32_t*>(&y)) : "r"(*reinterpret_cast<uint32_t*>(&x)));
  return y;
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// fp16 rasterizer: 128 threads, thread (tx, ty) owns pixels (2tx, ty) and
// (2tx+1, ty).  Every arithmetic step is the same fp16 operation as in the
// reference kernel, so images agree to the bit with it (up to the one
// hardware exp2 approximation both share).
constexpr int kF16Threads = kTilePixels / 2;

__global__ void __launch_bounds__(kF16Threads)
    k_blend_forward_f16(const uint2* __restrict__ ranges, const uint32_t* __restrict__ bucket_offsets,
                        const uint32_t* __restrict__ inst_prim, const float2* __restrict__ mean2d,
                        const PrimInfo16* __restrict__ prim_info, const DevCounts* __restrict__ counts,
                        DevCamera cam, __half* __restrict__ image, __half* __restrict__ alpha,
                        uint16_t* __restrict__ n_contrib, uint32_t* __restrict__ tile_max,
                        uint2* __restrict__ live_buckets, DevCounts* __restrict__ live_count,
                        uint4* __restrict__ ckpt) {
  // per primitive of the batch, as broadcast vector loads: (mx, my, cx, cy),
  // (cz, opacity, r, g) and b, every value duplicated into both halves
  __shared__ uint4 s_q0[kF16Threads], s_q1[kF16Threads];
  __shared__ __half2 s_b[kF16Threads];
  __shared__ uint32_t s_max[kF16Threads / 32];
  __shared__ uint32_t s_live[2];
  const uint32_t tid = threadIdx.x;
  const uint32_t tx = tid & 7u, ty = tid >> 3;
  const uint32_t lx = 2 * tx, ly = ty;
  const uint32_t tile = blockIdx.y * cam.grid_w + blockIdx.x;
  const uint32_t px = blockIdx.x * kTile + lx, py = blockIdx.y * kTile + ly;
  const uint32_t in0 = (px < cam.width && py < cam.height) ? 1u : 0u;
  const uint32_t in1 = (px + 1 < cam.width && py < cam.height) ? 1u : 0u;
  const uint32_t inside = in0 | (in1 << 16);

  const __half2 inv16 = __float2half2_rn(0.0625f);
  const __half2 h16 = __float2half2_rn(16.0f);
  const __half2 half_2 = __float2half2_rn(0.5f);
  const __half2 zero2 = __float2half2_rn(0.0f);
  const __half2 one2 = __float2half2_rn(1.0f);
  const __half2 scale2 = __float2half2_rn(255.0f);
  const __half2 unscale2 = __float2half2_rn(1.0f / 255.0f);
  const __half2 max_a2 = __float2half2_rn(kMaxAlphaF16);
  const __half min_t = __float2half_rd(kMinTransmittance * 255.0f);
  const __half2 min_t2 = __halves2half2(min_t, min_t);
  const __half2 log2e = __float2half2_rn(1.4426950409f);
  const __half2 s16_1 = __halves2half2(__float2half_rn(16.0f), __float2half_rn(1.0f));
  // pixel offsets in tile units: (x + 0.5) / 16 for both pixels, (y + 0.5) / 16
  const __half2 off0 = __hfma2(inv16, __halves2half2(__uint2half_rn(lx), __uint2half_rn(ly)),
                               __float2half2_rn(1.0f / 32.0f));
  const __half2 off_x = __halves2half2(__low2half(off0), __hadd(__low2half(inv16), __low2half(off0)));
  const __half2 off_y = __highs2half2(off0, off0);
  const float2 anchor = make_float2(static_cast<float>(blockIdx.x), static_cast<float>(blockIdx.y));

  const bool ok = counts->overflow == 0u;
  const uint2 r = ok ? ranges[tile] : make_uint2(0, 0);
  const uint32_t count = r.y - r.x;
  const uint32_t first_bucket = tile == 0 ? 0u : bucket_offsets[tile - 1];
  // checkpoint record of the pixel pair: 2 x (r,g | b,T) halves
  uint4* my_ckpt = ckpt + (static_cast<size_t>(first_bucket) * kTilePixels + tiled_index(ly, lx, 2)) / 2;

  __half2 cr = zero2, cg = zero2, cb = zero2, T = scale2;
  uint32_t n_seen = 0;        // two 16-bit counters
  uint32_t live = inside;     // 1 per unfinished pixel in each 16-bit half
  auto store_ckpt = [&](uint32_t bucket) {
    const uint32_t p0x = h2u(__lows2half2(cr, cg)), p0y = h2u(__lows2half2(cb, T));
    const uint32_t p1x = h2u(__highs2half2(cr, cg)), p1y = h2u(__highs2half2(cb, T));
    my_ckpt[static_cast<size_t>(bucket) * (kTilePixels / 2)] = make_uint4(p0x, p0y, p1x, p1y);
  };
  for (uint32_t start = 0; start < count; start += kF16Threads) {
    if (__syncthreads_count(live) == 0) break;
    const uint32_t k = start + tid;
    if (k < count) {
      const uint32_t p = inst_prim[r.x + k];
      const float2 m = mean2d[p];
      const float mx = m.x / 16.0f - anchor.x, my = m.y / 16.0f - anchor.y;
      const PrimInfo16 rec = prim_info[p];
      const __half2 cxy = __hmul2(rec.conic_xy, h16);
      const __half2 czo = __hmul2(rec.conic_z_opacity, s16_1);
      s_q0[tid] = make_uint4(h2u(__float2half2_rn(mx)), h2u(__float2half2_rn(my)), h2u(__lows2half2(cxy, cxy)),
                             h2u(__highs2half2(cxy, cxy)));
      s_q1[tid] = make_uint4(h2u(__lows2half2(czo, czo)), h2u(__highs2half2(czo, czo)),
                             h2u(__float2half2_rn(static_cast<float>(rec.rgb_pad.x))),
                             h2u(__float2half2_rn(static_cast<float>(rec.rgb_pad.y))));
      s_b[tid] = __float2half2_rn(static_cast<float>(rec.rgb_pad.z));
    }
    __syncthreads();
    const uint32_t batch = min(static_cast<uint32_t>(kF16Threads), count - start);
    uint32_t i = 0;
    while (live && i < batch) {
      store_ckpt((start + i) >> 5);
      const uint32_t j_end = min(i + 32u, batch);
      for (uint32_t j = i; j < j_end && live; ++j) {
        const uint4 q0 = s_q0[j], q1 = s_q1[j];
        const __half2 dx = __hsub2(u2h(q0.x), off_x);
        const __half2 dy = __hsub2(u2h(q0.y), off_y);
        const __half2 qx = __hmul2(dx, __hmul2(u2h(q0.z), dx));
        const __half2 qz = __hmul2(dy, __hmul2(u2h(q1.x), dy));
        const __half2 qy = __hmul2(dx, __hmul2(u2h(q0.w), dy));
        const __half2 power = __hmul2(__hfma2(half_2, __hadd2(qx, qz), qy), h16);
        const __half2 g = h2exp2_approx(__hmul2(__hneg2(power), log2e));
        const __half2 a = __hmin2(__hmul2(u2h(q1.y), g), max_a2);
        const __half2 Tn = __hfma2(__hneg2(a), T, T);
        // positive halves compare like their bit patterns
        const uint32_t accept = __vsetgeu2(h2u(Tn), h2u(min_t2));
        const uint32_t on = live & accept;
        const uint32_t mask = (on << 16) - on;  // 0xffff per enabled pixel
        const __half2 w = u2h(h2u(__hmul2(__hmul2(T, a), unscale2)) & mask);
        cr = __hfma2(u2h(q1.z), w, cr);
        cg = __hfma2(u2h(q1.w), w, cg);
        cb = __hfma2(s_b[j], w, cb);
        T = u2h(h2u(T) ^ (mask & (h2u(Tn) ^ h2u(T))));
        n_seen = __vaddus2(n_seen, live);
        live &= accept;
      }
      live &= __vsetltu2(n_seen, 0xffffffffu);
      i += 32u;
    }
    for (; i < batch; i += 32u) store_ckpt((start + i) >> 5);
  }
  const __half2 out_r = __hmul2(cr, unscale2), out_g = __hmul2(cg, unscale2), out_b = __hmul2(cb, unscale2);
  const __half2 out_t = __hmul2(T, unscale2);
  if (inside != 0u) {
    const uint32_t pi = tiled_index(py, px, cam.tiled_w);
    *reinterpret_cast<__half2*>(image + pi) = out_r;
    *reinterpret_cast<__half2*>(image + pi + cam.plane) = out_g;
    *reinterpret_cast<__half2*>(image + pi + 2 * cam.plane) = out_b;
    if (alpha != nullptr) *reinterpret_cast<__half2*>(alpha + pi) = __hsub2(one2, out_t);
    *reinterpret_cast<uint32_t*>(n_contrib + pi) = n_seen;
  }
  const uint32_t mine = max(n_seen & 0xffffu, n_seen >> 16);
  const uint32_t wmax = __reduce_max_sync(0xffffffffu, mine);
  if ((tid & 31u) == 0) s_max[tid >> 5] = wmax;
  __syncthreads();
  if (tid == 0) {
    uint32_t mx = 0;
    for (int w = 0; w < kF16Threads / 32; ++w) mx = max(mx, s_max[w]);
    tile_max[tile] = mx;
    publish_live_buckets(tile, mx, live_count, s_live);
  }
  __syncthreads();
  for (uint32_t j = tid; j < s_live[1]; j += kF16Threads) live_buckets[s_live[0] + j] = make_uint2(tile, j);
}

// ---------------------------------------------------------------- backward

constexpr int kBwdWarps = 8;
constexpr float kLog2e = 1.4426950408889634f;

// Per-pixel inputs of one bucket, fetched a chunk of 32 pixels ahead.
template <int kFp16>
struct PixelRaw {
  float ck[4];   // checkpoint (colour so far, T) at the start of the bucket
  float img[3];  // final colour
  float grad[3];
  uint32_t last;
  bool inside;
};

template <int kFp16>
__device__ __forceinline__ PixelRaw<kFp16> fetch_pixel(uint32_t i, uint32_t bucket, uint32_t gx, uint32_t gy,
                                                       const DevCamera& cam, const void* image_v,
                                                       const void* grad_v, const void* n_contrib_v,
                                                       const void* ckpt_v) {
  PixelRaw<kFp16> r{};
  uint32_t dx, dy;
  walk_pixel(i, dx, dy);
  const uint32_t px = gx * kTile + dx, py = gy * kTile + dy;
  r.inside = px < cam.width && py < cam.height;
  if (!r.inside) return r;
  const uint32_t pi = tiled_index(py, px, cam.tiled_w);
  if constexpr (kFp16) {
    const uint2 c = reinterpret_cast<const uint2*>(ckpt_v)[static_cast<size_t>(bucket) * kTilePixels + i];
    const float2 rg = __half22float2(u2h(c.x));
    const float2 bt = __half22float2(u2h(c.y));
    r.ck[0] = rg.x;
    r.ck[1] = rg.y;
    r.ck[2] = bt.x;
    r.ck[3] = bt.y;
    const __half* img = reinterpret_cast<const __half*>(image_v);
    const __half* gr = reinterpret_cast<const __half*>(grad_v);
#pragma unroll
    for (int c3 = 0; c3 < 3; ++c3) {
      r.img[c3] = __half2float(img[pi + c3 * cam.plane]);
      r.grad[c3] = __half2float(gr[pi + c3 * cam.plane]);
    }
  } else {
    const float4 c = reinterpret_cast<const float4*>(ckpt_v)[static_cast<size_t>(bucket) * kTilePixels + i];
    r.ck[0] = c.x;
    r.ck[1] = c.y;
    r.ck[2] = c.z;
    r.ck[3] = c.w;
    const float* img = reinterpret_cast<const float*>(image_v);
    const float* gr = reinterpret_cast<const float*>(grad_v);
#pragma unroll
    for (int c3 = 0; c3 < 3; ++c3) {
      r.img[c3] = img[pi + c3 * cam.plane];
      r.grad[c3] = gr[pi + c3 * cam.plane];
    }
    r.last = reinterpret_cast<const uint32_t*>(n_contrib_v)[pi];
  }
  return r;
}

// The state a pixel enters the bucket with: transmittance T, the colour
// still to come behind the current primitive dotted with dL/dpixel (adg),
// the pixel centre, dL/dpixel and (fp32 path) its contributor count.  fp16
// path: colour and the colour-behind are on the 0..255 scale.
template <int kFp16>
__device__ __forceinline__ void pixel_state(const PixelRaw<kFp16>& r, uint32_t i, uint32_t gx, uint32_t gy,
                                            float4& a4, float4& b4) {
  uint32_t dx, dy;
  walk_pixel(i, dx, dy);
  const float px = static_cast<float>(gx * kTile + dx), py = static_cast<float>(gy * kTile + dy);
  if (!r.inside) {
    a4 = make_float4(0.f, 0.f, px, py);
    b4 = make_float4(0.f, 0.f, 0.f, __uint_as_float(0u));
    return;
  }
  const float s = kFp16 ? 255.0f : 1.0f;
  const float a0 = r.img[0] * s - r.ck[0], a1 = r.img[1] * s - r.ck[1], a2 = r.img[2] * s - r.ck[2];
  const float adg = a0 * r.grad[0] + a1 * r.grad[1] + a2 * r.grad[2];
  const float T = kFp16 ? r.ck[3] * (1.0f / 255.0f) : r.ck[3];
  a4 = make_float4(T, adg, px, py);
  b4 = make_float4(r.grad[0], r.grad[1], r.grad[2], __uint_as_float(kFp16 ? 0xffffffffu : r.last));
}

// Packed fp32 pairs (sm_100 f32x2 instructions): two pixels per lane, each
// element rounded exactly like the scalar operation (ftz, as the rest of the
// fast-math build).
__device__ __forceinline__ uint64_t pk(float2 v) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(v.x), "f"(v.y));
  return r;
}
__device__ __forceinline__ float2 upk(uint64_t r) {
  float2 v;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
  return v;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  uint64_t d;
  asm("add.rn.ftz.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pk(a)), "l"(pk(b)));
  return upk(d);
}
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
  uint64_t d;
  asm("sub.rn.ftz.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pk(a)), "l"(pk(b)));
  return upk(d);
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  uint64_t d;
  asm("mul.rn.ftz.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pk(a)), "l"(pk(b)));
  return upk(d);
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.ftz.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(pk(a)), "l"(pk(b)), "l"(pk(c)));
  return upk(d);
}
__device__ __forceinline__ float2 dup2(float v) { return make_float2(v, v); }

template <int kFp16>
__device__ __forceinline__ void load_conic(uint32_t p, const float4* __restrict__ conic_opacity,
                                           const PrimInfo16* __restrict__ prim_info, float4& co) {
  if constexpr (kFp16) {
    const PrimInfo16 rec = prim_info[p];
    co = make_float4(__low2float(rec.conic_xy), __high2float(rec.conic_xy), __low2float(rec.conic_z_opacity),
                     __high2float(rec.conic_z_opacity));
  } else {
    co = conic_opacity[p];
  }
}

// kAbs: also accumulate sum |dL/dmean2d| (consumed only by densification).
template <int kFp16, bool kAbs>
__global__ void __launch_bounds__(32 * kBwdWarps)
    k_blend_backward(const uint2* __restrict__ ranges, const uint32_t* __restrict__ bucket_offsets,
                     const uint2* __restrict__ live_buckets, const uint32_t* __restrict__ inst_prim,
                     const float2* __restrict__ mean2d, const float4* __restrict__ conic_opacity,
                     const float* __restrict__ color, const PrimInfo16* __restrict__ prim_info,
                     const void* __restrict__ image_v, const void* __restrict__ grad_v,
                     const void* __restrict__ n_contrib_v, const void* __restrict__ ckpt_v,
                     const DevCounts* __restrict__ counts, DevCamera cam, float* __restrict__ helpers,
                     uint32_t* __restrict__ work) {
  // Two pixel streams per lane (pixels 0..127 and 128..255 of the tile),
  // evaluated together with packed fp32 pairs.  Per warp, the pixel pairs of
  // the current and the previous 32-step chunk sit in a ring of 64 records:
  // the constant part of a pixel (centre, dL/dpixel, contributor count) is
  // read by each lane from the ring at index (step - lane); only the
  // evolving state (T, -adg) travels from lane to lane, and lane 0 takes a
  // new pair's state from s_ta.
  __shared__ float4 s_pxy[kBwdWarps][64];  // (px A, px B, py A, py B)
  __shared__ float4 s_g01[kBwdWarps][64];  // (G.r A, G.r B, G.g A, G.g B)
  __shared__ float2 s_g2[kBwdWarps][64];   // (G.b A, G.b B)
  __shared__ uint2 s_last[kBwdWarps][kFp16 ? 1 : 64];
  __shared__ float4 s_ta[kBwdWarps][32];   // (T A, T B, -adg A, -adg B) entering the bucket
  if (counts->overflow != 0u) return;
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  const uint32_t n_live = counts->n_live_buckets;
  const uint32_t stride = gridDim.x * kBwdWarps;
  const float max_alpha = kFp16 ? __half2float(__float2half_rn(kMaxAlphaF16)) : kMaxAlphaF32;
  constexpr uint32_t kHalf = kTilePixels / 2;  // pixels per stream
  constexpr uint32_t kChunks = kHalf / 32;
  // lanes see the "previous chunk" half of the ring before the first chunk:
  // finite values there (their T = adg = 0 makes every term zero)
  s_pxy[warp][lane] = s_pxy[warp][32 + lane] = make_float4(0.f, 0.f, 0.f, 0.f);
  s_g01[warp][lane] = s_g01[warp][32 + lane] = make_float4(0.f, 0.f, 0.f, 0.f);
  s_g2[warp][lane] = s_g2[warp][32 + lane] = make_float2(0.f, 0.f);
  if constexpr (!kFp16) s_last[warp][lane] = s_last[warp][32 + lane] = make_uint2(0u, 0u);
  __syncwarp();

  // Buckets differ in cost (a bucket late in its tile sweeps pixels that
  // have mostly stopped), so a fixed share per warp leaves a tail of warps
  // still busy after the others ran out.  The first three quarters of the
  // list are dealt out by stride; the rest is taken kGrab buckets at a time
  // from the counter *work (zeroed before the launch), by whichever warps are
  // free.
  constexpr uint32_t kGrab = 4;
  const uint32_t n_static = n_live - n_live / 4;
  uint32_t item = blockIdx.x * kBwdWarps + warp, grab_end = 0;
  for (;;) {
    if (item >= n_static) {
      if (item >= grab_end) {
        uint32_t b = 0;
        if (lane == 0) b = atomicAdd(work, kGrab);
        item = n_static + __shfl_sync(0xffffffffu, b, 0);
        grab_end = item + kGrab;
      }
      if (item >= n_live) break;
    }
    const uint2 lb = live_buckets[item];
    const uint32_t tile = lb.x, tb = lb.y;
    const uint2 r = ranges[tile];
    const uint32_t bucket = (tile == 0 ? 0u : bucket_offsets[tile - 1]) + tb;
    const uint32_t count = r.y - r.x;
    const uint32_t tp = tb * kBucket + lane;
    const bool valid_prim = tp < count && (!kFp16 || tp <= 0xffffu);
    const uint32_t gx = tile % cam.grid_w, gy = tile / cam.grid_w;

    uint32_t p = 0;
    float mx = 0.f, my = 0.f, op = 0.f, ka = 0.f, kb = 0.f, kc = 0.f;
    float col0 = 0.f, col1 = 0.f, col2 = 0.f;
    if (valid_prim) {
      p = inst_prim[r.x + tp];
      const float2 m = mean2d[p];
      mx = m.x - 0.5f;
      my = m.y - 0.5f;
      float4 co;
      load_conic<kFp16>(p, conic_opacity, prim_info, co);
      op = co.w;
      // exponent in base 2: exp(-q) = 2^(-q log2 e)
      ka = 0.5f * kLog2e * co.x;
      kb = kLog2e * co.y;
      kc = 0.5f * kLog2e * co.z;
      if constexpr (kFp16) {
        const uchar4 c = prim_info[p].rgb_pad;
        col0 = static_cast<float>(c.x);
        col1 = static_cast<float>(c.y);
        col2 = static_cast<float>(c.z);
      } else {
        col0 = fmaxf(color[3 * p], 0.f);
        col1 = fmaxf(color[3 * p + 1], 0.f);
        col2 = fmaxf(color[3 * p + 2], 0.f);
      }
    }
    const float2 MX = dup2(mx), MY = dup2(my), OP = dup2(op), KA = dup2(ka), KB = dup2(kb), KC = dup2(kc);
    const float2 C0 = dup2(col0), C1 = dup2(col1), C2 = dup2(col2);
    // per-primitive sums, one partial per stream (added at the end)
    float2 g_op = dup2(0.f), g_ca = dup2(0.f), g_cb = dup2(0.f), g_cc = dup2(0.f);
    float2 g_c0 = dup2(0.f), g_c1 = dup2(0.f), g_c2 = dup2(0.f);
    float2 s_x = dup2(0.f), s_y = dup2(0.f);  // sums of dop * (mean - pixel)
    float2 g_mx = dup2(0.f), g_my = dup2(0.f), a_mx = dup2(0.f), a_my = dup2(0.f);
    // evolving state of the lane's two pixels (zero: no pixel)
    float2 T = dup2(0.f), nadg = dup2(0.f);

    for (uint32_t chunk = 0; chunk <= kChunks; ++chunk) {
      float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f), b4 = a4, c4 = a4, d4 = a4;
      if (chunk < kChunks) {
        const uint32_t ia = chunk * 32 + lane, ib = kHalf + ia;
        const PixelRaw<kFp16> ra = fetch_pixel<kFp16>(ia, bucket, gx, gy, cam, image_v, grad_v, n_contrib_v, ckpt_v);
        const PixelRaw<kFp16> rb = fetch_pixel<kFp16>(ib, bucket, gx, gy, cam, image_v, grad_v, n_contrib_v, ckpt_v);
        pixel_state<kFp16>(ra, ia, gx, gy, a4, b4);
        pixel_state<kFp16>(rb, ib, gx, gy, c4, d4);
      }
      const uint32_t slot = (chunk & 1u) * 32u + lane;
      s_pxy[warp][slot] = make_float4(a4.z, c4.z, a4.w, c4.w);
      s_g01[warp][slot] = make_float4(b4.x, d4.x, b4.y, d4.y);
      s_g2[warp][slot] = make_float2(b4.z, d4.z);
      if constexpr (!kFp16) s_last[warp][slot] = make_uint2(__float_as_uint(b4.w), __float_as_uint(d4.w));
      s_ta[warp][lane] = make_float4(a4.x, c4.x, -a4.y, -c4.y);
      __syncwarp();
      const uint32_t base = (chunk & 1u) * 32u + 64u;  // slot of step 0, lane 0, plus 64
#pragma unroll 4
      for (uint32_t st = 0; st < 32; ++st) {
        T.x = __shfl_up_sync(0xffffffffu, T.x, 1);
        T.y = __shfl_up_sync(0xffffffffu, T.y, 1);
        nadg.x = __shfl_up_sync(0xffffffffu, nadg.x, 1);
        nadg.y = __shfl_up_sync(0xffffffffu, nadg.y, 1);
        if (lane == 0) {
          const float4 ta = s_ta[warp][st];
          T = make_float2(ta.x, ta.y);
          nadg = make_float2(ta.z, ta.w);
        }
        const uint32_t ring = (base + st - lane) & 63u;
        const float4 pxy = s_pxy[warp][ring], g01 = s_g01[warp][ring];
        const float2 G2 = s_g2[warp][ring];
        const float2 G0 = make_float2(g01.x, g01.y), G1 = make_float2(g01.z, g01.w);
        const float2 ddx = sub2(MX, make_float2(pxy.x, pxy.y)), ddy = sub2(MY, make_float2(pxy.z, pxy.w));
        const float2 dxx = mul2(ddx, ddx), dxy = mul2(ddx, ddy), dyy = mul2(ddy, ddy);
        const float2 q = fma2(KB, dxy, fma2(KC, dyy, mul2(KA, dxx)));
        float2 a = mul2(OP, make_float2(exp2f(-fmaxf(q.x, 0.f)), exp2f(-fmaxf(q.y, 0.f))));
        a.x = fminf(a.x, max_alpha);
        a.y = fminf(a.y, max_alpha);
        if constexpr (!kFp16) {
          const uint2 last = s_last[warp][ring];
          a.x = tp < last.x ? a.x : 0.f;
          a.y = tp < last.y ? a.y : 0.f;
        }
        const float2 w = mul2(T, a);
        const float2 om = fma2(a, dup2(-1.0f), dup2(1.0f));
        const float2 cdg = fma2(C2, G2, fma2(C1, G1, mul2(C0, G0)));
        g_c0 = fma2(w, G0, g_c0);
        g_c1 = fma2(w, G1, g_c1);
        g_c2 = fma2(w, G2, g_c2);
        nadg = fma2(w, cdg, nadg);  // what lies behind this primitive (negated)
        const float2 ro = make_float2(1.0f / om.x, 1.0f / om.y);
        const float2 dop = mul2(a, fma2(T, cdg, mul2(nadg, ro)));
        g_op = add2(g_op, dop);
        g_ca = fma2(dop, dxx, g_ca);
        g_cb = fma2(dop, dxy, g_cb);
        g_cc = fma2(dop, dyy, g_cc);
        if constexpr (kAbs) {
          // (ca, cb, cc) = (2 ka, kb, 2 kc) / log2 e
          const float2 gmx = mul2(dop, fma2(dup2(2.0f * ka), ddx, mul2(KB, ddy)));
          const float2 gmy = mul2(dop, fma2(KB, ddx, mul2(dup2(2.0f * kc), ddy)));
          g_mx = add2(g_mx, gmx);
          g_my = add2(g_my, gmy);
          a_mx = add2(a_mx, make_float2(fabsf(gmx.x), fabsf(gmx.y)));
          a_my = add2(a_my, make_float2(fabsf(gmy.x), fabsf(gmy.y)));
        } else {
          s_x = fma2(dop, ddx, s_x);
          s_y = fma2(dop, ddy, s_y);
        }
        T = mul2(T, om);
      }
      __syncwarp();
    }
    float go = g_op.x + g_op.y, gca = g_ca.x + g_ca.y, gcb = g_cb.x + g_cb.y, gcc = g_cc.x + g_cc.y;
    float gc0 = g_c0.x + g_c0.y, gc1 = g_c1.x + g_c1.y, gc2 = g_c2.x + g_c2.y;
    float gmx_s = 0.f, gmy_s = 0.f, amx_s = 0.f, amy_s = 0.f;
    if constexpr (kAbs) {
      gmx_s = (g_mx.x + g_mx.y) * (1.0f / kLog2e);
      gmy_s = (g_my.x + g_my.y) * (1.0f / kLog2e);
      amx_s = (a_mx.x + a_mx.y) * (1.0f / kLog2e);
      amy_s = (a_my.x + a_my.y) * (1.0f / kLog2e);
    }
    const float sxs = s_x.x + s_x.y, sys = s_y.x + s_y.y;
    if (valid_prim) {
      if constexpr (!kAbs) {
        float4 co;
        load_conic<kFp16>(p, conic_opacity, prim_info, co);
        gmx_s = co.x * sxs + co.y * sys;
        gmy_s = co.y * sxs + co.z * sys;
      }
      if constexpr (!kFp16) {
        // colour clamped at zero passes no gradient
        if (color[3 * p] < 0.f) gc0 = 0.f;
        if (color[3 * p + 1] < 0.f) gc1 = 0.f;
        if (color[3 * p + 2] < 0.f) gc2 = 0.f;
      }
      // scale conventions: fp32 accumulates in [0,1] colour units; the fp16
      // path carries colour and the colour-behind scaled by 255 (reference
      // lines 1359-1369 divide by 255 at the end)
      const float sc = kFp16 ? (1.0f / 255.0f) : 1.0f;
      float* h = helpers + static_cast<size_t>(p) * kHelperFloats;
      atomicAdd(h + 0, -gmx_s * sc);
      atomicAdd(h + 1, -gmy_s * sc);
      if constexpr (kAbs) {
        atomicAdd(h + 2, amx_s * sc);
        atomicAdd(h + 3, amy_s * sc);
      }
      atomicAdd(h + 4, -0.5f * gca * sc);
      atomicAdd(h + 5, -0.5f * gcb * sc);
      atomicAdd(h + 6, -0.5f * gcc * sc);
      atomicAdd(h + 7, go * sc * (1.0f - op));
      atomicAdd(h + 8, gc0);
      atomicAdd(h + 9, gc1);
      atomicAdd(h + 10, gc2);
    }
    item += item < n_static ? stride : 1u;
  }
}

template <int kFp16, bool kAbs>
void run_blend_backward(const RasterState& s, const DevCamera& cam, const void* image, const void* grad_image,
                        cudaStream_t stream) {
  // persistent: as many blocks as are resident at once
  static int per_sm[64] = {};  // per device
  int dev = 0;
  cudaGetDevice(&dev);
  int& bps = per_sm[dev & 63];
  if (bps == 0) {
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&bps, k_blend_backward<kFp16, kAbs>, 32 * kBwdWarps, 0);
    if (bps <= 0) bps = 1;
  }
  cudaMemsetAsync(s.bwd_work, 0, sizeof(uint32_t), stream);
  k_blend_backward<kFp16, kAbs><<<s.num_sms * bps, 32 * kBwdWarps, 0, stream>>>(
      s.ranges, s.bucket_offsets, s.live_buckets, s.inst_prim[s.tile_result], s.mean2d, s.conic_opacity, s.color,
      s.prim_info, image, grad_image, s.n_contrib, s.ckpt, s.counts, cam, s.helpers, s.bwd_work);
}

}  // namespace

void launch_blend_forward(const RasterState& s, const DevCamera& cam, int fp16, void* image, void* alpha,
                          cudaStream_t stream) {
  const dim3 grid(cam.grid_w, cam.grid_h);
  const uint32_t* sorted_prim = s.inst_prim[s.tile_result];
  if (fp16)
    k_blend_forward_f16<<<grid, kF16Threads, 0, stream>>>(
        s.ranges, s.bucket_offsets, sorted_prim, s.mean2d, s.prim_info, s.counts, cam,
        reinterpret_cast<__half*>(image), reinterpret_cast<__half*>(alpha), reinterpret_cast<uint16_t*>(s.n_contrib),
        s.tile_max_contrib, s.live_buckets, s.counts, reinterpret_cast<uint4*>(s.ckpt));
  else
    k_blend_forward_f32<<<grid, kTilePixels, 0, stream>>>(
        s.ranges, s.bucket_offsets, sorted_prim, s.mean2d, s.conic_opacity, s.color, s.counts, cam,
        reinterpret_cast<float*>(image), reinterpret_cast<float*>(alpha), s.n_contrib, s.tile_max_contrib,
        s.live_buckets, s.counts, s.ckpt);
}

void launch_blend_backward(const RasterState& s, const DevCamera& cam, int fp16, const void* image,
                           const void* grad_image, int abs_grad, cudaStream_t stream) {
  if (fp16) {
    if (abs_grad)
      run_blend_backward<1, true>(s, cam, image, grad_image, stream);
    else
      run_blend_backward<1, false>(s, cam, image, grad_image, stream);
  } else {
    if (abs_grad)
      run_blend_backward<0, true>(s, cam, image, grad_image, stream);
    else
      run_blend_backward<0, false>(s, cam, image, grad_image, stream);
  }
}

}  // namespace tgs
