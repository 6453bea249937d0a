// tiles.cuh -- exact Gaussian/tile overlap tests used both when counting the
// tiles a Gaussian touches (preprocess) and when emitting its instances
// (binning).  Both call sites use these same functions, so counts and
// emitted instances always agree.
#pragma once

#include "common.cuh"

namespace tgs {

// Maximum of the Gaussian's exponent over the pixel rectangle of tile
// (tx, ty) compared against ln(255 * opacity): the StopThePop test
// (Radl et al. 2024), as used by tinygs
// (fastgs_ours/kernels_forward.cuh:49-84).  `mx, my` is the 2D mean shifted
// by -0.5 so that pixel centres sit on integer coordinates.  The arithmetic
// order follows the reference so that decisions coincide with it.
__device__ __forceinline__ bool tile_overlaps_f32(float mx, float my, float ca, float cb, float cc,
                                                  uint32_t tx, uint32_t ty, float thr) {
  const float x0 = static_cast<float>(tx * kTile), y0 = static_cast<float>(ty * kTile);
  const float x1 = static_cast<float>((tx + 1) * kTile - 1), y1 = static_cast<float>((ty + 1) * kTile - 1);
  const float dx0 = x0 - mx, dy0 = y0 - my;
  const float left = static_cast<float>(dx0 > 0.0f);
  const float above = static_cast<float>(dy0 > 0.0f);
  const float outx = left + static_cast<float>(mx > x1);
  const float outy = above + static_cast<float>(my > y1);
  if (outy + outx == 0.0f) return true;  // mean inside the tile
  // nearest corner, then slide along the tile edges towards the maximum
  const float cx = x1 + left * (x0 - x1);
  const float cy = y1 + above * (y0 - y1);
  const float ex = mx - cx, ey = my - cy;
  const float sx = copysignf(static_cast<float>(kTile - 1), dx0);
  const float sy = copysignf(static_cast<float>(kTile - 1), dy0);
  const float t0 = outy * __saturatef((sx * ca * ex + sx * cb * ey) / (sx * ca * sx));
  const float t1 = outx * __saturatef((sy * cb * ex + sy * cc * ey) / (sy * cc * sy));
  const float px = cx + t0 * sx, py = cy + t1 * sy;
  const float qx = mx - px, qy = my - py;
  const float power = 0.5f * (ca * qx * qx + cc * qy * qy) + cb * qx * qy;
  return power <= thr;
}

// Per-primitive tile-test inputs in one register bundle.
struct TileTest {
  float mx, my;        // mean2d - 0.5 (fp32 test)
  float ca, cb, cc;    // conic (fp16 test: the half conic widened)
  float xs, ys;        // (mean2d - 0.5) / 16 (fp16 test)
  __half2 c_xy, c_yz;  // fp16 test: conic component pairs of the edge numerator
  __half2 den;         // fp16 test: the edge denominator span^2 * (a, c)
  float thr;           // ln(255 * opacity)
};

// Half-precision variant of the same test used by the fp16 rasterizer
// (fastgs_ours_fp16/kernels_forward.cuh:123-169): the tile-relative
// distances and the edge parameter are evaluated in fp16 on the packed
// conic, the final exponent in fp32.  Same operation sequence and roundings
// as the reference so that instance lists coincide; the denominator
// step * step * (a, c) equals span^2 * (a, c) bit for bit (step = +-span, and
// rounding to nearest is symmetric in sign), so it is a per-primitive term.
__device__ __forceinline__ bool tile_overlaps_f16(const TileTest& p, uint32_t tx, uint32_t ty) {
  const __half2 zero = __float2half2_rn(0.0f);
  const __half span_h = __float2half_rd(static_cast<float>(kTile - 1) / static_cast<float>(kTile));
  const __half2 span = __halves2half2(span_h, span_h);
  const __half2 lo = __halves2half2(__float2half_rd(static_cast<float>(tx) - p.xs),
                                    __float2half_rd(static_cast<float>(ty) - p.ys));
  const __half2 hi = __hadd2(lo, span);
  const __half2 before = __hgtu2(lo, zero);  // 1.0 where the mean lies before the tile
  const __half2 after = __hltu2(hi, zero);   // 1.0 where it lies after it
  const __half2 outside = __hadd2(before, after);
  if (__hbeq2(outside, zero)) return true;
  // step sign from the sign of lo
  const uint32_t lo_bits = *reinterpret_cast<const uint32_t*>(&lo);
  const uint32_t span_bits = *reinterpret_cast<const uint32_t*>(&span);
  const uint32_t step_bits = (span_bits & 0x7fff7fffu) | (lo_bits & 0x80008000u);
  const __half2 step = *reinterpret_cast<const __half2*>(&step_bits);
  // distance from the nearest edge: -(lerp(hi, lo, before))
  const __half2 nb = __hneg2(before);
  const __half2 dist = __hneg2(__hfma2(before, lo, __hfma2(nb, hi, hi)));
  const __half2 dist_xx = __lows2half2(dist, dist);
  const __half2 dist_yy = __highs2half2(dist, dist);
  const __half2 num = __hadd2(__hmul2(__hmul2(step, p.c_xy), dist_xx), __hmul2(__hmul2(step, p.c_yz), dist_yy));
  const __half2 t = __hmul2_sat(__h2div(num, p.den), __lowhigh2highlow(outside));
  const float2 q = __half22float2(__hsub2(dist, __hmul2(t, step)));
  const float qx = q.x * static_cast<float>(kTile), qy = q.y * static_cast<float>(kTile);
  const float power = 0.5f * (p.ca * qx * qx + p.cc * qy * qy) + p.cb * qx * qy;
  return power <= p.thr;
}

// Bundle of the fp16 test from the packed conic (x, y | z, opacity).
__device__ __forceinline__ void tile_test_f16(TileTest& q, float mx, float my, __half2 conic_xy,
                                              __half2 conic_z_opacity) {
  q.mx = mx;
  q.my = my;
  q.xs = mx * (1.0f / kTile);
  q.ys = my * (1.0f / kTile);
  q.c_xy = conic_xy;
  q.c_yz = __halves2half2(__high2half(conic_xy), __low2half(conic_z_opacity));
  const __half2 c_xz = __halves2half2(__low2half(conic_xy), __low2half(conic_z_opacity));
  const __half span_h = __float2half_rd(static_cast<float>(kTile - 1) / static_cast<float>(kTile));
  const __half2 span = __halves2half2(span_h, span_h);
  q.den = __hmul2(__hmul2(span, span), c_xz);
  q.ca = __low2float(conic_xy);
  q.cb = __high2float(conic_xy);
  q.cc = __low2float(conic_z_opacity);
  q.thr = __logf(__high2float(conic_z_opacity) * 255.0f);
}

template <int kFp16>
__device__ __forceinline__ bool overlaps(const TileTest& p, uint32_t tx, uint32_t ty) {
  if constexpr (kFp16)
    return tile_overlaps_f16(p, tx, ty);
  else
    return tile_overlaps_f32(p.mx, p.my, p.ca, p.cb, p.cc, tx, ty, p.thr);
}

}  // namespace tgs
