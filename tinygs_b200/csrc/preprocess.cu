// preprocess.cu -- per-Gaussian projection (forward) and its chain rule
// (backward).
//
// Forward: cull, quaternion -> rotation, 3D covariance, EWA projection with
// the 0.3 px dilation, conic, SH colour, screen-space tile rectangle and the
// exact number of touched tiles.  Reference semantics:
// tinygs/src/rasterizer/fastgs_ours/kernels_forward.cuh:157-412 (fp32) and
// tinygs/src/rasterizer/fastgs_ours_fp16/kernels_forward.cuh:249-496 (fp16).
//
// Unlike the reference, visible Gaussians are not appended through an atomic
// counter: each block publishes its number of visible Gaussians and a
// separate compaction pass (binning.cu) writes the visible list in index
// order, so the depth sort that follows is fully deterministic.
#include "kernels.h"
#include "tiles.cuh"

namespace tgs {
namespace {

constexpr int kPreBlock = 256;

// Real spherical-harmonic basis up to degree 3 at the unit direction (x,y,z),
// normalisation constants of the standard real SH
// (fastgs_ours/kernels_forward.cuh:22-46).
__device__ __forceinline__ int sh_basis(float x, float y, float z, int active_bases, float b[15]) {
  b[0] = -0.48860251190291987f * y;
  b[1] = 0.48860251190291987f * z;
  b[2] = -0.48860251190291987f * x;
  if (active_bases <= 4) return 3;
  const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z;
  b[3] = 1.0925484305920792f * xy;
  b[4] = -1.0925484305920792f * yz;
  b[5] = 0.94617469575755997f * zz - 0.31539156525251999f;
  b[6] = -1.0925484305920792f * xz;
  b[7] = 0.54627421529603959f * xx - 0.54627421529603959f * yy;
  if (active_bases <= 9) return 8;
  b[8] = 0.59004358992664352f * y * (-3.0f * xx + yy);
  b[9] = 2.8906114426405538f * xy * z;
  b[10] = 0.45704579946446572f * y * (1.0f - 5.0f * zz);
  b[11] = 0.3731763325901154f * z * (5.0f * zz - 3.0f);
  b[12] = 0.45704579946446572f * x * (1.0f - 5.0f * zz);
  b[13] = 1.4453057213202769f * z * (xx - yy);
  b[14] = 0.59004358992664352f * x * (-xx + 3.0f * yy);
  return 15;
}

struct Cov3 {
  float m11, m12, m13, m22, m23, m33;
};

struct Rot {
  float r[3][3];
  float qxx, qyy, qzz, qxy, qxz, qyz, qrx, qry, qrz;
};

__device__ __forceinline__ Rot make_rotation(float qr, float qx, float qy, float qz, float qn) {
  Rot R;
  R.qxx = 2.0f * qx * qx / qn; R.qyy = 2.0f * qy * qy / qn; R.qzz = 2.0f * qz * qz / qn;
  R.qxy = 2.0f * qx * qy / qn; R.qxz = 2.0f * qx * qz / qn; R.qyz = 2.0f * qy * qz / qn;
  R.qrx = 2.0f * qr * qx / qn; R.qry = 2.0f * qr * qy / qn; R.qrz = 2.0f * qr * qz / qn;
  R.r[0][0] = 1.0f - (R.qyy + R.qzz); R.r[0][1] = R.qxy - R.qrz; R.r[0][2] = R.qry + R.qxz;
  R.r[1][0] = R.qrz + R.qxy; R.r[1][1] = 1.0f - (R.qxx + R.qzz); R.r[1][2] = R.qyz - R.qrx;
  R.r[2][0] = R.qxz - R.qry; R.r[2][1] = R.qrx + R.qyz; R.r[2][2] = 1.0f - (R.qxx + R.qyy);
  return R;
}

// Sigma = R diag(var) R^T (upper triangle); rs = R diag(var).
__device__ __forceinline__ Cov3 covariance(const Rot& R, const float var[3], float rs[3][3]) {
#pragma unroll
  for (int a = 0; a < 3; ++a)
#pragma unroll
    for (int b = 0; b < 3; ++b) rs[a][b] = R.r[a][b] * var[b];
  Cov3 c;
  c.m11 = rs[0][0] * R.r[0][0] + rs[0][1] * R.r[0][1] + rs[0][2] * R.r[0][2];
  c.m12 = rs[0][0] * R.r[1][0] + rs[0][1] * R.r[1][1] + rs[0][2] * R.r[1][2];
  c.m13 = rs[0][0] * R.r[2][0] + rs[0][1] * R.r[2][1] + rs[0][2] * R.r[2][2];
  c.m22 = rs[1][0] * R.r[1][0] + rs[1][1] * R.r[1][1] + rs[1][2] * R.r[1][2];
  c.m23 = rs[1][0] * R.r[2][0] + rs[1][1] * R.r[2][1] + rs[1][2] * R.r[2][2];
  c.m33 = rs[2][0] * R.r[2][0] + rs[2][1] * R.r[2][1] + rs[2][2] * R.r[2][2];
  return c;
}

// Rows of J*W of the EWA projection (J with the frustum-clamped tx, ty).
struct Ewa {
  float3 a1, a2;  // J W rows
  float3 b1, b2;  // (J W) Sigma rows
  float j11, j22, tx, ty;
};

__device__ __forceinline__ Ewa ewa(const DevCamera& cam, const Cov3& c, float x, float y, float depth) {
  const float cl = (-0.15f * cam.w - cam.cx) / cam.fx, cr = (1.15f * cam.w - cam.cx) / cam.fx;
  const float ct = (-0.15f * cam.h - cam.cy) / cam.fy, cb = (1.15f * cam.h - cam.cy) / cam.fy;
  Ewa e;
  e.tx = fminf(fmaxf(x, cl), cr);
  e.ty = fminf(fmaxf(y, ct), cb);
  e.j11 = cam.fx / depth;
  const float j13 = -e.j11 * e.tx;
  e.j22 = cam.fy / depth;
  const float j23 = -e.j22 * e.ty;
  e.a1 = make_float3(e.j11 * cam.r1.x + j13 * cam.r3.x, e.j11 * cam.r1.y + j13 * cam.r3.y,
                     e.j11 * cam.r1.z + j13 * cam.r3.z);
  e.a2 = make_float3(e.j22 * cam.r2.x + j23 * cam.r3.x, e.j22 * cam.r2.y + j23 * cam.r3.y,
                     e.j22 * cam.r2.z + j23 * cam.r3.z);
  e.b1 = make_float3(e.a1.x * c.m11 + e.a1.y * c.m12 + e.a1.z * c.m13,
                     e.a1.x * c.m12 + e.a1.y * c.m22 + e.a1.z * c.m23,
                     e.a1.x * c.m13 + e.a1.y * c.m23 + e.a1.z * c.m33);
  e.b2 = make_float3(e.a2.x * c.m11 + e.a2.y * c.m12 + e.a2.z * c.m13,
                     e.a2.x * c.m12 + e.a2.y * c.m22 + e.a2.z * c.m23,
                     e.a2.x * c.m13 + e.a2.y * c.m23 + e.a2.z * c.m33);
  return e;
}

__device__ __forceinline__ float dot3(float3 a, float3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }

__device__ __forceinline__ uint32_t clamp_bound(int v, uint32_t hi) {
  return min(hi, static_cast<uint32_t>(max(0, v)));
}

// Exact tile count with warp cooperation for large rectangles: the first
// kSequentialTiles tiles are tested by the owning lane, the rest by the
// whole warp, one Gaussian at a time.  Every lane must call this.
template <int kFp16>
__device__ uint32_t count_tiles(const TileTest& p, uint4 b, bool active) {
  const uint32_t width = b.y - b.x;
  const uint32_t total = active ? width * (b.w - b.z) : 0u;
  uint32_t count = 0;
  const uint32_t seq = min(total, kSequentialTiles);
  for (uint32_t k = 0; k < seq; ++k) {
    const uint32_t ty = b.z + k / width, tx = b.x + k % width;
    count += overlaps<kFp16>(p, tx, ty) ? 1u : 0u;
  }
  uint32_t big = __ballot_sync(0xffffffffu, total > kSequentialTiles);
  const uint32_t lane = lane_id();
  while (big) {
    const int src = __ffs(big) - 1;
    big &= big - 1;
    TileTest q;
    q.mx = __shfl_sync(0xffffffffu, p.mx, src);
    q.my = __shfl_sync(0xffffffffu, p.my, src);
    q.ca = __shfl_sync(0xffffffffu, p.ca, src);
    q.cb = __shfl_sync(0xffffffffu, p.cb, src);
    q.cc = __shfl_sync(0xffffffffu, p.cc, src);
    q.h_xy = __shfl_sync(0xffffffffu, p.h_xy, src);
    q.h_zw = __shfl_sync(0xffffffffu, p.h_zw, src);
    q.thr = __shfl_sync(0xffffffffu, p.thr, src);
    const uint32_t x0 = __shfl_sync(0xffffffffu, b.x, src);
    const uint32_t w = __shfl_sync(0xffffffffu, width, src);
    const uint32_t y0 = __shfl_sync(0xffffffffu, b.z, src);
    const uint32_t n = __shfl_sync(0xffffffffu, total, src);
    // n, w, x0, y0 are warp-uniform, so every lane runs the same rounds
    const uint32_t rounds = (n - kSequentialTiles + 31u) / 32u;
    uint32_t hits = 0;
    for (uint32_t r = 0; r < rounds; ++r) {
      const uint32_t k = kSequentialTiles + r * 32u + lane;
      const bool hit = k < n && overlaps<kFp16>(q, x0 + k % w, y0 + k / w);
      hits += __popc(__ballot_sync(0xffffffffu, hit));
    }
    if (lane == static_cast<uint32_t>(src)) count += hits;
  }
  return count;
}

template <int kFp16>
__global__ void __launch_bounds__(kPreBlock)
    k_preprocess(const float* __restrict__ means, const float* __restrict__ opacities,
                 const float4* __restrict__ rotations, const float* __restrict__ scales,
                 const float* __restrict__ sh0, const float* __restrict__ sh_rest, int active_bases,
                 uint32_t n, DevCamera cam, float4* __restrict__ dens, uint32_t* __restrict__ n_touched,
                 uint32_t* __restrict__ depth_key, ushort4* __restrict__ bounds,
                 float2* __restrict__ mean2d, float4* __restrict__ conic_opacity,
                 PrimInfo16* __restrict__ prim_info, float* __restrict__ color,
                 uint32_t* __restrict__ block_visible) {
  const uint32_t i = blockIdx.x * kPreBlock + threadIdx.x;
  const bool in_range = i < n;
  const uint32_t gi = in_range ? i : (n > 0 ? n - 1 : 0);

  // culling checks before the reference's first warp-level exit
  const float mx3 = means[3 * gi], my3 = means[3 * gi + 1], mz3 = means[3 * gi + 2];
  const float depth = cam.r3.x * mx3 + cam.r3.y * my3 + cam.r3.z * mz3 + cam.r3.w;
  bool active = in_range && !(depth < cam.near_plane || depth > cam.far_plane);
  float opacity;
  __half opacity_h = __float2half_rn(0.0f);
  if constexpr (kFp16) {
    // fp16 path: logit rounded to half, sigmoid in fp32, stored as half
    const __half raw = active ? __float2half_rn(opacities[gi]) : __float2half_rn(0.0f);
    opacity = 1.0f / (1.0f + __expf(-__half2float(raw)));
    if (opacity < kMinAlpha) active = false;
    opacity_h = __float2half_rn(opacity);
  } else {
    opacity = 1.0f / (1.0f + __expf(-opacities[gi]));
    if (opacity < kMinAlpha) active = false;
  }
  const float s0 = scales[3 * gi], s1 = scales[3 * gi + 1], s2 = scales[3 * gi + 2];
  float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
  if (!kFp16 || active) q = rotations[gi];
  const float qn = q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w;
  if (qn < 1e-8f) active = false;
  const bool warp_alive = __ballot_sync(0xffffffffu, active) != 0u;

  uint32_t touched = 0;
  uint4 rect = make_uint4(0, 0, 0, 0);
  float2 m2 = make_float2(0.f, 0.f);
  float3 conic = make_float3(0.f, 0.f, 0.f);
  TileTest tt{};
  if (warp_alive) {
    const float e0 = __expf(s0), e1 = __expf(s1), e2 = __expf(s2);
    const float var[3] = {e0 * e0, e1 * e1, e2 * e2};
    const Rot R = make_rotation(q.x, q.y, q.z, q.w, qn);
    float rs[3][3];
    const Cov3 c3 = covariance(R, var, rs);
    const float x = (cam.r1.x * mx3 + cam.r1.y * my3 + cam.r1.z * mz3 + cam.r1.w) / depth;
    const float y = (cam.r2.x * mx3 + cam.r2.y * my3 + cam.r2.z * mz3 + cam.r2.w) / depth;
    const Ewa e = ewa(cam, c3, x, y, depth);
    const float ca = dot3(e.b1, e.a1) + kDilation;
    const float cb = dot3(e.b1, e.a2);
    const float cc = dot3(e.b2, e.a2) + kDilation;
    const float det = ca * cc - cb * cb;
    if (det < 1e-8f) active = false;
    conic = make_float3(cc / det, -cb / det, ca / det);
    if (dens != nullptr && in_range) {
      // screen radius for densification; evaluated for every lane of a warp
      // that carried on, as in the reference (kernels_forward.cuh:342-348)
      const float mid = 0.5f * (ca + cc);
      const float l1 = mid + sqrtf(fmaxf(0.1f, mid * mid - det));
      const float l2 = mid - sqrtf(fmaxf(0.1f, mid * mid - det));
      const float rad = ceilf(3.f * sqrtf(fmaxf(l1, l2)));
      dens[gi].w = fmaxf(dens[gi].w, rad);
    }
    m2 = make_float2(x * cam.fx + cam.cx, y * cam.fy + cam.cy);
    __half2 hxy = __float2half2_rn(0.f), hzw = __float2half2_rn(0.f);
    float thr;
    if constexpr (kFp16) {
      hxy = __floats2half2_rn(conic.x, conic.y);
      hzw = __halves2half2(__float2half_rn(conic.z), opacity_h);
      thr = __logf(__half2float(opacity_h) * 255.0f);
    } else {
      thr = __logf(opacity * 255.0f);
    }
    const float fac = sqrtf(2.0f * thr);
    const float ex = fmaxf(fac * sqrtf(ca) - 0.5f, 0.0f);
    const float ey = fmaxf(fac * sqrtf(cc) - 0.5f, 0.0f);
    rect = make_uint4(clamp_bound(__float2int_rd((m2.x - ex) / static_cast<float>(kTile)), cam.grid_w),
                      clamp_bound(__float2int_ru((m2.x + ex) / static_cast<float>(kTile)), cam.grid_w),
                      clamp_bound(__float2int_rd((m2.y - ey) / static_cast<float>(kTile)), cam.grid_h),
                      clamp_bound(__float2int_ru((m2.y + ey) / static_cast<float>(kTile)), cam.grid_h));
    if ((rect.y - rect.x) * (rect.w - rect.z) == 0u) active = false;
    tt.mx = m2.x - 0.5f;
    tt.my = m2.y - 0.5f;
    tt.ca = conic.x;
    tt.cb = conic.y;
    tt.cc = conic.z;
    tt.h_xy = hxy;
    tt.h_zw = hzw;
    tt.thr = thr;
    if (__ballot_sync(0xffffffffu, active) != 0u) touched = count_tiles<kFp16>(tt, rect, active);
    if (!active) touched = 0;
  }

  if (in_range) {
    n_touched[i] = touched;
    if (touched > 0) {
      depth_key[i] = __float_as_uint(depth);
      bounds[i] = make_ushort4(static_cast<unsigned short>(rect.x), static_cast<unsigned short>(rect.y),
                               static_cast<unsigned short>(rect.z), static_cast<unsigned short>(rect.w));
      mean2d[i] = m2;
      // view-dependent colour
      float3 col = make_float3(0.5f + 0.28209479177387814f * sh0[3 * i],
                               0.5f + 0.28209479177387814f * sh0[3 * i + 1],
                               0.5f + 0.28209479177387814f * sh0[3 * i + 2]);
      if (active_bases > 1) {
        const float dx = mx3 - cam.pos.x, dy = my3 - cam.pos.y, dz = mz3 - cam.pos.z;
        const float inv = rsqrtf(dx * dx + dy * dy + dz * dz);
        float b[15];
        const int nb = sh_basis(dx * inv, dy * inv, dz * inv, active_bases, b);
        const float* rest = sh_rest + 45 * static_cast<size_t>(i);
        for (int k = 0; k < nb; ++k) {
          col.x += b[k] * rest[3 * k];
          col.y += b[k] * rest[3 * k + 1];
          col.z += b[k] * rest[3 * k + 2];
        }
      }
      if constexpr (kFp16) {
        PrimInfo16 rec;
        rec.conic_xy = tt.h_xy;
        rec.conic_z_opacity = tt.h_zw;
        rec.rgb_pad = make_uchar4(static_cast<unsigned char>(sat(col.x) * 255.0f),
                                  static_cast<unsigned char>(sat(col.y) * 255.0f),
                                  static_cast<unsigned char>(sat(col.z) * 255.0f), 0);
        rec.pad = 0;
        prim_info[i] = rec;
      } else {
        conic_opacity[i] = make_float4(conic.x, conic.y, conic.z, opacity);
        color[3 * i] = col.x;
        color[3 * i + 1] = col.y;
        color[3 * i + 2] = col.z;
      }
    }
  }
  // number of visible Gaussians of this block, for the compaction scan
  const uint32_t vis = __syncthreads_count(in_range && touched > 0);
  if (threadIdx.x == 0) block_visible[blockIdx.x] = vis;
}

// --------------------------------------------------------------- backward

// dL/d(direction) contributions of each SH basis function (derivatives of the
// real SH basis written out per band; fastgs_ours/kernels_backward.cuh:22-86).
__device__ __forceinline__ float3 sh_backward(const float* __restrict__ rest, float* __restrict__ g_rest,
                                              float3 gc, float3 dir_raw, int active_bases, bool accumulate,
                                              float3& g_dc_out) {
  g_dc_out = make_float3(0.28209479177387814f * gc.x, 0.28209479177387814f * gc.y,
                         0.28209479177387814f * gc.z);
  if (active_bases <= 1) {
    if (!accumulate)
      for (int k = 0; k < 45; ++k) g_rest[k] = 0.f;
    return make_float3(0.f, 0.f, 0.f);
  }
  const float inv = rsqrtf(dir_raw.x * dir_raw.x + dir_raw.y * dir_raw.y + dir_raw.z * dir_raw.z);
  const float x = dir_raw.x * inv, y = dir_raw.y * inv, z = dir_raw.z * inv;
  float b[15];
  const int nb = sh_basis(x, y, z, active_bases, b);
  float dbx[15], dby[15], dbz[15];
#pragma unroll
  for (int k = 0; k < 15; ++k) dbx[k] = dby[k] = dbz[k] = 0.f;
  dby[0] = -0.48860251190291987f;
  dbz[1] = 0.48860251190291987f;
  dbx[2] = -0.48860251190291987f;
  if (nb > 3) {
    dbx[3] = 1.0925484305920792f * y; dby[3] = 1.0925484305920792f * x;
    dby[4] = -1.0925484305920792f * z; dbz[4] = -1.0925484305920792f * y;
    dbz[5] = 1.8923493915151202f * z;
    dbx[6] = -1.0925484305920792f * z; dbz[6] = -1.0925484305920792f * x;
    dbx[7] = 1.0925484305920792f * x; dby[7] = -1.0925484305920792f * y;
  }
  if (nb > 8) {
    const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z;
    dbx[8] = -3.5402615395598609f * xy;
    dby[8] = -1.7701307697799304f * xx + 1.7701307697799304f * yy;
    dbx[9] = 2.8906114426405538f * yz; dby[9] = 2.8906114426405538f * xz; dbz[9] = 2.8906114426405538f * xy;
    dby[10] = 0.45704579946446572f - 2.2852289973223288f * zz; dbz[10] = -4.5704579946446566f * yz;
    dbz[11] = 5.597644988851731f * zz - 1.1195289977703462f;
    dbx[12] = 0.45704579946446572f - 2.2852289973223288f * zz; dbz[12] = -4.5704579946446566f * xz;
    dbx[13] = 2.8906114426405538f * xz; dby[13] = -2.8906114426405538f * yz;
    dbz[13] = 1.4453057213202769f * xx - 1.4453057213202769f * yy;
    dbx[14] = -1.7701307697799304f * xx + 1.7701307697799304f * yy; dby[14] = 3.5402615395598609f * xy;
  }
  float3 gd = make_float3(0.f, 0.f, 0.f);
  for (int k = 0; k < 15; ++k) {
    if (k < nb) {
      const float r0 = rest[3 * k], r1 = rest[3 * k + 1], r2 = rest[3 * k + 2];
      const float g0 = b[k] * gc.x, g1 = b[k] * gc.y, g2 = b[k] * gc.z;
      if (accumulate) {
        g_rest[3 * k] += g0; g_rest[3 * k + 1] += g1; g_rest[3 * k + 2] += g2;
      } else {
        g_rest[3 * k] = g0; g_rest[3 * k + 1] = g1; g_rest[3 * k + 2] = g2;
      }
      const float d = r0 * gc.x + r1 * gc.y + r2 * gc.z;
      gd.x += dbx[k] * d;
      gd.y += dby[k] * d;
      gd.z += dbz[k] * d;
    } else if (!accumulate) {
      g_rest[3 * k] = 0.f; g_rest[3 * k + 1] = 0.f; g_rest[3 * k + 2] = 0.f;
    }
  }
  // through the normalisation of the view direction
  const float xx = dir_raw.x * dir_raw.x, yy = dir_raw.y * dir_raw.y, zz = dir_raw.z * dir_raw.z;
  const float xy = dir_raw.x * dir_raw.y, xz = dir_raw.x * dir_raw.z, yz = dir_raw.y * dir_raw.z;
  const float ns = xx + yy + zz;
  const float r = rsqrtf(ns * ns * ns);
  return make_float3(((yy + zz) * gd.x - xy * gd.y - xz * gd.z) * r,
                     (-xy * gd.x + (xx + zz) * gd.y - yz * gd.z) * r,
                     (-xz * gd.x - yz * gd.y + (xx + yy) * gd.z) * r);
}

__device__ __forceinline__ void put(float* p, float v, bool acc) {
  if (acc) *p += v; else *p = v;
}

// Preprocess backward: conic -> 2D covariance -> 3D covariance -> (log-scale,
// quaternion); mean2d (+ frustum clamp mask) -> mean3d; colour -> SH (+ view
// direction) -> mean3d; densification accumulators.  Reference:
// fastgs_ours/kernels_backward.cuh:88-352 (including its 2D-covariance
// off-diagonal term without the factor 2, lines 210-214).
__global__ void __launch_bounds__(128)
    k_preprocess_backward(const float* __restrict__ means, const float4* __restrict__ rotations,
                          const float* __restrict__ scales, const float* __restrict__ sh_rest,
                          int active_bases, uint32_t n, DevCamera cam,
                          const uint32_t* __restrict__ n_touched, const float4* __restrict__ helpers,
                          float* __restrict__ g_means, float* __restrict__ g_opac,
                          float4* __restrict__ g_rot, float* __restrict__ g_scales,
                          float* __restrict__ g_sh0, float* __restrict__ g_sh_rest, int accumulate,
                          float4* __restrict__ dens, const DevCounts* __restrict__ counts) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const bool acc = accumulate != 0;
  // an overflowed forward left no valid backward scratch: treat as untouched
  if (n_touched[i] == 0 || counts->overflow != 0u) {
    if (!acc) {
      for (int k = 0; k < 3; ++k) {
        g_means[3 * i + k] = 0.f; g_scales[3 * i + k] = 0.f; g_sh0[3 * i + k] = 0.f;
      }
      g_opac[i] = 0.f;
      g_rot[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      float* gr = g_sh_rest + 45 * static_cast<size_t>(i);
      for (int k = 0; k < 45; ++k) gr[k] = 0.f;
    }
    return;
  }
  const float4 h0 = helpers[3 * i], h1 = helpers[3 * i + 1], h2 = helpers[3 * i + 2];
  const float gmx = h0.x, gmy = h0.y;
  const float gca = h1.x, gcb = h1.y, gcc = h1.z;
  const float gop = h1.w;
  const float3 gcol = make_float3(h2.x, h2.y, h2.z);

  const float m0 = means[3 * i], m1 = means[3 * i + 1], m2 = means[3 * i + 2];
  float3 g_dc;
  const float3 dmc = sh_backward(sh_rest + 45 * static_cast<size_t>(i), g_sh_rest + 45 * static_cast<size_t>(i),
                                 gcol, make_float3(m0 - cam.pos.x, m1 - cam.pos.y, m2 - cam.pos.z),
                                 active_bases, acc, g_dc);
  put(&g_sh0[3 * i], g_dc.x, acc);
  put(&g_sh0[3 * i + 1], g_dc.y, acc);
  put(&g_sh0[3 * i + 2], g_dc.z, acc);
  put(&g_opac[i], gop, acc);

  const float depth = cam.r3.x * m0 + cam.r3.y * m1 + cam.r3.z * m2 + cam.r3.w;
  const float x = (cam.r1.x * m0 + cam.r1.y * m1 + cam.r1.z * m2 + cam.r1.w) / depth;
  const float y = (cam.r2.x * m0 + cam.r2.y * m1 + cam.r2.z * m2 + cam.r2.w) / depth;
  const float e0 = __expf(scales[3 * i]), e1 = __expf(scales[3 * i + 1]), e2 = __expf(scales[3 * i + 2]);
  const float var[3] = {e0 * e0, e1 * e1, e2 * e2};
  const float4 q = rotations[i];
  const float qn = q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w;
  const Rot R = make_rotation(q.x, q.y, q.z, q.w, qn);
  float rs[3][3];
  const Cov3 c3 = covariance(R, var, rs);
  const Ewa e = ewa(cam, c3, x, y, depth);
  const float A = dot3(e.b1, e.a1) + kDilation, B = dot3(e.b1, e.a2), C = dot3(e.b2, e.a2) + kDilation;
  const float aa = A * A, bb = B * B, cc = C * C, ac = A * C, ab = A * B, bc = B * C;
  const float dr = 1.0f / (ac - bb + 1e-8f);
  const float dr2 = dr * dr;
  const float d2a = dr2 * (2.0f * bc * gcb - cc * gca - bb * gcc);
  const float d2b = dr2 * (bc * gca - (ac + bb) * gcb + ab * gcc);
  const float d2c = dr2 * (2.0f * ab * gcb - bb * gca - aa * gcc);
  const float3 a1 = e.a1, a2 = e.a2;
  const float d3[6] = {
      (a1.x * a1.x) * d2a + 2.0f * (a1.x * a2.x) * d2b + (a2.x * a2.x) * d2c,
      (a1.x * a1.y) * d2a + (a1.x * a2.y + a1.y * a2.x) * d2b + (a2.x * a2.y) * d2c,
      (a1.x * a1.z) * d2a + (a1.x * a2.z + a1.z * a2.x) * d2b + (a2.x * a2.z) * d2c,
      (a1.y * a1.y) * d2a + 2.0f * (a1.y * a2.y) * d2b + (a2.y * a2.y) * d2c,
      (a1.y * a1.z) * d2a + (a1.y * a2.z + a1.z * a2.y) * d2b + (a2.y * a2.z) * d2c,
      (a1.z * a1.z) * d2a + 2.0f * (a1.z * a2.z) * d2b + (a2.z * a2.z) * d2c};
  const float3 dj1 = make_float3(2.0f * (e.b1.x * d2a + e.b2.x * d2b), 2.0f * (e.b1.y * d2a + e.b2.y * d2b),
                                 2.0f * (e.b1.z * d2a + e.b2.z * d2b));
  const float3 dj2 = make_float3(2.0f * (e.b1.x * d2b + e.b2.x * d2c), 2.0f * (e.b1.y * d2b + e.b2.y * d2c),
                                 2.0f * (e.b1.z * d2b + e.b2.z * d2c));
  const float dj11 = cam.r1.x * dj1.x + cam.r1.y * dj1.y + cam.r1.z * dj1.z;
  const float dj22 = cam.r2.x * dj2.x + cam.r2.y * dj2.y + cam.r2.z * dj2.z;
  const float dj13 = cam.r3.x * dj1.x + cam.r3.y * dj1.y + cam.r3.z * dj1.z;
  const float dj23 = cam.r3.x * dj2.x + cam.r3.y * dj2.y + cam.r3.z * dj2.z;
  const float cl = (-0.15f * cam.w - cam.cx) / cam.fx, cr = (1.15f * cam.w - cam.cx) / cam.fx;
  const float ct = (-0.15f * cam.h - cam.cy) / cam.fy, cbm = (1.15f * cam.h - cam.cy) / cam.fy;
  const float dj13c = dj13 * ((x > cl && x < cr) ? 1.0f : 0.0f);
  const float dj23c = dj23 * ((y > ct && y < cbm) ? 1.0f : 0.0f);
  const float h1z = dj11 - 2.0f * e.tx * dj13c;
  const float h2z = dj22 - 2.0f * e.ty * dj23c;
  const float dc0 = e.j11 * (gmx - dj13c / depth);
  const float dc1 = e.j22 * (gmy - dj23c / depth);
  const float dc2 = -e.j11 * (x * gmx + h1z / depth) - e.j22 * (y * gmy + h2z / depth);
  put(&g_means[3 * i], (cam.r1.x * dc0 + cam.r2.x * dc1 + cam.r3.x * dc2) + dmc.x, acc);
  put(&g_means[3 * i + 1], (cam.r1.y * dc0 + cam.r2.y * dc1 + cam.r3.y * dc2) + dmc.y, acc);
  put(&g_means[3 * i + 2], (cam.r1.z * dc0 + cam.r2.z * dc1 + cam.r3.z * dc2) + dmc.z, acc);

  const float es[3] = {e0, e1, e2};
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const float dv = R.r[0][k] * R.r[0][k] * d3[0] + R.r[1][k] * R.r[1][k] * d3[3] +
                     R.r[2][k] * R.r[2][k] * d3[5] +
                     2.0f * (R.r[0][k] * R.r[1][k] * d3[1] + R.r[0][k] * R.r[2][k] * d3[2] +
                             R.r[1][k] * R.r[2][k] * d3[4]);
    put(&g_scales[3 * i + k], 2.0f * es[k] * es[k] * dv, acc);
  }
  float dR[3][3];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    dR[0][k] = 2.0f * (rs[0][k] * d3[0] + rs[1][k] * d3[1] + rs[2][k] * d3[2]);
    dR[1][k] = 2.0f * (rs[0][k] * d3[1] + rs[1][k] * d3[3] + rs[2][k] * d3[4]);
    dR[2][k] = 2.0f * (rs[0][k] * d3[2] + rs[1][k] * d3[4] + rs[2][k] * d3[5]);
  }
  const float dqxx = -dR[1][1] - dR[2][2], dqyy = -dR[0][0] - dR[2][2], dqzz = -dR[0][0] - dR[1][1];
  const float dqxy = dR[0][1] + dR[1][0], dqxz = dR[0][2] + dR[2][0], dqyz = dR[1][2] + dR[2][1];
  const float dqrx = dR[2][1] - dR[1][2], dqry = dR[0][2] - dR[2][0], dqrz = dR[1][0] - dR[0][1];
  const float hn = R.qxx * dqxx + R.qyy * dqyy + R.qzz * dqzz + R.qxy * dqxy + R.qxz * dqxz + R.qyz * dqyz +
                   R.qrx * dqrx + R.qry * dqry + R.qrz * dqrz;
  const float den = qn * __fsqrt_rn(qn);
  const float4 gq = make_float4(2.0f * (q.y * dqrx + q.z * dqry + q.w * dqrz - q.x * hn) / den,
                                2.0f * (2.0f * q.y * dqxx + q.z * dqxy + q.w * dqxz + q.x * dqrx - q.y * hn) / den,
                                2.0f * (2.0f * q.z * dqyy + q.y * dqxy + q.w * dqyz + q.x * dqry - q.z * hn) / den,
                                2.0f * (2.0f * q.w * dqzz + q.y * dqxz + q.z * dqyz + q.x * dqrz - q.w * hn) / den);
  if (acc) {
    float4 o = g_rot[i];
    g_rot[i] = make_float4(o.x + gq.x, o.y + gq.y, o.z + gq.z, o.w + gq.w);
  } else {
    g_rot[i] = gq;
  }
  if (dens != nullptr) {
    float4 d = dens[i];
    d.x += 1.0f;
    const float ux = gmx * (0.5f * cam.w), uy = gmy * (0.5f * cam.h);
    d.y += sqrtf(ux * ux + uy * uy);
    const float vx = h0.z * (0.5f * cam.w), vy = h0.w * (0.5f * cam.h);
    d.z += sqrtf(vx * vx + vy * vy);
    dens[i] = d;
  }
}

}  // namespace

void launch_preprocess(const RasterState& s, const GaussianPtrs& g, const DevCamera& cam, int fp16,
                       float4* dens, cudaStream_t stream) {
  const uint32_t n = static_cast<uint32_t>(g.n);
  const int active_bases = (g.sh_degree + 1) * (g.sh_degree + 1);
  const uint32_t blocks = (n + kPreBlock - 1) / kPreBlock;
  if (blocks == 0) return;
  if (fp16)
    k_preprocess<1><<<blocks, kPreBlock, 0, stream>>>(
        g.means, g.opacities, reinterpret_cast<const float4*>(g.rotations), g.scales, g.sh0, g.sh_rest,
        active_bases, n, cam, dens, s.n_touched, s.depth_key, s.bounds, s.mean2d, s.conic_opacity,
        s.prim_info, s.color, s.block_sums);
  else
    k_preprocess<0><<<blocks, kPreBlock, 0, stream>>>(
        g.means, g.opacities, reinterpret_cast<const float4*>(g.rotations), g.scales, g.sh0, g.sh_rest,
        active_bases, n, cam, dens, s.n_touched, s.depth_key, s.bounds, s.mean2d, s.conic_opacity,
        s.prim_info, s.color, s.block_sums);
}

void launch_preprocess_backward(const RasterState& s, const GaussianPtrs& g, const GaussianPtrs& grads,
                                const DevCamera& cam, int accumulate, float4* dens, cudaStream_t stream) {
  const uint32_t n = static_cast<uint32_t>(g.n);
  const int active_bases = (g.sh_degree + 1) * (g.sh_degree + 1);
  const uint32_t blocks = (n + 127) / 128;
  if (blocks == 0) return;
  k_preprocess_backward<<<blocks, 128, 0, stream>>>(
      g.means, reinterpret_cast<const float4*>(g.rotations), g.scales, g.sh_rest, active_bases, n, cam,
      s.n_touched, reinterpret_cast<const float4*>(s.helpers), grads.means, grads.opacities,
      reinterpret_cast<float4*>(grads.rotations), grads.scales, grads.sh0, grads.sh_rest, accumulate, dens, s.counts);
}

}  // namespace tgs
