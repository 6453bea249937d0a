// preprocess.cu -- per-Gaussian projection (forward) and its chain rule
// (backward).
//
// Forward: cull, quaternion -> rotation, 3D covariance, EWA projection with
// the 0.3 px dilation, conic, SH colour and screen-space tile rectangle (the
// exact tile tests and touched-tile counts are done during binning, per
// super-tile).  Reference semantics:
// tinygs/src/rasterizer/fastgs_ours/kernels_forward.cuh:157-412 (fp32) and
// tinygs/src/rasterizer/fastgs_ours_fp16/kernels_forward.cuh:249-496 (fp16).
//
// Unlike the reference, candidate Gaussians (culling passed, non-empty tile
// rectangle) are not appended through an atomic counter: each block
// publishes its number of candidates and a separate compaction pass
// (binning.cu) writes the list in index order, so the depth sort that follows
// is fully deterministic.
#include "kernels.h"
#include "tiles.cuh"

namespace tgs {
namespace {

constexpr int kPreBlock = 256;

// 16-byte (or 4-byte) asynchronous global -> shared copies (cp.async), so
// that the loads of a whole warp slice are in flight at once.
__device__ __forceinline__ void cp_async16(float* smem_dst, const float* gmem_src) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gmem_src));
}
__device__ __forceinline__ void cp_async4(float* smem_dst, const float* gmem_src) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(d), "l"(gmem_src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int kPending>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(kPending));
}


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

// Per-view outputs of the preprocess (one view's arena, possibly a peer's).
struct PreOut {
  uint32_t* n_touched;
  uint32_t* depth_key;
  ushort4* bounds;
  float2* mean2d;
  float4* conic_opacity;
  PrimInfo16* prim_info;
  float* color;
  float4* helpers;
  uint32_t* block_visible;
};

// One Gaussian's view-independent inputs, loaded once per thread.
struct PreIn {
  float mx3, my3, mz3, logit, s0, s1, s2;
  float4 q;
};

// Projection, culling, colour and records of Gaussian i for one camera, with
// the reference's operation order (fastgs_ours*/kernels_forward.cuh:157-412).
// Every thread of the block calls it (the candidate count is a block
// reduction).  The warp's SH rows are in `rest_rows` once the pending
// cp.async group has landed (waited for after the projection, so the copy
// overlaps it on the first call).
template <int kFp16>
__device__ __forceinline__ void preprocess_view(const PreIn& in, bool in_range, uint32_t i, uint32_t gi,
                                                const DevCamera& cam, const PreOut& o, float4* __restrict__ dens,
                                                const float* __restrict__ sh0, const float* rest_rows,
                                                int active_bases, uint32_t block_slot, int zero_helpers) {
  const uint32_t lane = threadIdx.x & 31u;
  // culling checks before the reference's first warp-level exit
  const float mx3 = in.mx3, my3 = in.my3, mz3 = in.mz3;
  const float depth = cam.r3.x * mx3 + cam.r3.y * my3 + cam.r3.z * mz3 + cam.r3.w;
  bool active = in_range && !(depth < cam.near_plane || depth > cam.far_plane);
  float opacity;
  __half opacity_h = __float2half_rn(0.0f);
  if constexpr (kFp16) {
    // fp16 path: logit rounded to half, sigmoid in fp32, stored as half
    const __half raw = active ? __float2half_rn(in.logit) : __float2half_rn(0.0f);
    opacity = 1.0f / (1.0f + __expf(-__half2float(raw)));
    if (opacity < kMinAlpha) active = false;
    opacity_h = __float2half_rn(opacity);
  } else {
    opacity = 1.0f / (1.0f + __expf(-in.logit));
    if (opacity < kMinAlpha) active = false;
  }
  const float s0 = in.s0, s1 = in.s1, s2 = in.s2;
  // (the fp16 reference reads the rotation of active Gaussians only)
  const float4 q = (!kFp16 || active) ? in.q : make_float4(0.f, 0.f, 0.f, 0.f);
  const float qn = q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w;
  if (qn < 1e-8f) active = false;
  const bool warp_alive = __ballot_sync(0xffffffffu, active) != 0u;

  uint4 rect = make_uint4(0, 0, 0, 0);
  float2 m2 = make_float2(0.f, 0.f);
  float3 conic = make_float3(0.f, 0.f, 0.f);
  __half2 hxy = __float2half2_rn(0.f), hzw = __float2half2_rn(0.f);
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
  }
  const bool candidate = in_range && warp_alive && active;

  cp_async_wait<0>();
  __syncwarp();

  if (in_range) {
    o.n_touched[i] = 0;  // binning adds the hits of each super-tile
    o.bounds[i] = candidate ? make_ushort4(static_cast<unsigned short>(rect.x), static_cast<unsigned short>(rect.y),
                                           static_cast<unsigned short>(rect.z), static_cast<unsigned short>(rect.w))
                            : make_ushort4(0, 0, 0, 0);
    if (candidate) {
      o.depth_key[i] = __float_as_uint(depth);
      // the blend backward accumulates into these (zero_helpers == 0: the
      // view's own rank clears them locally instead)
      if (zero_helpers) {
        const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
        o.helpers[3 * i] = z;
        o.helpers[3 * i + 1] = z;
        o.helpers[3 * i + 2] = z;
      }
      o.mean2d[i] = m2;
      // view-dependent colour
      float3 col = make_float3(0.5f + 0.28209479177387814f * sh0[3 * i],
                               0.5f + 0.28209479177387814f * sh0[3 * i + 1],
                               0.5f + 0.28209479177387814f * sh0[3 * i + 2]);
      if (active_bases > 1) {
        const float dx = mx3 - cam.pos.x, dy = my3 - cam.pos.y, dz = mz3 - cam.pos.z;
        const float inv = rsqrtf(dx * dx + dy * dy + dz * dz);
        float b[15] = {};
        const int nb = sh_basis(dx * inv, dy * inv, dz * inv, active_bases, b);
        const float* rest = rest_rows + 45 * lane;  // 45 words apart: no bank conflicts
#pragma unroll
        for (int k = 0; k < 15; ++k) {
          if (k < nb) {
            col.x += b[k] * rest[3 * k];
            col.y += b[k] * rest[3 * k + 1];
            col.z += b[k] * rest[3 * k + 2];
          }
        }
      }
      if constexpr (kFp16) {
        PrimInfo16 rec;
        rec.conic_xy = hxy;
        rec.conic_z_opacity = hzw;
        rec.rgb_pad = make_uchar4(static_cast<unsigned char>(sat(col.x) * 255.0f),
                                  static_cast<unsigned char>(sat(col.y) * 255.0f),
                                  static_cast<unsigned char>(sat(col.z) * 255.0f), 0);
        rec.pad = 0;
        o.prim_info[i] = rec;
      } else {
        o.conic_opacity[i] = make_float4(conic.x, conic.y, conic.z, opacity);
        o.color[3 * i] = col.x;
        o.color[3 * i + 1] = col.y;
        o.color[3 * i + 2] = col.z;
      }
    }
  }
  // number of candidates of this block, for the compaction scan
  const uint32_t vis = __syncthreads_count(candidate);
  if (threadIdx.x == 0) o.block_visible[block_slot] = vis;
}

// Loads of Gaussian i (clamped to a valid index) and the start of the
// coalesced copy of its warp's higher-order SH rows into `rows` (one row per
// lane would touch 32 cache lines per load instruction; rows of culled
// Gaussians are copied too).
__device__ __forceinline__ PreIn preprocess_load(const float* __restrict__ means, const float* __restrict__ opacities,
                                                 const float4* __restrict__ rotations,
                                                 const float* __restrict__ scales, const float* __restrict__ sh_rest,
                                                 int active_bases, uint32_t n, uint32_t i, int rest_vec, float* rows,
                                                 uint32_t& gi) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t first = i - lane;
  if (active_bases > 1 && first < n) {
    const uint32_t cnt = min(32u, n - first);
    const float* src = sh_rest + 45 * static_cast<size_t>(first);
    if (rest_vec && cnt == 32u) {
      for (uint32_t e = lane; e < 32u * 45u / 4u; e += 32u) cp_async16(rows + 4 * e, src + 4 * e);
    } else {
      for (uint32_t e = lane; e < cnt * 45u; e += 32u) cp_async4(rows + e, src + e);
    }
  }
  cp_async_commit();
  gi = i < n ? i : (n > 0 ? n - 1 : 0);
  PreIn in;
  in.mx3 = means[3 * gi];
  in.my3 = means[3 * gi + 1];
  in.mz3 = means[3 * gi + 2];
  in.logit = opacities[gi];
  in.s0 = scales[3 * gi];
  in.s1 = scales[3 * gi + 1];
  in.s2 = scales[3 * gi + 2];
  in.q = rotations[gi];
  return in;
}

// Preprocess of Gaussians [first_block * kPreBlock, n) for `count` views:
// one view for a single GPU; every rank's view for the owner split, whose
// records go to each view's arena (peers' arenas over NVLink).  The
// parameters and SH rows are read once for all views; the views are taken
// in `order` (each rank starts with a different one, so the ranks' stores go
// to different GPUs at any moment).  The single-view and the owner-split
// paths run this same kernel, so their records are the same bit for bit.
struct PreViews {
  DevCamera cam[kMaxDpRanks];
  PreOut out[kMaxDpRanks];
  int order[kMaxDpRanks];
  int count;
};

template <int kFp16>
__global__ void __launch_bounds__(kPreBlock)
    k_preprocess_views(const float* __restrict__ means, const float* __restrict__ opacities,
                       const float4* __restrict__ rotations, const float* __restrict__ scales,
                       const float* __restrict__ sh0, const float* __restrict__ sh_rest, int active_bases,
                       uint32_t n, const __grid_constant__ PreViews views, float4* __restrict__ dens, int rest_vec,
                       uint32_t first_block, int zero_helpers) {
  __shared__ __align__(16) float s_rest[kPreBlock / 32][32 * 45];
  const uint32_t i = (first_block + blockIdx.x) * kPreBlock + threadIdx.x;
  float* rows = s_rest[threadIdx.x >> 5];
  uint32_t gi;
  const PreIn in = preprocess_load(means, opacities, rotations, scales, sh_rest, active_bases, n, i, rest_vec, rows, gi);
  for (int j = 0; j < views.count; ++j) {
    const int k = views.order[j];
    preprocess_view<kFp16>(in, i < n, i, gi, views.cam[k], views.out[k], dens, sh0, rows, active_bases,
                           first_block + blockIdx.x, zero_helpers);
  }
}

// --------------------------------------------------------------- backward

// The backward works on one warp's 32 consecutive Gaussians at a time.  The
// 59 parameter floats of those Gaussians are staged in shared memory by
// coalesced asynchronous copies (slice layout per warp, in floats: means 96,
// opacity 32, rotation 128, log-scale 96, sh0 96, sh1..3 1440).  Each lane
// computes its Gaussian's gradients: the 14 geometry and sh0 floats go to a
// shared gradient slice; the 45 higher-band SH gradients are the outer
// product of the 15 basis values and dL/dcolour, so only those 18 floats are
// kept.  The write-out (gradients, or the Adam step) then streams every
// segment with coalesced, 16-byte accesses.
constexpr int kWarpGaussians = 32;
constexpr int kSliceFloats = 59 * kWarpGaussians;  // 1888
constexpr int kGeomFloats = 14 * kWarpGaussians;   // 448: segments 0..4
constexpr int kShStride = 19;                      // 15 basis + 3 dL/dcolour, odd: no bank conflicts
constexpr int kShFloats = kShStride * kWarpGaussians;
constexpr int kWarpFloats = kSliceFloats + kGeomFloats + kShFloats;  // 2944
constexpr int kBwdWarps = 4;
__host__ __device__ constexpr int seg_width(int k) {
  return k == 0 ? 3 : k == 1 ? 1 : k == 2 ? 4 : k == 3 ? 3 : k == 4 ? 3 : 45;
}
__host__ __device__ constexpr int seg_off(int k) {
  return k == 0 ? 0 : k == 1 ? 96 : k == 2 ? 128 : k == 3 ? 256 : k == 4 ? 352 : 448;
}

struct SegPtrs {
  float* p[6];
};

struct AdamArgs {
  float lr[6];
  float decay[6];
  int kind[6];
  float beta1, beta2, eps, gscale, bc1, bc2_sqrt, max_g;
};

struct RouteArgs {
  float* inbox[kMaxDpRanks];
  int64_t lo[kMaxDpRanks + 1];
  int64_t slice_pad;
  int world, rank;
  // warps start at the next rank's slice and end with this rank's own, so the
  // stores crossing NVLink go out first (overlapping the local slice's work)
  // and the ranks begin with different owners
  uint32_t warp_shift;
};

// SH colour backward (fastgs_ours/kernels_backward.cuh:22-86): writes the 45
// higher-band gradients and returns dL/dposition through the view direction.
__device__ __forceinline__ float3 sh_backward_slice(const float* __restrict__ rest, float* __restrict__ sb,
                                                    float3 gc, float3 dir_raw, int active_bases) {
  // sb: 15 basis values (zero past the active band) then dL/dcolour; the
  // gradient of rest[k][c] is sb[k] * sb[15 + c]
  sb[15] = gc.x;
  sb[16] = gc.y;
  sb[17] = gc.z;
  if (active_bases <= 1) {
#pragma unroll
    for (int k = 0; k < 15; ++k) sb[k] = 0.f;
    return make_float3(0.f, 0.f, 0.f);
  }
  const float inv = rsqrtf(dir_raw.x * dir_raw.x + dir_raw.y * dir_raw.y + dir_raw.z * dir_raw.z);
  const float x = dir_raw.x * inv, y = dir_raw.y * inv, z = dir_raw.z * inv;
  float b[15] = {};
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
#pragma unroll
  for (int k = 0; k < 15; ++k) {
    if (k < nb) {
      sb[k] = b[k];
      const float d = rest[3 * k] * gc.x + rest[3 * k + 1] * gc.y + rest[3 * k + 2] * gc.z;
      gd.x += dbx[k] * d;
      gd.y += dby[k] * d;
      gd.z += dbz[k] * d;
    } else {
      sb[k] = 0.f;
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

// All parameter gradients of one Gaussian from its screen-space gradients:
// conic -> 2D covariance -> 3D covariance -> (log-scale, quaternion);
// mean2d (+ frustum clamp mask) -> mean3d; colour -> SH (+ view direction)
// -> mean3d.  Reference: fastgs_ours/kernels_backward.cuh:88-352, including
// its 2D-covariance off-diagonal term without the factor 2 (lines 210-214,
// consistent with its halved dL/dconic.y) and its raw-quaternion gradient
// divided by |q|^3 (lines 328-332).  th / g are the warp's parameter and
// geometry-gradient slices (stride per segment: its width times 32), sb the
// lane's basis / dL/dcolour row.
__device__ __forceinline__ void gaussian_backward(const float* __restrict__ th, float* __restrict__ g,
                                                  float* __restrict__ sb, int lane, const float4 h0,
                                                  const float4 h1, const float4 h2, int active_bases,
                                                  const DevCamera& cam) {
  const float gmx = h0.x, gmy = h0.y;
  const float gca = h1.x, gcb = h1.y, gcc = h1.z;
  const float3 gcol = make_float3(h2.x, h2.y, h2.z);
  const float* tm = th + 3 * lane;
  const float m0 = tm[0], m1 = tm[1], m2 = tm[2];
  const float* tr = th + 128 + 4 * lane;
  const float4 q = make_float4(tr[0], tr[1], tr[2], tr[3]);
  const float* ts = th + 256 + 3 * lane;
  float* g_means = g + 3 * lane;
  float* g_rot = g + 128 + 4 * lane;
  float* g_scales = g + 256 + 3 * lane;
  float* g_sh0 = g + 352 + 3 * lane;
  const float3 dmc = sh_backward_slice(th + 448 + 45 * lane, sb, gcol,
                                       make_float3(m0 - cam.pos.x, m1 - cam.pos.y, m2 - cam.pos.z), active_bases);
  g_sh0[0] = 0.28209479177387814f * gcol.x;
  g_sh0[1] = 0.28209479177387814f * gcol.y;
  g_sh0[2] = 0.28209479177387814f * gcol.z;
  g[96 + lane] = h1.w;  // opacity: already times (1 - opacity)

  const float depth = cam.r3.x * m0 + cam.r3.y * m1 + cam.r3.z * m2 + cam.r3.w;
  const float x = (cam.r1.x * m0 + cam.r1.y * m1 + cam.r1.z * m2 + cam.r1.w) / depth;
  const float y = (cam.r2.x * m0 + cam.r2.y * m1 + cam.r2.z * m2 + cam.r2.w) / depth;
  const float e0 = __expf(ts[0]), e1 = __expf(ts[1]), e2 = __expf(ts[2]);
  const float var[3] = {e0 * e0, e1 * e1, e2 * e2};
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
  g_means[0] = (cam.r1.x * dc0 + cam.r2.x * dc1 + cam.r3.x * dc2) + dmc.x;
  g_means[1] = (cam.r1.y * dc0 + cam.r2.y * dc1 + cam.r3.y * dc2) + dmc.y;
  g_means[2] = (cam.r1.z * dc0 + cam.r2.z * dc1 + cam.r3.z * dc2) + dmc.z;
  const float es[3] = {e0, e1, e2};
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const float dv = R.r[0][k] * R.r[0][k] * d3[0] + R.r[1][k] * R.r[1][k] * d3[3] +
                     R.r[2][k] * R.r[2][k] * d3[5] +
                     2.0f * (R.r[0][k] * R.r[1][k] * d3[1] + R.r[0][k] * R.r[2][k] * d3[2] +
                             R.r[1][k] * R.r[2][k] * d3[4]);
    g_scales[k] = 2.0f * es[k] * es[k] * dv;
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
  g_rot[0] = 2.0f * (q.y * dqrx + q.z * dqry + q.w * dqrz - q.x * hn) / den;
  g_rot[1] = 2.0f * (2.0f * q.y * dqxx + q.z * dqxy + q.w * dqxz + q.x * dqrx - q.y * hn) / den;
  g_rot[2] = 2.0f * (2.0f * q.z * dqyy + q.y * dqxy + q.w * dqyz + q.x * dqry - q.z * hn) / den;
  g_rot[3] = 2.0f * (2.0f * q.w * dqzz + q.y * dqxz + q.z * dqyz + q.x * dqrz - q.w * hn) / den;
}

__device__ __forceinline__ float lerp_adam(float v0, float v1, float t) {
  // fma form of v0 + t (v1 - v0), simple_adam.cu:24-26
  return fmaf(t, v1, fmaf(-t, v0, v0));
}

// Adam update of one element (simple_adam.cu:105-152).
__device__ __forceinline__ void adam_element(float& th, float g_raw, float& m, float& v, float lr, int kind,
                                             float decay, const AdamArgs& a) {
  float g = a.gscale * g_raw;
  if (kind == 1) {
    const float sg = 1.0f / (1.0f + __expf(-th));
    g = g + decay * (sg * (1.0f - sg));
  } else if (kind == 2) {
    g = g + decay * __expf(th);
  }
  if (a.max_g != 0.0f) g = copysignf(fminf(fabsf(g), a.max_g), g);
  m = lerp_adam(m, g, 1.0f - a.beta1);
  v = lerp_adam(v, g * g, 1.0f - a.beta2);
  const float mh = m / a.bc1;
  const float den = sqrtf(v) / a.bc2_sqrt + a.eps;
  th -= mh * lr / den;
}

// Copy the warp's slice of six segments (rows of `cnt` Gaussians) into
// shared memory.  Full slices of 16-byte aligned segments move in 16-byte
// chunks; anything else in 4-byte ones.
__device__ __forceinline__ void stage_slice(const SegPtrs& src, float* dst, uint32_t first, uint32_t cnt,
                                            uint32_t lane, bool vec) {
#pragma unroll
  for (int k = 0; k < 6; ++k) {
    const int w = seg_width(k);
    const float* s = src.p[k] + static_cast<size_t>(first) * w;
    float* d = dst + seg_off(k);
    const uint32_t count = cnt * w;
    if (vec) {
      for (uint32_t e = 4 * lane; e < count; e += 128) cp_async16(d + e, s + e);
    } else {
      for (uint32_t e = lane; e < count; e += 32) cp_async4(d + e, s + e);
    }
  }
}

// Gradient of element e of segment k of the warp slice.
template <int k>
__device__ __forceinline__ float slice_grad(const float* __restrict__ g, const float* __restrict__ sb, uint32_t e) {
  if constexpr (k < 5) {
    return g[seg_off(k) + e];
  } else {
    const uint32_t gl = e / 45u, r = e - 45u * gl, band = r / 3u, c = r - 3u * band;
    return sb[gl * kShStride + band] * sb[gl * kShStride + 15 + c];
  }
}

// Write-out of segment k: gradients (=, or += when accumulate) or, when
// kAdam, the Adam step on (params, exp_avg, exp_avg_sq) plus the optional
// gradient store.
// Owner of Gaussian gi under gradient routing: the last rank whose slice
// starts at or before it (empty slices are skipped that way).
__device__ __forceinline__ int route_owner(const RouteArgs& r, int64_t gi) {
  int s = r.world - 1;
  while (s > 0 && r.lo[s] > gi) --s;
  return s;
}

// Destination of gradient element `elem` (index within segment k, i.e.
// Gaussian * width + component) under gradient routing: slot `rank` of the
// inbox of the rank whose slice holds the Gaussian.
template <int k>
__device__ __forceinline__ float* routed_dst(const RouteArgs& r, int64_t elem) {
  constexpr int w = seg_width(k);
  const int s = route_owner(r, elem / w);
  int64_t seg_base = 0;
#pragma unroll
  for (int j = 0; j < k; ++j) seg_base += seg_width(j) * r.slice_pad;
  return r.inbox[s] + r.rank * 59 * r.slice_pad + seg_base + (elem - r.lo[s] * w);
}

// Routed write-out of a full, 16-byte aligned warp slice through the bulk
// copy engine: segments 0..4 of the gradients already sit in shared memory
// in the arenas' layout (g), segment 5 (the rank-1 SH gradient) is written
// out into the no longer needed parameter staging area, then one lane hands
// every (segment, owner) piece to cp.async.bulk, so the warp does not wait on
// the stores crossing NVLink.  Pieces start and end on multiples of four
// Gaussians (warp slices start on multiples of 32, owner slices on multiples
// of four), so every address and size is a multiple of 16 bytes.
__device__ __forceinline__ void route_warp_bulk(const RouteArgs& r, float* th, const float* g, const float* sb,
                                                uint32_t first, uint32_t lane) {
  for (uint32_t e = lane; e < 45u * kWarpGaussians; e += 32) th[seg_off(5) + e] = slice_grad<5>(g, sb, e);
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
  __syncwarp();
  if (lane == 0) {
    int64_t g0 = first;
    const int64_t end = static_cast<int64_t>(first) + kWarpGaussians;
    while (g0 < end) {
      const int s = route_owner(r, g0);
      const int64_t g1 = min(end, r.lo[s + 1]);
      float* slot = r.inbox[s] + static_cast<int64_t>(r.rank) * 59 * r.slice_pad;
      int64_t seg_base = 0;
#pragma unroll
      for (int k = 0; k < 6; ++k) {
        const int w = seg_width(k);
        const float* src = (k < 5 ? g : th) + seg_off(k) + (g0 - first) * w;
        float* dst = slot + seg_base + (g0 - r.lo[s]) * w;
        const uint32_t bytes = static_cast<uint32_t>((g1 - g0) * w * 4);
        const uint32_t saddr = static_cast<uint32_t>(__cvta_generic_to_shared(src));
        asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(dst), "r"(saddr),
                     "r"(bytes)
                     : "memory");
        seg_base += w * r.slice_pad;
      }
      g0 = g1;
    }
    asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
    // the shared-memory sources are read before the warp's slot is freed
    asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");
  }
  __syncwarp();
}

// Adam write-out of a full, 16-byte aligned warp slice with the moment
// loads grouped, so that a warp waits on L2 about three times per slice
// instead of once per segment and batch.  Segments 0..4 are 112 16-byte
// chunks whose staged values (theta, gradients) sit back to back in shared
// memory (chunk c at float 4c), taken in four rounds of 32 chunks; each round
// spans at most two segments (kLo, kHi).  Segment 5 (sh_rest) is 360 chunks,
// taken in batches of four per lane with the next batch's moments loaded
// before the current batch is computed.
__host__ __device__ constexpr uint32_t seg_chunk0(int k) { return static_cast<uint32_t>(seg_off(k)) / 4u; }

struct ChunkRef {
  float* p;
  float* m;
  float* v;
  float* g;
  float lr, decay;
  int kind;
};

template <int kLo, int kHi>
__device__ __forceinline__ ChunkRef chunk_ref(const SegPtrs& params, const SegPtrs& grads, const SegPtrs& exp_avg,
                                              const SegPtrs& exp_avg_sq, const AdamArgs& adam, uint32_t first,
                                              uint32_t c) {
  const bool hi = kLo != kHi && c >= seg_chunk0(kHi);
  const size_t lo_off = static_cast<size_t>(first) * seg_width(kLo) + 4u * (c - seg_chunk0(kLo));
  const size_t hi_off = static_cast<size_t>(first) * seg_width(kHi) + 4u * (c - seg_chunk0(kHi));
  ChunkRef r;
  r.p = hi ? params.p[kHi] + hi_off : params.p[kLo] + lo_off;
  r.m = hi ? exp_avg.p[kHi] + hi_off : exp_avg.p[kLo] + lo_off;
  r.v = hi ? exp_avg_sq.p[kHi] + hi_off : exp_avg_sq.p[kLo] + lo_off;
  float* glo = grads.p[kLo];
  float* ghi = grads.p[kHi];
  r.g = hi ? (ghi != nullptr ? ghi + hi_off : nullptr) : (glo != nullptr ? glo + lo_off : nullptr);
  r.lr = hi ? adam.lr[kHi] : adam.lr[kLo];
  r.decay = hi ? adam.decay[kHi] : adam.decay[kLo];
  r.kind = hi ? adam.kind[kHi] : adam.kind[kLo];
  return r;
}

__device__ __forceinline__ void adam_chunk(const ChunkRef& r, float4 t, float4 m, float4 v, float4 gv,
                                           const AdamArgs& adam) {
  adam_element(t.x, gv.x, m.x, v.x, r.lr, r.kind, r.decay, adam);
  adam_element(t.y, gv.y, m.y, v.y, r.lr, r.kind, r.decay, adam);
  adam_element(t.z, gv.z, m.z, v.z, r.lr, r.kind, r.decay, adam);
  adam_element(t.w, gv.w, m.w, v.w, r.lr, r.kind, r.decay, adam);
  *reinterpret_cast<float4*>(r.p) = t;
  *reinterpret_cast<float4*>(r.m) = m;
  *reinterpret_cast<float4*>(r.v) = v;
  if (r.g != nullptr) *reinterpret_cast<float4*>(r.g) = gv;
}

template <int kLo, int kHi>
__device__ __forceinline__ void geom_round(const SegPtrs& params, const SegPtrs& grads, const SegPtrs& exp_avg,
                                           const SegPtrs& exp_avg_sq, const AdamArgs& adam, const float* th,
                                           const float* g, uint32_t first, uint32_t c, float4 m, float4 v) {
  if (c >= seg_chunk0(5)) return;
  const ChunkRef r = chunk_ref<kLo, kHi>(params, grads, exp_avg, exp_avg_sq, adam, first, c);
  adam_chunk(r, reinterpret_cast<const float4*>(th)[c], m, v, reinterpret_cast<const float4*>(g)[c], adam);
}

__device__ __forceinline__ float4 rest_grad4(const float* sb, uint32_t e4) {
  return make_float4(slice_grad<5>(nullptr, sb, 4 * e4), slice_grad<5>(nullptr, sb, 4 * e4 + 1),
                     slice_grad<5>(nullptr, sb, 4 * e4 + 2), slice_grad<5>(nullptr, sb, 4 * e4 + 3));
}

// kSum: the higher-band SH gradients are read from `sb` as a plain slice
// segment (the multi-view sum) instead of being formed from basis x colour.
template <bool kSum = false>
__device__ __forceinline__ void adam_slice_v16(const SegPtrs& params, const SegPtrs& grads, const SegPtrs& exp_avg,
                                               const SegPtrs& exp_avg_sq, const AdamArgs& adam, const float* th,
                                               const float* g, const float* sb, uint32_t first, uint32_t lane) {
  constexpr uint32_t kRestChunks = 45u * kWarpGaussians / 4u;  // 360
  constexpr int kBatch = 4;
  constexpr uint32_t kRestRounds = (kRestChunks + 31u) / 32u;  // 12 (the last one: lanes < 8)
  const size_t rest_base = static_cast<size_t>(first) * 45u;
  const float* RM = exp_avg.p[5] + rest_base;
  const float* RV = exp_avg_sq.p[5] + rest_base;
  // moments of segments 0..4 and of the first sh_rest batch
  float4 gm[4], gvv[4], rm[kBatch], rv[kBatch];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t c = 32u * j + lane;
    if (c < seg_chunk0(5)) {
      const ChunkRef r = j == 0   ? chunk_ref<0, 1>(params, grads, exp_avg, exp_avg_sq, adam, first, c)
                         : j == 1 ? chunk_ref<2, 2>(params, grads, exp_avg, exp_avg_sq, adam, first, c)
                         : j == 2 ? chunk_ref<3, 4>(params, grads, exp_avg, exp_avg_sq, adam, first, c)
                                  : chunk_ref<4, 4>(params, grads, exp_avg, exp_avg_sq, adam, first, c);
      gm[j] = *reinterpret_cast<const float4*>(r.m);
      gvv[j] = *reinterpret_cast<const float4*>(r.v);
    }
  }
#pragma unroll
  for (int q = 0; q < kBatch; ++q) {
    const uint32_t e4 = 32u * q + lane;
    rm[q] = reinterpret_cast<const float4*>(RM)[e4];
    rv[q] = reinterpret_cast<const float4*>(RV)[e4];
  }
  geom_round<0, 1>(params, grads, exp_avg, exp_avg_sq, adam, th, g, first, lane, gm[0], gvv[0]);
  geom_round<2, 2>(params, grads, exp_avg, exp_avg_sq, adam, th, g, first, 32u + lane, gm[1], gvv[1]);
  geom_round<3, 4>(params, grads, exp_avg, exp_avg_sq, adam, th, g, first, 64u + lane, gm[2], gvv[2]);
  geom_round<4, 4>(params, grads, exp_avg, exp_avg_sq, adam, th, g, first, 96u + lane, gm[3], gvv[3]);
  // sh_rest
  ChunkRef rr;
  rr.lr = adam.lr[5];
  rr.decay = adam.decay[5];
  rr.kind = adam.kind[5];
  const float* ts = th + seg_off(5);
#pragma unroll
  for (uint32_t b0 = 0; b0 < kRestRounds; b0 += kBatch) {
    float4 nm[kBatch], nv[kBatch];
    if (b0 + kBatch < kRestRounds) {
#pragma unroll
      for (int q = 0; q < kBatch; ++q) {
        const uint32_t e4 = 32u * (b0 + kBatch + q) + lane;
        if (e4 < kRestChunks) {
          nm[q] = reinterpret_cast<const float4*>(RM)[e4];
          nv[q] = reinterpret_cast<const float4*>(RV)[e4];
        }
      }
    }
#pragma unroll
    for (int q = 0; q < kBatch; ++q) {
      const uint32_t e4 = 32u * (b0 + q) + lane;
      if (e4 < kRestChunks) {
        rr.p = params.p[5] + rest_base + 4u * e4;
        rr.m = exp_avg.p[5] + rest_base + 4u * e4;
        rr.v = exp_avg_sq.p[5] + rest_base + 4u * e4;
        rr.g = grads.p[5] != nullptr ? grads.p[5] + rest_base + 4u * e4 : nullptr;
        adam_chunk(rr, reinterpret_cast<const float4*>(ts)[e4], rm[q], rv[q],
                   kSum ? reinterpret_cast<const float4*>(sb)[e4] : rest_grad4(sb, e4), adam);
      }
    }
    if (b0 + kBatch < kRestRounds) {
#pragma unroll
      for (int q = 0; q < kBatch; ++q) {
        rm[q] = nm[q];
        rv[q] = nv[q];
      }
    }
  }
}

// Gradient element e of segment k: kSum reads the higher-band SH gradients
// from `sb` as a plain segment (the multi-view sum).
template <int k, bool kSum>
__device__ __forceinline__ float grad_of(const float* __restrict__ g, const float* __restrict__ sb, uint32_t e) {
  if constexpr (kSum && k == 5) {
    return sb[e];
  } else {
    return slice_grad<k>(g, sb, e);
  }
}

template <bool kAdam, int k, bool kRoute = false, bool kSum = false>
__device__ __forceinline__ void write_segment(const SegPtrs& params, const SegPtrs& grads, const SegPtrs& exp_avg,
                                              const SegPtrs& exp_avg_sq, const AdamArgs& adam, int accumulate,
                                              const float* __restrict__ th, const float* __restrict__ g,
                                              const float* __restrict__ sb, uint32_t first, uint32_t cnt,
                                              uint32_t lane, bool v16, const RouteArgs& route) {
  constexpr int w = seg_width(k);
  const size_t base = static_cast<size_t>(first) * w;
  const uint32_t count = cnt * w;
  if constexpr (kRoute) {
    // overwrite into the owners' inboxes; a slice boundary is a multiple of
    // four Gaussians, so no 16-byte chunk straddles two owners
    if (v16) {
      for (uint32_t e4 = lane; e4 < count / 4; e4 += 32) {
        const float4 gv = make_float4(slice_grad<k>(g, sb, 4 * e4), slice_grad<k>(g, sb, 4 * e4 + 1),
                                      slice_grad<k>(g, sb, 4 * e4 + 2), slice_grad<k>(g, sb, 4 * e4 + 3));
        *reinterpret_cast<float4*>(routed_dst<k>(route, static_cast<int64_t>(base) + 4 * e4)) = gv;
      }
    } else {
      for (uint32_t e = lane; e < count; e += 32)
        *routed_dst<k>(route, static_cast<int64_t>(base) + e) = slice_grad<k>(g, sb, e);
    }
    return;
  }
  float* G = grads.p[k] != nullptr ? grads.p[k] + base : nullptr;
  if constexpr (kAdam) {
    const float* ts = th + seg_off(k);
    float* P = params.p[k] + base;
    float* M = exp_avg.p[k] + base;
    float* V = exp_avg_sq.p[k] + base;
    const float lr = adam.lr[k], decay = adam.decay[k];
    const int kind = adam.kind[k];
    if (v16) {
#pragma unroll 4
      for (uint32_t e4 = lane; e4 < count / 4; e4 += 32) {
        float4 t = reinterpret_cast<const float4*>(ts)[e4];
        float4 m = reinterpret_cast<const float4*>(M)[e4];
        float4 v = reinterpret_cast<const float4*>(V)[e4];
        const float4 gv = make_float4(grad_of<k, kSum>(g, sb, 4 * e4), grad_of<k, kSum>(g, sb, 4 * e4 + 1),
                                      grad_of<k, kSum>(g, sb, 4 * e4 + 2), grad_of<k, kSum>(g, sb, 4 * e4 + 3));
        adam_element(t.x, gv.x, m.x, v.x, lr, kind, decay, adam);
        adam_element(t.y, gv.y, m.y, v.y, lr, kind, decay, adam);
        adam_element(t.z, gv.z, m.z, v.z, lr, kind, decay, adam);
        adam_element(t.w, gv.w, m.w, v.w, lr, kind, decay, adam);
        reinterpret_cast<float4*>(P)[e4] = t;
        reinterpret_cast<float4*>(M)[e4] = m;
        reinterpret_cast<float4*>(V)[e4] = v;
        if (G != nullptr) reinterpret_cast<float4*>(G)[e4] = gv;
      }
    } else {
      for (uint32_t e = lane; e < count; e += 32) {
        float t = ts[e], m = M[e], v = V[e];
        const float gv = grad_of<k, kSum>(g, sb, e);
        adam_element(t, gv, m, v, lr, kind, decay, adam);
        P[e] = t;
        M[e] = m;
        V[e] = v;
        if (G != nullptr) G[e] = gv;
      }
    }
  } else {
    if (v16) {
      for (uint32_t e4 = lane; e4 < count / 4; e4 += 32) {
        float4 gv = make_float4(slice_grad<k>(g, sb, 4 * e4), slice_grad<k>(g, sb, 4 * e4 + 1),
                                slice_grad<k>(g, sb, 4 * e4 + 2), slice_grad<k>(g, sb, 4 * e4 + 3));
        if (accumulate) {
          // untouched Gaussians keep their gradient (+= 0)
          const float4 o = reinterpret_cast<const float4*>(G)[e4];
          gv = make_float4(o.x + gv.x, o.y + gv.y, o.z + gv.z, o.w + gv.w);
        }
        reinterpret_cast<float4*>(G)[e4] = gv;
      }
    } else {
      for (uint32_t e = lane; e < count; e += 32) {
        const float gv = slice_grad<k>(g, sb, e);
        G[e] = accumulate ? G[e] + gv : gv;
      }
    }
  }
}

// kAdam == false: gradients written (or added, accumulate) to `grads`.
// kAdam == true: the Adam step is applied to params / exp_avg / exp_avg_sq
// directly from the shared-memory gradients (the gradient arena is written
// only if `grads` is given), which is tgs_raster_backward(accumulate = 0)
// followed by tgs_adam_step without the gradient round trip through HBM.
// The moments of the warp's Gaussians are prefetched into L2 (bulk
// prefetch) at the start, so their reads in the write-out hit L2.
template <bool kAdam, bool kRoute = false>
__global__ void __launch_bounds__(32 * kBwdWarps, 4)
    k_preprocess_backward(SegPtrs params, SegPtrs grads, SegPtrs exp_avg, SegPtrs exp_avg_sq, AdamArgs adam,
                          int accumulate, int vec, int active_bases, uint32_t n, DevCamera cam,
                          const uint32_t* __restrict__ n_touched, const float4* __restrict__ helpers,
                          float4* __restrict__ dens, const DevCounts* __restrict__ counts, RouteArgs route,
                          uint32_t base) {
  __shared__ __align__(16) float smem[kBwdWarps * kWarpFloats];
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  uint32_t wi = blockIdx.x * kBwdWarps + warp;
  // Gaussians [base, n): base is a multiple of 32
  const uint32_t n_warps = (n - base + kWarpGaussians - 1) / kWarpGaussians;
  if (wi >= n_warps) return;
  if constexpr (kRoute) {
    wi += route.warp_shift;
    if (wi >= n_warps) wi -= n_warps;
  }
  const uint32_t first = base + wi * kWarpGaussians;
  const uint32_t cnt = min(static_cast<uint32_t>(kWarpGaussians), n - first);
  const bool v16 = vec != 0 && cnt == kWarpGaussians;
  float* th = smem + warp * kWarpFloats;
  float* g = th + kSliceFloats;
  float* sb = g + kGeomFloats;
  if constexpr (kAdam) {
    if (v16) {
#pragma unroll
      for (int k = 0; k < 6; ++k) {
        if (lane == static_cast<uint32_t>(k) || lane == static_cast<uint32_t>(k + 6)) {
          const float* ptr = (lane < 6u ? exp_avg.p[k] : exp_avg_sq.p[k]) + static_cast<size_t>(first) * seg_width(k);
          const uint32_t bytes = 4u * kWarpGaussians * seg_width(k);
          asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(ptr), "r"(bytes) : "memory");
        }
      }
    }
  }
  stage_slice(params, th, first, cnt, lane, v16);
  cp_async_commit();
  // the per-Gaussian loads go out together with the staging copies (the
  // screen-space gradients of an untouched Gaussian are loaded and unused)
  const uint32_t i = first + lane;
  const bool ok = counts->overflow == 0u;
  uint32_t nt = 0;
  float4 h0{}, h1{}, h2{}, d{};
  if (lane < cnt) {
    nt = n_touched[i];
    h0 = helpers[3 * i];
    h1 = helpers[3 * i + 1];
    h2 = helpers[3 * i + 2];
    if (dens != nullptr) d = dens[i];
  }
  cp_async_wait<0>();
  __syncwarp();
  const bool touched = ok && lane < cnt && nt > 0;
  float* my_sb = sb + kShStride * lane;
  if (touched) {
    gaussian_backward(th, g, my_sb, lane, h0, h1, h2, active_bases, cam);
    if (dens != nullptr) {
      d.x += 1.0f;
      const float ux = h0.x * (0.5f * cam.w), uy = h0.y * (0.5f * cam.h);
      d.y += sqrtf(ux * ux + uy * uy);
      const float vx = h0.z * (0.5f * cam.w), vy = h0.w * (0.5f * cam.h);
      d.z += sqrtf(vx * vx + vy * vy);
      dens[i] = d;
    }
  } else {
#pragma unroll
    for (int k = 0; k < 5; ++k) {
#pragma unroll
      for (int c = 0; c < seg_width(k); ++c) g[seg_off(k) + seg_width(k) * lane + c] = 0.f;
    }
#pragma unroll
    for (int c = 0; c < 18; ++c) my_sb[c] = 0.f;
  }
  __syncwarp();
  if (kRoute && v16) {
    route_warp_bulk(route, th, g, sb, first, lane);
  } else if (kAdam && v16) {
    adam_slice_v16(params, grads, exp_avg, exp_avg_sq, adam, th, g, sb, first, lane);
  } else {
    write_segment<kAdam, 0, kRoute>(params, grads, exp_avg, exp_avg_sq, adam, accumulate, th, g, sb, first, cnt,
                                      lane, v16, route);
    write_segment<kAdam, 1, kRoute>(params, grads, exp_avg, exp_avg_sq, adam, accumulate, th, g, sb, first, cnt,
                                      lane, v16, route);
    write_segment<kAdam, 2, kRoute>(params, grads, exp_avg, exp_avg_sq, adam, accumulate, th, g, sb, first, cnt,
                                      lane, v16, route);
    write_segment<kAdam, 3, kRoute>(params, grads, exp_avg, exp_avg_sq, adam, accumulate, th, g, sb, first, cnt,
                                      lane, v16, route);
    write_segment<kAdam, 4, kRoute>(params, grads, exp_avg, exp_avg_sq, adam, accumulate, th, g, sb, first, cnt,
                                      lane, v16, route);
    write_segment<kAdam, 5, kRoute>(params, grads, exp_avg, exp_avg_sq, adam, accumulate, th, g, sb, first, cnt,
                                      lane, v16, route);
  }
  // (routed stores: the kernel's completion orders them before the
  // collective that the owners wait on; no per-warp system fence, which
  // would hold every warp until its stores crossed NVLink)
}

// Owner-split backward: one rank's slice of Gaussians, the per-Gaussian
// backward of every rank's view, summed in view order, then Adam.
struct ViewsArgs {
  DevCamera cam[kMaxDpRanks];
  const uint32_t* n_touched[kMaxDpRanks];
  const float4* helpers[kMaxDpRanks];
  const DevCounts* counts[kMaxDpRanks];
  int world;
};
// per warp: the slice staging, one view's gradients, and the running sum of
// the 45 higher-band SH gradients of its 32 Gaussians (the 14 others are
// summed in registers, one Gaussian per lane)
constexpr int kViewsWarpFloats = kWarpFloats + 45 * kWarpGaussians;  // 4384
constexpr size_t kViewsSmemBytes = sizeof(float) * kViewsWarpFloats * kBwdWarps;

// Position of geometry gradient j (0..13: means 3, opacity, rotation 4,
// scales 3, sh0 3) of `lane`'s Gaussian in the warp's gradient slice.
__device__ __forceinline__ uint32_t geom_pos(int j, uint32_t lane) {
  return j < 3 ? seg_off(0) + 3u * lane + j
       : j < 4 ? seg_off(1) + lane
       : j < 8 ? seg_off(2) + 4u * lane + (j - 4)
       : j < 11 ? seg_off(3) + 3u * lane + (j - 8)
                : seg_off(4) + 3u * lane + (j - 11);
}

// The sum runs as acc = g_0, acc = acc + g_1, ..., the order in which
// tgs_raster_backward(accumulate) over the views in turn would add the
// gradients into one arena, so the Adam step sees the same sums; the
// screen-space inputs of view k + 1 (peer memory in a multi-GPU run) are
// loaded while view k is computed.
__global__ void __launch_bounds__(32 * kBwdWarps, 3)
    k_views_backward_adam(SegPtrs params, SegPtrs grads, SegPtrs exp_avg, SegPtrs exp_avg_sq, AdamArgs adam,
                          int vec, int active_bases, uint32_t n, uint32_t base, float4* __restrict__ dens,
                          ViewsArgs views) {
  extern __shared__ __align__(16) float vsmem[];
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  const uint32_t wi = blockIdx.x * kBwdWarps + warp;
  const uint32_t n_warps = (n - base + kWarpGaussians - 1) / kWarpGaussians;
  if (wi >= n_warps) return;
  const uint32_t first = base + wi * kWarpGaussians;
  const uint32_t cnt = min(static_cast<uint32_t>(kWarpGaussians), n - first);
  const bool v16 = vec != 0 && cnt == kWarpGaussians;
  float* th = vsmem + warp * kViewsWarpFloats;
  float* g = th + kSliceFloats;
  float* sb = g + kGeomFloats;
  float* rest_sum = sb + kShFloats;
  if (v16) {
#pragma unroll
    for (int k = 0; k < 6; ++k) {
      if (lane == static_cast<uint32_t>(k) || lane == static_cast<uint32_t>(k + 6)) {
        const float* ptr = (lane < 6u ? exp_avg.p[k] : exp_avg_sq.p[k]) + static_cast<size_t>(first) * seg_width(k);
        const uint32_t bytes = 4u * kWarpGaussians * seg_width(k);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(ptr), "r"(bytes) : "memory");
      }
    }
  }
  stage_slice(params, th, first, cnt, lane, v16);
  cp_async_commit();
  const uint32_t i = first + lane;
  const bool live = lane < cnt;
  uint32_t nt = 0;
  float4 h0{}, h1{}, h2{}, d{};
  if (live) {
    nt = views.n_touched[0][i];
    h0 = views.helpers[0][3 * i];
    h1 = views.helpers[0][3 * i + 1];
    h2 = views.helpers[0][3 * i + 2];
    if (dens != nullptr) d = dens[i];
  }
  cp_async_wait<0>();
  __syncwarp();
  float* my_sb = sb + kShStride * lane;
  float acc[14];
  bool any_touched = false;
  for (int k = 0; k < views.world; ++k) {
    uint32_t nt_next = 0;
    float4 n0{}, n1{}, n2{};
    if (k + 1 < views.world && live) {
      nt_next = views.n_touched[k + 1][i];
      n0 = views.helpers[k + 1][3 * i];
      n1 = views.helpers[k + 1][3 * i + 1];
      n2 = views.helpers[k + 1][3 * i + 2];
    }
    const bool touched = views.counts[k]->overflow == 0u && live && nt > 0;
    if (touched) {
      const DevCamera& cam = views.cam[k];
      gaussian_backward(th, g, my_sb, lane, h0, h1, h2, active_bases, cam);
      if (dens != nullptr) {
        d.x += 1.0f;
        const float ux = h0.x * (0.5f * cam.w), uy = h0.y * (0.5f * cam.h);
        d.y += sqrtf(ux * ux + uy * uy);
        const float vx = h0.z * (0.5f * cam.w), vy = h0.w * (0.5f * cam.h);
        d.z += sqrtf(vx * vx + vy * vy);
      }
      any_touched = true;
    } else {
#pragma unroll
      for (int j = 0; j < 14; ++j) g[geom_pos(j, lane)] = 0.f;
#pragma unroll
      for (int c = 0; c < 18; ++c) my_sb[c] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < 14; ++j) {
      const float x = g[geom_pos(j, lane)];
      acc[j] = k == 0 ? x : acc[j] + x;
    }
    __syncwarp();  // every lane's basis and colour gradients are in place
    for (uint32_t e = lane; e < 45u * kWarpGaussians; e += 32) {
      const float x = slice_grad<5>(g, sb, e);
      rest_sum[e] = k == 0 ? x : rest_sum[e] + x;
    }
    __syncwarp();  // sb is rewritten by the next view
    nt = nt_next;
    h0 = n0;
    h1 = n1;
    h2 = n2;
  }
#pragma unroll
  for (int j = 0; j < 14; ++j) g[geom_pos(j, lane)] = acc[j];
  if (dens != nullptr && any_touched) dens[i] = d;
  __syncwarp();
  if (v16) {
    adam_slice_v16<true>(params, grads, exp_avg, exp_avg_sq, adam, th, g, rest_sum, first, lane);
  } else {
    write_segment<true, 0, false, true>(params, grads, exp_avg, exp_avg_sq, adam, 0, th, g, rest_sum, first, cnt,
                                        lane, false, RouteArgs{});
    write_segment<true, 1, false, true>(params, grads, exp_avg, exp_avg_sq, adam, 0, th, g, rest_sum, first, cnt,
                                        lane, false, RouteArgs{});
    write_segment<true, 2, false, true>(params, grads, exp_avg, exp_avg_sq, adam, 0, th, g, rest_sum, first, cnt,
                                        lane, false, RouteArgs{});
    write_segment<true, 3, false, true>(params, grads, exp_avg, exp_avg_sq, adam, 0, th, g, rest_sum, first, cnt,
                                        lane, false, RouteArgs{});
    write_segment<true, 4, false, true>(params, grads, exp_avg, exp_avg_sq, adam, 0, th, g, rest_sum, first, cnt,
                                        lane, false, RouteArgs{});
    write_segment<true, 5, false, true>(params, grads, exp_avg, exp_avg_sq, adam, 0, th, g, rest_sum, first, cnt,
                                        lane, false, RouteArgs{});
  }
}

PreOut pre_out(const RasterState& s) {
  return PreOut{s.n_touched, s.depth_key, s.bounds, s.mean2d, s.conic_opacity, s.prim_info, s.color,
                reinterpret_cast<float4*>(s.helpers), s.block_sums};
}

}  // namespace

void launch_preprocess(const RasterState& s, const GaussianPtrs& g, const DevCamera& cam, int fp16,
                       float4* dens, cudaStream_t stream, int64_t first, int64_t last, int zero_helpers) {
  // Gaussians [first, last) (last < 0: to g.n); first is a multiple of the
  // block size so every block's candidate count has one writer
  const int order = 0;
  launch_preprocess_views(&s, &cam, &order, 1, g, fp16, dens, stream, first, last < 0 ? g.n : last, zero_helpers);
}

void launch_preprocess_views(const RasterState* views, const DevCamera* cams, const int* order, int count,
                             const GaussianPtrs& g, int fp16, float4* dens, cudaStream_t stream, int64_t first,
                             int64_t last, int zero_helpers) {
  const uint32_t n = static_cast<uint32_t>(last);
  const uint32_t first_block = static_cast<uint32_t>(first / kPreBlock);
  const int active_bases = (g.sh_degree + 1) * (g.sh_degree + 1);
  const uint32_t blocks = n > first_block * kPreBlock ? (n - first_block * kPreBlock + kPreBlock - 1) / kPreBlock : 0;
  if (blocks == 0 || count <= 0) return;
  const int rest_vec = (reinterpret_cast<uintptr_t>(g.sh_rest) & 15u) == 0;
  PreViews v{};
  v.count = count;
  for (int k = 0; k < count; ++k) {
    v.cam[k] = cams[k];
    v.out[k] = pre_out(views[k]);
    v.order[k] = order[k];
  }
  if (fp16)
    k_preprocess_views<1><<<blocks, kPreBlock, 0, stream>>>(
        g.means, g.opacities, reinterpret_cast<const float4*>(g.rotations), g.scales, g.sh0, g.sh_rest,
        active_bases, n, v, dens, rest_vec, first_block, zero_helpers);
  else
    k_preprocess_views<0><<<blocks, kPreBlock, 0, stream>>>(
        g.means, g.opacities, reinterpret_cast<const float4*>(g.rotations), g.scales, g.sh0, g.sh_rest,
        active_bases, n, v, dens, rest_vec, first_block, zero_helpers);
}

void launch_preprocess_backward(const RasterState& s, const GaussianPtrs& g, const GaussianPtrs& grads,
                                const DevCamera& cam, int accumulate, float4* dens, cudaStream_t stream,
                                const GaussianPtrs* exp_avg, const GaussianPtrs* exp_avg_sq,
                                const AdamStepArgs* adam, const GradRoute* route, int64_t first, int64_t last) {
  // Gaussians [first, last) (last < 0: to g.n); first is a multiple of 32
  const uint32_t n = static_cast<uint32_t>(last < 0 ? g.n : last);
  const uint32_t base = static_cast<uint32_t>(first);
  if (n <= base) return;
  const int active_bases = (g.sh_degree + 1) * (g.sh_degree + 1);
  const uint32_t per_block = kBwdWarps * kWarpGaussians;
  const uint32_t blocks = (n - base + per_block - 1) / per_block;
  auto segs = [](const GaussianPtrs& x) {
    SegPtrs p{{x.means, x.opacities, x.rotations, x.scales, x.sh0, x.sh_rest}};
    return p;
  };
  auto aligned = [](const SegPtrs& p) {
    for (float* q : p.p)
      if (q != nullptr && (reinterpret_cast<uintptr_t>(q) & 15u) != 0) return false;
    return true;
  };
  AdamArgs a{};
  SegPtrs m{}, v{};
  if (adam != nullptr) {
    for (int k = 0; k < 6; ++k) {
      a.lr[k] = adam->lr[k];
      a.decay[k] = adam->decay[k];
      a.kind[k] = adam->kind[k];
    }
    a.beta1 = adam->beta1;
    a.beta2 = adam->beta2;
    a.eps = adam->eps;
    a.gscale = adam->gradient_scale;
    a.bc1 = adam->bc1;
    a.bc2_sqrt = adam->bc2_sqrt;
    a.max_g = adam->max_grad_1;
    m = segs(*exp_avg);
    v = segs(*exp_avg_sq);
    const int vec = aligned(segs(g)) && aligned(m) && aligned(v) && aligned(segs(grads));
    k_preprocess_backward<true><<<blocks, 32 * kBwdWarps, 0, stream>>>(
        segs(g), segs(grads), m, v, a, 0, vec, active_bases, n, cam, s.n_touched,
        reinterpret_cast<const float4*>(s.helpers), dens, s.counts, RouteArgs{}, base);
  } else if (route != nullptr) {
    RouteArgs r{};
    bool vec = aligned(segs(g));
    for (int k = 0; k < route->world; ++k) {
      r.inbox[k] = route->inbox[k];
      vec = vec && (reinterpret_cast<uintptr_t>(route->inbox[k]) & 15u) == 0;
    }
    for (int k = 0; k <= route->world; ++k) r.lo[k] = route->lo[k];
    r.slice_pad = route->slice_pad;
    r.world = route->world;
    r.rank = route->rank;
    const uint32_t n_warps = (n + kWarpGaussians - 1) / kWarpGaussians;
    const int64_t next_lo = route->lo[(route->rank + 1) % route->world];
    r.warp_shift = static_cast<uint32_t>(next_lo / kWarpGaussians) % n_warps;
    vec = vec && route->slice_pad % 4 == 0;
    k_preprocess_backward<false, true><<<blocks, 32 * kBwdWarps, 0, stream>>>(
        segs(g), segs(grads), m, v, a, 0, vec ? 1 : 0, active_bases, n, cam, s.n_touched,
        reinterpret_cast<const float4*>(s.helpers), dens, s.counts, r, base);
  } else {
    const int vec = aligned(segs(g)) && aligned(segs(grads));
    k_preprocess_backward<false><<<blocks, 32 * kBwdWarps, 0, stream>>>(
        segs(g), segs(grads), m, v, a, accumulate, vec, active_bases, n, cam, s.n_touched,
        reinterpret_cast<const float4*>(s.helpers), dens, s.counts, RouteArgs{}, base);
  }
}

void launch_views_backward_adam(const RasterState* const* views, const DevCamera* cams, int world,
                                const GaussianPtrs& g, const GaussianPtrs* grads, const GaussianPtrs& exp_avg,
                                const GaussianPtrs& exp_avg_sq, const AdamStepArgs& adam, float4* dens,
                                cudaStream_t stream, int64_t first, int64_t last) {
  const uint32_t n = static_cast<uint32_t>(last);
  const uint32_t base = static_cast<uint32_t>(first);
  if (n <= base || world < 1 || world > kMaxDpRanks) return;
  static const bool attr_set = [] {
    return cudaFuncSetAttribute(k_views_backward_adam, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(kViewsSmemBytes)) == cudaSuccess;
  }();
  (void)attr_set;
  auto segs = [](const GaussianPtrs& x) {
    SegPtrs p{{x.means, x.opacities, x.rotations, x.scales, x.sh0, x.sh_rest}};
    return p;
  };
  auto aligned = [](const SegPtrs& p) {
    for (float* q : p.p)
      if (q != nullptr && (reinterpret_cast<uintptr_t>(q) & 15u) != 0) return false;
    return true;
  };
  AdamArgs a{};
  for (int k = 0; k < 6; ++k) {
    a.lr[k] = adam.lr[k];
    a.decay[k] = adam.decay[k];
    a.kind[k] = adam.kind[k];
  }
  a.beta1 = adam.beta1;
  a.beta2 = adam.beta2;
  a.eps = adam.eps;
  a.gscale = adam.gradient_scale;
  a.bc1 = adam.bc1;
  a.bc2_sqrt = adam.bc2_sqrt;
  a.max_g = adam.max_grad_1;
  ViewsArgs va{};
  for (int k = 0; k < world; ++k) {
    va.cam[k] = cams[k];
    va.n_touched[k] = views[k]->n_touched;
    va.helpers[k] = reinterpret_cast<const float4*>(views[k]->helpers);
    va.counts[k] = views[k]->counts;
  }
  va.world = world;
  const SegPtrs gr = grads != nullptr ? segs(*grads) : SegPtrs{};
  const SegPtrs m = segs(exp_avg), v = segs(exp_avg_sq);
  const int vec = aligned(segs(g)) && aligned(m) && aligned(v) && aligned(gr);
  const int active_bases = (g.sh_degree + 1) * (g.sh_degree + 1);
  const uint32_t per_block = kBwdWarps * kWarpGaussians;
  const uint32_t blocks = (n - base + per_block - 1) / per_block;
  k_views_backward_adam<<<blocks, 32 * kBwdWarps, kViewsSmemBytes, stream>>>(segs(g), gr, m, v, a, vec,
                                                                           active_bases, n, base, dens, va);
}

}  // namespace tgs
