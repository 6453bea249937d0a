// ref_raster_f32.cu -- the reference's fp32 rasterizer
// (tinygs/src/rasterizer/fastgs_ours/) driven through its raw entry points,
// with the helper buffers FastGSRasterizer::backward allocates and zeroes
// (fastgs.cu:316-331).  Test infrastructure (oracle/_ref build).
#include <tuple>

#include "fastgs_ours/backward.h"
#include "fastgs_ours/buffer_utils.h"
#include "fastgs_ours/forward.h"
#include "ref_common.h"

#define REF_NS fast_gs::rasterization
#define REF_IMG_T float
#define REF_SUFFIX f32
#define REF_IS_FP16 0

namespace tgsref {

// Helper arrays of the fp32 backward, carved from one blob: grad_mean2d
// float2[N], grad_conic float3[N], grad_color float3[N], absgrad float2[N].
struct HelpersF32 {
  float2* grad_mean2d;
  float* grad_conic;
  float3* grad_color;
  float2* absgrad;
};
static HelpersF32 helpers_f32(RefHandle* h, int n, bool grow) {
  const size_t a = 256 * ((8ull * n + 255) / 256), b = 256 * ((12ull * n + 255) / 256);
  char* base = grow ? h->grow(RefHandle::kHelper, 2 * a + 2 * b) : h->blob[RefHandle::kHelper];
  HelpersF32 r;
  r.grad_mean2d = reinterpret_cast<float2*>(base);
  r.grad_conic = reinterpret_cast<float*>(base + a);
  r.grad_color = reinterpret_cast<float3*>(base + a + b);
  r.absgrad = reinterpret_cast<float2*>(base + a + 2 * b);
  return r;
}

static bool locate_extra_f32(RefHandle* h, REF_NS::PerPrimitiveBuffers& P, int which, const void** ptr,
                             size_t* bytes) {
  const int n = h->n;
  switch (which) {
    case TGSREF_CONIC_OPACITY: *ptr = P.conic_opacity; *bytes = 16ull * n; return true;
    case TGSREF_COLOR: *ptr = P.color; *bytes = 12ull * n; return true;
    default: break;
  }
  if (h->blob[RefHandle::kHelper] == nullptr) return false;
  HelpersF32 hp = helpers_f32(h, n, false);
  switch (which) {
    case TGSREF_GRAD_MEAN2D: *ptr = hp.grad_mean2d; *bytes = 8ull * n; return true;
    case TGSREF_ABSGRAD_MEAN2D: *ptr = hp.absgrad; *bytes = 8ull * n; return true;
    case TGSREF_GRAD_CONIC: *ptr = hp.grad_conic; *bytes = 12ull * n; return true;
    case TGSREF_GRAD_COLOR: *ptr = hp.grad_color; *bytes = 12ull * n; return true;
    default: return false;
  }
}

void backward_f32(RefHandle* h, const TgsRefGaussians* g, const TgsRefCamera* cam, const void* image,
                  const void* grad_image, const TgsRefGaussians* gr, void* dens, cudaStream_t stream) {
  const int n = static_cast<int>(g->n);
  HelpersF32 hp = helpers_f32(h, n, true);
  check(cudaMemsetAsync(h->blob[RefHandle::kHelper], 0, h->cap[RefHandle::kHelper], stream), "memset helpers");
  const int active_bases = (g->sh_degree + 1) * (g->sh_degree + 1);
  fast_gs::rasterization::backward(
      static_cast<const float*>(grad_image), static_cast<const float*>(image),
      reinterpret_cast<const float3*>(g->means), reinterpret_cast<const float3*>(g->scales),
      reinterpret_cast<const float4*>(g->rotations), reinterpret_cast<const float3*>(g->sh_rest), h->pose_w2c(),
      h->pose_cam(), h->blob[RefHandle::kPrim], h->blob[RefHandle::kTile], h->blob[RefHandle::kInst],
      h->blob[RefHandle::kBucket], reinterpret_cast<float3*>(gr->means), reinterpret_cast<float3*>(gr->scales),
      reinterpret_cast<float4*>(gr->rotations), gr->opacities, reinterpret_cast<float3*>(gr->sh0),
      reinterpret_cast<float3*>(gr->sh_rest), hp.grad_mean2d, hp.grad_conic, hp.grad_color, h->pose_grad(),
      nullptr, reinterpret_cast<tinygs::DensificationInfo*>(dens), hp.absgrad, n, h->n_visible, h->n_instances,
      h->n_buckets, h->prim_selector, h->inst_selector, active_bases, 15, cam->width, cam->height, cam->fx,
      cam->fy, cam->cx, cam->cy, stream);
}

}  // namespace tgsref

#include "ref_raster.inc"
