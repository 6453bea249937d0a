// ref_raster_f16.cu -- the reference's fp16 rasterizer
// (tinygs/src/rasterizer/fastgs_ours_fp16/) driven through its raw entry
// points (FastGSRasterizer::forward/backward, fastgs.cu:142-189,272-313).
// Test infrastructure (oracle/_ref build).
#include <tuple>

#include "fastgs_ours_fp16/backward.h"
#include "fastgs_ours_fp16/buffer_utils.h"
#include "fastgs_ours_fp16/forward.h"
#include "ref_common.h"

#define REF_NS tinygs::fast_gs_fp16
#define REF_IMG_T __half
#define REF_SUFFIX f16
#define REF_IS_FP16 1

namespace tgsref {

static bool locate_extra_f16(RefHandle* h, REF_NS::PerPrimitiveBuffers& P, int which, const void** ptr,
                             size_t* bytes) {
  const int n = h->n;
  switch (which) {
    case TGSREF_CONIC_OPACITY: *ptr = P.primitive_infos; *bytes = sizeof(*P.primitive_infos) * (size_t)n; return true;
    case TGSREF_PRIM_INFO_GRAD:
      *ptr = P.primitive_info_gradients;
      *bytes = sizeof(*P.primitive_info_gradients) * (size_t)n;
      return true;
    default: return false;
  }
}

void backward_f16(RefHandle* h, const TgsRefGaussians* g, const TgsRefCamera* cam, const void* image,
                  const void* grad_image, const TgsRefGaussians* gr, void* dens, cudaStream_t stream) {
  const int active_bases = (g->sh_degree + 1) * (g->sh_degree + 1);
  tinygs::fast_gs_fp16::backward(
      static_cast<const tinygs::float16_t*>(grad_image), static_cast<const tinygs::float16_t*>(image),
      reinterpret_cast<const float3*>(g->means), reinterpret_cast<const float3*>(g->scales),
      reinterpret_cast<const float4*>(g->rotations), reinterpret_cast<const float3*>(g->sh_rest), h->pose_w2c(),
      h->pose_cam(), h->blob[RefHandle::kPrim], h->blob[RefHandle::kTile], h->blob[RefHandle::kInst],
      h->blob[RefHandle::kBucket], reinterpret_cast<float3*>(gr->means), reinterpret_cast<float3*>(gr->scales),
      reinterpret_cast<float4*>(gr->rotations), gr->opacities, reinterpret_cast<float3*>(gr->sh0),
      reinterpret_cast<float3*>(gr->sh_rest), h->pose_grad(), nullptr,
      reinterpret_cast<tinygs::DensificationInfo*>(dens), static_cast<int>(g->n), h->n_visible, h->n_instances,
      h->n_buckets, h->prim_selector, h->inst_selector, active_bases, 15, cam->width, cam->height, cam->fx,
      cam->fy, cam->cx, cam->cy, stream);
}

}  // namespace tgsref

#include "ref_raster.inc"
