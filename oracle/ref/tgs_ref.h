/* tgs_ref.h -- C interface of oracle/_ref/libtgs_ref.so: the reference's own
 * CUDA kernels (Adversarr/tinygs tinygs/src/rasterizer/fastgs_ours/,
 * fastgs_ours_fp16/, loss/l1.cu, loss/fused_ssim.cu), compiled unchanged from
 * their sources, driven through their own raw entry points
 * (fast_gs::rasterization::forward/backward, fastgs_ours/forward.h:13-45,
 * backward.h:13-53; tinygs::fast_gs_fp16::forward/backward; L1Loss and
 * FusedSSIMLoss::evaluate).
 *
 * Test infrastructure only: the parity tests and bench.py's reference arm
 * load it to produce the reference's outputs on the same inputs as the
 * product.  Nothing in the product links it. */
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same field order and meaning as TgsCamera (include/tgs_abi.h). */
typedef struct TgsRefCamera {
  int32_t width, height;
  float fx, fy, cx, cy;
  float near_plane, far_plane;
  float w2c[16]; /* row-major world-to-camera matrix */
} TgsRefCamera;

/* Device pointers of the six SoA parameter (or gradient) arrays, laid out as
 * the reference's GPUGaussian3d (means float3, opacities float, rotations
 * float4 (w,x,y,z), scales float3, sh0 float3, sh_rest 15 x float3). */
typedef struct TgsRefGaussians {
  float* means;
  float* opacities;
  float* rotations;
  float* scales;
  float* sh0;
  float* sh_rest;
  int64_t n;
  int32_t sh_degree;
} TgsRefGaussians;

/* Buffers tgsref_copy can read back (the reference's own scratch). */
enum {
  TGSREF_N_TOUCHED = 0,        /* uint32[N] */
  TGSREF_SORTED_PRIMS = 1,     /* uint32[V], depth order */
  TGSREF_SORTED_DEPTH_KEYS = 2,/* uint32[V] */
  TGSREF_INST_KEYS = 3,        /* fp32 path uint16[I], fp16 path uint32[I], sorted by tile */
  TGSREF_INST_PRIMS = 4,       /* uint32[I] */
  TGSREF_TILE_RANGES = 5,      /* uint32[T][2] */
  TGSREF_BUCKET_OFFSETS = 6,   /* uint32[T], inclusive */
  TGSREF_TILE_MAX_CONTRIB = 7, /* fp32 uint32[T], fp16 uint16[T] */
  TGSREF_N_CONTRIB = 8,        /* fp32 uint32[T*256], fp16 uint16[T*256] */
  TGSREF_MEAN2D = 9,           /* float32[N][2] */
  TGSREF_CONIC_OPACITY = 10,   /* fp32: float32[N][4]; fp16: PrimitiveInfo 16 B [N] */
  TGSREF_COLOR = 11,           /* fp32: float32[N][3] */
  TGSREF_BOUNDS = 12,          /* uint16[N][4] */
  TGSREF_CKPT = 13,            /* fp32 float32[B*256][4], fp16 4 x half [B*256] */
  TGSREF_GRAD_MEAN2D = 14,     /* fp32 path helpers after backward: float32[N][2] */
  TGSREF_ABSGRAD_MEAN2D = 15,  /* float32[N][2] */
  TGSREF_GRAD_CONIC = 16,      /* float32[N][3] */
  TGSREF_GRAD_COLOR = 17,      /* float32[N][3] */
  TGSREF_PRIM_INFO_GRAD = 18,  /* fp16 path: PrimitiveInfoGradient[N] */
  TGSREF_ALPHA = 19,           /* fp32 float32[P] / fp16 half[P] (padded plane) */
  TGSREF_BUCKET_TILE = 20      /* uint32[B*256] (only [b*256] used by the reference) */
};

int tgsref_create(void** handle);
void tgsref_destroy(void* handle);

/* One forward of the reference rasterizer (precision by fp16 != 0; the image
 * is float32 or half, tiled CHW).  dens may be NULL.  counts[0..2] = visible
 * primitives, instances, buckets.  Returns 0 or a CUDA error code; a C++
 * exception of the reference code returns -1 with its message in
 * tgsref_last_error(). */
int tgsref_forward(void* handle, int32_t fp16, const TgsRefGaussians* g, const TgsRefCamera* cam, void* image,
                   void* dens, void* stream, int32_t counts[3]);

/* One backward after tgsref_forward on the same handle.  grads are added into
 * (the caller zeroes them), as the reference does. */
int tgsref_backward(void* handle, int32_t fp16, const TgsRefGaussians* g, const TgsRefCamera* cam,
                    const void* image, const void* grad_image, const TgsRefGaussians* grads, void* dens,
                    void* stream);

/* Copies buffer `which` of the last forward/backward to host memory; returns
 * the number of bytes copied (at most max_bytes), or -1. */
int64_t tgsref_copy(void* handle, int32_t which, void* host_dst, int64_t max_bytes);

/* L1Loss::evaluate / FusedSSIMLoss::evaluate (accumulate into loss and grad
 * with the given scale = weight * grad_scaler). */
int tgsref_l1(int32_t fp16, int32_t width, int32_t height, const void* pred, const void* target, void* loss,
              void* grad, float scale, void* stream);
int tgsref_ssim(void* handle, int32_t fp16, int32_t width, int32_t height, const void* pred, const void* target,
                void* loss, void* grad, float scale, void* stream);

/* The reference's SimpleAdam (tinygs/src/optim/simple_adam.cu) over its own
 * parameter and gradient containers of n Gaussians (zero-filled; fill them
 * through the pointers tgsref_adam_arrays returns).  config_json: the
 * optimizer's JSON configuration (GaussianOptimizationParams and
 * SimpleAdamParameters keys), or NULL for the defaults. */
int tgsref_adam_create(int64_t n, int32_t sh_degree, const char* config_json, void** handle);
void tgsref_adam_destroy(void* handle);
int tgsref_adam_arrays(void* handle, TgsRefGaussians* params, TgsRefGaussians* grads);
/* SimpleAdam::step(gradient_scale, stream). */
int tgsref_adam_step(void* handle, float gradient_scale, void* stream);

const char* tgsref_last_error(void);

#ifdef __cplusplus
}
#endif
