/*
 * tgs_oracle.h -- CPU restatement of the tinygs training hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the checker the parity tests, smoke()
 * and bench.py's cpu_baseline leg compare the CUDA path against; it is never
 * linked into, loaded by or called from the product library.
 *
 * Parity status: UNPINNED.  The reference ships no golden vectors or
 * known-answer tests for this path and its CUDA sources cannot be built here
 * (they need glm, nlohmann_json, spdlog and NVTX fetched by CMake), so this
 * restatement is anchored only on the reference source it cites, function
 * by function, and on self-consistency checks (finite differences).
 *
 * All buffers are host memory.  Image buffers use the reference's 8x8-tiled
 * CHW layout (tinygs/include/tinygs/common.hpp:389-408).
 */
#ifndef TGS_ORACLE_H
#define TGS_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct OrcCamera {
    int32_t width, height;
    float fx, fy, cx, cy, near_plane, far_plane;
    float w2c[16]; /* row-major */
} OrcCamera;

/* Per-Gaussian preprocess outputs (all n entries written; culled => n_touched 0). */
typedef struct OrcPrimitives {
    uint32_t* n_touched;     /* [n]    */
    uint16_t* bounds;        /* [n][4] x_min, x_max, y_min, y_max (tiles) */
    float* mean2d;           /* [n][2] */
    float* conic_opacity;    /* [n][4] fp32 path: conic (a,b,c), opacity     */
    float* color;            /* [n][3] unclamped SH colour                     */
    uint32_t* depth_key;     /* [n]    float bits of the view-space depth      */
    uint8_t* fragile;        /* [n]    1 if a cull/bound/tile decision lies
                                       within the tolerance of its threshold   */
    uint8_t* prim_info;      /* [n][16] fp16 path packed record or NULL        */
} OrcPrimitives;

void orc_camera_position(const OrcCamera* cam, float out[3]);

/* fastgs_ours/kernels_forward.cuh:157-412 (fp16 == 0),
 * fastgs_ours_fp16/kernels_forward.cuh:249-496 (fp16 == 1). */
void orc_preprocess(int64_t n, const float* means, const float* opacities,
                    const float* rotations, const float* scales,
                    const float* sh0, const float* sh_rest, int32_t sh_degree,
                    const OrcCamera* cam, int32_t fp16, OrcPrimitives* out,
                    float* dens /* [n][4] or NULL */, int32_t n_threads);

/* Depth ordering + instance creation + stable tile sort + ranges
 * (fastgs_ours/forward.cu:146-250, kernels_forward.cuh:414-567).
 * Visible Gaussians are ordered by (depth, index).  Returns the number of
 * instances, or -1 if `cap` was too small.  ranges: [n_tiles][2]. */
/* Touched-tile count of every Gaussian recomputed from its stored record
 * (the test create_instances repeats); 0 where prim->n_touched is 0.
 * fragile[i] (if given) flags a tile test within `band` (relative to
 * max(|threshold|, 1)) of its threshold. */
void orc_count_tiles(int64_t n, const OrcPrimitives* prim, const OrcCamera* cam, int32_t fp16,
                     uint32_t* out, uint8_t* fragile /* or NULL */, float band, int32_t n_threads);

/* Optional per-pixel flags set by the blend forwards for decisions within
 * `band` (relative) of their thresholds; NULL turns the recording off. */
void orc_set_pixel_fragile(uint8_t* buf, float band);

int64_t orc_binning(int64_t n, const OrcPrimitives* prim, const OrcCamera* cam,
                    int32_t fp16, uint32_t* inst_tile, uint32_t* inst_prim,
                    int64_t cap, uint32_t* ranges, uint32_t* sorted_visible,
                    uint32_t* n_visible);

/* Per-tile bucket offsets (inclusive scan of ceil(count/32)); returns total. */
int64_t orc_bucket_offsets(const uint32_t* ranges, int32_t n_tiles,
                           uint32_t* bucket_offsets);

/* fp32 blend forward, fastgs_ours/kernels_forward.cuh:569-715.
 * ckpt: [n_buckets][256][4] (rgb, T) or NULL. */
void orc_blend_forward_f32(const OrcCamera* cam, const uint32_t* ranges,
                           const uint32_t* inst_prim, const float* mean2d,
                           const float* conic_opacity, const float* color,
                           float* image, float* alpha, uint32_t* n_contrib,
                           uint32_t* tile_max_contrib,
                           const uint32_t* bucket_offsets, float* ckpt,
                           int32_t n_threads);

/* fp32 blend backward, fastgs_ours/kernels_backward.cuh:675-927.
 * Outputs are accumulated (+=): grad_mean2d [n][2], absgrad [n][2],
 * grad_conic [3][n] (SoA), grad_opacity [n], grad_color [n][3]. */
void orc_blend_backward_f32(const OrcCamera* cam, int64_t n,
                            const uint32_t* ranges, const uint32_t* inst_prim,
                            const float* mean2d, const float* conic_opacity,
                            const float* color, const float* image,
                            const float* grad_image, const uint32_t* n_contrib,
                            const uint32_t* tile_max_contrib,
                            const uint32_t* bucket_offsets, const float* ckpt,
                            float* grad_mean2d, float* absgrad_mean2d,
                            float* grad_conic, float* grad_opacity,
                            float* grad_color, int32_t n_threads);

/* fp16 blend forward, fastgs_ours_fp16/kernels_forward.cuh:917-1171, with
 * half arithmetic emulated (IEEE RN; ex2.approx is replaced by a correctly
 * rounded exp2, the one op that is not bit-exact).
 * image/alpha are fp16 bit patterns; ckpt: [n_buckets][256][4] fp16 bits
 * (r,g,b,T scaled by 255); n_contrib uint16. */
void orc_blend_forward_f16(const OrcCamera* cam, const uint32_t* ranges,
                           const uint32_t* inst_prim, const float* mean2d,
                           const uint8_t* prim_info, uint16_t* image,
                           uint16_t* alpha, uint16_t* n_contrib,
                           uint16_t* tile_max_contrib,
                           const uint32_t* bucket_offsets, uint16_t* ckpt,
                           int32_t n_threads);

/* fp16-path blend backward semantics (fastgs_ours_fp16/kernels_backward.cuh:
 * 861-1389 as compiled, i.e. without TINYGS_SAFE_MATH) evaluated in fp32.
 * image/grad_image fp16 bits.  Outputs accumulated (+=) as for fp32, but
 * grad_conic here is [n][3] and grad_color [n][3]. */
void orc_blend_backward_f16(const OrcCamera* cam, int64_t n,
                            const uint32_t* ranges, const uint32_t* inst_prim,
                            const float* mean2d, const uint8_t* prim_info,
                            const uint16_t* image, const uint16_t* grad_image,
                            const uint16_t* tile_max_contrib,
                            const uint32_t* bucket_offsets,
                            const uint16_t* ckpt, float* grad_mean2d,
                            float* absgrad_mean2d, float* grad_conic,
                            float* grad_opacity, float* grad_color,
                            int32_t n_threads);

/* Preprocess backward, fastgs_ours/kernels_backward.cuh:22-352 (fp32 path,
 * grad_conic SoA [3][n]) or fastgs_ours_fp16/kernels_backward.cuh:93-359
 * (conic_soa == 0: grad_conic [n][3]).  Gradients accumulated (+=). */
void orc_preprocess_backward(
    int64_t n, const float* means, const float* rotations, const float* scales,
    const float* sh_rest, int32_t sh_degree, const OrcCamera* cam,
    const uint32_t* n_touched, const float* grad_mean2d,
    const float* grad_conic, int32_t conic_soa, const float* absgrad_mean2d,
    const float* grad_color, float* g_means, float* g_rotations,
    float* g_scales, float* g_sh0, float* g_sh_rest, float* dens,
    int32_t n_threads);

/* L1 term, tinygs/src/loss/l1.cu:19-151 (fp32 buffers). */
void orc_l1_f32(int32_t width, int32_t height, const float* pred,
                const float* target, float* loss_map, float* grad, float scale);

/* Fused SSIM fwd+bwd, tinygs/src/loss/fused_ssim.cu:55-442,797-916 (fp32
 * buffers; inputs are staged through fp16 as the reference does). */
void orc_ssim_f32(int32_t width, int32_t height, const float* pred,
                  const float* target, float* loss_map, float* grad,
                  float scale, int32_t n_threads);

/* fp16 buffers: tinygs/src/loss/l1.cu:72-106, fused_ssim.cu:445-763. */
void orc_l1_f16(int32_t width, int32_t height, const uint16_t* pred,
                const uint16_t* target, uint16_t* loss_map, uint16_t* grad,
                float scale);
void orc_ssim_f16(int32_t width, int32_t height, const uint16_t* pred,
                  const uint16_t* target, uint16_t* loss_map, uint16_t* grad,
                  float scale, int32_t n_threads);

/* Adam over one parameter array, tinygs/src/optim/simple_adam.cu:105-213.
 * decay_kind 0 none, 1 opacity (sigmoid'), 2 scale (exp). */
void orc_adam(int64_t count, float* theta, const float* grad, float* m,
              float* v, float lr, float beta1, float beta2, float eps,
              float gradient_scale, float bias_correction1,
              float bias_correction2_sqrt, float max_grad_1,
              int32_t decay_kind, float decay);

/* ------------------------------------------------------ densification */

/* PCG32 (M. E. O'Neill, "PCG: A Family of Simple Fast Space-Efficient
 * Statistically Good Algorithms for Random Number Generation", 2014: 64-bit
 * LCG state, XSH-RR 32-bit output), seeded and advanced as
 * tinygs/include/tinygs/random/pcg32.hpp:40-150 does. */
typedef struct OrcPcg32 {
    uint64_t state;
    uint64_t inc;
} OrcPcg32;
void orc_pcg32_seed(OrcPcg32* r, uint64_t initstate, uint64_t initseq);
uint32_t orc_pcg32_next_uint(OrcPcg32* r);
float orc_pcg32_next_float(OrcPcg32* r);
void orc_pcg32_advance(OrcPcg32* r, uint64_t delta);
/* generate_random_logistic(rng, n, out, 0, 1), random/device.cuh:38-79:
 * element idx is draw (idx % T) * 4 + idx / T of the stream, T the number of
 * threads its launch has; the generator then advances by n. */
void orc_random_logistic(OrcPcg32* r, int64_t n, float* out);

/* The six parameter arrays of one set (parameters, gradients or a moment),
 * each holding `capacity` Gaussians. */
typedef struct OrcSet {
    float* means;      /* [cap][3] */
    float* opacities;  /* [cap]    */
    float* rotations;  /* [cap][4] (w, x, y, z) */
    float* scales;     /* [cap][3] */
    float* sh0;        /* [cap][3] */
    float* sh_rest;    /* [cap][45] */
} OrcSet;

typedef struct OrcDensifyConfig {
    float duplicate_grad_threshold;
    float duplicate_scale_threshold;
    float pruning_opacity_threshold;
    float pruning_scale_threshold;
    float max_screen_size;
    float scene_scale;
    float grad_scaler;
    int32_t absgrad;
    int32_t refine_every;
    int32_t start_refine;
    int32_t end_refine;
    int32_t reset_every;
    int32_t image_width;
    int32_t image_height;
    int32_t _pad;
    int64_t max_num_gaussians;
} OrcDensifyConfig;

/* DefaultStrategy::step_impl at strategy step `step`
 * (tinygs/src/strategy/default.cu:40-69): refine (duplicate, default.cu:75-296,
 * then prune, :298-345, with the stable compaction of gpu_gaussian.cu:117-160
 * and simple_adam.cu:841-906; appended Gaussians get zero gradients and
 * moments, strategy.cpp:34-46, simple_adam.cu:908-924) and the opacity reset
 * (default.cu:26-38, simple_adam.cu:981-985).  dens is [n][4] (counter,
 * grad, absgrad, max radius) and is zeroed after a refine.  Sets whose
 * pointers are NULL are skipped.  Returns the new Gaussian count, or -1 if
 * the growth would pass `capacity` (nothing is modified then). */
int64_t orc_densify_step(int64_t n, int64_t capacity, OrcSet params, OrcSet grads, OrcSet exp_avg,
                         OrcSet exp_avg_sq, float* dens, const OrcDensifyConfig* cfg, int32_t step,
                         OrcPcg32* rng);

/* Timing samples only: blend stages process every `stride`-th tile. */
void orc_set_tile_stride(int32_t stride);

/* Finite-difference checks only: smooth fp32 forward (see tgs_oracle.c). */
void orc_set_smooth_forward(int32_t on);
/* fp16 path: width of the band around the tile-test threshold inside which
 * a decision is marked fragile, relative to max(|threshold|, 1); <= 0
 * restores the default 2e-2. */
void orc_set_fragile_f16(float rel);

/* IEEE binary16 helpers used by the fp16 emulation. */
uint16_t orc_f2h(float f);
float orc_h2f(uint16_t h);

/* Morton order of the means (tinygs/src/orchestrator.cu:26-100): perm[i] is
 * the Gaussian that moves to row i. */
void orc_morton_order(int64_t n, const float* means, uint32_t* perm);

#ifdef __cplusplus
}
#endif
#endif
