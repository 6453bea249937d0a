/*
 * tgs_abi.h -- C ABI of the B200-native tinygs training hot path.
 *
 * Every entry point is `extern "C"`, takes plain pointers and sizes and
 * returns an int status (TGS_OK == 0).  No exception and no C++ type crosses
 * this boundary.  All device work is enqueued on the caller's stream; no
 * entry point synchronises the host unless its comment says so.
 *
 * Reference interfaces replaced (paths inside Adversarr/tinygs):
 *   rasterizer  RasterizerBase::forward/backward
 *                 tinygs/include/tinygs/rasterizer/rasterizer.hpp:38-58
 *               raw API fast_gs::rasterization::forward/backward
 *                 tinygs/src/rasterizer/fastgs_ours/forward.h:13-45,
 *                 tinygs/src/rasterizer/fastgs_ours/backward.h:13-53,
 *                 tinygs/src/rasterizer/fastgs.cu:89-384 (fp32/fp16 dispatch)
 *   loss        LossBase::evaluate(LossContext, float scale)
 *                 tinygs/include/tinygs/loss/loss.hpp:6-28,
 *                 tinygs/src/loss/l1.cu:109-151,
 *                 tinygs/src/loss/fused_ssim.cu:797-916
 *   optimizer   OptimizerBase::step(float scale, cudaStream_t)
 *                 tinygs/include/tinygs/optim/optim.hpp:39-92,
 *                 tinygs/src/optim/simple_adam.cu:457-580
 *   model state GPUGaussian3d (SoA parameter arrays)
 *                 tinygs/include/tinygs/core/gpu_gaussian.hpp:9-73
 *
 * Image buffers use the reference's physical layout: CHW planes, each plane
 * padded to multiples of 8 in x and y and stored as 8x8 tiles,
 *   idx = ((y>>3)*(Wp>>3) + (x>>3))*64 + (y&7)*8 + (x&7),  plane stride Wp*Hp
 * (tinygs/include/tinygs/common.hpp:389-408, core/image.hpp:51-59).
 */
#ifndef TGS_ABI_H
#define TGS_ABI_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TGS_API __attribute__((visibility("default")))
#else
#define TGS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
#define TGS_OK                    0
#define TGS_ERR_INVALID_ARGUMENT  1  /* null pointer, bad size, bad dtype     */
#define TGS_ERR_CUDA              2  /* a CUDA runtime call failed            */
#define TGS_ERR_CAPACITY          3  /* a device buffer bound was exceeded    */
#define TGS_ERR_OUT_OF_MEMORY     4  /* cudaMalloc failed at handle creation  */
#define TGS_ERR_NO_FORWARD        5  /* backward called without a forward     */
#define TGS_ERR_UNSUPPORTED       6  /* combination not implemented           */
#define TGS_ERR_DEVICE_TIMEOUT    7  /* a bounded device wait gave up         */

/* Image / rasterizer arithmetic type (reference tinygs::DataType, image.hpp:6-11). */
#define TGS_FLOAT32 0
#define TGS_FLOAT16 1
#define TGS_UINT8   2  /* image data path only */

/* Layouts of 8-bit host images (tgs_image_from_u8). */
#define TGS_IMAGE_TILED_CHW 0  /* channel planes of 8x8 tiles, padded to multiples of 8 (Image, image.hpp) */
#define TGS_IMAGE_HWC       1  /* decoded rows, 3 (RGB) or 4 (RGBA) bytes per pixel, no padding */

/* Opaque stream handle: a cudaStream_t passed through as a pointer. */
typedef void* tgs_stream_t;

/* SoA parameter (or gradient, or moment) arrays of one Gaussian model, all
 * device pointers of fp32, exactly the reference GPUGaussian3d layout:
 *   means     [n][3]   world position
 *   opacities [n]      logit of opacity
 *   rotations [n][4]   quaternion stored (w, x, y, z)
 *   scales    [n][3]   log of the axis scales
 *   sh0       [n][3]   SH band-0 coefficients (RGB)
 *   sh_rest   [n][15][3] SH bands 1..3, always 15 per Gaussian
 * `sh_degree` (0..3) selects the active bands; storage is always 15.  */
typedef struct TgsGaussians {
    float* means;
    float* opacities;
    float* rotations;
    float* scales;
    float* sh0;
    float* sh_rest;
    int64_t n;
    int32_t sh_degree;
    int32_t _pad;
} TgsGaussians;

/* One pinhole view.  `w2c` is the 4x4 world-to-camera matrix in row-major
 * order (row r at w2c[4r..4r+3]); OpenCV convention (z forward, y down).
 * The reference takes glm matrices K (column-major, fx=K[0][0], fy=K[1][1],
 * cx=K[2][0], cy=K[2][1]) and w2c and uploads transpose(w2c)
 * (tinygs/src/rasterizer/fastgs.cu:95-126); this struct carries the same
 * numbers by value, so no pose upload is needed.  */
typedef struct TgsCamera {
    int32_t width;
    int32_t height;
    float fx, fy, cx, cy;
    float near_plane;   /* reference default 0.01 (orchestrator.hpp:45) */
    float far_plane;    /* reference default 100  (orchestrator.hpp:46) */
    float w2c[16];
} TgsCamera;

/* Per-Gaussian densification statistics, 16 B, reference
 * tinygs::DensificationInfo (tinygs/include/tinygs/core/gaussian.hpp:18-23). */
typedef struct TgsDensificationInfo {
    float accum_counter;
    float accum_grad_mean2d;
    float accum_absgrad_mean2d;
    float max_radii_screen;
} TgsDensificationInfo;

/* ------------------------------------------------------------- rasterizer */

/* Capacity bounds fixed at creation.  All scratch is allocated once from
 * these; no step allocates.  max_instances == 0 selects 16 * max_gaussians. */
typedef struct TgsRasterCaps {
    int64_t max_gaussians;
    int32_t max_width;
    int32_t max_height;
    int64_t max_instances;
} TgsRasterCaps;

/* Counts of the last forward.  Written on the device; read by
 * tgs_raster_counts().  n_visible counts the Gaussians that passed culling
 * with a non-empty tile rectangle (a superset of those that touch a tile,
 * whose per-Gaussian tile counts are debug buffer 0).  `overflow` != 0 means
 * a capacity bound was hit and the outputs of that forward are invalid (grow
 * the caps and rerun). */
typedef struct TgsRasterCounts {
    uint32_t n_visible;
    uint32_t n_instances;
    uint32_t n_buckets;
    uint32_t overflow;
} TgsRasterCounts;

typedef struct TgsRaster TgsRaster;

/* Replaces FastGSRasterizer construction + its scratch blobs
 * (tinygs/src/rasterizer/fastgs.cu:26-87).  Uses the current CUDA device. */
TGS_API int tgs_raster_create(const TgsRasterCaps* caps, TgsRaster** out);
TGS_API int tgs_raster_destroy(TgsRaster* r);

/* Device bytes held by the handle (all scratch, allocated at creation). */
TGS_API int tgs_raster_workspace_bytes(const TgsRaster* r, size_t* bytes);

/* Forward render.  Replaces RasterizerBase::forward / FastGSRasterizer::forward
 * (tinygs/src/rasterizer/fastgs.cu:89-236) and the kernels of
 * fastgs_ours/forward.cu:20-292 (dtype TGS_FLOAT32) or
 * fastgs_ours_fp16/forward.cu:20-290 (dtype TGS_FLOAT16).
 *   image  [3][Hp*Wp] of dtype, written
 *   alpha  [Hp*Wp] of dtype, written; may be NULL
 *   dens   [n] densification info, max_radii_screen updated; may be NULL
 * The handle keeps the per-view state the backward needs.  No host sync. */
TGS_API int tgs_raster_forward(TgsRaster* r, const TgsGaussians* params,
                       const TgsCamera* cam, int32_t dtype, void* image,
                       void* alpha, TgsDensificationInfo* dens,
                       tgs_stream_t stream);

/* Backward.  Replaces RasterizerBase::backward / FastGSRasterizer::backward
 * (tinygs/src/rasterizer/fastgs.cu:238-384) and the kernels of
 * fastgs_ours/backward.cu:211-349 or fastgs_ours_fp16/backward.cu:211-342.
 *   image       the image written by the matching forward
 *   grad_image  dL/dimage, same layout and dtype
 *   grads       gradient arrays (same layout as params)
 *   accumulate  1: grads += dL/dparams (reference semantics, grads must be
 *               zeroed by the caller at the start of an accumulation cycle);
 *               0: grads = dL/dparams for every Gaussian (no zeroing needed)
 *   dens        densification accumulators updated; may be NULL  */
TGS_API int tgs_raster_backward(TgsRaster* r, const TgsGaussians* params,
                        const TgsCamera* cam, int32_t dtype, const void* image,
                        const void* grad_image, TgsGaussians* grads,
                        int32_t accumulate, TgsDensificationInfo* dens,
                        tgs_stream_t stream);

/* Copies the counts of the last forward to the host.  Synchronises `stream`. */
TGS_API int tgs_raster_counts(TgsRaster* r, TgsRasterCounts* out, tgs_stream_t stream);

/* Debug / parity access to the intermediate state of the last forward
 * (device pointers owned by the handle, valid until the next forward):
 *   which = 0 n_touched_tiles   uint32[n]
 *         = 1 (not kept: the tile of each instance follows from the ranges)
 *         = 2 instance prim ids  uint32[n_instances]   (tile-major, depth order)
 *         = 3 tile ranges        uint32[2*n_tiles]      [start, end)
 *         = 4 per-pixel contribution counts  uint32[Hp*Wp] (fp32 path)
 *                                            uint16[Hp*Wp] (fp16 path)
 *         = 5 mean2d             float[2*n]
 *         = 6 conic_opacity      float[4*n]  (fp32 path)
 *         = 7 color              float[3*n]  (fp32 path)
 *         = 8 primitive info     16 B * n    (fp16 path, packed record)
 *         = 9 screen bounds      uint16[4*n]
 *         =10 depth-sorted visible prim ids  uint32[n_visible]
 *         =11 backward scratch   float[12*n]  (dL/dmean2d, |dL/dmean2d|,
 *                                dL/dconic, dL/dopacity, dL/dcolor, pad)
 *         =12 per-tile max contribution count  uint32[n_tiles]
 *         =13 per-tile inclusive bucket offsets uint32[n_tiles]
 *         =14 depth keys (float bits)          uint32[n]
 *         =15 bucket checkpoints [n_buckets][256] float4 (fp32 path) or
 *             4 x fp16 (r, g, b, 255*T) (fp16 path)  */
TGS_API int tgs_raster_debug_buffer(TgsRaster* r, int32_t which, void** dev_ptr,
                            size_t* bytes);

/* ---------------------------------------------------------- densification
 * DefaultStrategy (tinygs/src/strategy/default.cu:26-345): clone / split the
 * Gaussians whose mean view-space gradient is large, prune transparent,
 * oversized or degenerate ones, reset opacities periodically.  Arrays are
 * updated in place within their capacity (the reference reallocates every
 * array on each refine, gpu_gaussian.cu:117-171, simple_adam.cu:841-924). */
typedef struct TgsDensifyConfig {     /* StrategyParams, strategy.hpp:9-29 */
    float duplicate_grad_threshold;   /* 2e-4 */
    float duplicate_scale_threshold;  /* 0.01 */
    float pruning_opacity_threshold;  /* 0.005 */
    float pruning_scale_threshold;    /* 0.1 */
    float max_screen_size;            /* 10 */
    float scene_scale;
    float grad_scaler;                /* RasterizeContext::grad_scaler */
    int32_t absgrad;
    int32_t refine_every;             /* 100 */
    int32_t start_refine;             /* 500 */
    int32_t end_refine;               /* 15000 */
    int32_t reset_every;              /* 3000 */
    int32_t image_width;              /* camera of the step (prune by screen size) */
    int32_t image_height;
    int32_t _pad;
    int64_t max_num_gaussians;        /* soft cap: refine grows only below it */
} TgsDensifyConfig;

/* PCG32 generator state (pcg32.hpp:40-150); seed with tgs_pcg32_seed. */
typedef struct TgsPcg32 {
    uint64_t state;
    uint64_t inc;
} TgsPcg32;

typedef struct TgsDensifier TgsDensifier;

/* pcg32::seed(initstate, initseq) (pcg32.hpp:50-56); DefaultStrategy seeds
 * with StrategyParams::seed (42) and initseq 1. */
TGS_API void tgs_pcg32_seed(TgsPcg32* rng, uint64_t initstate, uint64_t initseq);

/* Scratch for densification of sets of up to `capacity` Gaussians (one
 * cudaMalloc).  No counterpart in the reference, which allocates its flag and
 * index vectors on every refine (default.cu:79-236). */
TGS_API int tgs_densify_create(int64_t capacity, TgsDensifier** out);
TGS_API int tgs_densify_destroy(TgsDensifier* d);

/* One DefaultStrategy::step_impl at strategy step `step` (default.cu:40-69):
 * at refine steps duplicate (default.cu:75-296: clones appended in ascending
 * source order, split offsets from generate_random_logistic over `rng`) then
 * prune (:298-345, stable compaction of params, grads and both moments;
 * appended rows get zero gradients and moments); at reset steps the opacity
 * reset (:26-38) with the opacity moments zeroed.  The six arrays of each set
 * hold `capacity` Gaussians (their n fields are ignored); *n is the live count
 * in and out; grads may be NULL.  dens ([*n] records) is zeroed after a
 * refine.  A refine synchronises `stream` to read the growth and survivor
 * counts (the reference synchronises every step, default.cu:42).  Growth past
 * the capacity returns TGS_ERR_CAPACITY with nothing modified. */
TGS_API int tgs_densify_step(TgsDensifier* d, TgsGaussians* params, TgsGaussians* grads,
                             TgsGaussians* exp_avg, TgsGaussians* exp_avg_sq,
                             TgsDensificationInfo* dens, const TgsDensifyConfig* cfg,
                             int32_t step, TgsPcg32* rng, int64_t* n, tgs_stream_t stream);

/* Stage timing for profiling.  When enabled, forward and backward record a
 * CUDA event between their stages on the caller's stream (no host sync).
 * tgs_raster_stage_times() waits for those events and returns the elapsed
 * milliseconds of the stages of the last forward and backward:
 *   [0] preprocess  [1] binning (compaction, sorts, instances, ranges)
 *   [2] blend forward  [3] blend backward
 *   [4] per-Gaussian backward (with the Adam update when fused). */
TGS_API int tgs_raster_set_stage_timing(TgsRaster* r, int32_t enable);
TGS_API int tgs_raster_stage_times(TgsRaster* r, float* out_ms5);

/* ------------------------------------------------------------------- loss */

/* L1 term.  Replaces L1Loss::evaluate (tinygs/src/loss/l1.cu:109-151):
 *   loss_map += s*|sat(pred)-target|, grad += s*sign(sat(pred)-target),
 *   s = scale / (3*W*H), over every physical element (padding included).
 * loss_map and grad may each be NULL. dtype TGS_FLOAT32 or TGS_FLOAT16. */
TGS_API int tgs_loss_l1(int32_t dtype, int32_t width, int32_t height, const void* pred,
                const void* target, void* loss_map, void* grad, float scale,
                tgs_stream_t stream);

typedef struct TgsLoss TgsLoss;

/* Scratch for the SSIM partial-derivative maps, sized for max_w x max_h. */
TGS_API int tgs_loss_create(int32_t max_width, int32_t max_height, TgsLoss** out);
TGS_API int tgs_loss_destroy(TgsLoss* l);

/* Fused SSIM term.  Replaces FusedSSIMLoss::evaluate
 * (tinygs/src/loss/fused_ssim.cu:797-916): 11-tap Gaussian window
 * (sigma 1.5), C1 = 1e-4, C2 = 9e-4, zero padding,
 *   loss_map += s*(1-ssim), grad -= s*dssim/dpred,  s = scale/(W*H).
 * grad may be NULL (forward only); loss_map must not be NULL. */
TGS_API int tgs_loss_fused_ssim(TgsLoss* l, int32_t dtype, int32_t width,
                        int32_t height, const void* pred, const void* target,
                        void* loss_map, void* grad, float scale,
                        tgs_stream_t stream);

/* Both terms of the reference's default loss mix in one call, equal to
 * tgs_loss_l1(scale_l1) followed by tgs_loss_fused_ssim(scale_ssim), plus an
 * optional device scalar: if loss_sum != NULL, *loss_sum (fp32, device) is
 * set to the sum of this call's loss contributions (no host sync). */
TGS_API int tgs_loss_l1_ssim(TgsLoss* l, int32_t dtype, int32_t width, int32_t height,
                     const void* pred, const void* target, void* loss_map,
                     void* grad, float scale_l1, float scale_ssim,
                     float* loss_sum, tgs_stream_t stream);

/* Accumulation mode of tgs_loss_l1_ssim on this handle (no counterpart in
 * the reference, whose loss adds into buffers its trainer zeroes every step).
 * accumulate != 0 (the default): loss_map and grad are added into, as in the
 * reference.  accumulate == 0: tgs_loss_l1_ssim writes every element of the
 * padded loss_map and grad (the values the accumulate mode would leave in
 * zeroed buffers), so the caller needs no per-step zeroing; it requires
 * scale_l1 != 0 or the padding pixels' values (zero) still being written. */
TGS_API int tgs_loss_set_accumulate(TgsLoss* l, int32_t accumulate);

/* Largest padded image (Wp * Hp pixels, e.g. 512 x 512) that
 * tgs_loss_l1_ssim_noalloc accepts. */
#define TGS_NOALLOC_MAX_PIXELS 262144

/* tgs_loss_l1_ssim for callers that cannot allocate device memory -- hosts
 * whose memory pool owns all device memory, or code that must not allocate
 * where it runs.  No counterpart in the reference.  It takes no TgsLoss
 * handle: the SSIM partial-derivative maps live in a fixed array inside the
 * library (9 MiB held by every GPU that loads it, until exit) instead of
 * memory the caller allocates; the caller still passes inputs and outputs.
 * Same arguments and results as tgs_loss_l1_ssim without its first argument.
 * Returns TGS_ERR_CAPACITY if Wp * Hp exceeds TGS_NOALLOC_MAX_PIXELS.  Every
 * call looks up the array's device address on the current device (make the
 * first call before any stream capture).  The array is placed in device
 * memory when the library's device code loads on a device, which with lazy
 * module loading is the library's first call there: make that call before
 * the host's pool reserves all free device memory.  Every call on a device
 * shares the array: calls whose GPU work may overlap race on it and must be
 * serialised.  Calls no cudaMalloc or cudaFree. */
TGS_API int tgs_loss_l1_ssim_noalloc(int32_t dtype, int32_t width,
                                     int32_t height, const void* pred,
                                     const void* target, void* loss_map,
                                     void* grad, float scale_l1,
                                     float scale_ssim, float* loss_sum,
                                     tgs_stream_t stream);

/* PSNR of pred against target, left on the device: out[0] = MSE over the
 * 3 W H real values (pred saturated to [0, 1]), out[1] = -10 log10(MSE) (100
 * for MSE 0).  Replaces PsnrMetric::evaluate (tinygs/src/loss/psnr.cu:72-128),
 * which allocates, reduces with thrust and returns the value to the host;
 * this call allocates nothing and does not synchronise.  workspace: 8 bytes
 * of device memory (a double accumulator).  dtype TGS_FLOAT32 / TGS_FLOAT16,
 * images in the tiled layout with zero padding. */
TGS_API int tgs_metric_psnr(int32_t dtype, int32_t width, int32_t height, const void* pred,
                            const void* target, void* workspace, float* out, tgs_stream_t stream);

/* ------------------------------------------------------------- data path */

/* An 8-bit image already on the device (src) into the rasterizer's tiled
 * layout in dst_dtype (TGS_FLOAT32 / TGS_FLOAT16: value / 255, fp16 rounded
 * to nearest; TGS_UINT8: the bytes).
 *   layout TGS_IMAGE_TILED_CHW: src holds src_channels (3 or 4) padded tiled
 *     planes, converted element for element, padding included; src and dst
 *     16-byte aligned.  Replaces the same-shape branch of
 *     DataLoaderBase::transfer_gpu (tinygs/src/dataloader/dataloader.cu:
 *     257-297) and its kernels (:26-104).
 *   layout TGS_IMAGE_HWC: src holds height rows of width pixels of
 *     src_channels bytes (RGB or RGBA; alpha is dropped); dst receives 3
 *     padded tiled planes, padding zero.  This is the reorder that
 *     PngFolderDataset does on the host while loading
 *     (tinygs/src/dataset/png_folder.cpp:60-69), moved to the device.
 * Asynchronous on `stream`; nothing is allocated. */
TGS_API int tgs_image_from_u8(const uint8_t* src, int32_t layout, int32_t src_channels, int32_t width,
                              int32_t height, void* dst, int32_t dst_dtype, tgs_stream_t stream);

/* A tiled 8-bit image of src_width x src_height with `channels` (3 or 4)
 * planes resized into dst (TGS_FLOAT32 / TGS_FLOAT16, dst_width x
 * dst_height, padding written as zero).  blur_state NULL: nearest source
 * pixel (dataloader.cu:107-120).  Otherwise the stochastic blur of the
 * reference's resize branch (dataloader.cu:122-186, 299-322): each
 * destination element draws its source pixel from the block it covers with
 * its own PCG32 state, blur_state[c * plane + tiled index] (at least
 * channels x padded destination plane entries), which is advanced in place.
 * Asynchronous on `stream`. */
TGS_API int tgs_image_resize_u8(const uint8_t* src, int32_t src_width, int32_t src_height, int32_t channels,
                                void* dst, int32_t dst_dtype, int32_t dst_width, int32_t dst_height,
                                uint64_t* blur_state, tgs_stream_t stream);

/* blur_state[i] = (a << 32) | b, a and b the outputs 2i and 2i + 1 of
 * pcg32(seed, 1): DataLoaderBase::reset's initialisation (dataloader.cu:
 * 361-378, seed 0 there), computed in parallel by jumping ahead. */
TGS_API int tgs_image_blur_state_init(uint64_t* blur_state, int64_t n, uint64_t seed, tgs_stream_t stream);

/* ---------------------------------------------------- checkpoint / resume */

/* Counters that a resumed run needs besides the arrays. */
typedef struct TgsTrainState {
    uint64_t step;           /* training steps done (TrainingState::current_step) */
    uint64_t adam_step;      /* SimpleAdam's step count (bias correction) */
    uint64_t strategy_step;  /* the densification strategy's step count */
    TgsPcg32 rng;            /* the strategy's random stream */
} TgsTrainState;

/* Write the live rows (params->n) of the parameters, of both Adam moments
 * (exp_avg and exp_avg_sq both given, or both NULL) and of the
 * densification statistics (dens, may be NULL), with *state, to `path` (a
 * temporary file renamed over it when complete).  Device memory is read on
 * `stream`, which is synchronised.  The reference offers only a callback
 * hook for this (Orchestrator::set_checkpoint_callback,
 * tinygs/src/orchestrator.cu:291-293,433-435) and a PLY export of the
 * parameters (core/pointcloud.cpp:111); with this file a resumed run
 * continues bit for bit. */
TGS_API int tgs_checkpoint_save(const char* path, const TgsGaussians* params, const TgsGaussians* exp_avg,
                                const TgsGaussians* exp_avg_sq, const TgsDensificationInfo* dens,
                                const TgsTrainState* state, tgs_stream_t stream);

/* Header of a checkpoint: Gaussian count, SH degree, flags (bit 0 moments,
 * bit 1 densification statistics) and the counters.  Any pointer may be
 * NULL.  TGS_ERR_INVALID_ARGUMENT for a missing or foreign file. */
TGS_API int tgs_checkpoint_info(const char* path, int64_t* n, int32_t* sh_degree, uint32_t* flags,
                                TgsTrainState* state);

/* Read a checkpoint into arrays with room for `capacity` Gaussians
 * (TGS_ERR_CAPACITY if the file holds more).  exp_avg / exp_avg_sq / dens
 * may be NULL to skip those arrays; asking for arrays the file does not hold
 * is TGS_ERR_UNSUPPORTED.  The whole file is read and its hash checked
 * before device memory is written: a truncated or damaged file returns
 * TGS_ERR_INVALID_ARGUMENT and leaves the arrays as they were.  On success
 * params->n (and the moments' n) and params->sh_degree are set from the
 * file and *state (may be NULL) receives the counters; `stream` is
 * synchronised. */
TGS_API int tgs_checkpoint_load(const char* path, int64_t capacity, TgsGaussians* params, TgsGaussians* exp_avg,
                                TgsGaussians* exp_avg_sq, TgsDensificationInfo* dens, TgsTrainState* state,
                                tgs_stream_t stream);

/* -------------------------------------------------------------- optimizer */

/* Hyper-parameters, reference GaussianOptimizationParams + SimpleAdamParameters
 * (tinygs/include/tinygs/optim/optim.hpp:8-37, simple_adam.hpp:8-27). */
typedef struct TgsAdamConfig {
    float beta1;          /* 0.9   */
    float beta2;          /* 0.999 */
    float epsilon;        /* 1e-8  */
    float max_grad_1;     /* |g| clip per element, 0 disables (ref default 1) */
    float means_lr;       /* times scene_scale * global_lr                    */
    float shs_lr;         /* sh0: shs_lr*global_lr; sh_rest: *0.05 in addition */
    float opacities_lr;
    float scales_lr;
    float rotations_lr;
    float opacities_l1;   /* L1 decay on opacity (ref default 0)             */
    float scales_l1;      /* L1 decay on scale   (ref default 0)             */
    float scene_scale;
    float global_lr;
    int32_t decay_reduction_mean; /* 1: decay weights divided by n ("mean") */
} TgsAdamConfig;

/* One Adam step over all six parameter arrays in one launch.  Replaces
 * SimpleAdam::step_adam (tinygs/src/optim/simple_adam.cu:457-580):
 *   g = gradient_scale*grad (+ decay), clipped to +-max_grad_1,
 *   m = lerp(m, g, 1-b1), v = lerp(v, g^2, 1-b2),
 *   theta -= (m/bc1)*lr / (sqrt(v)/sqrt(bc2) + eps),
 * with bc1 = 1-b1^step and bc2 = 1-b2^step computed in double on the host.
 * `step` is the 1-based step count after increment (reference
 * m_global_steps).  m and v use the TgsGaussians layout.  If zero_grads != 0
 * the gradient arrays are zeroed in the same pass. */
TGS_API int tgs_adam_step(const TgsGaussians* params, const TgsGaussians* grads,
                  const TgsGaussians* exp_avg, const TgsGaussians* exp_avg_sq,
                  const TgsAdamConfig* cfg, uint32_t step,
                  float gradient_scale, int32_t zero_grads,
                  tgs_stream_t stream);

/* Backward and optimizer step in one pass: equal to
 *   tgs_raster_backward(accumulate = 0) into a gradient arena, followed by
 *   tgs_adam_step(..., zero_grads = 0)
 * (the reference's FastGSRasterizer::backward then SimpleAdam::step with a
 * single view per step, orchestrator.cu:373-403), but each Gaussian's 59
 * gradients go from the backward straight into its Adam update without being
 * stored and re-read.  `grads` may be NULL (no gradient output) or receive
 * the gradients as tgs_raster_backward would write them.  For several views
 * per step (accumulation or multi-GPU all-reduce) use the separate calls. */
TGS_API int tgs_raster_backward_adam(TgsRaster* r, const TgsGaussians* params,
                                     const TgsCamera* cam, int32_t dtype,
                                     const void* image, const void* grad_image,
                                     TgsGaussians* grads,
                                     const TgsGaussians* exp_avg,
                                     const TgsGaussians* exp_avg_sq,
                                     const TgsAdamConfig* cfg, uint32_t step,
                                     float gradient_scale,
                                     TgsDensificationInfo* dens,
                                     tgs_stream_t stream);

/* ------------------------------------------------------------------ misc */

/* Zero a Gaussian array set (the reference's m_gradients->memset(0),
 * tinygs/src/orchestrator.cu:351-353). */
TGS_API int tgs_gaussians_zero(const TgsGaussians* g, tgs_stream_t stream);

/* ------------------------------------------------------ rows of a set
 * Row operations on a set of Gaussian arrays (parameters, gradients or an
 * Adam moment).  None allocates; sets may not overlap unless stated. */

/* dst row i <- src row idx[i] for every array, i < n (idx on the device).
 * Replaces GPUGaussian3d::reorder (tinygs/src/core/gpu_gaussian.cu:273-311)
 * and SimpleAdam::reorder (tinygs/src/optim/simple_adam.cu:1036-1099),
 * which gather into newly allocated vectors; here into a caller-owned set. */
TGS_API int tgs_arena_gather(const TgsGaussians* src, TgsGaussians* dst, const uint32_t* idx, int64_t n,
                             tgs_stream_t stream);

/* Workspace of tgs_arena_keep_index / tgs_arena_compact for n rows. */
TGS_API int tgs_arena_compact_workspace_bytes(int64_t n, size_t* bytes);

/* Indices of the rows with keep[i] != 0, in increasing order, into idx_out;
 * their number into *n_kept (device).  The mapping step of
 * GPUGaussian3d::remove / SimpleAdam::remove (thrust::copy_if over a
 * counting iterator, gpu_gaussian.cu:117-160, simple_adam.cu:841-903). */
TGS_API int tgs_arena_keep_index(const uint8_t* keep, int64_t n, void* workspace, size_t workspace_bytes,
                                 uint32_t* idx_out, uint32_t* n_kept, tgs_stream_t stream);

/* Stable compaction: dst rows 0..*n_kept-1 <- the src rows with
 * keep[i] != 0, in order; *n_kept (device) receives their number.
 * Replaces GPUGaussian3d::remove and SimpleAdam::remove (same lines), which
 * reallocate every array; no host synchronisation. */
TGS_API int tgs_arena_compact(const TgsGaussians* src, TgsGaussians* dst, const uint8_t* keep, int64_t n,
                              void* workspace, size_t workspace_bytes, uint32_t* n_kept, tgs_stream_t stream);

/* Rows rows[0..count) of every array (segment == -1) or of one array
 * (segment 0..5: means, opacities, rotations, scales, sh0, sh_rest) set to
 * `value`.  SimpleAdam::reset(indices, n) zeroes both moments' rows
 * (simple_adam.cu:944-982); SimpleAdam::reset_opacity zeroes the opacity
 * moments (simple_adam.cu:984-987, a fill of segment 1). */
TGS_API int tgs_arena_fill_rows(TgsGaussians* set, const int32_t* rows, int64_t count, float value,
                                int32_t segment, tgs_stream_t stream);

/* dst[i] <- src[idx[i]] of the densification records (the gather of
 * Orchestrator::reorder_gaussians, tinygs/src/orchestrator.cu:1024-1036). */
TGS_API int tgs_dens_gather(const TgsDensificationInfo* src, TgsDensificationInfo* dst, const uint32_t* idx,
                            int64_t n, tgs_stream_t stream);

/* Workspace of tgs_morton_order for n Gaussians. */
TGS_API int tgs_morton_workspace_bytes(int64_t n, size_t* bytes);

/* The reference's Morton order (reorder(), tinygs/src/orchestrator.cu:26-100):
 * bounding box of the means, inverse extents 1/max(max-min, 1e-8) in IEEE
 * float, each coordinate normalised, clamped to [0, 1] and truncated to 10
 * bits (x 1023), a 30-bit Morton code (x in bits 3i, y 3i+1, z 3i+2), and a
 * stable sort by code.  perm[i] is the index of the Gaussian that moves to
 * row i (apply with tgs_arena_gather / tgs_dens_gather).  means: [n][3]. */
TGS_API int tgs_morton_order(const float* means, int64_t n, void* workspace, size_t workspace_bytes,
                             uint32_t* perm, tgs_stream_t stream);

/* Human-readable text for a status code (static storage). */
TGS_API const char* tgs_status_string(int status);

/* Library version string, e.g. "tinygs-b200 0.1 sm_100a". */
TGS_API const char* tgs_version(void);

/* ------------------------------------------------ multi-GPU (one process per GPU)
 * The reference trains on one GPU; several views per optimizer step are its
 * gradient accumulation (Orchestrator::train_step with accumulate_grad_steps,
 * orchestrator.cu:343-403).  Here the views of one step are rendered on
 * several GPUs and the accumulation + Adam is one kernel over NVLink peer
 * memory.  No counterpart functions in the reference. */
typedef struct TgsIpcHandle {
    char bytes[64];
} TgsIpcHandle;

/* Zeroed device memory another process can map (CUDA IPC). */
TGS_API int tgs_shared_alloc(size_t bytes, void** ptr, TgsIpcHandle* handle);
TGS_API int tgs_shared_free(void* ptr);
/* Maps another process's tgs_shared_alloc memory into this one. */
TGS_API int tgs_shared_open(const TgsIpcHandle* handle, void** peer_ptr);
TGS_API int tgs_shared_close(void* peer_ptr);

/* Rank `rank` of `world` (<= 8) owns the Gaussians [rank*n/world,
 * (rank+1)*n/world) (rounded to multiples of 4): it sums their gradients over
 * the ranks' gradient arenas (grads_per_rank[r], summed in rank order as the
 * reference's accumulation adds views), applies the Adam step of
 * tgs_adam_step with its own exp_avg / exp_avg_sq rows, and stores the new
 * parameters into every rank's parameter arena (params_per_rank[r]).  The
 * per-rank pointers must be valid in this process (tgs_shared_open).  The
 * caller orders the call after every rank's backward and before every
 * rank's next forward (for example with a collective on `stream`). */
TGS_API int tgs_dp_reduce_adam(const TgsGaussians* params_per_rank, const TgsGaussians* grads_per_rank,
                               int32_t world, int32_t rank, TgsGaussians* exp_avg,
                               TgsGaussians* exp_avg_sq, const TgsAdamConfig* cfg, uint32_t step,
                               float gradient_scale, tgs_stream_t stream);

/* tgs_dp_reduce_adam through NVLink SHARP: params_mc / grads_mc are the
 * multicast addresses of the parameter and gradient arenas (segment pointers
 * in the layout of `params`, e.g. from a multicast object bound to every
 * rank's arena); the slice's gradient sum is read with one reducing load
 * through the switch and the new parameters are stored to every rank with
 * one multicast store.  `params` are this rank's parameters (read).  For more
 * than two ranks the switch's summation order can change the last bit of the
 * summed gradient. */
TGS_API int tgs_dp_reduce_adam_multicast(const TgsGaussians* params_mc, const TgsGaussians* grads_mc,
                                         TgsGaussians* params, int32_t world, int32_t rank,
                                         TgsGaussians* exp_avg, TgsGaussians* exp_avg_sq,
                                         const TgsAdamConfig* cfg, uint32_t step, float gradient_scale,
                                         tgs_stream_t stream);

/* Gradient routing for several GPUs: the backward of tgs_raster_backward
 * (overwrite mode) with each Gaussian's gradients stored into the gradient
 * inbox of the rank whose slice holds it (inbox_per_rank[s], mapped into this
 * process), into slot `rank`, while the kernel computes them -- the transfer
 * the exchange would do afterwards overlaps the backward.  An inbox holds
 * `world` slots, each laid out like a parameter arena of `slice_pad`
 * Gaussians (segments back to back, slice_pad rows each); slices as in
 * tgs_dp_reduce_adam. */
TGS_API int tgs_raster_backward_routed(TgsRaster* r, const TgsGaussians* params, const TgsCamera* cam,
                                       int32_t dtype, const void* image, const void* grad_image,
                                       float* const* inbox_per_rank, int64_t slice_pad, int32_t world,
                                       int32_t rank, TgsDensificationInfo* dens, tgs_stream_t stream);

/* ---- owner-split data parallelism (no counterpart in the reference; its
 * accumulate_grad_steps = world, orchestrator.cu:343-403, with the views of
 * one optimizer step rendered on `world` GPUs).  Rank r owns the Gaussians
 * [first_r, last_r) -- their parameters and Adam moments -- and renders view
 * r.  Per step: every owner preprocesses its slice for every rank's view and
 * stores the screen-space records into that rank's handle
 * (tgs_raster_preprocess_views); after a collective, every rank bins and
 * blends its view from the records of all n Gaussians
 * (tgs_raster_forward_gathered), evaluates the loss and runs the blend
 * backward into its handle (tgs_raster_backward_screen); after a second
 * collective, every owner runs the per-Gaussian backward of its slice for
 * every view, reading the screen-space gradients from the views' handles,
 * sums them in view order and applies Adam (tgs_raster_backward_views_adam).
 * Only screen-space records and gradients cross NVLink, and nothing is
 * broadcast.  Every handle must have the same capacities; slice starts are
 * multiples of 256. */

/* Exports the handle's device memory for the other ranks (CUDA IPC; open it
 * with tgs_shared_open). */
TGS_API int tgs_raster_share(TgsRaster* r, TgsIpcHandle* out);
/* The handle's device memory in this process (for rank == this rank). */
TGS_API int tgs_raster_arena(TgsRaster* r, void** arena);
/* arenas[k]: rank k's handle memory valid in this process (this rank's own
 * from tgs_raster_arena, the others' from tgs_shared_open). */
TGS_API int tgs_raster_attach_views(TgsRaster* r, void* const* arenas, int32_t world, int32_t rank);
/* Preprocess of the Gaussians [first, last) for the `world` views cams[k],
 * each into rank k's handle (peer stores); dens (this owner's records,
 * may be NULL) takes the maximum screen radius over the views. */
TGS_API int tgs_raster_preprocess_views(TgsRaster* r, const TgsGaussians* params, const TgsCamera* cams,
                                        int32_t dtype, int64_t first, int64_t last, TgsDensificationInfo* dens,
                                        tgs_stream_t stream);
/* Binning and blending of this rank's view from the records of all n
 * Gaussians that the owners stored into this handle. */
TGS_API int tgs_raster_forward_gathered(TgsRaster* r, int64_t n, const TgsCamera* cam, int32_t dtype,
                                        void* image, void* alpha, tgs_stream_t stream);
/* Blend backward of this rank's view: per-Gaussian screen-space gradients
 * into this handle (absgrad != 0: also the absolute-gradient sums). */
TGS_API int tgs_raster_backward_screen(TgsRaster* r, const TgsCamera* cam, int32_t dtype, const void* image,
                                       const void* grad_image, int32_t absgrad, tgs_stream_t stream);
/* Per-Gaussian backward of the Gaussians [first, last) for the `world`
 * views (screen-space gradients read from the views' handles), summed in
 * view order on chip, then the Adam step of tgs_adam_step on those rows of
 * params / exp_avg / exp_avg_sq with the gradient sum -- one pass over the
 * slice.  grads (may be NULL) receives the sums of those rows.  dens (may
 * be NULL) accumulates over the views. */
TGS_API int tgs_raster_backward_views_adam(TgsRaster* r, const TgsGaussians* params, const TgsCamera* cams,
                                           int64_t first, int64_t last, TgsGaussians* grads,
                                           const TgsGaussians* exp_avg, const TgsGaussians* exp_avg_sq,
                                           const TgsAdamConfig* cfg, uint32_t step, float gradient_scale,
                                           TgsDensificationInfo* dens, tgs_stream_t stream);

/* The owner's half of the routed exchange: the slice's gradients are the sum
 * of this rank's inbox slots (local memory, rank order), then the Adam step
 * and the parameter stores into every rank as in tgs_dp_reduce_adam. */
TGS_API int tgs_dp_inbox_adam(const TgsGaussians* params_per_rank, const float* inbox, int64_t slice_pad,
                              int32_t world, int32_t rank, TgsGaussians* exp_avg, TgsGaussians* exp_avg_sq,
                              const TgsAdamConfig* cfg, uint32_t step, float gradient_scale,
                              tgs_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* TGS_ABI_H */
