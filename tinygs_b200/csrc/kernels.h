// kernels.h -- host-side launchers of the device kernels (internal interface
// between the C ABI in abi.cu and the kernel translation units).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "common.cuh"

namespace tgs {

struct GaussianPtrs {
  float* means;
  float* opacities;
  float* rotations;
  float* scales;
  float* sh0;
  float* sh_rest;
  int64_t n;
  int32_t sh_degree;
};

// Scratch of one rasterizer handle; every pointer is a device allocation
// sized at creation.
struct RasterState {
  int64_t cap_n = 0;        // Gaussians
  int64_t cap_inst = 0;     // instances
  int64_t cap_buckets = 0;  // 32-primitive buckets
  int32_t max_w = 0, max_h = 0;
  int64_t max_tiles = 0;
  int64_t max_pixels = 0;   // padded pixels

  // per Gaussian
  uint32_t* n_touched = nullptr;
  uint32_t* depth_key = nullptr;
  ushort4* bounds = nullptr;
  float2* mean2d = nullptr;
  float4* conic_opacity = nullptr;  // fp32 path; aliases prim_info storage
  PrimInfo16* prim_info = nullptr;  // fp16 path
  float* color = nullptr;           // [n][3] fp32 path
  float* helpers = nullptr;         // [n][12] backward scratch
  uint32_t* vis_key[2] = {nullptr, nullptr};
  uint32_t* vis_idx[2] = {nullptr, nullptr};
  uint32_t* block_sums = nullptr;   // block partial sums for scans
  // per (Gaussian, super-tile) entry
  int64_t cap_entries = 0;
  uint16_t* ent_key[2] = {nullptr, nullptr};   // super-tile id (double-buffered for the sort)
  uint32_t* ent_prim[2] = {nullptr, nullptr};
  uint32_t* masks = nullptr;                   // hit mask over the 8x4 tiles of the super-tile
  int ent_result = 0;
  // per super-tile and per chunk of its entries
  int64_t max_super = 0;
  int64_t cap_chunks = 0;
  uint2* super_ranges = nullptr;
  uint32_t* super_chunk = nullptr;   // first chunk of each super-tile
  uint4* chunks = nullptr;           // (super-tile, first entry, end entry)
  uint32_t* chunk_counts = nullptr;  // [chunk][32] hits per tile, then first-slot offsets
  uint32_t* sub_offsets = nullptr;   // [chunk][kSubChunks][32] slots of a sub-chunk's tile runs within its chunk
  // per instance, in final (tile, depth, index) order (the tile of an
  // instance follows from the tile ranges)
  uint32_t* inst_prim[2] = {nullptr, nullptr};  // only [0] is allocated
  // radix sort scratch
  uint32_t* sort_hist = nullptr;    // [256][sort_max_blocks]
  uint32_t* sort_digit_total = nullptr;  // [256]
  int64_t sort_max_blocks = 0;
  // per tile
  uint2* ranges = nullptr;
  uint32_t* tile_total = nullptr;
  uint32_t* bucket_offsets = nullptr;
  uint32_t* tile_max_contrib = nullptr;
  // per pixel
  uint32_t* n_contrib = nullptr;    // uint32 (fp32 path) or uint16 (fp16 path)
  // per bucket
  uint2* live_buckets = nullptr;    // (tile, bucket in tile) of the buckets the backward runs
  float4* ckpt = nullptr;           // [buckets][256] float4 (fp32) or uint2 (fp16)
  // counts
  DevCounts* counts = nullptr;
  uint32_t* bwd_work = nullptr;     // work counter of the persistent backward

  // state of the last forward
  int have_forward = 0;
  int last_dtype = 0;
  int64_t last_n = 0;
  uint32_t last_tile_passes = 0;  // parity of the tile sort result
  int depth_result = 0;           // which vis buffer holds the sorted list
  int tile_result = 0;            // which inst buffer holds the sorted list
  int num_sms = 148;
};

DevCamera make_camera(int width, int height, float fx, float fy, float cx, float cy,
                      float near_plane, float far_plane, const float w2c[16]);

// Scratch of the stable LSD radix sort (binning.cu): per-digit block counts
// [256][max_blocks] (max_blocks = ceil(capacity / kSortTileItems)) and the
// 256 digit totals.
struct SortScratch {
  uint32_t* hist;
  uint32_t* digit_total;
  int64_t max_blocks;
  int num_sms;
};

// Stable sort of (key, value) pairs by the low `total_bits` bits of the
// keys, 8 bits per pass; *count_ptr (device) pairs of at most `capacity`.
// The sorted pairs end in keys[result], vals[result].
void sort_pairs_u32(uint32_t* keys[2], uint32_t* vals[2], const uint32_t* count_ptr, int64_t capacity,
                    int total_bits, int& result, const SortScratch& ss, cudaStream_t stream);

// forward stages (preprocess.cu, binning.cu, blend.cu)
// zero_helpers == 0: the backward accumulators of the candidates are left
// for the caller to clear (the owner split clears them on the view's rank)
void launch_preprocess(const RasterState& s, const GaussianPtrs& g, const DevCamera& cam,
                       int fp16, float4* dens, cudaStream_t stream, int64_t first = 0, int64_t last = -1,
                       int zero_helpers = 1);
// Gaussians [first, last) projected into `count` views (cams[k], records
// into views[k]'s arena), taken in `order`; parameters read once.
// zero_helpers == 0 leaves the views' backward accumulators to their ranks
// (the owner split).  launch_preprocess is the one-view case.
void launch_preprocess_views(const RasterState* views, const DevCamera* cams, const int* order, int count,
                             const GaussianPtrs& g, int fp16, float4* dens, cudaStream_t stream, int64_t first,
                             int64_t last, int zero_helpers);
void launch_binning(RasterState& s, int64_t n, const DevCamera& cam, int fp16, cudaStream_t stream);
void launch_blend_forward(const RasterState& s, const DevCamera& cam, int fp16, void* image,
                          void* alpha, cudaStream_t stream);
// backward stages
// abs_grad: also accumulate sum |dL/dmean2d| (densification statistics)
void launch_blend_backward(const RasterState& s, const DevCamera& cam, int fp16, const void* image,
                           const void* grad_image, int abs_grad, cudaStream_t stream);
// Optimizer step fused into the preprocess backward (per-segment learning
// rate, decay kind and weight in the reference's segment order).
struct GradRoute;  // below: multi-GPU gradient routing
struct AdamStepArgs {
  float lr[6];
  float decay[6];
  int kind[6];
  float beta1, beta2, eps, gradient_scale, bc1, bc2_sqrt, max_grad_1;
};
// adam == nullptr: gradients written to `grads` (+= if accumulate).
// adam != nullptr: Adam applied to g/exp_avg/exp_avg_sq; grads written only
// where its pointers are non-null.
void launch_preprocess_backward(const RasterState& s, const GaussianPtrs& g,
                                const GaussianPtrs& grads, const DevCamera& cam, int accumulate,
                                float4* dens, cudaStream_t stream, const GaussianPtrs* exp_avg = nullptr,
                                const GaussianPtrs* exp_avg_sq = nullptr, const AdamStepArgs* adam = nullptr,
                                const GradRoute* route = nullptr, int64_t first = 0, int64_t last = -1);
// Owner split: Gaussians [first, last) back-propagated through the views of
// all `world` ranks (views[k]: rank k's handle state, cams[k] its camera),
// summed in view order, then Adam; grads (may be null) receives the sums.
void launch_views_backward_adam(const RasterState* const* views, const DevCamera* cams, int world,
                                const GaussianPtrs& g, const GaussianPtrs* grads, const GaussianPtrs& exp_avg,
                                const GaussianPtrs& exp_avg_sq, const AdamStepArgs& adam, float4* dens,
                                cudaStream_t stream, int64_t first, int64_t last);

// losses (loss.cu)
void launch_l1(int fp16, int width, int height, const void* pred, const void* target,
               void* loss_map, void* grad, float scale, cudaStream_t stream);
void launch_ssim(int fp16, int width, int height, const void* pred, const void* target,
                 void* loss_map, void* grad, float scale_ssim, float scale_l1, float* partials,
                 float* loss_sum, cudaStream_t stream, int accumulate = 1);

// data-parallel Adam over peer memory (adam.cu): params/grads hold one
// entry per rank (pointers valid in this process)
constexpr int kMaxDpRanks = 8;
// First Gaussian of rank r's slice (multiples of four, so every slice's rows
// start 16-byte aligned); dp_slice_begin(n, world, world) == n.
inline int64_t dp_slice_begin(int64_t n, int world, int r) {
  return r >= world ? n : (n * r / world) / 4 * 4;
}
// grads_are_slices: grads[r] hold only this rank's slice (row 0 = the
// slice's first Gaussian), as in the gradient inbox
void launch_dp_adam(const GaussianPtrs* params, const GaussianPtrs* grads, int world, int rank,
                    const GaussianPtrs& m, const GaussianPtrs& v, const AdamStepArgs& adam, cudaStream_t stream,
                    bool grads_are_slices = false);
// Gradient routing of the per-Gaussian backward: Gaussian i's gradients go
// to the inbox of the rank whose slice holds it, into slot `rank`.  An inbox
// holds `world` slots, each laid out like a parameter arena of `slice_pad`
// Gaussians.
struct GradRoute {
  float* inbox[kMaxDpRanks];
  int64_t lo[kMaxDpRanks + 1];
  int64_t slice_pad;
  int world, rank;
};

// the same over the multicast addresses of the gradient and parameter
// arenas (NVLink SHARP); `own` are this rank's parameters
void launch_dp_adam_mc(const GaussianPtrs& params_mc, const GaussianPtrs& grads_mc, const GaussianPtrs& own,
                       int world, int rank, const GaussianPtrs& m, const GaussianPtrs& v, const AdamStepArgs& adam,
                       cudaStream_t stream);

// optimizer (adam.cu)
struct AdamSegment {
  float* theta;
  const float* grad;
  float* m;
  float* v;
  int64_t count;
  float lr;
  int decay_kind;  // 0 none, 1 opacity, 2 scale
  float decay;
};
void launch_adam(const AdamSegment* segs, int n_segs, float beta1, float beta2, float eps,
                 float gradient_scale, float bc1, float bc2_sqrt, float max_grad_1,
                 int zero_grads, cudaStream_t stream);

}  // namespace tgs
