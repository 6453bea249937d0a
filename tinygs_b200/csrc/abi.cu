// abi.cu -- the extern "C" boundary (include/tgs_abi.h).  Validates
// arguments, owns the per-handle scratch arena and sequences the kernels on
// the caller's stream.  No entry point allocates after handle creation and
// none synchronises the host except tgs_raster_counts.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>

#include "../../include/tgs_abi.h"
#include "kernels.h"

namespace tgs {

DevCamera make_camera(int width, int height, float fx, float fy, float cx, float cy, float near_plane,
                      float far_plane, const float w2c[16]) {
  DevCamera c{};
  c.r1 = make_float4(w2c[0], w2c[1], w2c[2], w2c[3]);
  c.r2 = make_float4(w2c[4], w2c[5], w2c[6], w2c[7]);
  c.r3 = make_float4(w2c[8], w2c[9], w2c[10], w2c[11]);
  // camera centre = translation of inverse(w2c), evaluated in double
  // (the reference takes c2w[3] of glm::inverse(w2c), fastgs.cu:97-100)
  double r[3][3], t[3];
  for (int i = 0; i < 3; ++i) {
    for (int j = 0; j < 3; ++j) r[i][j] = w2c[4 * i + j];
    t[i] = w2c[4 * i + 3];
  }
  const double c00 = r[1][1] * r[2][2] - r[1][2] * r[2][1];
  const double c01 = r[1][2] * r[2][0] - r[1][0] * r[2][2];
  const double c02 = r[1][0] * r[2][1] - r[1][1] * r[2][0];
  const double det = r[0][0] * c00 + r[0][1] * c01 + r[0][2] * c02;
  double inv[3][3];
  inv[0][0] = c00 / det;
  inv[0][1] = (r[0][2] * r[2][1] - r[0][1] * r[2][2]) / det;
  inv[0][2] = (r[0][1] * r[1][2] - r[0][2] * r[1][1]) / det;
  inv[1][0] = c01 / det;
  inv[1][1] = (r[0][0] * r[2][2] - r[0][2] * r[2][0]) / det;
  inv[1][2] = (r[0][2] * r[1][0] - r[0][0] * r[1][2]) / det;
  inv[2][0] = c02 / det;
  inv[2][1] = (r[0][1] * r[2][0] - r[0][0] * r[2][1]) / det;
  inv[2][2] = (r[0][0] * r[1][1] - r[0][1] * r[1][0]) / det;
  float pos[3];
  for (int i = 0; i < 3; ++i) pos[i] = static_cast<float>(-(inv[i][0] * t[0] + inv[i][1] * t[1] + inv[i][2] * t[2]));
  c.pos = make_float3(pos[0], pos[1], pos[2]);
  c.fx = fx;
  c.fy = fy;
  c.cx = cx;
  c.cy = cy;
  c.near_plane = near_plane;
  c.far_plane = far_plane;
  c.w = static_cast<float>(width);
  c.h = static_cast<float>(height);
  c.width = static_cast<uint32_t>(width);
  c.height = static_cast<uint32_t>(height);
  c.grid_w = (c.width + kTile - 1) / kTile;
  c.grid_h = (c.height + kTile - 1) / kTile;
  c.tiled_w = (c.width + 7u) >> 3;
  c.tiled_h = (c.height + 7u) >> 3;
  c.plane = c.tiled_w * c.tiled_h * 64u;
  return c;
}

}  // namespace tgs

using namespace tgs;

struct TgsRaster {
  RasterState s;
  void* arena = nullptr;
  size_t arena_bytes = 0;
  int device = 0;
  // owner-split data parallelism: the arenas of every rank's handle (same
  // capacities, hence the same layout), valid in this process
  char* peer_arena[kMaxDpRanks] = {};
  int world = 1, rank = 0;
  // stage timing (profiling only): events between the stages
  bool timing = false;
  cudaEvent_t ev[7] = {};
  bool fwd_timed = false, bwd_timed = false;
};

namespace {
void mark(TgsRaster* r, int k, cudaStream_t st) {
  if (r->timing) cudaEventRecord(r->ev[k], st);
}
}  // namespace

struct TgsLoss {
  float* partials = nullptr;
  int32_t max_w = 0, max_h = 0;
  int32_t accumulate = 1;  // tgs_loss_l1_ssim adds into loss_map / grad
};

namespace {

GaussianPtrs to_ptrs(const TgsGaussians* g) {
  GaussianPtrs p;
  p.means = g->means;
  p.opacities = g->opacities;
  p.rotations = g->rotations;
  p.scales = g->scales;
  p.sh0 = g->sh0;
  p.sh_rest = g->sh_rest;
  p.n = g->n;
  p.sh_degree = g->sh_degree;
  return p;
}

bool gaussians_ok(const TgsGaussians* g) {
  if (g == nullptr || g->n < 0) return false;
  if (g->n == 0) return true;
  return g->means && g->opacities && g->rotations && g->scales && g->sh0 && g->sh_rest && g->sh_degree >= 0 &&
         g->sh_degree <= 3 && (reinterpret_cast<uintptr_t>(g->rotations) & 15u) == 0;
}

bool camera_ok(const TgsCamera* c) {
  return c != nullptr && c->width > 0 && c->height > 0 && std::isfinite(c->fx) && std::isfinite(c->fy) &&
         c->fx != 0.f && c->fy != 0.f;
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? TGS_OK : TGS_ERR_CUDA; }

// Bump allocator over one device allocation.
struct Carver {
  char* base;
  size_t off = 0;
  template <typename T>
  T* take(size_t count) {
    off = (off + 255u) & ~static_cast<size_t>(255u);
    T* p = reinterpret_cast<T*>(base ? base + off : nullptr);
    off += count * sizeof(T);
    return p;
  }
};

void carve(RasterState& s, char* base, size_t& bytes) {
  Carver c{base};
  const size_t n = static_cast<size_t>(s.cap_n > 0 ? s.cap_n : 1);
  const size_t ni = static_cast<size_t>(s.cap_inst > 0 ? s.cap_inst : 1);
  const size_t nb = static_cast<size_t>(s.cap_buckets > 0 ? s.cap_buckets : 1);
  const size_t nt = static_cast<size_t>(s.max_tiles);
  const size_t np = static_cast<size_t>(s.max_pixels);
  s.n_touched = c.take<uint32_t>(n);
  s.depth_key = c.take<uint32_t>(n);
  s.bounds = c.take<ushort4>(n);
  s.mean2d = c.take<float2>(n);
  s.conic_opacity = c.take<float4>(n);
  s.prim_info = reinterpret_cast<PrimInfo16*>(s.conic_opacity);
  s.color = c.take<float>(3 * n);
  s.helpers = c.take<float>(kHelperFloats * n);
  s.vis_key[0] = c.take<uint32_t>(n);
  s.vis_key[1] = c.take<uint32_t>(n);
  s.vis_idx[0] = c.take<uint32_t>(n);
  s.vis_idx[1] = c.take<uint32_t>(n);
  s.block_sums = c.take<uint32_t>((n + 255) / 256 + 1);
  s.inst_prim[0] = c.take<uint32_t>(ni);
  const size_t ne = static_cast<size_t>(s.cap_entries > 0 ? s.cap_entries : 1);
  const size_t ns = static_cast<size_t>(s.max_super);
  s.ent_key[0] = c.take<uint16_t>(ne);
  s.ent_key[1] = c.take<uint16_t>(ne);
  s.ent_prim[0] = c.take<uint32_t>(ne);
  s.ent_prim[1] = c.take<uint32_t>(ne);
  s.masks = c.take<uint32_t>(ne);
  s.super_ranges = c.take<uint2>(ns);
  s.super_chunk = c.take<uint32_t>(ns);
  s.cap_chunks = static_cast<int64_t>(ne / kChunk + ns + 1);
  s.chunks = c.take<uint4>(static_cast<size_t>(s.cap_chunks));
  s.chunk_counts = c.take<uint32_t>(static_cast<size_t>(s.cap_chunks) * kSuperTiles);
  s.sub_offsets = c.take<uint32_t>(static_cast<size_t>(s.cap_chunks) * kSubChunks * kSuperTiles);
  s.tile_total = c.take<uint32_t>(nt);
  s.sort_max_blocks = static_cast<int64_t>((std::max(n, ne) + kSortTileItems - 1) / kSortTileItems);
  s.sort_hist = c.take<uint32_t>(256 * static_cast<size_t>(s.sort_max_blocks));
  s.sort_digit_total = c.take<uint32_t>(256);
  s.ranges = c.take<uint2>(nt);
  s.bucket_offsets = c.take<uint32_t>(nt);
  s.tile_max_contrib = c.take<uint32_t>(nt);
  s.n_contrib = c.take<uint32_t>(np);
  s.live_buckets = c.take<uint2>(nb);
  s.ckpt = c.take<float4>(nb * kTilePixels);
  s.counts = c.take<DevCounts>(1);
  s.bwd_work = c.take<uint32_t>(4);
  bytes = c.off + 256;
}

// Per-segment learning rates and decays of SimpleAdam::step_adam
// (simple_adam.cu:468-577), segment order means, opacities, rotations,
// scales, sh0, sh_rest; the higher SH bands use 0.05 * shs_lr (line 19, 571).
void adam_segments(const TgsAdamConfig* cfg, int64_t n, uint32_t step, float gradient_scale, AdamStepArgs* out) {
  const float g_scale = cfg->decay_reduction_mean ? 1.0f / static_cast<float>(n) : 1.0f;
  const float op_decay = cfg->opacities_l1 * g_scale, sc_decay = cfg->scales_l1 * g_scale;
  const float lr[6] = {cfg->means_lr * cfg->scene_scale * cfg->global_lr, cfg->opacities_lr * cfg->global_lr,
                       cfg->rotations_lr * cfg->global_lr,               cfg->scales_lr * cfg->global_lr,
                       cfg->shs_lr * cfg->global_lr,                     cfg->shs_lr * 0.05f * cfg->global_lr};
  for (int k = 0; k < 6; ++k) {
    out->lr[k] = lr[k];
    out->decay[k] = 0.f;
    out->kind[k] = 0;
  }
  if (op_decay != 0.f) {
    out->kind[1] = 1;
    out->decay[1] = op_decay;
  }
  if (sc_decay != 0.f) {
    out->kind[3] = 2;
    out->decay[3] = sc_decay;
  }
  out->beta1 = cfg->beta1;
  out->beta2 = cfg->beta2;
  out->eps = cfg->epsilon;
  out->gradient_scale = gradient_scale;
  out->bc1 = static_cast<float>(1.0 - std::pow(static_cast<double>(cfg->beta1), static_cast<double>(step)));
  out->bc2_sqrt =
      static_cast<float>(std::sqrt(1.0 - std::pow(static_cast<double>(cfg->beta2), static_cast<double>(step))));
  out->max_grad_1 = cfg->max_grad_1;
}

}  // namespace

extern "C" {

const char* tgs_status_string(int status) {
  switch (status) {
    case TGS_OK: return "ok";
    case TGS_ERR_INVALID_ARGUMENT: return "invalid argument";
    case TGS_ERR_CUDA: return "CUDA error";
    case TGS_ERR_CAPACITY: return "capacity exceeded";
    case TGS_ERR_OUT_OF_MEMORY: return "out of device memory";
    case TGS_ERR_NO_FORWARD: return "backward without a matching forward";
    case TGS_ERR_UNSUPPORTED: return "unsupported";
    case TGS_ERR_DEVICE_TIMEOUT: return "device wait timed out";
    default: return "unknown status";
  }
}

const char* tgs_version(void) { return "tinygs-b200 0.1 sm_100a"; }

int tgs_raster_create(const TgsRasterCaps* caps, TgsRaster** out) {
  if (caps == nullptr || out == nullptr || caps->max_gaussians < 0 || caps->max_width <= 0 ||
      caps->max_height <= 0 || caps->max_instances < 0)
    return TGS_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  const int64_t gw = (caps->max_width + kTile - 1) / kTile, gh = (caps->max_height + kTile - 1) / kTile;
  if (gw * gh > 65535) return TGS_ERR_UNSUPPORTED;  // 16-bit tile ids
  if (caps->max_gaussians > 0x7fffffffLL) return TGS_ERR_UNSUPPORTED;
  TgsRaster* r = new (std::nothrow) TgsRaster();
  if (r == nullptr) return TGS_ERR_OUT_OF_MEMORY;
  RasterState& s = r->s;
  s.cap_n = caps->max_gaussians;
  s.cap_inst = caps->max_instances > 0 ? caps->max_instances : 16 * std::max<int64_t>(caps->max_gaussians, 1);
  if (s.cap_inst > 0x7fffffffLL) s.cap_inst = 0x7fffffffLL;
  s.max_w = caps->max_width;
  s.max_h = caps->max_height;
  s.max_tiles = gw * gh;
  s.cap_buckets = s.cap_inst / kBucket + s.max_tiles;
  // (Gaussian, super-tile) entries: at least one per Gaussian, about 1.5 in
  // typical scenes; each entry with a hit carries at least one instance
  s.cap_entries = std::min<int64_t>(0x7fffffffLL, 2 * std::max<int64_t>(s.cap_n, 1) + s.cap_inst / 2);
  s.max_super = ((gw + kSuperW - 1) / kSuperW) * ((gh + kSuperH - 1) / kSuperH);
  s.max_pixels = static_cast<int64_t>((caps->max_width + 7) / 8 * 8) * ((caps->max_height + 7) / 8 * 8);
  cudaGetDevice(&r->device);
  cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, r->device);
  size_t bytes = 0;
  carve(s, nullptr, bytes);
  void* mem = nullptr;
  if (cudaMalloc(&mem, bytes) != cudaSuccess) {
    cudaGetLastError();
    delete r;
    return TGS_ERR_OUT_OF_MEMORY;
  }
  r->arena = mem;
  r->arena_bytes = bytes;
  carve(s, static_cast<char*>(mem), bytes);
  if (cudaMemset(s.counts, 0, sizeof(DevCounts)) != cudaSuccess) {
    cudaFree(mem);
    delete r;
    return TGS_ERR_CUDA;
  }
  *out = r;
  return TGS_OK;
}

int tgs_raster_destroy(TgsRaster* r) {
  if (r == nullptr) return TGS_ERR_INVALID_ARGUMENT;
  int st = TGS_OK;
  for (cudaEvent_t e : r->ev)
    if (e != nullptr) cudaEventDestroy(e);
  if (r->arena != nullptr) st = cuda_status(cudaFree(r->arena));
  delete r;
  return st;
}

int tgs_raster_workspace_bytes(const TgsRaster* r, size_t* bytes) {
  if (r == nullptr || bytes == nullptr) return TGS_ERR_INVALID_ARGUMENT;
  *bytes = r->arena_bytes;
  return TGS_OK;
}

int tgs_raster_forward(TgsRaster* r, const TgsGaussians* params, const TgsCamera* cam, int32_t dtype, void* image,
                       void* alpha, TgsDensificationInfo* dens, tgs_stream_t stream) {
  if (r == nullptr || !gaussians_ok(params) || !camera_ok(cam) || image == nullptr) return TGS_ERR_INVALID_ARGUMENT;
  if (dtype != TGS_FLOAT32 && dtype != TGS_FLOAT16) return TGS_ERR_INVALID_ARGUMENT;
  RasterState& s = r->s;
  if (params->n > s.cap_n || cam->width > s.max_w || cam->height > s.max_h) return TGS_ERR_CAPACITY;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const DevCamera dc = make_camera(cam->width, cam->height, cam->fx, cam->fy, cam->cx, cam->cy, cam->near_plane,
                                   cam->far_plane, cam->w2c);
  const GaussianPtrs g = to_ptrs(params);
  cudaMemsetAsync(s.counts, 0, sizeof(DevCounts), st);
  s.have_forward = 0;
  mark(r, 0, st);
  if (g.n > 0) launch_preprocess(s, g, dc, dtype == TGS_FLOAT16, reinterpret_cast<float4*>(dens), st);
  mark(r, 1, st);
  launch_binning(s, g.n, dc, dtype == TGS_FLOAT16, st);
  mark(r, 2, st);
  launch_blend_forward(s, dc, dtype == TGS_FLOAT16, image, alpha, st);
  mark(r, 3, st);
  r->fwd_timed = r->timing;
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return TGS_ERR_CUDA;
  s.have_forward = 1;
  s.last_dtype = dtype;
  s.last_n = g.n;
  return TGS_OK;
}

int tgs_raster_backward(TgsRaster* r, const TgsGaussians* params, const TgsCamera* cam, int32_t dtype,
                        const void* image, const void* grad_image, TgsGaussians* grads, int32_t accumulate,
                        TgsDensificationInfo* dens, tgs_stream_t stream) {
  if (r == nullptr || !gaussians_ok(params) || !camera_ok(cam) || image == nullptr || grad_image == nullptr ||
      !gaussians_ok(grads))
    return TGS_ERR_INVALID_ARGUMENT;
  RasterState& s = r->s;
  if (!s.have_forward || s.last_dtype != dtype || s.last_n != params->n || grads->n != params->n)
    return TGS_ERR_NO_FORWARD;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const DevCamera dc = make_camera(cam->width, cam->height, cam->fx, cam->fy, cam->cx, cam->cy, cam->near_plane,
                                   cam->far_plane, cam->w2c);
  mark(r, 4, st);
  launch_blend_backward(s, dc, dtype == TGS_FLOAT16, image, grad_image, dens != nullptr, st);
  mark(r, 5, st);
  if (params->n > 0)
    launch_preprocess_backward(s, to_ptrs(params), to_ptrs(grads), dc, accumulate, reinterpret_cast<float4*>(dens),
                               st);
  mark(r, 6, st);
  r->bwd_timed = r->timing;
  return cuda_status(cudaGetLastError());
}

int tgs_raster_backward_adam(TgsRaster* r, const TgsGaussians* params, const TgsCamera* cam, int32_t dtype,
                             const void* image, const void* grad_image, TgsGaussians* grads,
                             const TgsGaussians* exp_avg, const TgsGaussians* exp_avg_sq, const TgsAdamConfig* cfg,
                             uint32_t step, float gradient_scale, TgsDensificationInfo* dens, tgs_stream_t stream) {
  if (r == nullptr || !gaussians_ok(params) || !camera_ok(cam) || image == nullptr || grad_image == nullptr ||
      !gaussians_ok(exp_avg) || !gaussians_ok(exp_avg_sq) || cfg == nullptr || step == 0 ||
      (grads != nullptr && !gaussians_ok(grads)))
    return TGS_ERR_INVALID_ARGUMENT;
  RasterState& s = r->s;
  if (!s.have_forward || s.last_dtype != dtype || s.last_n != params->n || exp_avg->n != params->n ||
      exp_avg_sq->n != params->n || (grads != nullptr && grads->n != params->n))
    return TGS_ERR_NO_FORWARD;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const DevCamera dc = make_camera(cam->width, cam->height, cam->fx, cam->fy, cam->cx, cam->cy, cam->near_plane,
                                   cam->far_plane, cam->w2c);
  mark(r, 4, st);
  launch_blend_backward(s, dc, dtype == TGS_FLOAT16, image, grad_image, dens != nullptr, st);
  mark(r, 5, st);
  if (params->n > 0) {
    AdamStepArgs a{};
    adam_segments(cfg, params->n, step, gradient_scale, &a);
    GaussianPtrs none{};
    none.n = params->n;
    const GaussianPtrs gp = grads != nullptr ? to_ptrs(grads) : none;
    const GaussianPtrs m = to_ptrs(exp_avg), v = to_ptrs(exp_avg_sq);
    launch_preprocess_backward(s, to_ptrs(params), gp, dc, 0, reinterpret_cast<float4*>(dens), st, &m, &v, &a);
  }
  mark(r, 6, st);
  r->bwd_timed = r->timing;
  return cuda_status(cudaGetLastError());
}

int tgs_raster_set_stage_timing(TgsRaster* r, int32_t enable) {
  if (r == nullptr) return TGS_ERR_INVALID_ARGUMENT;
  if (enable && r->ev[0] == nullptr)
    for (cudaEvent_t& e : r->ev)
      if (cudaEventCreate(&e) != cudaSuccess) return TGS_ERR_CUDA;
  r->timing = enable != 0;
  r->fwd_timed = r->bwd_timed = false;
  return TGS_OK;
}

int tgs_raster_stage_times(TgsRaster* r, float* out) {
  if (r == nullptr || out == nullptr) return TGS_ERR_INVALID_ARGUMENT;
  for (int k = 0; k < 5; ++k) out[k] = 0.f;
  if (r->fwd_timed) {
    if (cudaEventSynchronize(r->ev[3]) != cudaSuccess) return TGS_ERR_CUDA;
    for (int k = 0; k < 3; ++k) cudaEventElapsedTime(&out[k], r->ev[k], r->ev[k + 1]);
  }
  if (r->bwd_timed) {
    if (cudaEventSynchronize(r->ev[6]) != cudaSuccess) return TGS_ERR_CUDA;
    cudaEventElapsedTime(&out[3], r->ev[4], r->ev[5]);
    cudaEventElapsedTime(&out[4], r->ev[5], r->ev[6]);
  }
  return TGS_OK;
}

int tgs_raster_counts(TgsRaster* r, TgsRasterCounts* out, tgs_stream_t stream) {
  if (r == nullptr || out == nullptr) return TGS_ERR_INVALID_ARGUMENT;
  DevCounts h{};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(&h, r->s.counts, sizeof(DevCounts), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return TGS_ERR_CUDA;
  out->n_visible = h.n_visible;
  out->n_instances = h.n_instances;
  out->n_buckets = h.n_buckets;
  out->overflow = h.overflow;
  return TGS_OK;
}

int tgs_raster_debug_buffer(TgsRaster* r, int32_t which, void** dev_ptr, size_t* bytes) {
  if (r == nullptr || dev_ptr == nullptr || bytes == nullptr) return TGS_ERR_INVALID_ARGUMENT;
  RasterState& s = r->s;
  const size_t n = static_cast<size_t>(s.cap_n);
  switch (which) {
    case 0: *dev_ptr = s.n_touched; *bytes = 4 * n; break;
    case 2: *dev_ptr = s.inst_prim[s.tile_result]; *bytes = 4 * static_cast<size_t>(s.cap_inst); break;
    case 3: *dev_ptr = s.ranges; *bytes = 8 * static_cast<size_t>(s.max_tiles); break;
    case 4: *dev_ptr = s.n_contrib; *bytes = 4 * static_cast<size_t>(s.max_pixels); break;
    case 5: *dev_ptr = s.mean2d; *bytes = 8 * n; break;
    case 6: *dev_ptr = s.conic_opacity; *bytes = 16 * n; break;
    case 7: *dev_ptr = s.color; *bytes = 12 * n; break;
    case 8: *dev_ptr = s.prim_info; *bytes = 16 * n; break;
    case 9: *dev_ptr = s.bounds; *bytes = 8 * n; break;
    case 10: *dev_ptr = s.vis_idx[s.depth_result]; *bytes = 4 * n; break;
    case 11: *dev_ptr = s.helpers; *bytes = 4 * kHelperFloats * n; break;
    case 12: *dev_ptr = s.tile_max_contrib; *bytes = 4 * static_cast<size_t>(s.max_tiles); break;
    case 13: *dev_ptr = s.bucket_offsets; *bytes = 4 * static_cast<size_t>(s.max_tiles); break;
    case 14: *dev_ptr = s.depth_key; *bytes = 4 * n; break;
    case 15: *dev_ptr = s.ckpt; *bytes = 16 * kTilePixels * static_cast<size_t>(s.cap_buckets); break;
    default: return TGS_ERR_INVALID_ARGUMENT;
  }
  return TGS_OK;
}

int tgs_loss_l1(int32_t dtype, int32_t width, int32_t height, const void* pred, const void* target, void* loss_map,
                void* grad, float scale, tgs_stream_t stream) {
  if ((dtype != TGS_FLOAT32 && dtype != TGS_FLOAT16) || width <= 0 || height <= 0 || pred == nullptr ||
      target == nullptr)
    return TGS_ERR_INVALID_ARGUMENT;
  launch_l1(dtype == TGS_FLOAT16, width, height, pred, target, loss_map, grad, scale,
            static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError());
}

int tgs_loss_create(int32_t max_width, int32_t max_height, TgsLoss** out) {
  if (out == nullptr || max_width <= 0 || max_height <= 0) return TGS_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  TgsLoss* l = new (std::nothrow) TgsLoss();
  if (l == nullptr) return TGS_ERR_OUT_OF_MEMORY;
  const size_t px = static_cast<size_t>((max_width + 7) / 8 * 8) * ((max_height + 7) / 8 * 8);
  if (cudaMalloc(&l->partials, sizeof(float) * 9 * px) != cudaSuccess) {
    cudaGetLastError();
    delete l;
    return TGS_ERR_OUT_OF_MEMORY;
  }
  l->max_w = max_width;
  l->max_h = max_height;
  *out = l;
  return TGS_OK;
}

int tgs_loss_destroy(TgsLoss* l) {
  if (l == nullptr) return TGS_ERR_INVALID_ARGUMENT;
  const int st = cuda_status(cudaFree(l->partials));
  delete l;
  return st;
}

int tgs_loss_fused_ssim(TgsLoss* l, int32_t dtype, int32_t width, int32_t height, const void* pred,
                        const void* target, void* loss_map, void* grad, float scale, tgs_stream_t stream) {
  if (l == nullptr || (dtype != TGS_FLOAT32 && dtype != TGS_FLOAT16) || width <= 0 || height <= 0 ||
      pred == nullptr || target == nullptr || loss_map == nullptr)
    return TGS_ERR_INVALID_ARGUMENT;
  if (width > l->max_w || height > l->max_h) return TGS_ERR_CAPACITY;
  launch_ssim(dtype == TGS_FLOAT16, width, height, pred, target, loss_map, grad, scale, 0.0f, l->partials, nullptr,
              static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError());
}

int tgs_loss_l1_ssim(TgsLoss* l, int32_t dtype, int32_t width, int32_t height, const void* pred,
                     const void* target, void* loss_map, void* grad, float scale_l1, float scale_ssim,
                     float* loss_sum, tgs_stream_t stream) {
  if (l == nullptr || (dtype != TGS_FLOAT32 && dtype != TGS_FLOAT16) || width <= 0 || height <= 0 ||
      pred == nullptr || target == nullptr)
    return TGS_ERR_INVALID_ARGUMENT;
  if (width > l->max_w || height > l->max_h) return TGS_ERR_CAPACITY;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (loss_sum != nullptr) cudaMemsetAsync(loss_sum, 0, sizeof(float), st);
  if (scale_l1 == 0.0f && scale_ssim == 0.0f && l->accumulate) return cuda_status(cudaGetLastError());
  launch_ssim(dtype == TGS_FLOAT16, width, height, pred, target, loss_map, grad, scale_ssim, scale_l1, l->partials,
              loss_sum, st, l->accumulate);
  return cuda_status(cudaGetLastError());
}

int tgs_loss_set_accumulate(TgsLoss* l, int32_t accumulate) {
  if (l == nullptr) return TGS_ERR_INVALID_ARGUMENT;
  l->accumulate = accumulate != 0 ? 1 : 0;
  return TGS_OK;
}

int tgs_adam_step(const TgsGaussians* params, const TgsGaussians* grads, const TgsGaussians* exp_avg,
                  const TgsGaussians* exp_avg_sq, const TgsAdamConfig* cfg, uint32_t step, float gradient_scale,
                  int32_t zero_grads, tgs_stream_t stream) {
  if (!gaussians_ok(params) || !gaussians_ok(grads) || !gaussians_ok(exp_avg) || !gaussians_ok(exp_avg_sq) ||
      cfg == nullptr || step == 0)
    return TGS_ERR_INVALID_ARGUMENT;
  const int64_t n = params->n;
  if (grads->n != n || exp_avg->n != n || exp_avg_sq->n != n) return TGS_ERR_INVALID_ARGUMENT;
  if (n == 0) return TGS_OK;
  const float bc1 = static_cast<float>(1.0 - std::pow(static_cast<double>(cfg->beta1), static_cast<double>(step)));
  const float bc2 =
      static_cast<float>(std::sqrt(1.0 - std::pow(static_cast<double>(cfg->beta2), static_cast<double>(step))));
  const float g_scale = cfg->decay_reduction_mean ? 1.0f / static_cast<float>(n) : 1.0f;
  const float op_decay = cfg->opacities_l1 * g_scale, sc_decay = cfg->scales_l1 * g_scale;
  AdamSegment seg[6] = {
      {params->means, grads->means, exp_avg->means, exp_avg_sq->means, 3 * n,
       cfg->means_lr * cfg->scene_scale * cfg->global_lr, 0, 0.f},
      {params->opacities, grads->opacities, exp_avg->opacities, exp_avg_sq->opacities, n,
       cfg->opacities_lr * cfg->global_lr, op_decay != 0.f ? 1 : 0, op_decay},
      {params->rotations, grads->rotations, exp_avg->rotations, exp_avg_sq->rotations, 4 * n,
       cfg->rotations_lr * cfg->global_lr, 0, 0.f},
      {params->scales, grads->scales, exp_avg->scales, exp_avg_sq->scales, 3 * n, cfg->scales_lr * cfg->global_lr,
       sc_decay != 0.f ? 2 : 0, sc_decay},
      {params->sh0, grads->sh0, exp_avg->sh0, exp_avg_sq->sh0, 3 * n, cfg->shs_lr * cfg->global_lr, 0, 0.f},
      // the reference scales the higher SH bands' rate by 0.05 (simple_adam.cu:19,571)
      {params->sh_rest, grads->sh_rest, exp_avg->sh_rest, exp_avg_sq->sh_rest, 45 * n,
       cfg->shs_lr * 0.05f * cfg->global_lr, 0, 0.f},
  };
  launch_adam(seg, 6, cfg->beta1, cfg->beta2, cfg->epsilon, gradient_scale, bc1, bc2, cfg->max_grad_1, zero_grads,
              static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError());
}

int tgs_gaussians_zero(const TgsGaussians* g, tgs_stream_t stream) {
  if (!gaussians_ok(g)) return TGS_ERR_INVALID_ARGUMENT;
  const size_t n = static_cast<size_t>(g->n);
  if (n == 0) return TGS_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaMemsetAsync(g->means, 0, 12 * n, st);
  cudaMemsetAsync(g->opacities, 0, 4 * n, st);
  cudaMemsetAsync(g->rotations, 0, 16 * n, st);
  cudaMemsetAsync(g->scales, 0, 12 * n, st);
  cudaMemsetAsync(g->sh0, 0, 12 * n, st);
  cudaMemsetAsync(g->sh_rest, 0, 180 * n, st);
  return cuda_status(cudaGetLastError());
}


int tgs_shared_alloc(size_t bytes, void** ptr, TgsIpcHandle* handle) {
  if (ptr == nullptr || handle == nullptr || bytes == 0) return TGS_ERR_INVALID_ARGUMENT;
  *ptr = nullptr;
  if (cudaMalloc(ptr, bytes) != cudaSuccess) {
    cudaGetLastError();
    return TGS_ERR_OUT_OF_MEMORY;
  }
  if (cudaMemset(*ptr, 0, bytes) != cudaSuccess) return TGS_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, *ptr) != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return TGS_ERR_CUDA;
  }
  static_assert(sizeof(h) <= sizeof(handle->bytes), "IPC handle size");
  std::memcpy(handle->bytes, &h, sizeof(h));
  return TGS_OK;
}

int tgs_shared_free(void* ptr) { return ptr == nullptr ? TGS_ERR_INVALID_ARGUMENT : cuda_status(cudaFree(ptr)); }

int tgs_shared_open(const TgsIpcHandle* handle, void** peer_ptr) {
  if (handle == nullptr || peer_ptr == nullptr) return TGS_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->bytes, sizeof(h));
  if (cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    *peer_ptr = nullptr;
    return TGS_ERR_CUDA;
  }
  return TGS_OK;
}

int tgs_shared_close(void* peer_ptr) {
  return peer_ptr == nullptr ? TGS_ERR_INVALID_ARGUMENT : cuda_status(cudaIpcCloseMemHandle(peer_ptr));
}

int tgs_dp_reduce_adam(const TgsGaussians* params_per_rank, const TgsGaussians* grads_per_rank, int32_t world,
                       int32_t rank, TgsGaussians* exp_avg, TgsGaussians* exp_avg_sq, const TgsAdamConfig* cfg,
                       uint32_t step, float gradient_scale, tgs_stream_t stream) {
  if (params_per_rank == nullptr || grads_per_rank == nullptr || world < 1 || world > kMaxDpRanks || rank < 0 ||
      rank >= world || cfg == nullptr || step == 0 || !gaussians_ok(exp_avg) || !gaussians_ok(exp_avg_sq))
    return TGS_ERR_INVALID_ARGUMENT;
  const int64_t n = params_per_rank[rank].n;
  GaussianPtrs p[kMaxDpRanks], g[kMaxDpRanks];
  for (int r = 0; r < world; ++r) {
    if (!gaussians_ok(&params_per_rank[r]) || !gaussians_ok(&grads_per_rank[r]) || params_per_rank[r].n != n ||
        grads_per_rank[r].n != n)
      return TGS_ERR_INVALID_ARGUMENT;
    p[r] = to_ptrs(&params_per_rank[r]);
    g[r] = to_ptrs(&grads_per_rank[r]);
  }
  if (exp_avg->n != n || exp_avg_sq->n != n) return TGS_ERR_INVALID_ARGUMENT;
  if (n == 0) return TGS_OK;
  AdamStepArgs a{};
  adam_segments(cfg, n, step, gradient_scale, &a);
  launch_dp_adam(p, g, world, rank, to_ptrs(exp_avg), to_ptrs(exp_avg_sq), a, static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError());
}

int tgs_dp_reduce_adam_multicast(const TgsGaussians* params_mc, const TgsGaussians* grads_mc,
                                 TgsGaussians* params, int32_t world, int32_t rank, TgsGaussians* exp_avg,
                                 TgsGaussians* exp_avg_sq, const TgsAdamConfig* cfg, uint32_t step,
                                 float gradient_scale, tgs_stream_t stream) {
  if (!gaussians_ok(params_mc) || !gaussians_ok(grads_mc) || !gaussians_ok(params) || world < 1 ||
      world > kMaxDpRanks || rank < 0 || rank >= world || cfg == nullptr || step == 0 || !gaussians_ok(exp_avg) ||
      !gaussians_ok(exp_avg_sq))
    return TGS_ERR_INVALID_ARGUMENT;
  const int64_t n = params->n;
  if (params_mc->n != n || grads_mc->n != n || exp_avg->n != n || exp_avg_sq->n != n) return TGS_ERR_INVALID_ARGUMENT;
  if (n == 0) return TGS_OK;
  AdamStepArgs a{};
  adam_segments(cfg, n, step, gradient_scale, &a);
  launch_dp_adam_mc(to_ptrs(params_mc), to_ptrs(grads_mc), to_ptrs(params), world, rank, to_ptrs(exp_avg),
                    to_ptrs(exp_avg_sq), a, static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError());
}

int tgs_raster_backward_routed(TgsRaster* r, const TgsGaussians* params, const TgsCamera* cam, int32_t dtype,
                               const void* image, const void* grad_image, float* const* inbox_per_rank,
                               int64_t slice_pad, int32_t world, int32_t rank, TgsDensificationInfo* dens,
                               tgs_stream_t stream) {
  if (r == nullptr || !gaussians_ok(params) || !camera_ok(cam) || image == nullptr || grad_image == nullptr ||
      inbox_per_rank == nullptr || world < 1 || world > kMaxDpRanks || rank < 0 || rank >= world)
    return TGS_ERR_INVALID_ARGUMENT;
  RasterState& s = r->s;
  if (!s.have_forward || s.last_dtype != dtype || s.last_n != params->n) return TGS_ERR_NO_FORWARD;
  GradRoute route{};
  for (int k = 0; k < world; ++k) {
    if (inbox_per_rank[k] == nullptr) return TGS_ERR_INVALID_ARGUMENT;
    route.inbox[k] = inbox_per_rank[k];
  }
  for (int k = 0; k <= world; ++k) route.lo[k] = dp_slice_begin(params->n, world, k);
  for (int k = 0; k < world; ++k)
    if (route.lo[k + 1] - route.lo[k] > slice_pad) return TGS_ERR_CAPACITY;
  route.slice_pad = slice_pad;
  route.world = world;
  route.rank = rank;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const DevCamera dc = make_camera(cam->width, cam->height, cam->fx, cam->fy, cam->cx, cam->cy, cam->near_plane,
                                   cam->far_plane, cam->w2c);
  mark(r, 4, st);
  launch_blend_backward(s, dc, dtype == TGS_FLOAT16, image, grad_image, dens != nullptr, st);
  mark(r, 5, st);
  if (params->n > 0) {
    GaussianPtrs none{};
    none.n = params->n;
    launch_preprocess_backward(s, to_ptrs(params), none, dc, 0, reinterpret_cast<float4*>(dens), st, nullptr,
                               nullptr, nullptr, &route);
  }
  mark(r, 6, st);
  r->bwd_timed = r->timing;
  return cuda_status(cudaGetLastError());
}

int tgs_dp_inbox_adam(const TgsGaussians* params_per_rank, const float* inbox, int64_t slice_pad, int32_t world,
                      int32_t rank, TgsGaussians* exp_avg, TgsGaussians* exp_avg_sq, const TgsAdamConfig* cfg,
                      uint32_t step, float gradient_scale, tgs_stream_t stream) {
  if (params_per_rank == nullptr || inbox == nullptr || world < 1 || world > kMaxDpRanks || rank < 0 ||
      rank >= world || cfg == nullptr || step == 0 || !gaussians_ok(exp_avg) || !gaussians_ok(exp_avg_sq))
    return TGS_ERR_INVALID_ARGUMENT;
  const int64_t n = params_per_rank[rank].n;
  if (dp_slice_begin(n, world, rank + 1) - dp_slice_begin(n, world, rank) > slice_pad) return TGS_ERR_CAPACITY;
  GaussianPtrs p[kMaxDpRanks], g[kMaxDpRanks];
  const int widths[6] = {3, 1, 4, 3, 3, 45};
  for (int r = 0; r < world; ++r) {
    if (!gaussians_ok(&params_per_rank[r]) || params_per_rank[r].n != n) return TGS_ERR_INVALID_ARGUMENT;
    p[r] = to_ptrs(&params_per_rank[r]);
    // slot r of the inbox: an arena of slice_pad Gaussians
    float* slot = const_cast<float*>(inbox) + static_cast<int64_t>(r) * 59 * slice_pad;
    float* seg[6];
    int64_t off = 0;
    for (int k = 0; k < 6; ++k) {
      seg[k] = slot + off;
      off += widths[k] * slice_pad;
    }
    g[r] = GaussianPtrs{seg[0], seg[1], seg[2], seg[3], seg[4], seg[5], n, 0};
  }
  if (exp_avg->n != n || exp_avg_sq->n != n) return TGS_ERR_INVALID_ARGUMENT;
  if (n == 0) return TGS_OK;
  AdamStepArgs a{};
  adam_segments(cfg, n, step, gradient_scale, &a);
  launch_dp_adam(p, g, world, rank, to_ptrs(exp_avg), to_ptrs(exp_avg_sq), a, static_cast<cudaStream_t>(stream),
                 true);
  return cuda_status(cudaGetLastError());
}


// ------------------------------------------------------- owner-split views

namespace {
// The handle state of rank k's view: every scratch pointer rebased onto
// rank k's arena (identical capacities give identical carving).
RasterState view_state(const TgsRaster* r, int k) {
  RasterState v = r->s;
  size_t bytes = 0;
  carve(v, r->peer_arena[k], bytes);
  return v;
}

bool slice_ok(const TgsRaster* r, const TgsGaussians* params, int64_t first, int64_t last) {
  return first >= 0 && first <= last && last <= params->n && first % 256 == 0 && params->n <= r->s.cap_n;
}
}  // namespace

int tgs_raster_share(TgsRaster* r, TgsIpcHandle* out) {
  if (r == nullptr || out == nullptr) return TGS_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, r->arena) != cudaSuccess) {
    cudaGetLastError();
    return TGS_ERR_CUDA;
  }
  std::memcpy(out->bytes, &h, sizeof(h));
  return TGS_OK;
}

int tgs_raster_arena(TgsRaster* r, void** arena) {
  if (r == nullptr || arena == nullptr) return TGS_ERR_INVALID_ARGUMENT;
  *arena = r->arena;
  return TGS_OK;
}

int tgs_raster_attach_views(TgsRaster* r, void* const* arenas, int32_t world, int32_t rank) {
  if (r == nullptr || arenas == nullptr || world < 1 || world > kMaxDpRanks || rank < 0 || rank >= world)
    return TGS_ERR_INVALID_ARGUMENT;
  for (int k = 0; k < world; ++k) {
    if (arenas[k] == nullptr) return TGS_ERR_INVALID_ARGUMENT;
    r->peer_arena[k] = static_cast<char*>(arenas[k]);
  }
  for (int k = world; k < kMaxDpRanks; ++k) r->peer_arena[k] = nullptr;
  r->world = world;
  r->rank = rank;
  return TGS_OK;
}

int tgs_raster_preprocess_views(TgsRaster* r, const TgsGaussians* params, const TgsCamera* cams, int32_t dtype,
                                int64_t first, int64_t last, TgsDensificationInfo* dens, tgs_stream_t stream) {
  if (r == nullptr || !gaussians_ok(params) || cams == nullptr || (dtype != TGS_FLOAT32 && dtype != TGS_FLOAT16) ||
      r->peer_arena[0] == nullptr || !slice_ok(r, params, first, last))
    return TGS_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const GaussianPtrs g = to_ptrs(params);
  for (int k = 0; k < r->world; ++k) {
    const TgsCamera* c = &cams[k];
    if (!camera_ok(c) || c->width > r->s.max_w || c->height > r->s.max_h) return TGS_ERR_INVALID_ARGUMENT;
  }
  // one launch for all views (the slice's parameters are read once); every
  // rank starts with the next rank's view and ends with its own, so that at
  // any moment the ranks' record stores go to different GPUs (in view order
  // every rank would store into rank 0's arena first); the records of
  // different views are disjoint, so the order changes nothing.  The views'
  // backward accumulators are cleared by their ranks
  // (tgs_raster_forward_gathered), not across NVLink.
  RasterState vs[kMaxDpRanks];
  DevCamera dcs[kMaxDpRanks];
  int order[kMaxDpRanks];
  for (int k = 0; k < r->world; ++k) {
    const TgsCamera* c = &cams[k];
    vs[k] = view_state(r, k);
    dcs[k] = make_camera(c->width, c->height, c->fx, c->fy, c->cx, c->cy, c->near_plane, c->far_plane, c->w2c);
    order[k] = (r->rank + 1 + k) % r->world;
  }
  if (last > first)
    launch_preprocess_views(vs, dcs, order, r->world, g, dtype == TGS_FLOAT16, reinterpret_cast<float4*>(dens), st,
                            first, last, 0);
  return cuda_status(cudaGetLastError());
}

int tgs_raster_forward_gathered(TgsRaster* r, int64_t n, const TgsCamera* cam, int32_t dtype, void* image,
                                void* alpha, tgs_stream_t stream) {
  if (r == nullptr || n < 0 || !camera_ok(cam) || image == nullptr || (dtype != TGS_FLOAT32 && dtype != TGS_FLOAT16))
    return TGS_ERR_INVALID_ARGUMENT;
  RasterState& s = r->s;
  if (n > s.cap_n || cam->width > s.max_w || cam->height > s.max_h) return TGS_ERR_CAPACITY;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const DevCamera dc = make_camera(cam->width, cam->height, cam->fx, cam->fy, cam->cx, cam->cy, cam->near_plane,
                                   cam->far_plane, cam->w2c);
  cudaMemsetAsync(s.counts, 0, sizeof(DevCounts), st);
  cudaMemsetAsync(s.helpers, 0, sizeof(float) * kHelperFloats * static_cast<size_t>(n), st);
  s.have_forward = 0;
  mark(r, 0, st);
  mark(r, 1, st);
  launch_binning(s, n, dc, dtype == TGS_FLOAT16, st);
  mark(r, 2, st);
  launch_blend_forward(s, dc, dtype == TGS_FLOAT16, image, alpha, st);
  mark(r, 3, st);
  r->fwd_timed = r->timing;
  if (cudaGetLastError() != cudaSuccess) return TGS_ERR_CUDA;
  s.have_forward = 1;
  s.last_dtype = dtype;
  s.last_n = n;
  return TGS_OK;
}

int tgs_raster_backward_screen(TgsRaster* r, const TgsCamera* cam, int32_t dtype, const void* image,
                               const void* grad_image, int32_t absgrad, tgs_stream_t stream) {
  if (r == nullptr || !camera_ok(cam) || image == nullptr || grad_image == nullptr) return TGS_ERR_INVALID_ARGUMENT;
  RasterState& s = r->s;
  if (!s.have_forward || s.last_dtype != dtype) return TGS_ERR_NO_FORWARD;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const DevCamera dc = make_camera(cam->width, cam->height, cam->fx, cam->fy, cam->cx, cam->cy, cam->near_plane,
                                   cam->far_plane, cam->w2c);
  mark(r, 4, st);
  launch_blend_backward(s, dc, dtype == TGS_FLOAT16, image, grad_image, absgrad != 0, st);
  mark(r, 5, st);
  mark(r, 6, st);
  r->bwd_timed = r->timing;
  return cuda_status(cudaGetLastError());
}

int tgs_raster_backward_views_adam(TgsRaster* r, const TgsGaussians* params, const TgsCamera* cams, int64_t first,
                                   int64_t last, TgsGaussians* grads, const TgsGaussians* exp_avg,
                                   const TgsGaussians* exp_avg_sq, const TgsAdamConfig* cfg, uint32_t step,
                                   float gradient_scale, TgsDensificationInfo* dens, tgs_stream_t stream) {
  if (r == nullptr || !gaussians_ok(params) || cams == nullptr || (grads != nullptr && !gaussians_ok(grads)) ||
      !gaussians_ok(exp_avg) || !gaussians_ok(exp_avg_sq) || cfg == nullptr || step == 0 ||
      r->peer_arena[0] == nullptr || !slice_ok(r, params, first, last) ||
      (grads != nullptr && grads->n != params->n) || exp_avg->n != params->n || exp_avg_sq->n != params->n)
    return TGS_ERR_INVALID_ARGUMENT;
  if (last == first) return TGS_OK;
  RasterState vs[kMaxDpRanks];
  const RasterState* vp[kMaxDpRanks];
  DevCamera dc[kMaxDpRanks];
  for (int k = 0; k < r->world; ++k) {
    const TgsCamera* c = &cams[k];
    if (!camera_ok(c)) return TGS_ERR_INVALID_ARGUMENT;
    dc[k] = make_camera(c->width, c->height, c->fx, c->fy, c->cx, c->cy, c->near_plane, c->far_plane, c->w2c);
    vs[k] = view_state(r, k);
    vp[k] = &vs[k];
  }
  AdamStepArgs a{};
  adam_segments(cfg, params->n, step, gradient_scale, &a);
  const GaussianPtrs g = to_ptrs(params), m = to_ptrs(exp_avg), v = to_ptrs(exp_avg_sq);
  GaussianPtrs gr{};
  if (grads != nullptr) gr = to_ptrs(grads);
  launch_views_backward_adam(vp, dc, r->world, g, grads != nullptr ? &gr : nullptr, m, v, a,
                             reinterpret_cast<float4*>(dens), static_cast<cudaStream_t>(stream), first, last);
  return cuda_status(cudaGetLastError());
}

}  // extern "C"
