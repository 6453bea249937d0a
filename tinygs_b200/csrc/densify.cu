// densify.cu -- the densification strategy of the training loop (clone /
// split Gaussians with large view-space gradients, prune transparent or
// oversized ones, periodic opacity reset), in place inside arrays that were
// allocated with room to grow.
//
// Reference: DefaultStrategy, tinygs/src/strategy/default.cu:26-345, with the
// array surgery of GPUGaussian3d::remove/append (src/core/gpu_gaussian.cu:
// 117-171), SimpleAdam::remove/duplicate/reset_opacity
// (src/optim/simple_adam.cu:841-924,981-985) and the random split offsets of
// generate_random_logistic (include/tinygs/random/device.cuh:38-79) over a
// PCG32 stream (include/tinygs/random/pcg32.hpp).  Same decisions, the same
// order (stable compaction, clones appended in ascending source order) and
// the same random stream; unlike the reference nothing is reallocated: the
// caller's arrays hold `capacity` Gaussians and the live count moves within
// them.
#include <cstring>
#include <new>

#include "kernels.h"
#include "tgs_abi.h"

namespace tgs {
namespace {

constexpr int kBlock = 256;
// common.hpp:358-364 (compiled with fast math, as the reference is)
__device__ __forceinline__ float logistic(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float logit(float x) {
  return -logf(1.0f / fminf(fmaxf(x, 1e-9f), 1.0f - 1e-9f) - 1.0f);
}

struct Set {
  float* p[6];  // means, opacities, rotations, scales, sh0, sh_rest
};
__host__ __device__ constexpr int seg_width(int k) {
  return k == 0 ? 3 : k == 1 ? 1 : k == 2 ? 4 : k == 3 ? 3 : k == 4 ? 3 : 45;
}

// Exclusive scan of per-block counts in place (one block of 1024 threads);
// the total goes to *total.
__global__ void __launch_bounds__(1024) k_scan_counts(uint32_t* __restrict__ sums, uint32_t count,
                                                      uint32_t* __restrict__ total) {
  __shared__ uint32_t warp_sums[32];
  const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5;
  const uint32_t per = (count + 1023u) / 1024u;
  const uint32_t begin = min(count, t * per), end = min(count, begin + per);
  uint32_t local = 0;
  for (uint32_t k = begin; k < end; ++k) local += sums[k];
  uint32_t x = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= static_cast<uint32_t>(o)) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= static_cast<uint32_t>(o)) w += y;
    }
    warp_sums[lane] = w;
  }
  __syncthreads();
  uint32_t run = (warp == 0 ? 0u : warp_sums[warp - 1]) + x - local;
  for (uint32_t k = begin; k < end; ++k) {
    const uint32_t v = sums[k];
    sums[k] = run;
    run += v;
  }
  if (t == 1023) *total = warp_sums[31];
}

// Ordered list of the flagged indices (stable compaction of 0..n-1).
__global__ void __launch_bounds__(kBlock) k_flag_list(const uint8_t* __restrict__ flags, uint32_t n,
                                                      const uint32_t* __restrict__ block_offsets,
                                                      uint32_t* __restrict__ list) {
  __shared__ uint32_t warp_sums[kBlock / 32];
  const uint32_t i = blockIdx.x * kBlock + threadIdx.x, lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  const bool f = i < n && flags[i] != 0;
  const uint32_t b = __ballot_sync(0xffffffffu, f);
  if (lane == 0) warp_sums[warp] = __popc(b);
  __syncthreads();
  uint32_t before = block_offsets[blockIdx.x];
  for (uint32_t w = 0; w < warp; ++w) before += warp_sums[w];
  if (f) list[before + __popc(b & ((1u << lane) - 1u))] = i;
}

// default.cu:151-175: 1 = clone, 2 = split
__global__ void __launch_bounds__(kBlock)
    k_grow_flags(const float4* __restrict__ dens, const float* __restrict__ scales, uint32_t n, float grow_grad,
                 float grow_scale, int absgrad, uint8_t* __restrict__ flags, uint32_t* __restrict__ block_counts) {
  const uint32_t i = blockIdx.x * kBlock + threadIdx.x;
  uint8_t f = 0;
  if (i < n) {
    const float4 d = dens[i];
    const float grad = __fdiv_rn(absgrad ? d.z : d.y, fmaxf(d.x, 1.0f));
    if (grad > grow_grad && d.x > 0.0f) {
      const float mx = fmaxf(fmaxf(expf(scales[3 * i]), expf(scales[3 * i + 1])), expf(scales[3 * i + 2]));
      f = mx > grow_scale ? 2 : 1;
    }
    flags[i] = f;
  }
  const uint32_t c = __syncthreads_count(f != 0);
  if (threadIdx.x == 0) block_counts[blockIdx.x] = c;
}

// generate_random_logistic: element idx is draw (idx % T) * 4 + idx / T of
// the stream, T the thread count of the reference's launch.
__global__ void k_logistic(Pcg rng, uint32_t count, uint32_t threads, float* __restrict__ out) {
  const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= count) return;
  Pcg g = rng;
  g.advance(static_cast<uint64_t>(idx % threads) * 4u + idx / threads);
  out[idx] = logit(g.next_float()) * 1.0f * 0.551328895f + 0.0f;
}

// default.cu:239-295: the means, scales and opacities of the appended rows
// (clone: copies; split: both halves moved and shrunk); the appended rows of
// gradients and moments are zeroed by the caller
__global__ void __launch_bounds__(kBlock)
    k_duplicate(const uint32_t* __restrict__ grow_src, const uint8_t* __restrict__ flags, uint32_t n_grow,
                uint32_t n0, Set params, const float* __restrict__ rnd) {
  const uint32_t k = blockIdx.x * kBlock + threadIdx.x;
  if (k >= n_grow) return;
  const uint32_t src = grow_src[k], dst = n0 + k;
  float* means = params.p[0];
  float* opac = params.p[1];
  float* rot = params.p[2];
  float* scales = params.p[3];
  // (rotations and SH rows: k_duplicate_rows; gradient and moment rows:
  // zeroed by the caller)
  if (flags[src] == 1) {
    for (int c = 0; c < 3; ++c) {
      means[3 * dst + c] = means[3 * src + c];
      scales[3 * dst + c] = scales[3 * src + c];
    }
    opac[dst] = opac[src];
  } else {
    // glm::mat3 built column by column from (w, x, y, z), column-major product
    const float r = rot[4 * src], x = rot[4 * src + 1], y = rot[4 * src + 2], z = rot[4 * src + 3];
    const float c0[3] = {1.f - 2.f * (y * y + z * z), 2.f * (x * y - r * z), 2.f * (x * z + r * y)};
    const float c1[3] = {2.f * (x * y + r * z), 1.f - 2.f * (x * x + z * z), 2.f * (y * z - r * x)};
    const float c2[3] = {2.f * (x * z - r * y), 2.f * (y * z + r * x), 1.f - 2.f * (x * x + y * y)};
    const float act[3] = {expf(scales[3 * src]), expf(scales[3 * src + 1]), expf(scales[3 * src + 2])};
    const float new_op = 1.0f - sqrtf(1.0f - logistic(opac[src]));
    float v1[3], v2[3];
    for (int c = 0; c < 3; ++c) {
      v1[c] = rnd[6 * k + c] * (act[c] + 1e-5f);
      v2[c] = rnd[6 * k + 3 + c] * (act[c] + 1e-5f);
    }
    for (int c = 0; c < 3; ++c) {
      const float off1 = c0[c] * v1[0] + c1[c] * v1[1] + c2[c] * v1[2];
      const float off2 = c0[c] * v2[0] + c1[c] * v2[1] + c2[c] * v2[2];
      const float base = means[3 * src + c];
      means[3 * dst + c] = base + off1;
      means[3 * src + c] = base + off2;
    }
    for (int c = 0; c < 3; ++c) {
      const float ns = logf(act[c] / 1.6f);
      scales[3 * dst + c] = ns;
      scales[3 * src + c] = ns;
    }
    const float lo = logit(new_op);
    opac[dst] = lo;
    opac[src] = lo;
  }
}

// Rows of width W: destination rows [0, cnt) of `dst` (a contiguous block)
// taken from rows s_rows[0..cnt) of `src`; the lanes of a warp run over the
// block's elements, so stores are coalesced and reads coalesced within a row.
template <int W>
__device__ __forceinline__ void copy_rows(const float* __restrict__ src, float* __restrict__ dst,
                                          const uint32_t* s_rows, uint32_t cnt, uint32_t lane) {
  for (uint32_t e = lane; e < cnt * W; e += 32u) {
    const uint32_t r = e / W, c = e - r * W;
    dst[e] = src[static_cast<size_t>(s_rows[r]) * W + c];
  }
}

constexpr int kRowWarps = 8;

// The appended rows' rotations and SH coefficients (copies of their source
// rows), one warp per 32 appended rows.
__global__ void __launch_bounds__(32 * kRowWarps)
    k_duplicate_rows(const uint32_t* __restrict__ grow_src, uint32_t n_grow, uint32_t n0, Set params) {
  __shared__ uint32_t s_rows[kRowWarps][32];
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  const uint32_t wb = (blockIdx.x * kRowWarps + warp) * 32u;
  if (wb >= n_grow) return;
  const uint32_t cnt = min(32u, n_grow - wb);
  if (lane < cnt) s_rows[warp][lane] = grow_src[wb + lane];
  __syncwarp();
  const size_t d = static_cast<size_t>(n0) + wb;
  copy_rows<4>(params.p[2], params.p[2] + 4 * d, s_rows[warp], cnt, lane);
  copy_rows<3>(params.p[4], params.p[4] + 3 * d, s_rows[warp], cnt, lane);
  copy_rows<45>(params.p[5], params.p[5] + 45 * d, s_rows[warp], cnt, lane);
}

// default.cu:309-332
__global__ void __launch_bounds__(kBlock)
    k_alive(const float* __restrict__ opac, const float* __restrict__ scales, const float4* __restrict__ rot,
            const float4* __restrict__ dens, uint32_t n, uint32_t n0, float ws_thr, float ss_thr, int prune_large,
            float min_opacity, uint8_t* __restrict__ keep, uint32_t* __restrict__ block_counts) {
  const uint32_t i = blockIdx.x * kBlock + threadIdx.x;
  bool alive = false;
  if (i < n) {
    const float mx = fmaxf(fmaxf(expf(scales[3 * i]), expf(scales[3 * i + 1])), expf(scales[3 * i + 2]));
    const bool not_large_ws = mx < ws_thr;
    const bool not_large_ss = i >= n0 || dens[i].w < ss_thr;
    const bool not_transparent = logistic(opac[i]) > min_opacity;
    const float4 q = rot[i];
    const bool not_degenerate = fabsf(q.x) + fabsf(q.y) + fabsf(q.z) + fabsf(q.w) > 1.1920929e-07f;
    alive = not_transparent && ((not_large_ws && not_large_ss) || !prune_large) && not_degenerate;
    keep[i] = alive ? 1 : 0;
  }
  const uint32_t c = __syncthreads_count(alive);
  if (threadIdx.x == 0) block_counts[blockIdx.x] = c;
}

// rows of the kept list gathered into scratch (copied back by the host), one
// warp per 32 kept rows of width W
template <int W>
__global__ void __launch_bounds__(32 * kRowWarps)
    k_gather_rows(const float* __restrict__ src, float* __restrict__ dst, const uint32_t* __restrict__ list,
                  uint32_t n_rows) {
  __shared__ uint32_t s_rows[kRowWarps][32];
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  for (uint32_t wb = (blockIdx.x * kRowWarps + warp) * 32u; wb < n_rows; wb += gridDim.x * kRowWarps * 32u) {
    const uint32_t cnt = min(32u, n_rows - wb);
    if (lane < cnt) s_rows[warp][lane] = list[wb + lane];
    __syncwarp();
    copy_rows<W>(src, dst + static_cast<size_t>(wb) * W, s_rows[warp], cnt, lane);
    __syncwarp();  // s_rows is refilled for the next 32 rows
  }
}

void gather_rows(const float* src, float* dst, const uint32_t* list, uint32_t n_rows, int width, int blocks,
                 cudaStream_t st) {
  switch (width) {
    case 1: k_gather_rows<1><<<blocks, 32 * kRowWarps, 0, st>>>(src, dst, list, n_rows); break;
    case 3: k_gather_rows<3><<<blocks, 32 * kRowWarps, 0, st>>>(src, dst, list, n_rows); break;
    case 4: k_gather_rows<4><<<blocks, 32 * kRowWarps, 0, st>>>(src, dst, list, n_rows); break;
    default: k_gather_rows<45><<<blocks, 32 * kRowWarps, 0, st>>>(src, dst, list, n_rows); break;
  }
}

// default.cu:26-38 and SimpleAdam::reset_opacity
__global__ void k_reset_opacity(float* __restrict__ opac, float* __restrict__ m, float* __restrict__ v, uint32_t n,
                                float cap) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  opac[i] = logit(fminf(logistic(opac[i]), cap));
  if (m != nullptr) m[i] = 0.f;
  if (v != nullptr) v[i] = 0.f;
}

}  // namespace
}  // namespace tgs

using namespace tgs;

struct TgsDensifier {
  int64_t capacity = 0;
  int device = 0;
  int num_sms = 148;
  void* arena = nullptr;
  uint8_t* flags = nullptr;
  uint32_t* list = nullptr;
  uint32_t* block_counts = nullptr;
  uint32_t* total = nullptr;
  float* rnd = nullptr;
  float* scratch = nullptr;
  uint32_t* host_total = nullptr;  // pinned
};

namespace {
Set to_set(const TgsGaussians* g) {
  Set s{};
  if (g != nullptr) {
    s.p[0] = g->means;
    s.p[1] = g->opacities;
    s.p[2] = g->rotations;
    s.p[3] = g->scales;
    s.p[4] = g->sh0;
    s.p[5] = g->sh_rest;
  }
  return s;
}

int read_total(TgsDensifier* d, cudaStream_t st, uint32_t* out) {
  if (cudaMemcpyAsync(d->host_total, d->total, sizeof(uint32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return TGS_ERR_CUDA;
  *out = *d->host_total;
  return TGS_OK;
}
}  // namespace

extern "C" {

void tgs_pcg32_seed(TgsPcg32* rng, uint64_t initstate, uint64_t initseq) {
  const Pcg g = Pcg::seeded(initstate, initseq);
  rng->state = g.state;
  rng->inc = g.inc;
}

int tgs_densify_create(int64_t capacity, TgsDensifier** out) {
  if (out == nullptr || capacity <= 0 || capacity > 0x7fffffffLL) return TGS_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  auto* d = new (std::nothrow) TgsDensifier();
  if (d == nullptr) return TGS_ERR_OUT_OF_MEMORY;
  d->capacity = capacity;
  cudaGetDevice(&d->device);
  cudaDeviceGetAttribute(&d->num_sms, cudaDevAttrMultiProcessorCount, d->device);
  const size_t cap = static_cast<size_t>(capacity);
  const size_t blocks = (cap + kBlock - 1) / kBlock + 1;
  auto up = [](size_t b) { return (b + 255u) & ~static_cast<size_t>(255u); };
  const size_t sz_flags = up(cap), sz_list = up(4 * cap), sz_blocks = up(4 * blocks), sz_total = 256,
               sz_rnd = up(4 * 6 * cap), sz_scratch = up(4 * 45 * cap);
  const size_t bytes = sz_flags + sz_list + sz_blocks + sz_total + sz_rnd + sz_scratch;
  if (cudaMalloc(&d->arena, bytes) != cudaSuccess) {
    cudaGetLastError();
    delete d;
    return TGS_ERR_OUT_OF_MEMORY;
  }
  char* b = static_cast<char*>(d->arena);
  d->flags = reinterpret_cast<uint8_t*>(b);
  b += sz_flags;
  d->list = reinterpret_cast<uint32_t*>(b);
  b += sz_list;
  d->block_counts = reinterpret_cast<uint32_t*>(b);
  b += sz_blocks;
  d->total = reinterpret_cast<uint32_t*>(b);
  b += sz_total;
  d->rnd = reinterpret_cast<float*>(b);
  b += sz_rnd;
  d->scratch = reinterpret_cast<float*>(b);
  if (cudaMallocHost(&d->host_total, sizeof(uint32_t)) != cudaSuccess) {
    cudaFree(d->arena);
    delete d;
    return TGS_ERR_OUT_OF_MEMORY;
  }
  *out = d;
  return TGS_OK;
}

int tgs_densify_destroy(TgsDensifier* d) {
  if (d == nullptr) return TGS_ERR_INVALID_ARGUMENT;
  cudaFree(d->arena);
  cudaFreeHost(d->host_total);
  delete d;
  return TGS_OK;
}

int tgs_densify_step(TgsDensifier* d, TgsGaussians* params, TgsGaussians* grads, TgsGaussians* exp_avg,
                     TgsGaussians* exp_avg_sq, TgsDensificationInfo* dens, const TgsDensifyConfig* cfg, int32_t step,
                     TgsPcg32* rng, int64_t* n_inout, tgs_stream_t stream) {
  if (d == nullptr || params == nullptr || dens == nullptr || cfg == nullptr || rng == nullptr ||
      n_inout == nullptr || *n_inout < 0 || *n_inout > d->capacity || cfg->refine_every <= 0)
    return TGS_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const Set P = to_set(params), G = to_set(grads), M = to_set(exp_avg), V = to_set(exp_avg_sq);
  float4* dn = reinterpret_cast<float4*>(dens);
  uint32_t n = static_cast<uint32_t>(*n_inout);
  const bool refine = step % cfg->refine_every == 0 && step >= cfg->start_refine && step <= cfg->end_refine;
  if (refine) {
    const uint32_t n0 = n;
    uint32_t grows = 0;
    const uint32_t blocks0 = (n0 + kBlock - 1) / kBlock;
    if (static_cast<int64_t>(n0) < cfg->max_num_gaussians && n0 > 0) {
      k_grow_flags<<<blocks0, kBlock, 0, st>>>(dn, P.p[3], n0, cfg->duplicate_grad_threshold * cfg->grad_scaler,
                                               cfg->duplicate_scale_threshold * cfg->scene_scale, cfg->absgrad,
                                               d->flags, d->block_counts);
      k_scan_counts<<<1, 1024, 0, st>>>(d->block_counts, blocks0, d->total);
      const int rc = read_total(d, st, &grows);
      if (rc != TGS_OK) return rc;
    }
    if (static_cast<int64_t>(n0) + grows > d->capacity) return TGS_ERR_CAPACITY;
    if (static_cast<uint64_t>(grows) * 6u > 0xffffffffull) return TGS_ERR_UNSUPPORTED;
    if (grows > 0) {
      k_flag_list<<<blocks0, kBlock, 0, st>>>(d->flags, n0, d->block_counts, d->list);
      const uint32_t count = 6 * grows;
      const uint32_t work = (count + 3u) / 4u;
      const uint32_t threads = (work + 127u) / 128u * 128u;  // the reference's launch: 128-thread blocks
      Pcg g{rng->state, rng->inc};
      k_logistic<<<(count + 255u) / 256u, 256, 0, st>>>(g, count, threads, d->rnd);
      g.advance(count);
      rng->state = g.state;
      rng->inc = g.inc;
      k_duplicate<<<(grows + kBlock - 1) / kBlock, kBlock, 0, st>>>(d->list, d->flags, grows, n0, P, d->rnd);
      const uint32_t row_warps = (grows + 31u) / 32u;
      k_duplicate_rows<<<(row_warps + kRowWarps - 1) / kRowWarps, 32 * kRowWarps, 0, st>>>(d->list, grows, n0, P);
      // gradients and moments of the appended rows are zero
      const Set zero_sets[3] = {G, M, V};
      for (const Set& zs : zero_sets)
        for (int seg = 0; seg < 6; ++seg)
          if (zs.p[seg] != nullptr)
            cudaMemsetAsync(zs.p[seg] + static_cast<size_t>(n0) * seg_width(seg), 0,
                            sizeof(float) * seg_width(seg) * static_cast<size_t>(grows), st);
    }
    n = n0 + grows;
    // prune
    uint32_t kept = 0;
    const uint32_t blocks = (n + kBlock - 1) / kBlock;
    if (n > 0) {
      const int32_t side = cfg->image_width > cfg->image_height ? cfg->image_width : cfg->image_height;
      k_alive<<<blocks, kBlock, 0, st>>>(P.p[1], P.p[3], reinterpret_cast<const float4*>(P.p[2]), dn, n, n0,
                                         cfg->pruning_scale_threshold * cfg->scene_scale,
                                         static_cast<float>(side) * cfg->max_screen_size, step > cfg->reset_every,
                                         cfg->pruning_opacity_threshold, d->flags, d->block_counts);
      k_scan_counts<<<1, 1024, 0, st>>>(d->block_counts, blocks, d->total);
      const int rc = read_total(d, st, &kept);
      if (rc != TGS_OK) return rc;
    }
    // an empty survivor set leaves the arrays as they are (strategy.cpp:21)
    if (kept > 0 && kept < n) {
      k_flag_list<<<blocks, kBlock, 0, st>>>(d->flags, n, d->block_counts, d->list);
      const Set sets[4] = {P, G, M, V};
      for (const Set& s : sets)
        for (int seg = 0; seg < 6; ++seg) {
          float* p = s.p[seg];
          if (p == nullptr) continue;
          const int w = seg_width(seg);
          gather_rows(p, d->scratch, d->list, kept, w, d->num_sms * 8, st);
          cudaMemcpyAsync(p, d->scratch, sizeof(float) * w * static_cast<size_t>(kept), cudaMemcpyDeviceToDevice,
                          st);
        }
      n = kept;
    }
    cudaMemsetAsync(dens, 0, sizeof(TgsDensificationInfo) * static_cast<size_t>(n), st);
  }
  if (cfg->reset_every > 0 && step % cfg->reset_every == 0 && step >= cfg->start_refine && step < cfg->end_refine &&
      n > 0) {
    k_reset_opacity<<<(n + 255u) / 256u, 256, 0, st>>>(P.p[1], M.p[1], V.p[1], n,
                                                       2.0f * cfg->pruning_opacity_threshold);
  }
  *n_inout = n;
  return cudaGetLastError() == cudaSuccess ? TGS_OK : TGS_ERR_CUDA;
}

}  // extern "C"
