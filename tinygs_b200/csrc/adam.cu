// adam.cu -- one fused Adam step over all six Gaussian parameter arrays.
//
// The reference launches one kernel per parameter array
// (tinygs/src/optim/simple_adam.cu:457-580, kernels adam / adam_f32x4 at
// :105-213).  Here a single grid-stride launch walks the six segments as one
// virtual array in 16-byte chunks (float4 loads/stores of theta, grad, m, v),
// with the per-segment learning rate and decay looked up per chunk; segment
// tails that are not a multiple of four floats are handled element-wise
// (the reference's f32x4 kernel reads and writes up to three floats past
// the end there).  Optionally the gradient is zeroed in the same pass.
#include "kernels.h"

namespace tgs {
namespace {

constexpr int kMaxSegs = 8;

struct SegTable {
  float* theta[kMaxSegs];
  const float* grad[kMaxSegs];
  float* m[kMaxSegs];
  float* v[kMaxSegs];
  int64_t count[kMaxSegs];
  int64_t chunk_begin[kMaxSegs + 1];  // prefix of ceil(count/4)
  float lr[kMaxSegs];
  float decay[kMaxSegs];
  int decay_kind[kMaxSegs];
  int vec_ok[kMaxSegs];
  int n;
};

struct AdamScalars {
  float beta1, beta2, eps, gscale, bc1, bc2_sqrt, max_g;
  int zero_grads;
};

__device__ __forceinline__ float lerp_ref(float v0, float v1, float t) {
  // fma form of v0 + t (v1 - v0), simple_adam.cu:24-26
  return fmaf(t, v1, fmaf(-t, v0, v0));
}

__device__ __forceinline__ void adam_one(float& th, float g_raw, float& m, float& v, float lr, int kind, float decay,
                                         const AdamScalars& a) {
  float g = a.gscale * g_raw;
  if (kind == 1) {
    const float s = 1.0f / (1.0f + __expf(-th));
    g = g + decay * (s * (1.0f - s));
  } else if (kind == 2) {
    g = g + decay * __expf(th);
  }
  if (a.max_g != 0.0f) g = copysignf(fminf(fabsf(g), a.max_g), g);
  m = lerp_ref(m, g, 1.0f - a.beta1);
  v = lerp_ref(v, g * g, 1.0f - a.beta2);
  const float mh = m / a.bc1;
  const float den = sqrtf(v) / a.bc2_sqrt + a.eps;
  th -= mh * lr / den;
}

__global__ void __launch_bounds__(256) k_adam(SegTable t, AdamScalars a, int64_t total_chunks) {
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < total_chunks;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int s = 0;
#pragma unroll
    for (int k = 1; k < kMaxSegs; ++k)
      if (k < t.n && c >= t.chunk_begin[k]) s = k;
    const int64_t e0 = (c - t.chunk_begin[s]) * 4;
    const int64_t cnt = t.count[s];
    const float lr = t.lr[s], decay = t.decay[s];
    const int kind = t.decay_kind[s];
    if (t.vec_ok[s] && e0 + 4 <= cnt) {
      float4 th = *reinterpret_cast<const float4*>(t.theta[s] + e0);
      const float4 g = *reinterpret_cast<const float4*>(t.grad[s] + e0);
      float4 m = *reinterpret_cast<const float4*>(t.m[s] + e0);
      float4 v = *reinterpret_cast<const float4*>(t.v[s] + e0);
      adam_one(th.x, g.x, m.x, v.x, lr, kind, decay, a);
      adam_one(th.y, g.y, m.y, v.y, lr, kind, decay, a);
      adam_one(th.z, g.z, m.z, v.z, lr, kind, decay, a);
      adam_one(th.w, g.w, m.w, v.w, lr, kind, decay, a);
      *reinterpret_cast<float4*>(t.theta[s] + e0) = th;
      *reinterpret_cast<float4*>(t.m[s] + e0) = m;
      *reinterpret_cast<float4*>(t.v[s] + e0) = v;
      if (a.zero_grads) *reinterpret_cast<float4*>(const_cast<float*>(t.grad[s]) + e0) = make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
      for (int64_t e = e0; e < min(e0 + 4, cnt); ++e) {
        float th = t.theta[s][e], m = t.m[s][e], v = t.v[s][e];
        adam_one(th, t.grad[s][e], m, v, lr, kind, decay, a);
        t.theta[s][e] = th;
        t.m[s][e] = m;
        t.v[s][e] = v;
        if (a.zero_grads) const_cast<float*>(t.grad[s])[e] = 0.f;
      }
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Data-parallel step over peer memory: this rank's slice of every segment
// gets the sum of all ranks' gradients (peer loads, rank order, the same
// order as the reference's accumulation into one arena), the Adam update on
// this rank's moments, and the new parameters stored into every rank's
// parameter arena (peer stores).
struct PeerTable {
  float* params[kMaxDpRanks][6];
  const float* grads[kMaxDpRanks][6];
  int64_t goff[6];  // gradient arrays indexed by (element - goff)
  float* m[6];
  float* v[6];
  int64_t lo[6];
  int64_t hi[6];
  int64_t chunk_begin[7];
  float lr[6];
  float decay[6];
  int kind[6];
  int world, rank, vec;
};

// One 16-byte chunk of the slice: segment, element offset and its data.
struct DpChunk {
  int s;
  int64_t e0;
  bool vec;
  float4 g, th, m, v;
};

__device__ __forceinline__ DpChunk dp_load(const PeerTable& t, int64_t c) {
  DpChunk k{};
  k.s = 0;
#pragma unroll
  for (int q = 1; q < 6; ++q)
    if (c >= t.chunk_begin[q]) k.s = q;
  k.e0 = t.lo[k.s] + (c - t.chunk_begin[k.s]) * 4;
  k.vec = t.vec && k.e0 + 4 <= t.hi[k.s];
  if (k.vec) {
    const int64_t ge = k.e0 - t.goff[k.s];
    k.g = *reinterpret_cast<const float4*>(t.grads[0][k.s] + ge);
#pragma unroll
    for (int r = 1; r < kMaxDpRanks; ++r) {
      if (r >= t.world) break;
      const float4 q = *reinterpret_cast<const float4*>(t.grads[r][k.s] + ge);
      k.g.x += q.x;
      k.g.y += q.y;
      k.g.z += q.z;
      k.g.w += q.w;
    }
    k.th = *reinterpret_cast<const float4*>(t.params[t.rank][k.s] + k.e0);
    k.m = *reinterpret_cast<const float4*>(t.m[k.s] + k.e0);
    k.v = *reinterpret_cast<const float4*>(t.v[k.s] + k.e0);
  }
  return k;
}

__device__ __forceinline__ void dp_finish(const PeerTable& t, DpChunk& k, const AdamScalars& a) {
  const float lr = t.lr[k.s], decay = t.decay[k.s];
  const int kind = t.kind[k.s];
  if (k.vec) {
    adam_one(k.th.x, k.g.x, k.m.x, k.v.x, lr, kind, decay, a);
    adam_one(k.th.y, k.g.y, k.m.y, k.v.y, lr, kind, decay, a);
    adam_one(k.th.z, k.g.z, k.m.z, k.v.z, lr, kind, decay, a);
    adam_one(k.th.w, k.g.w, k.m.w, k.v.w, lr, kind, decay, a);
    *reinterpret_cast<float4*>(t.m[k.s] + k.e0) = k.m;
    *reinterpret_cast<float4*>(t.v[k.s] + k.e0) = k.v;
#pragma unroll
    for (int r = 0; r < kMaxDpRanks; ++r) {
      if (r >= t.world) break;
      *reinterpret_cast<float4*>(t.params[r][k.s] + k.e0) = k.th;
    }
  } else {
    // scalar tail (a slice end that is not a multiple of four floats)
    for (int64_t e = k.e0; e < min(k.e0 + 4, t.hi[k.s]); ++e) {
      float g = t.grads[0][k.s][e - t.goff[k.s]];
      for (int r = 1; r < t.world; ++r) g += t.grads[r][k.s][e - t.goff[k.s]];
      float th = t.params[t.rank][k.s][e], m = t.m[k.s][e], v = t.v[k.s][e];
      adam_one(th, g, m, v, lr, kind, decay, a);
      t.m[k.s][e] = m;
      t.v[k.s][e] = v;
      for (int r = 0; r < t.world; ++r) t.params[r][k.s][e] = th;
    }
  }
}

// Two chunks per thread and iteration, both loaded before either is
// updated, so that more peer loads are in flight.
__global__ void __launch_bounds__(256) k_dp_adam(PeerTable t, AdamScalars a, int64_t total_chunks) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < total_chunks;
       c += 2 * stride) {
    DpChunk k0 = dp_load(t, c);
    const bool has1 = c + stride < total_chunks;
    DpChunk k1{};
    if (has1) k1 = dp_load(t, c + stride);
    dp_finish(t, k0, a);
    if (has1) dp_finish(t, k1, a);
  }
  // the stores into the other ranks' memory are complete before this
  // kernel is; the caller's collective orders them before the next forward
  __threadfence_system();
}

// Same step through NVLink SHARP: the slice's gradients are read already
// summed over the ranks by the switch (multimem.ld_reduce on the gradient
// arenas' multicast address) and the new parameters are written to every
// rank at once (multimem.st on the parameter arenas' multicast address).
// The sum's order is the switch's, so for more than two ranks it can differ
// from the rank-order sum in the last bit.
struct McTable {
  float* mc_params[6];
  const float* mc_grads[6];
  const float* own[6];
  float* m[6];
  float* v[6];
  int64_t lo[6];
  int64_t hi[6];
  int64_t chunk_begin[7];
  float lr[6];
  float decay[6];
  int kind[6];
};

__device__ __forceinline__ float4 mc_ld_reduce4(const float* p) {
  float4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];\n"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p)
               : "memory");
  return r;
}
__device__ __forceinline__ float mc_ld_reduce1(const float* p) {
  float r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.f32 %0, [%1];\n" : "=f"(r) : "l"(p) : "memory");
  return r;
}
__device__ __forceinline__ void mc_st4(float* p, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"l"(p), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void mc_st1(float* p, float v) {
  asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;\n" ::"l"(p), "f"(v) : "memory");
}

// Four chunks per thread and iteration: the reducing loads of all four are
// issued before any update, to keep more of them in flight through the
// switch.
constexpr int kMcUnroll = 4;

__global__ void __launch_bounds__(256) k_dp_adam_mc(McTable t, AdamScalars a, int64_t total_chunks) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t c0 = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c0 < total_chunks;
       c0 += kMcUnroll * stride) {
    int seg[kMcUnroll];
    int64_t e0[kMcUnroll];
    bool full[kMcUnroll];
    float4 g[kMcUnroll];
#pragma unroll
    for (int u = 0; u < kMcUnroll; ++u) {
      const int64_t c = c0 + u * stride;
      seg[u] = 0;
      e0[u] = 0;
      full[u] = false;
      if (c < total_chunks) {
#pragma unroll
        for (int k = 1; k < 6; ++k)
          if (c >= t.chunk_begin[k]) seg[u] = k;
        e0[u] = t.lo[seg[u]] + (c - t.chunk_begin[seg[u]]) * 4;
        full[u] = e0[u] + 4 <= t.hi[seg[u]];
        if (full[u]) g[u] = mc_ld_reduce4(t.mc_grads[seg[u]] + e0[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < kMcUnroll; ++u) {
      const int64_t c = c0 + u * stride;
      if (c >= total_chunks) continue;
      const int s = seg[u];
      const float lr = t.lr[s], decay = t.decay[s];
      const int kind = t.kind[s];
      if (full[u]) {
        float4 th = *reinterpret_cast<const float4*>(t.own[s] + e0[u]);
        float4 m = *reinterpret_cast<const float4*>(t.m[s] + e0[u]);
        float4 v = *reinterpret_cast<const float4*>(t.v[s] + e0[u]);
        adam_one(th.x, g[u].x, m.x, v.x, lr, kind, decay, a);
        adam_one(th.y, g[u].y, m.y, v.y, lr, kind, decay, a);
        adam_one(th.z, g[u].z, m.z, v.z, lr, kind, decay, a);
        adam_one(th.w, g[u].w, m.w, v.w, lr, kind, decay, a);
        *reinterpret_cast<float4*>(t.m[s] + e0[u]) = m;
        *reinterpret_cast<float4*>(t.v[s] + e0[u]) = v;
        mc_st4(t.mc_params[s] + e0[u], th);
      } else {
        for (int64_t e = e0[u]; e < min(e0[u] + 4, t.hi[s]); ++e) {
          const float gs = mc_ld_reduce1(t.mc_grads[s] + e);
          float th = t.own[s][e], m = t.m[s][e], v = t.v[s][e];
          adam_one(th, gs, m, v, lr, kind, decay, a);
          t.m[s][e] = m;
          t.v[s][e] = v;
          mc_st1(t.mc_params[s] + e, th);
        }
      }
    }
  }
  __threadfence_system();
}

}  // namespace

void launch_dp_adam_mc(const GaussianPtrs& params_mc, const GaussianPtrs& grads_mc, const GaussianPtrs& own,
                       int world, int rank, const GaussianPtrs& m, const GaussianPtrs& v, const AdamStepArgs& adam,
                       cudaStream_t stream) {
  McTable t{};
  const int64_t n = own.n;
  const int64_t lo_g = dp_slice_begin(n, world, rank), hi_g = dp_slice_begin(n, world, rank + 1);
  const int widths[6] = {3, 1, 4, 3, 3, 45};
  float* pm[6] = {params_mc.means, params_mc.opacities, params_mc.rotations, params_mc.scales, params_mc.sh0,
                  params_mc.sh_rest};
  float* gm[6] = {grads_mc.means, grads_mc.opacities, grads_mc.rotations, grads_mc.scales, grads_mc.sh0,
                  grads_mc.sh_rest};
  float* ow[6] = {own.means, own.opacities, own.rotations, own.scales, own.sh0, own.sh_rest};
  float* mp[6] = {m.means, m.opacities, m.rotations, m.scales, m.sh0, m.sh_rest};
  float* vp[6] = {v.means, v.opacities, v.rotations, v.scales, v.sh0, v.sh_rest};
  int64_t chunks = 0;
  for (int k = 0; k < 6; ++k) {
    t.mc_params[k] = pm[k];
    t.mc_grads[k] = gm[k];
    t.own[k] = ow[k];
    t.m[k] = mp[k];
    t.v[k] = vp[k];
    t.lo[k] = lo_g * widths[k];
    t.hi[k] = hi_g * widths[k];
    t.lr[k] = adam.lr[k];
    t.decay[k] = adam.decay[k];
    t.kind[k] = adam.kind[k];
    t.chunk_begin[k] = chunks;
    chunks += (t.hi[k] - t.lo[k] + 3) / 4;
  }
  t.chunk_begin[6] = chunks;
  if (chunks <= 0) return;
  AdamScalars a{adam.beta1, adam.beta2, adam.eps, adam.gradient_scale, adam.bc1, adam.bc2_sqrt, adam.max_grad_1, 0};
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (chunks + 255) / 256;
  const int blocks = static_cast<int>(want < sms * 8 ? want : sms * 8);
  k_dp_adam_mc<<<blocks, 256, 0, stream>>>(t, a, chunks);
}

void launch_dp_adam(const GaussianPtrs* params, const GaussianPtrs* grads, int world, int rank,
                    const GaussianPtrs& m, const GaussianPtrs& v, const AdamStepArgs& adam, cudaStream_t stream,
                    bool grads_are_slices) {
  PeerTable t{};
  t.world = world;
  t.rank = rank;
  const int64_t n = params[rank].n;
  const int64_t lo_g = dp_slice_begin(n, world, rank), hi_g = dp_slice_begin(n, world, rank + 1);
  const int widths[6] = {3, 1, 4, 3, 3, 45};
  bool vec = true;
  for (int r = 0; r < world; ++r) {
    float* pp[6] = {params[r].means, params[r].opacities, params[r].rotations, params[r].scales, params[r].sh0,
                    params[r].sh_rest};
    float* gp[6] = {grads[r].means, grads[r].opacities, grads[r].rotations, grads[r].scales, grads[r].sh0,
                    grads[r].sh_rest};
    for (int k = 0; k < 6; ++k) {
      t.params[r][k] = pp[k];
      t.grads[r][k] = gp[k];
      vec = vec && aligned16(pp[k]) && aligned16(gp[k]);
    }
  }
  float* mp[6] = {m.means, m.opacities, m.rotations, m.scales, m.sh0, m.sh_rest};
  float* vp[6] = {v.means, v.opacities, v.rotations, v.scales, v.sh0, v.sh_rest};
  int64_t chunks = 0;
  for (int k = 0; k < 6; ++k) {
    t.m[k] = mp[k];
    t.v[k] = vp[k];
    vec = vec && aligned16(mp[k]) && aligned16(vp[k]);
    t.lo[k] = lo_g * widths[k];
    t.hi[k] = hi_g * widths[k];
    t.goff[k] = grads_are_slices ? t.lo[k] : 0;
    t.lr[k] = adam.lr[k];
    t.decay[k] = adam.decay[k];
    t.kind[k] = adam.kind[k];
    t.chunk_begin[k] = chunks;
    chunks += (t.hi[k] - t.lo[k] + 3) / 4;
  }
  t.chunk_begin[6] = chunks;
  t.vec = vec ? 1 : 0;
  if (chunks <= 0) return;
  AdamScalars a{adam.beta1, adam.beta2, adam.eps, adam.gradient_scale, adam.bc1, adam.bc2_sqrt, adam.max_grad_1, 0};
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (chunks + 255) / 256;
  const int blocks = static_cast<int>(want < sms * 8 ? want : sms * 8);
  k_dp_adam<<<blocks, 256, 0, stream>>>(t, a, chunks);
}

void launch_adam(const AdamSegment* segs, int n_segs, float beta1, float beta2, float eps, float gradient_scale,
                 float bc1, float bc2_sqrt, float max_grad_1, int zero_grads, cudaStream_t stream) {
  SegTable t{};
  t.n = n_segs;
  int64_t chunks = 0;
  for (int k = 0; k < n_segs && k < kMaxSegs; ++k) {
    t.theta[k] = segs[k].theta;
    t.grad[k] = segs[k].grad;
    t.m[k] = segs[k].m;
    t.v[k] = segs[k].v;
    t.count[k] = segs[k].count;
    t.lr[k] = segs[k].lr;
    t.decay[k] = segs[k].decay;
    t.decay_kind[k] = segs[k].decay_kind;
    t.vec_ok[k] = aligned16(segs[k].theta) && aligned16(segs[k].grad) && aligned16(segs[k].m) &&
                  aligned16(segs[k].v);
    t.chunk_begin[k] = chunks;
    chunks += (segs[k].count + 3) / 4;
  }
  for (int k = n_segs; k <= kMaxSegs; ++k) t.chunk_begin[k < kMaxSegs + 1 ? k : kMaxSegs] = chunks;
  if (chunks == 0) return;
  AdamScalars a{beta1, beta2, eps, gradient_scale, bc1, bc2_sqrt, max_grad_1, zero_grads};
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (chunks + 255) / 256;
  const int blocks = static_cast<int>(want < sms * 8 ? want : sms * 8);
  k_adam<<<blocks, 256, 0, stream>>>(t, a, chunks);
}

}  // namespace tgs
