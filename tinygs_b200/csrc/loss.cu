// loss.cu -- L1 and fused SSIM terms of the photometric loss, forward and
// backward, on 8x8-tiled CHW images in fp32 or fp16.
//
// References: tinygs/src/loss/l1.cu:19-151 and
// tinygs/src/loss/fused_ssim.cu:55-916 (11-tap Gaussian window, sigma 1.5,
// C1 = 0.01^2, C2 = 0.03^2, zero padding; the fp32 forward stages both images
// as fp16 in shared memory, which this implementation keeps because it
// changes the result at the 1e-3 level).
//
// Layout of the work: one CTA per 32x32 output tile and channel (grid.z = 3).
// The forward loads the 42x48 window once as aligned 8-pixel segments, runs
// the horizontal then the vertical pass of the five moment images in shared
// memory (four outputs per thread from a 14-value register window in each
// pass), writes the SSIM loss and the three per-pixel partial derivatives;
// the L1 term of the same pixels is fused into this pass.  The backward
// filters the partial-derivative maps the same way and finishes dL/dpred.
#include <cstring>

#include "kernels.h"

namespace tgs {
namespace {

constexpr int kHalo = 5;

__constant__ float c_gauss[11] = {0.001028380123898387f, 0.0075987582094967365f, 0.036000773310661316f,
                                  0.10936068743467331f,  0.21300552785396576f,   0.26601171493530273f,
                                  0.21300552785396576f,  0.10936068743467331f,   0.036000773310661316f,
                                  0.0075987582094967365f, 0.001028380123898387f};

template <int kFp16>
__device__ __forceinline__ float load_px(const void* p, uint32_t i) {
  if constexpr (kFp16)
    return __half2float(reinterpret_cast<const __half*>(p)[i]);
  else
    return reinterpret_cast<const float*>(p)[i];
}

template <int kFp16>
__device__ __forceinline__ void add_px(void* p, uint32_t i, float v, float s) {
  // p[i] += v * s, rounding once per update like the reference kernels
  if constexpr (kFp16) {
    __half* h = reinterpret_cast<__half*>(p);
    h[i] = __float2half_rn(fmaf(v, s, __half2float(h[i])));
  } else {
    float* f = reinterpret_cast<float*>(p);
    f[i] = fmaf(v, s, f[i]);
  }
}

// the image type's rounding of v (fp16: round to nearest half)
template <int kFp16>
__device__ __forceinline__ float round_px(float v) {
  if constexpr (kFp16)
    return __half2float(__float2half_rn(v));
  else
    return v;
}

template <int kFp16>
__device__ __forceinline__ void store_px(void* p, uint32_t i, float v) {
  if constexpr (kFp16)
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else
    reinterpret_cast<float*>(p)[i] = v;
}

__device__ __forceinline__ float block_sum_256(float v) {
  __shared__ float ws[8];
  v += __shfl_xor_sync(0xffffffffu, v, 16);
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  if ((threadIdx.x & 31u) == 0) ws[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x == 0)
    for (int w = 0; w < 8; ++w) t += ws[w];
  return t;
}

// Standalone L1 over every physical element (padding included), l1.cu:19-106.
template <int kFp16>
__global__ void k_l1(uint32_t total, const void* __restrict__ pred, const void* __restrict__ target,
                     void* __restrict__ loss_map, void* __restrict__ grad, float s) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const float d = sat(load_px<kFp16>(pred, i)) - load_px<kFp16>(target, i);
    if (loss_map != nullptr) add_px<kFp16>(loss_map, i, fabsf(d), s);
    if (grad != nullptr) add_px<kFp16>(grad, i, copysignf(1.0f, d), s);
  }
}

// Shared tile geometry of both SSIM passes: 32x32 output pixels of one
// channel per CTA; the input window is 42 rows (5-pixel halo) by 48 columns
// (six 8-pixel row segments of the tiled layout, x0 - 8 .. x0 + 40), so every
// global load is one aligned 8-pixel segment.
constexpr int kOut = 32;
constexpr int kInH = kOut + 2 * kHalo;  // 42
constexpr int kInW = kOut + 16;         // 48
constexpr int kSegs = kInW / 8;         // 6
// shared-memory row strides padded by one word: the horizontal pass has
// lanes on four rows (and eight column groups) at once, which an unpadded
// 32- or 48-word stride maps onto the same eight banks
constexpr int kInStride = kInW + 1;
constexpr int kSumStride = kOut + 1;

__device__ __forceinline__ bool segment_of(const DevCamera& cam, int x0, int y0, int r, int sg, uint32_t& idx,
                                           int& gx0) {
  const int gy = y0 - kHalo + r;
  gx0 = x0 - 8 + 8 * sg;
  if (gy < 0 || gy >= static_cast<int>(cam.height) || gx0 < 0 || gx0 >= static_cast<int>(cam.width)) return false;
  idx = tiled_index(static_cast<uint32_t>(gy), static_cast<uint32_t>(gx0), cam.tiled_w);
  return true;
}

// Horizontal 11-tap sums of four consecutive outputs from 14 inputs.
template <int kM>
__device__ __forceinline__ void taps4(const float (&in)[kM][14], float (&out)[kM][4]) {
#pragma unroll
  for (int m = 0; m < kM; ++m)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float acc = 0.f;
#pragma unroll
      for (int d = 0; d < 11; ++d) acc += in[m][k + d] * c_gauss[d];
      out[m][k] = acc;
    }
}

// SSIM forward (+ fused L1).  Moments mu_p, E[p^2], mu_t, E[t^2], E[pt] by
// separable 11x11 Gaussian filtering of the half-precision window.
template <int kFp16>
__global__ void __launch_bounds__(256)
    k_ssim_forward(DevCamera cam, const void* __restrict__ pred, const void* __restrict__ target,
                   void* __restrict__ loss_map, void* __restrict__ grad, float s_ssim, float s_l1,
                   float* __restrict__ partials, float* __restrict__ loss_sum, int accumulate) {
  __shared__ __half2 tile[kInH][kInStride];  // (pred, target)
  __shared__ float hsum[5][kInH][kSumStride];
  const int x0 = blockIdx.x * kOut, y0 = blockIdx.y * kOut;
  const uint32_t ch = blockIdx.z * cam.plane;
  const int W = static_cast<int>(cam.width), H = static_cast<int>(cam.height);
  // load: one 8-pixel segment per (row, segment)
  for (int k = threadIdx.x; k < kInH * kSegs; k += 256) {
    const int r = k / kSegs, sg = k % kSegs;
    uint32_t idx;
    int gx0;
    __half2 v[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) v[q] = __float2half2_rn(0.f);
    if (segment_of(cam, x0, y0, r, sg, idx, gx0)) {
      __half p[8], t[8];
      if constexpr (kFp16) {
        const uint4 pv = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(pred) + ch + idx);
        const uint4 tv = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(target) + ch + idx);
        memcpy(p, &pv, 16);
        memcpy(t, &tv, 16);
      } else {
        const float4* pf = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(pred) + ch + idx);
        const float4* tf = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(target) + ch + idx);
        const float4 p0 = pf[0], p1 = pf[1], t0 = tf[0], t1 = tf[1];
        const float pa[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        const float ta[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          p[q] = __float2half_rn(pa[q]);
          t[q] = __float2half_rn(ta[q]);
        }
      }
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (gx0 + q < W) v[q] = __halves2half2(p[q], t[q]);
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) tile[r][8 * sg + q] = v[q];
  }
  __syncthreads();
  // horizontal: four consecutive outputs per item (output x reads window
  // columns x + 3 .. x + 13)
  for (int it = threadIdx.x; it < kInH * (kOut / 4); it += 256) {
    const int r = it / (kOut / 4), c0 = 4 * (it % (kOut / 4));
    float in[5][14];
#pragma unroll
    for (int j = 0; j < 14; ++j) {
      const float2 xy = __half22float2(tile[r][c0 + 3 + j]);
      in[0][j] = xy.x;
      in[1][j] = xy.x * xy.x;
      in[2][j] = xy.y;
      in[3][j] = xy.y * xy.y;
      in[4][j] = xy.x * xy.y;
    }
    float out[5][4];
    taps4<5>(in, out);
#pragma unroll
    for (int m = 0; m < 5; ++m)
#pragma unroll
      for (int k = 0; k < 4; ++k) hsum[m][r][c0 + k] = out[m][k];
  }
  __syncthreads();
  // vertical: lane = column, warp = group of four rows
  const int c = threadIdx.x & 31, q0 = 4 * (threadIdx.x >> 5);
  float in[5][14];
#pragma unroll
  for (int m = 0; m < 5; ++m)
#pragma unroll
    for (int j = 0; j < 14; ++j) in[m][j] = hsum[m][q0 + j][c];
  float o[5][4];
  taps4<5>(in, o);
  const int px = x0 + c;
  float contrib = 0.f;
  const uint32_t plane3 = 3 * cam.plane;
  // every global load of the four pixels first, then the arithmetic, then
  // the stores; fp16 images inside the picture come from the staged window
  // (exact), the L1 term's padding pixels from memory
  // accumulate == 0: every pixel of the padded extent is written (from zero)
  uint32_t pis[4];
  bool l1_on[4], in_img[4], in_pad[4];
  float pv[4], tv[4], lm[4], gr[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int py = y0 + q0 + k;
    pis[k] = ch + tiled_index(static_cast<uint32_t>(py), static_cast<uint32_t>(px), cam.tiled_w);
    in_pad[k] = static_cast<uint32_t>(px) < cam.tiled_w * 8u && static_cast<uint32_t>(py) < cam.tiled_h * 8u;
    l1_on[k] = s_l1 != 0.f && in_pad[k];
    in_img[k] = px < W && py < H;
    pv[k] = tv[k] = lm[k] = gr[k] = 0.f;
    if (l1_on[k]) {
      if (kFp16 && in_img[k]) {
        const float2 v = __half22float2(tile[q0 + k + kHalo][c + 8]);
        pv[k] = v.x;
        tv[k] = v.y;
      } else {
        pv[k] = load_px<kFp16>(pred, pis[k]);
        tv[k] = load_px<kFp16>(target, pis[k]);
      }
      if (grad != nullptr && accumulate) gr[k] = load_px<kFp16>(grad, pis[k]);
    }
    if (loss_map != nullptr && accumulate && (l1_on[k] || in_img[k])) lm[k] = load_px<kFp16>(loss_map, pis[k]);
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t pi = pis[k];
    float lmv = lm[k];
    // fused L1 term over the padded physical extent (l1.cu:117-129); applied
    // first, as the reference evaluates the L1 loss before the SSIM loss;
    // each update of the loss map and the gradient rounds once to the image
    // type, like two separate read-modify-writes
    if (l1_on[k]) {
      const float d = sat(pv[k]) - tv[k];
      contrib += fabsf(d) * s_l1;
      lmv = round_px<kFp16>(fmaf(fabsf(d), s_l1, lmv));
      if (grad != nullptr) store_px<kFp16>(grad, pi, round_px<kFp16>(fmaf(copysignf(1.0f, d), s_l1, gr[k])));
    } else if (!accumulate && grad != nullptr && in_pad[k]) {
      store_px<kFp16>(grad, pi, 0.0f);
    }
    if (in_img[k]) {
      const float C1 = 0.01f * 0.01f, C2 = 0.03f * 0.03f;
      const float mu1 = o[0][k], mu2 = o[2][k];
      const float m11 = mu1 * mu1, m22 = mu2 * mu2;
      const float sg1 = o[1][k] - m11, sg2 = o[3][k] - m22, sg12 = o[4][k] - mu1 * mu2;
      const float A = m11 + m22 + C1, B = sg1 + sg2 + C2;
      const float Cc = 2.f * mu1 * mu2 + C1, D = 2.f * sg12 + C2;
      const float val = (Cc * D) / (A * B);
      lmv = round_px<kFp16>(fmaf(1.0f - val, s_ssim, lmv));
      contrib += (1.0f - val) * s_ssim;
      if (partials != nullptr) {
        partials[pi] = (mu2 * 2.f * D) / (A * B) - (mu2 * 2.f * Cc) / (A * B) - (mu1 * 2.f * Cc * D) / (A * A * B) +
                       (mu1 * 2.f * Cc * D) / (A * B * B);
        partials[pi + plane3] = (-Cc * D) / (A * B * B);
        partials[pi + 2 * plane3] = (2.f * Cc) / (A * B);
      }
    }
    if (loss_map != nullptr && (l1_on[k] || in_img[k] || (!accumulate && in_pad[k]))) store_px<kFp16>(loss_map, pi, lmv);
  }
  if (loss_sum != nullptr) {
    const float t = block_sum_256(contrib);
    if (threadIdx.x == 0) atomicAdd(loss_sum, t);
  }
}

// SSIM backward: dL/dpred = -s * (G*d_mu + 2 p G*d_s1 + t G*d_s12), the three
// partial-derivative maps filtered with the same separable window.
template <int kFp16>
__global__ void __launch_bounds__(256)
    k_ssim_backward(DevCamera cam, const void* __restrict__ pred, const void* __restrict__ target,
                    void* __restrict__ grad, float s_ssim, const float* __restrict__ partials) {
  __shared__ float tile[3][kInH][kInStride];
  __shared__ float hsum[3][kInH][kSumStride];
  const int x0 = blockIdx.x * kOut, y0 = blockIdx.y * kOut;
  const uint32_t ch = blockIdx.z * cam.plane;
  const uint32_t plane3 = 3 * cam.plane;
  const int W = static_cast<int>(cam.width), H = static_cast<int>(cam.height);
  for (int k = threadIdx.x; k < 3 * kInH * kSegs; k += 256) {
    const int m = k / (kInH * kSegs), rs = k % (kInH * kSegs);
    const int r = rs / kSegs, sg = rs % kSegs;
    uint32_t idx;
    int gx0;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (segment_of(cam, x0, y0, r, sg, idx, gx0)) {
      const float4* src = reinterpret_cast<const float4*>(partials + ch + idx + m * plane3);
      const float4 a = src[0], b = src[1];
      const float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (gx0 + q < W) v[q] = f[q];
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) tile[m][r][8 * sg + q] = v[q];
  }
  __syncthreads();
  for (int it = threadIdx.x; it < kInH * (kOut / 4); it += 256) {
    const int r = it / (kOut / 4), c0 = 4 * (it % (kOut / 4));
    float in[3][14];
#pragma unroll
    for (int m = 0; m < 3; ++m)
#pragma unroll
      for (int j = 0; j < 14; ++j) in[m][j] = tile[m][r][c0 + 3 + j];
    float out[3][4];
    taps4<3>(in, out);
#pragma unroll
    for (int m = 0; m < 3; ++m)
#pragma unroll
      for (int k = 0; k < 4; ++k) hsum[m][r][c0 + k] = out[m][k];
  }
  __syncthreads();
  const int c = threadIdx.x & 31, q0 = 4 * (threadIdx.x >> 5);
  float in[3][14];
#pragma unroll
  for (int m = 0; m < 3; ++m)
#pragma unroll
    for (int j = 0; j < 14; ++j) in[m][j] = hsum[m][q0 + j][c];
  float o[3][4];
  taps4<3>(in, o);
  const int px = x0 + c;
  if (px >= W) return;
  uint32_t pis[4];
  float p1[4], p2[4], g0[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int py = y0 + q0 + k;
    pis[k] = ch + tiled_index(static_cast<uint32_t>(py), static_cast<uint32_t>(px), cam.tiled_w);
    p1[k] = p2[k] = g0[k] = 0.f;
    if (py < H) {
      p1[k] = load_px<kFp16>(pred, pis[k]);
      p2[k] = load_px<kFp16>(target, pis[k]);
      g0[k] = load_px<kFp16>(grad, pis[k]);
    }
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (y0 + q0 + k >= H) break;
    const float dL = o[0][k] + (2.f * p1[k]) * o[1][k] + p2[k] * o[2][k];
    store_px<kFp16>(grad, pis[k], round_px<kFp16>(fmaf(dL, -s_ssim, g0[k])));
  }
}

}  // namespace

static DevCamera image_geometry(int width, int height) {
  DevCamera c{};
  c.width = static_cast<uint32_t>(width);
  c.height = static_cast<uint32_t>(height);
  c.tiled_w = (c.width + 7u) >> 3;
  c.tiled_h = (c.height + 7u) >> 3;
  c.plane = c.tiled_w * c.tiled_h * 64u;
  return c;
}

void launch_l1(int fp16, int width, int height, const void* pred, const void* target, void* loss_map, void* grad,
               float scale, cudaStream_t stream) {
  const DevCamera g = image_geometry(width, height);
  const uint32_t total = 3u * g.plane;
  const float s = scale / static_cast<float>(width * height * 3);
  const uint32_t blocks = min((total + 255u) / 256u, 148u * 16u);
  if (fp16)
    k_l1<1><<<blocks, 256, 0, stream>>>(total, pred, target, loss_map, grad, s);
  else
    k_l1<0><<<blocks, 256, 0, stream>>>(total, pred, target, loss_map, grad, s);
}

// scale_l1 == 0 disables the fused L1 term; grad == nullptr skips the backward.
void launch_ssim(int fp16, int width, int height, const void* pred, const void* target, void* loss_map,
                 void* grad, float scale_ssim, float scale_l1, float* partials, float* loss_sum,
                 cudaStream_t stream, int accumulate) {
  const DevCamera g = image_geometry(width, height);
  const dim3 grid((width + kOut - 1) / kOut, (height + kOut - 1) / kOut, 3);
  const float s_ssim = scale_ssim / static_cast<float>(width * height);
  const float s_l1 = scale_l1 / static_cast<float>(width * height * 3);
  float* parts = grad != nullptr ? partials : nullptr;
  if (fp16) {
    k_ssim_forward<1><<<grid, 256, 0, stream>>>(g, pred, target, loss_map, grad, s_ssim, s_l1, parts, loss_sum,
                                                accumulate);
    if (grad != nullptr) k_ssim_backward<1><<<grid, 256, 0, stream>>>(g, pred, target, grad, s_ssim, partials);
  } else {
    k_ssim_forward<0><<<grid, 256, 0, stream>>>(g, pred, target, loss_map, grad, s_ssim, s_l1, parts, loss_sum,
                                                accumulate);
    if (grad != nullptr) k_ssim_backward<0><<<grid, 256, 0, stream>>>(g, pred, target, grad, s_ssim, partials);
  }
}

}  // namespace tgs
