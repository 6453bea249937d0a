// image.cu -- the data path of the training loop: 8-bit images from the
// host turned into the rasterizer's tiled CHW layout (fp32 / fp16 / u8) on
// the device, with the reference's resize modes.
//
// Reference: DataLoaderBase::transfer_gpu (tinygs/src/dataloader/
// dataloader.cu:218-339) and its kernels (:26-186): same-shape conversion
// c / 255 (v * (1.0f/255.0f), rounded to half for fp16), nearest resize and
// the stochastic-blur resize that draws one source pixel per destination
// pixel and channel from a per-element PCG32 state (:122-186), the states
// initialised by one sequential pcg32(0, 1) stream (:361-378).  The HWC ->
// tiled reorder that the reference does on the host while loading a PNG
// (tinygs/src/dataset/png_folder.cpp:60-69) is done here on the device, so
// the host ships decoded rows as they come (3 or 4 bytes per pixel).
//
// Layout: channel planes of 8x8 pixel tiles, tiles row-major, pixels within
// a tile row-major (include/tinygs/common.hpp:367-413); planes are
// padded_width x padded_height (multiples of 8).  The HWC reorder and the
// resize write padding pixels as zero; the same-layout conversion converts
// the source's padding with the rest, as the reference does.
#include "kernels.h"
#include "tgs_abi.h"

namespace tgs {
namespace {

constexpr float kU8Scale = 1.0f / 255.0f;

__host__ __device__ inline uint32_t pad8(uint32_t x) { return (x + 7u) & ~7u; }

__device__ __forceinline__ uint32_t tiled_index(uint32_t y, uint32_t x, uint32_t tiles_w) {
  return (((y >> 3) * tiles_w + (x >> 3)) << 6) + ((y & 7u) << 3) + (x & 7u);
}

template <int kOut>
__device__ __forceinline__ void put(void* dst, size_t i, uint32_t v) {
  if constexpr (kOut == TGS_FLOAT32) {
    static_cast<float*>(dst)[i] = kU8Scale * static_cast<float>(v);
  } else if constexpr (kOut == TGS_FLOAT16) {
    static_cast<__half*>(dst)[i] = __float2half_rn(kU8Scale * static_cast<float>(v));
  } else {
    static_cast<uint8_t*>(dst)[i] = static_cast<uint8_t>(v);
  }
}

// Same layout, same shape: 16 bytes in, 16 elements out per thread and
// iteration (the padded plane is a multiple of 64 elements).
template <int kOut>
__global__ void __launch_bounds__(256) k_convert_tiled(const uint4* __restrict__ src, void* __restrict__ dst,
                                                       size_t chunks) {
  for (size_t c = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; c < chunks;
       c += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint4 w = src[c];
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
    if constexpr (kOut == TGS_FLOAT32) {
      float4* o = static_cast<float4*>(dst) + 4 * c;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t u = words[k];
        o[k] = make_float4(kU8Scale * static_cast<float>(u & 0xffu), kU8Scale * static_cast<float>((u >> 8) & 0xffu),
                           kU8Scale * static_cast<float>((u >> 16) & 0xffu), kU8Scale * static_cast<float>(u >> 24));
      }
    } else if constexpr (kOut == TGS_FLOAT16) {
      uint4* o = static_cast<uint4*>(dst) + 2 * c;
      uint32_t h[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t u = words[k];
        const __half2 lo = __halves2half2(__float2half_rn(kU8Scale * static_cast<float>(u & 0xffu)),
                                          __float2half_rn(kU8Scale * static_cast<float>((u >> 8) & 0xffu)));
        const __half2 hi = __halves2half2(__float2half_rn(kU8Scale * static_cast<float>((u >> 16) & 0xffu)),
                                          __float2half_rn(kU8Scale * static_cast<float>(u >> 24)));
        memcpy(&h[2 * k], &lo, 4);
        memcpy(&h[2 * k + 1], &hi, 4);
      }
      o[0] = make_uint4(h[0], h[1], h[2], h[3]);
      o[1] = make_uint4(h[4], h[5], h[6], h[7]);
    } else {
      static_cast<uint4*>(dst)[c] = w;
    }
  }
}

// HWC rows -> tiled CHW.  A block takes one band of 8 rows and up to 32
// tiles of it (256 columns): the band's bytes are read row by row
// (coalesced) into shared memory, then each output channel's run of
// 32 x 64 tiled elements -- contiguous in the destination -- is written
// coalesced.
constexpr int kBandTiles = 32;
template <int kOut>
__global__ void __launch_bounds__(256) k_hwc_to_tiled(const uint8_t* __restrict__ src, int channels_in,
                                                      uint32_t width, uint32_t height, void* __restrict__ dst) {
  __shared__ uint8_t band[8][kBandTiles * 8 * 4];
  const uint32_t tiles_w = pad8(width) >> 3;
  const uint32_t plane = pad8(width) * pad8(height);
  const uint32_t ty = blockIdx.y, tx0 = blockIdx.x * kBandTiles;
  const uint32_t x0 = tx0 * 8;
  const uint32_t cols = min(static_cast<uint32_t>(kBandTiles * 8), width > x0 ? width - x0 : 0u);
  const uint32_t row_bytes = cols * static_cast<uint32_t>(channels_in);
  for (uint32_t r = 0; r < 8; ++r) {
    const uint32_t y = ty * 8 + r;
    if (y >= height) break;
    const uint8_t* row = src + (static_cast<size_t>(y) * width + x0) * channels_in;
    for (uint32_t b = threadIdx.x; b < row_bytes; b += blockDim.x) band[r][b] = row[b];
  }
  __syncthreads();
  const uint32_t n_tiles = min(static_cast<uint32_t>(kBandTiles), tiles_w - tx0);
  const size_t run0 = (static_cast<size_t>(ty) * tiles_w + tx0) << 6;
  for (int c = 0; c < 3; ++c) {
    for (uint32_t e = threadIdx.x; e < n_tiles * 64u; e += blockDim.x) {
      const uint32_t t = e >> 6, iy = (e >> 3) & 7u, ix = e & 7u;
      const uint32_t xl = t * 8 + ix, y = ty * 8 + iy;
      const uint32_t v = (xl < cols && y < height) ? band[iy][xl * channels_in + c] : 0u;
      put<kOut>(dst, static_cast<size_t>(c) * plane + run0 + e, v);
    }
  }
}

// (uint32_t)((float)x * (float)src / (float)dst) of the reference, in IEEE
// single precision whatever the build's fast-math setting
__device__ __forceinline__ uint32_t src_coord(uint32_t x, uint32_t src, uint32_t dst) {
  return min(__float2uint_rz(__fdiv_rn(__fmul_rn(static_cast<float>(x), static_cast<float>(src)),
                                       static_cast<float>(dst))),
             src - 1u);
}

// Tiled u8 source -> tiled destination of another shape, one thread per
// destination pixel (padding included, written as zero).  kBlur: the
// stochastic blur of dataloader.cu:122-186 (per element: pcg32(state, 1),
// dx then dy drawn as next_uint() % span, state written back); otherwise
// nearest (dataloader.cu:107-120).
template <int kOut, bool kBlur>
__global__ void __launch_bounds__(256) k_resize_tiled(const uint8_t* __restrict__ src, uint32_t src_w, uint32_t src_h,
                                                      void* __restrict__ dst, uint32_t dst_w, uint32_t dst_h,
                                                      int channels, uint64_t* __restrict__ state) {
  const uint32_t x = blockIdx.x * 16 + (threadIdx.x & 15u);
  const uint32_t y = blockIdx.y * 16 + (threadIdx.x >> 4);
  const uint32_t dtw = pad8(dst_w) >> 3, stw = pad8(src_w) >> 3;
  if (x >= pad8(dst_w) || y >= pad8(dst_h)) return;
  const uint32_t dplane = pad8(dst_w) * pad8(dst_h), splane = pad8(src_w) * pad8(src_h);
  const uint32_t di = tiled_index(y, x, dtw);
  if (x >= dst_w || y >= dst_h) {
    for (int c = 0; c < channels; ++c) put<kOut>(dst, static_cast<size_t>(c) * dplane + di, 0u);
    return;
  }
  const uint32_t sx = src_coord(x, src_w, dst_w), sy = src_coord(y, src_h, dst_h);
  if constexpr (!kBlur) {
    const uint32_t si = tiled_index(sy, sx, stw);
    for (int c = 0; c < channels; ++c)
      put<kOut>(dst, static_cast<size_t>(c) * dplane + di, src[static_cast<size_t>(c) * splane + si]);
  } else {
    const uint32_t span_x = src_coord(x + 1, src_w, dst_w) - sx + 1u;
    const uint32_t span_y = src_coord(y + 1, src_h, dst_h) - sy + 1u;
    for (int c = 0; c < channels; ++c) {
      const size_t o = static_cast<size_t>(c) * dplane + di;
      Pcg g = Pcg::seeded(state[o], 1u);
      const uint32_t dx = g.next_uint() % span_x;
      const uint32_t dy = g.next_uint() % span_y;
      const uint32_t si = tiled_index(sy + dy, sx + dx, stw);
      put<kOut>(dst, o, src[static_cast<size_t>(c) * splane + si]);
      state[o] = g.state;
    }
  }
}

// state[i] = (u << 32) | l with u, l the (2i)th and (2i+1)th outputs of
// pcg32(seed, 1): the reference's sequential host loop, each element
// jumping ahead to its own position.
__global__ void __launch_bounds__(256) k_blur_state_init(uint64_t* __restrict__ state, size_t n, Pcg base) {
  const size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  if (i >= n) return;
  Pcg g = base;
  g.advance(2u * static_cast<uint64_t>(i));
  const uint64_t up = g.next_uint();
  const uint64_t lo = g.next_uint();
  state[i] = (up << 32) | lo;
}

int grid_for(size_t work, int per_block) {
  const size_t b = (work + per_block - 1) / per_block;
  return static_cast<int>(b < 148u * 16u ? (b > 0 ? b : 1) : 148u * 16u);
}

template <int kOut>
void launch_from_u8(const uint8_t* src, int layout, int channels, uint32_t w, uint32_t h, void* dst,
                    cudaStream_t st) {
  if (layout == TGS_IMAGE_TILED_CHW) {
    const size_t chunks = static_cast<size_t>(pad8(w)) * pad8(h) * channels / 16u;
    k_convert_tiled<kOut><<<grid_for(chunks, 256), 256, 0, st>>>(reinterpret_cast<const uint4*>(src), dst, chunks);
  } else {
    const dim3 grid((pad8(w) / 8 + kBandTiles - 1) / kBandTiles, pad8(h) / 8);
    k_hwc_to_tiled<kOut><<<grid, 256, 0, st>>>(src, channels, w, h, dst);
  }
}

template <int kOut>
void launch_resize(const uint8_t* src, uint32_t sw, uint32_t sh, int channels, void* dst, uint32_t dw,
                   uint32_t dh, uint64_t* state, cudaStream_t st) {
  const dim3 grid((pad8(dw) + 15) / 16, (pad8(dh) + 15) / 16);
  if (state != nullptr)
    k_resize_tiled<kOut, true><<<grid, 256, 0, st>>>(src, sw, sh, dst, dw, dh, channels, state);
  else
    k_resize_tiled<kOut, false><<<grid, 256, 0, st>>>(src, sw, sh, dst, dw, dh, channels, nullptr);
}

bool size_ok(int32_t w, int32_t h) { return w > 0 && h > 0 && w <= 16384 && h <= 16384; }

}  // namespace
}  // namespace tgs

using namespace tgs;

extern "C" {

int tgs_image_from_u8(const uint8_t* src, int32_t layout, int32_t src_channels, int32_t width, int32_t height,
                      void* dst, int32_t dst_dtype, tgs_stream_t stream) {
  if (src == nullptr || dst == nullptr || !size_ok(width, height)) return TGS_ERR_INVALID_ARGUMENT;
  if (layout == TGS_IMAGE_TILED_CHW) {
    if (src_channels != 3 && src_channels != 4) return TGS_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(src) & 15u) != 0 || (reinterpret_cast<uintptr_t>(dst) & 15u) != 0)
      return TGS_ERR_INVALID_ARGUMENT;
  } else if (layout == TGS_IMAGE_HWC) {
    if (src_channels != 3 && src_channels != 4) return TGS_ERR_INVALID_ARGUMENT;
  } else {
    return TGS_ERR_INVALID_ARGUMENT;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint32_t w = static_cast<uint32_t>(width), h = static_cast<uint32_t>(height);
  switch (dst_dtype) {
    case TGS_FLOAT32: launch_from_u8<TGS_FLOAT32>(src, layout, src_channels, w, h, dst, st); break;
    case TGS_FLOAT16: launch_from_u8<TGS_FLOAT16>(src, layout, src_channels, w, h, dst, st); break;
    case TGS_UINT8: launch_from_u8<TGS_UINT8>(src, layout, src_channels, w, h, dst, st); break;
    default: return TGS_ERR_INVALID_ARGUMENT;
  }
  return cudaGetLastError() == cudaSuccess ? TGS_OK : TGS_ERR_CUDA;
}

int tgs_image_resize_u8(const uint8_t* src, int32_t src_width, int32_t src_height, int32_t channels, void* dst,
                        int32_t dst_dtype, int32_t dst_width, int32_t dst_height, uint64_t* blur_state,
                        tgs_stream_t stream) {
  if (src == nullptr || dst == nullptr || !size_ok(src_width, src_height) || !size_ok(dst_width, dst_height) ||
      (channels != 3 && channels != 4))
    return TGS_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint32_t sw = src_width, sh = src_height, dw = dst_width, dh = dst_height;
  switch (dst_dtype) {
    case TGS_FLOAT32: launch_resize<TGS_FLOAT32>(src, sw, sh, channels, dst, dw, dh, blur_state, st); break;
    case TGS_FLOAT16: launch_resize<TGS_FLOAT16>(src, sw, sh, channels, dst, dw, dh, blur_state, st); break;
    default: return TGS_ERR_INVALID_ARGUMENT;
  }
  return cudaGetLastError() == cudaSuccess ? TGS_OK : TGS_ERR_CUDA;
}

int tgs_image_blur_state_init(uint64_t* state, int64_t n, uint64_t seed, tgs_stream_t stream) {
  if (state == nullptr || n < 0) return TGS_ERR_INVALID_ARGUMENT;
  if (n == 0) return TGS_OK;
  const Pcg base = Pcg::seeded(seed, 1u);
  const size_t count = static_cast<size_t>(n);
  k_blur_state_init<<<static_cast<unsigned>((count + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      state, count, base);
  return cudaGetLastError() == cudaSuccess ? TGS_OK : TGS_ERR_CUDA;
}

}  // extern "C"
