// metrics.cu -- device-side training metrics with no host synchronisation.
//
// PSNR replaces PsnrMetric::evaluate (tinygs/src/loss/psnr.cu:72-128), which
// allocates a squared-difference buffer, reduces it with thrust and returns
// the value to the host (a synchronisation per call).  Here one pass over
// the image accumulates the squared differences per block in double and adds
// the block sums into a double accumulator; a second one-thread launch turns
// the sum into the PSNR, both left on the device for the caller to read when
// it wants (the reference's record_trajectory synchronises every step,
// orchestrator.cu:596-605, 763-807).
#include <algorithm>
#include <cmath>

#include "../../include/tgs_abi.h"
#include "kernels.h"

namespace tgs {
namespace {

constexpr int kThreads = 256;

template <int kFp16>
__global__ void __launch_bounds__(kThreads)
    k_sq_diff_sum(const void* __restrict__ pred, const void* __restrict__ target, uint32_t n,
                  double* __restrict__ acc) {
  double local = 0.0;
  for (uint32_t i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads) {
    float p, t;
    if constexpr (kFp16) {
      p = __half2float(static_cast<const __half*>(pred)[i]);
      t = __half2float(static_cast<const __half*>(target)[i]);
    } else {
      p = static_cast<const float*>(pred)[i];
      t = static_cast<const float*>(target)[i];
    }
    // psnr.cu:24-33: the prediction is saturated to [0, 1] first
    const float d = __fsub_rn(__saturatef(p), t);
    local += static_cast<double>(__fmul_rn(d, d));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) local += __shfl_xor_sync(0xffffffffu, local, o);
  __shared__ double s[kThreads / 32];
  if ((threadIdx.x & 31u) == 0) s[threadIdx.x >> 5] = local;
  __syncthreads();
  if (threadIdx.x == 0) {
    double b = 0.0;
    for (int w = 0; w < kThreads / 32; ++w) b += s[w];
    atomicAdd(acc, b);
  }
}

// out[0] = MSE over the real pixels (3 W H values; the padding holds zeros on
// both sides and adds nothing), out[1] = PSNR = -10 log10(MSE), 100 for a
// perfect match (psnr.cu:117-127).
__global__ void k_psnr_final(const double* __restrict__ acc, double npix, float* __restrict__ out) {
  const double mse = *acc / npix;
  out[0] = static_cast<float>(mse);
  out[1] = mse == 0.0 ? 100.0f : static_cast<float>(-10.0 * log10(mse));
}

}  // namespace
}  // namespace tgs

using namespace tgs;

extern "C" int tgs_metric_psnr(int32_t dtype, int32_t width, int32_t height, const void* pred, const void* target,
                               void* workspace, float* out, tgs_stream_t stream) {
  if ((dtype != TGS_FLOAT32 && dtype != TGS_FLOAT16) || width <= 0 || height <= 0 || pred == nullptr ||
      target == nullptr || workspace == nullptr || out == nullptr)
    return TGS_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint32_t n = 3u * static_cast<uint32_t>((width + 7) / 8 * 8) * static_cast<uint32_t>((height + 7) / 8 * 8);
  double* acc = static_cast<double*>(workspace);
  cudaMemsetAsync(acc, 0, sizeof(double), s);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uint32_t blocks = std::min<uint32_t>((n + kThreads - 1) / kThreads, static_cast<uint32_t>(sms) * 4u);
  if (dtype == TGS_FLOAT16)
    k_sq_diff_sum<1><<<blocks, kThreads, 0, s>>>(pred, target, n, acc);
  else
    k_sq_diff_sum<0><<<blocks, kThreads, 0, s>>>(pred, target, n, acc);
  k_psnr_final<<<1, 1, 0, s>>>(acc, 3.0 * width * height, out);
  return cudaGetLastError() == cudaSuccess ? TGS_OK : TGS_ERR_CUDA;
}
