// noalloc.cu -- tgs_loss_l1_ssim_noalloc: the fused L1 + SSIM loss for
// callers that cannot allocate device memory.
//
// Some hosts own every byte of device memory themselves (a framework's
// caching allocator or memory pool, an embedding engine with a fixed budget)
// or run the loss where allocation is not allowed at all; such callers can
// neither call cudaMalloc nor hold a TgsLoss handle, whose creation
// allocates the SSIM partial-derivative maps.  This entry point keeps those
// maps in a fixed array of device memory that belongs to the library itself
// instead.  The caller still passes inputs and outputs.
//
// The array is a file-scope __device__ variable: every GPU that loads this
// library holds it (TGS_NOALLOC_MAX_PIXELS * 9 floats, 9 MiB) until the
// process exits, and every call on a device shares it.  It needs no clearing
// between calls: the forward pass writes each map entry it later reads.
// Calls whose work overlaps on the GPU (different streams, no ordering) race
// on the array and must be serialised by the caller.
//
// The array is placed in device memory when the library's device code is
// loaded on a device.  With lazy module loading (the CUDA default) that is
// the first call of this library on that device; a host that lets its own
// pool reserve all free device memory must make that first call (for
// example one warm-up call of this entry point) before the pool reserves
// it, or the load fails and the call returns TGS_ERR_CUDA.
#include "../../include/tgs_abi.h"
#include "kernels.h"

namespace {

// Three partial-derivative maps for each of the three channels.
static __device__ __align__(256) float g_ssim_scratch[9 * static_cast<size_t>(TGS_NOALLOC_MAX_PIXELS)];

// The host-side name of a __device__ array is not a device address.  The
// device address is looked up on every call, with the caller's device
// current: the lookup allocates nothing and costs about a microsecond, and a
// cached address would go stale when the module is loaded again at another
// address (after cudaDeviceReset, or in another driver-API context).
int scratch_for_current_device(float** out) {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_ssim_scratch) != cudaSuccess) {
    cudaGetLastError();
    return TGS_ERR_CUDA;
  }
  *out = static_cast<float*>(p);
  return TGS_OK;
}

}  // namespace

extern "C" int tgs_loss_l1_ssim_noalloc(int32_t dtype, int32_t width, int32_t height, const void* pred,
                                        const void* target, void* loss_map, void* grad, float scale_l1,
                                        float scale_ssim, float* loss_sum, tgs_stream_t stream) {
  if ((dtype != TGS_FLOAT32 && dtype != TGS_FLOAT16) || width <= 0 || height <= 0 || pred == nullptr ||
      target == nullptr)
    return TGS_ERR_INVALID_ARGUMENT;
  const int64_t padded = static_cast<int64_t>((width + 7) / 8 * 8) * ((height + 7) / 8 * 8);
  if (padded > TGS_NOALLOC_MAX_PIXELS) return TGS_ERR_CAPACITY;
  float* scratch = nullptr;
  const int st = scratch_for_current_device(&scratch);
  if (st != TGS_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (loss_sum != nullptr) cudaMemsetAsync(loss_sum, 0, sizeof(float), s);
  if (scale_l1 != 0.0f || scale_ssim != 0.0f)
    tgs::launch_ssim(dtype == TGS_FLOAT16, width, height, pred, target, loss_map, grad, scale_ssim, scale_l1,
                     scratch, loss_sum, s);
  return cudaGetLastError() == cudaSuccess ? TGS_OK : TGS_ERR_CUDA;
}
