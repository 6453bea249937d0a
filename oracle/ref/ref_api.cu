// ref_api.cu -- the extern "C" functions of libtgs_ref.so (tgs_ref.h) and
// the reference's L1Loss / FusedSSIMLoss driven through LossBase::evaluate
// (tinygs/src/loss/l1.cu:109-151, fused_ssim.cu:797-916).  Exceptions of the
// reference code are caught here and reported through tgsref_last_error().
// Test infrastructure (oracle/_ref build).
#include <cstring>
#include <string>

#include "ref_common.h"
#include "tinygs/loss/fused_ssim.hpp"
#include "tinygs/loss/l1.hpp"

namespace {
thread_local std::string g_err;

template <typename F>
int guarded(F&& f) {
  try {
    f();
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
      g_err = cudaGetErrorString(e);
      return static_cast<int>(e);
    }
    return 0;
  } catch (const std::exception& ex) {
    g_err = ex.what();
    cudaGetLastError();  // a failed call must not be reported again by the next one
    return -1;
  }
}

tinygs::Image image_view(int fp16, int w, int h, const void* p) {
  tinygs::ImageShape s{static_cast<uint32_t>(w), static_cast<uint32_t>(h), 3u};
  return tinygs::Image(s, fp16 ? tinygs::DataType::Float16 : tinygs::DataType::Float32, const_cast<void*>(p));
}
}  // namespace

tgsref::RefHandle::~RefHandle() {
  cudaDeviceSynchronize();
  for (auto& b : blob)
    if (b) cudaFree(b);
  if (pose) cudaFree(pose);
  if (zero_copy) cudaFreeHost(zero_copy);
  if (helper) cudaStreamDestroy(helper);
  for (auto& e : ev)
    if (e) cudaEventDestroy(e);
  delete static_cast<tinygs::FusedSSIMLoss*>(ssim);
}

extern "C" {

int tgsref_create(void** handle) {
  return guarded([&] { *handle = new tgsref::RefHandle(); });
}

void tgsref_destroy(void* handle) { delete static_cast<tgsref::RefHandle*>(handle); }

int tgsref_forward(void* handle, int32_t fp16, const TgsRefGaussians* g, const TgsRefCamera* cam, void* image,
                   void* dens, void* stream, int32_t counts[3]) {
  auto* h = static_cast<tgsref::RefHandle*>(handle);
  const int st = guarded([&] {
    if (fp16)
      tgsref::forward_f16(h, g, cam, image, dens, static_cast<cudaStream_t>(stream));
    else
      tgsref::forward_f32(h, g, cam, image, dens, static_cast<cudaStream_t>(stream));
    tgsref::check(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "forward sync");
  });
  counts[0] = h->n_visible;
  counts[1] = h->n_instances;
  counts[2] = h->n_buckets;
  return st;
}

int tgsref_backward(void* handle, int32_t fp16, const TgsRefGaussians* g, const TgsRefCamera* cam,
                    const void* image, const void* grad_image, const TgsRefGaussians* grads, void* dens,
                    void* stream) {
  auto* h = static_cast<tgsref::RefHandle*>(handle);
  return guarded([&] {
    if (fp16)
      tgsref::backward_f16(h, g, cam, image, grad_image, grads, dens, static_cast<cudaStream_t>(stream));
    else
      tgsref::backward_f32(h, g, cam, image, grad_image, grads, dens, static_cast<cudaStream_t>(stream));
    tgsref::check(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "backward sync");
  });
}

int64_t tgsref_copy(void* handle, int32_t which, void* host_dst, int64_t max_bytes) {
  auto* h = static_cast<tgsref::RefHandle*>(handle);
  const void* p = nullptr;
  size_t bytes = 0;
  const bool ok = h->fp16 ? tgsref::locate_f16(h, which, &p, &bytes) : tgsref::locate_f32(h, which, &p, &bytes);
  if (!ok || p == nullptr) return -1;
  if (static_cast<int64_t>(bytes) > max_bytes) bytes = static_cast<size_t>(max_bytes);
  if (bytes == 0) return 0;
  if (cudaMemcpy(host_dst, p, bytes, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  return static_cast<int64_t>(bytes);
}

int tgsref_l1(int32_t fp16, int32_t width, int32_t height, const void* pred, const void* target, void* loss,
              void* grad, float scale, void* stream) {
  return guarded([&] {
    tinygs::L1Loss l1;
    tinygs::LossContext ctx{image_view(fp16, width, height, pred), image_view(fp16, width, height, target),
                            image_view(fp16, width, height, loss), image_view(fp16, width, height, grad),
                            static_cast<cudaStream_t>(stream)};
    l1.evaluate(ctx, scale);
    tgsref::check(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "l1 sync");
  });
}

int tgsref_ssim(void* handle, int32_t fp16, int32_t width, int32_t height, const void* pred, const void* target,
                void* loss, void* grad, float scale, void* stream) {
  auto* h = static_cast<tgsref::RefHandle*>(handle);
  return guarded([&] {
    if (h->ssim == nullptr) h->ssim = new tinygs::FusedSSIMLoss();
    tinygs::LossContext ctx{image_view(fp16, width, height, pred), image_view(fp16, width, height, target),
                            image_view(fp16, width, height, loss), image_view(fp16, width, height, grad),
                            static_cast<cudaStream_t>(stream)};
    static_cast<tinygs::FusedSSIMLoss*>(h->ssim)->evaluate(ctx, scale);
    tgsref::check(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "ssim sync");
  });
}

const char* tgsref_last_error(void) { return g_err.c_str(); }

}  // extern "C"
