// ref_common.h -- the handle shared by the reference-harness translation
// units: growing scratch blobs (the reference's per-primitive / per-tile /
// per-instance / per-bucket buffers, handed to it through its allocator
// callbacks as FastGSRasterizer::Impl::alloc does, fastgs.cu:71-78), the
// pose block, the helper stream, events and the mapped count page.
// Test infrastructure (oracle/_ref build).
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <algorithm>
#include <string>
#include <vector>

#include "tgs_ref.h"

namespace tgsref {

inline size_t padded_plane(int w, int h) { return (size_t)((w + 7) / 8 * 8) * ((h + 7) / 8 * 8); }

inline void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

struct RefHandle {
  enum { kPrim = 0, kTile, kInst, kBucket, kAlpha, kHelper, kNumBlobs };
  char* blob[kNumBlobs] = {};
  size_t cap[kNumBlobs] = {};
  float* pose = nullptr;      // w2c rows (4 x float4) | cam position (float3) | grad w2c (16 floats)
  char* zero_copy = nullptr;  // mapped pinned page for the reference's counts
  cudaStream_t helper = nullptr;
  cudaEvent_t ev[3] = {};
  int n = 0, width = 0, height = 0, fp16 = 0;
  int n_visible = 0, n_instances = 0, n_buckets = 0, prim_selector = 0, inst_selector = 0;
  void* ssim = nullptr;  // FusedSSIMLoss, created on first use

  RefHandle() {
    check(cudaMalloc(&pose, 64 * sizeof(float)), "cudaMalloc pose");
    check(cudaMemset(pose, 0, 64 * sizeof(float)), "cudaMemset pose");
    check(cudaHostAlloc(&zero_copy, 1024, cudaHostAllocMapped), "cudaHostAlloc");
    check(cudaStreamCreateWithFlags(&helper, cudaStreamNonBlocking), "cudaStreamCreate");
    for (auto& e : ev) check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
  }
  ~RefHandle();

  // Grows blob k to at least `bytes` (zero-filled when new); never shrinks.
  char* grow(int k, size_t bytes) {
    if (bytes > cap[k]) {
      check(cudaDeviceSynchronize(), "sync before grow");
      if (blob[k]) cudaFree(blob[k]);
      blob[k] = nullptr;
      const cudaError_t e = cudaMalloc(&blob[k], bytes);
      if (e != cudaSuccess) {
        cudaGetLastError();
        size_t free_b = 0, total_b = 0;
        cudaMemGetInfo(&free_b, &total_b);
        blob[k] = nullptr;
        cap[k] = 0;
        throw std::runtime_error("cudaMalloc of blob " + std::to_string(k) + " (" + std::to_string(bytes) +
                                 " bytes, " + std::to_string(free_b) + " free): " + cudaGetErrorString(e));
      }
      check(cudaMemset(blob[k], 0, bytes), "cudaMemset blob");
      cap[k] = bytes;
    }
    return blob[k];
  }

  const float4* pose_w2c() const { return reinterpret_cast<const float4*>(pose); }
  const float3* pose_cam() const { return reinterpret_cast<const float3*>(pose + 16); }
  float4* pose_grad() const { return reinterpret_cast<float4*>(pose + 32); }

  // The pose block of FastGSRasterizer::forward (fastgs.cu:95-106): the four
  // rows of w2c as float4 and the camera centre, the translation of
  // inverse(w2c) (evaluated here in double).
  void upload_pose(const TgsRefCamera& c, cudaStream_t s) {
    float host[20];
    for (int i = 0; i < 16; ++i) host[i] = c.w2c[i];
    double r[3][3], t[3];
    for (int i = 0; i < 3; ++i) {
      for (int j = 0; j < 3; ++j) r[i][j] = c.w2c[4 * i + j];
      t[i] = c.w2c[4 * i + 3];
    }
    // camera centre = -R^-1 t, with R^-1 from the adjugate
    double adj[3][3];
    adj[0][0] = r[1][1] * r[2][2] - r[1][2] * r[2][1];
    adj[0][1] = r[0][2] * r[2][1] - r[0][1] * r[2][2];
    adj[0][2] = r[0][1] * r[1][2] - r[0][2] * r[1][1];
    adj[1][0] = r[1][2] * r[2][0] - r[1][0] * r[2][2];
    adj[1][1] = r[0][0] * r[2][2] - r[0][2] * r[2][0];
    adj[1][2] = r[0][2] * r[1][0] - r[0][0] * r[1][2];
    adj[2][0] = r[1][0] * r[2][1] - r[1][1] * r[2][0];
    adj[2][1] = r[0][1] * r[2][0] - r[0][0] * r[2][1];
    adj[2][2] = r[0][0] * r[1][1] - r[0][1] * r[1][0];
    const double det = r[0][0] * adj[0][0] + r[0][1] * adj[1][0] + r[0][2] * adj[2][0];
    for (int i = 0; i < 3; ++i)
      host[16 + i] = static_cast<float>(-(adj[i][0] * t[0] + adj[i][1] * t[1] + adj[i][2] * t[2]) / det);
    host[19] = 0.0f;
    check(cudaMemcpyAsync(pose, host, sizeof(host), cudaMemcpyHostToDevice, s), "pose upload");
    check(cudaStreamSynchronize(s), "pose upload sync");
  }
};

// Per-precision entry points (ref_raster_f32.cu, ref_raster_f16.cu).
void forward_f32(RefHandle*, const TgsRefGaussians*, const TgsRefCamera*, void*, void*, cudaStream_t);
void forward_f16(RefHandle*, const TgsRefGaussians*, const TgsRefCamera*, void*, void*, cudaStream_t);
void backward_f32(RefHandle*, const TgsRefGaussians*, const TgsRefCamera*, const void*, const void*,
                  const TgsRefGaussians*, void*, cudaStream_t);
void backward_f16(RefHandle*, const TgsRefGaussians*, const TgsRefCamera*, const void*, const void*,
                  const TgsRefGaussians*, void*, cudaStream_t);
bool locate_f32(RefHandle*, int, const void**, size_t*);
bool locate_f16(RefHandle*, int, const void**, size_t*);

}  // namespace tgsref
