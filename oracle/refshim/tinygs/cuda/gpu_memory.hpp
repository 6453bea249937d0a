// Stand-in for tinygs/include/tinygs/cuda/gpu_memory.hpp: a typed,
// owning, move-only device buffer (GPUBuffer) as the reference's loss and
// optimizer classes use it.  Test infrastructure (oracle/_ref build).
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <stdexcept>
#include "tinygs/cuda/common_host.hpp"

namespace tinygs {

template <typename T>
class GPUBuffer {
 public:
  GPUBuffer() = default;
  GPUBuffer(cudaStream_t, size_t n) : m_n(n) {
    if (n && cudaMalloc(reinterpret_cast<void**>(&m_data), n * sizeof(T)) != cudaSuccess)
      throw std::runtime_error("GPUBuffer: cudaMalloc failed");
  }
  explicit GPUBuffer(size_t n) : GPUBuffer(nullptr, n) {}
  GPUBuffer(const GPUBuffer&) = delete;
  GPUBuffer& operator=(const GPUBuffer&) = delete;
  GPUBuffer(GPUBuffer&& o) noexcept : m_data(o.m_data), m_n(o.m_n) { o.m_data = nullptr; o.m_n = 0; }
  GPUBuffer& operator=(GPUBuffer&& o) noexcept {
    if (this != &o) {
      release();
      m_data = o.m_data; m_n = o.m_n;
      o.m_data = nullptr; o.m_n = 0;
    }
    return *this;
  }
  ~GPUBuffer() { release(); }
  T* data() const { return m_data; }
  size_t size() const { return m_n; }
  size_t get_bytes() const { return m_n * sizeof(T); }
  explicit operator bool() const { return m_data != nullptr; }
  void memset_async(cudaStream_t s, int v) { if (m_data) cudaMemsetAsync(m_data, v, m_n * sizeof(T), s); }

 private:
  void release() { if (m_data) cudaFree(m_data); m_data = nullptr; }
  T* m_data = nullptr;
  size_t m_n = 0;
};

}  // namespace tinygs
