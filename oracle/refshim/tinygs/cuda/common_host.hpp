// Stand-in for tinygs/include/tinygs/cuda/common_host.hpp (the parts the
// hot-path kernels use).  Test infrastructure (oracle/_ref build).
#pragma once
#include <cuda_runtime.h>
#include <stdexcept>
#include <string>
#include "tinygs/common.hpp"

// common_host.hpp:104-110: throw on a failed runtime call.
#define CUDA_CHECK_THROW(x)                                                                       \
  do {                                                                                            \
    cudaError_t _tgs_ref_result = (x);                                                            \
    if (_tgs_ref_result != cudaSuccess)                                                           \
      throw std::runtime_error(std::string(FILE_LINE " " #x " failed: ") +                       \
                               cudaGetErrorString(_tgs_ref_result));                              \
  } while (0)

#define CUDA_CHECK_PRINT(x)                                                                       \
  do {                                                                                            \
    cudaError_t _tgs_ref_result = (x);                                                            \
    if (_tgs_ref_result != cudaSuccess) fprintf(stderr, "%s\n", cudaGetErrorString(_tgs_ref_result)); \
  } while (0)

namespace tinygs {
// common_host.hpp:449-453: a no-op unless the NVTX sync option is on (it is off).
inline void maybe_sync(cudaStream_t = 0) {}
}  // namespace tinygs

#include <cstdio>
#include <utility>

// A stand-in for the fmt::format calls in the reference's error messages:
// the message keeps its format string; the arguments are dropped.
namespace fmt {
template <typename... Args>
inline std::string format(const char* f, Args&&...) { return std::string(f); }
}  // namespace fmt

namespace tinygs {

// common_host.hpp:452-453: string -> value conversion, specialised per type.
template <typename T>
T from_string(const std::string& str);

// common.hpp (N_THREADS_LINEAR, n_blocks_linear): 1-D launches of 128 threads.
constexpr uint32_t N_THREADS_LINEAR = 128;
template <typename T>
constexpr TINYGS_HOST_DEVICE uint32_t n_blocks_linear(T n, uint32_t threads = N_THREADS_LINEAR) {
  return (uint32_t)((n + (T)threads - 1) / (T)threads);
}

#if defined(__CUDACC__)
// common_host.hpp:342-348: kernel(n, args...) over ceil(n / 128) blocks of 128.
template <typename K, typename T, typename... Types>
inline void linear_kernel(K kernel, uint32_t shmem, cudaStream_t stream, T n, Types... args) {
  if (n <= 0) return;
  kernel<<<n_blocks_linear(n), N_THREADS_LINEAR, shmem, stream>>>(n, args...);
}
#endif

}  // namespace tinygs
