// Stand-in for tinygs/include/tinygs/cuda/vec.hpp: the reference's loss
// kernels include it without using it; its optimizer stores parameters as
// glm vectors (2-4 floats, 4-byte aligned, broadcast and component
// constructors) and takes glm::length of them.  Only that subset is here.
// Test infrastructure (oracle/_ref build).
#pragma once
#include <cmath>
#include "tinygs/common.hpp"

namespace glm {
template <int N, typename T>
struct vec;
template <typename T>
struct vec<2, T> {
  T x, y;
  TINYGS_HOST_DEVICE vec() : x(0), y(0) {}
  TINYGS_HOST_DEVICE explicit vec(T s) : x(s), y(s) {}
  TINYGS_HOST_DEVICE vec(T a, T b) : x(a), y(b) {}
  TINYGS_HOST_DEVICE T& operator[](int i) { return (&x)[i]; }
  TINYGS_HOST_DEVICE const T& operator[](int i) const { return (&x)[i]; }
};
template <typename T>
struct vec<3, T> {
  T x, y, z;
  TINYGS_HOST_DEVICE vec() : x(0), y(0), z(0) {}
  TINYGS_HOST_DEVICE explicit vec(T s) : x(s), y(s), z(s) {}
  TINYGS_HOST_DEVICE vec(T a, T b, T c) : x(a), y(b), z(c) {}
  TINYGS_HOST_DEVICE T& operator[](int i) { return (&x)[i]; }
  TINYGS_HOST_DEVICE const T& operator[](int i) const { return (&x)[i]; }
};
template <typename T>
struct vec<4, T> {
  T x, y, z, w;
  TINYGS_HOST_DEVICE vec() : x(0), y(0), z(0), w(0) {}
  TINYGS_HOST_DEVICE explicit vec(T s) : x(s), y(s), z(s), w(s) {}
  TINYGS_HOST_DEVICE vec(T a, T b, T c, T d) : x(a), y(b), z(c), w(d) {}
  TINYGS_HOST_DEVICE T& operator[](int i) { return (&x)[i]; }
  TINYGS_HOST_DEVICE const T& operator[](int i) const { return (&x)[i]; }
};
using fvec2 = vec<2, float>;
using fvec3 = vec<3, float>;
using fvec4 = vec<4, float>;
using ivec3 = vec<3, int>;
using uvec3 = vec<3, unsigned int>;

// Euclidean norm of the components (of a scalar: its absolute value).
template <typename T>
TINYGS_HOST_DEVICE T length(T x) {
  return x < T(0) ? -x : x;
}
template <int N, typename T>
TINYGS_HOST_DEVICE T length(const vec<N, T>& v) {
  T s = 0;
  for (int i = 0; i < N; ++i) s += v[i] * v[i];
  return std::sqrt(s);
}
}  // namespace glm

namespace tinygs {
using vec2 = glm::fvec2;
using vec3 = glm::fvec3;
using vec4 = glm::fvec4;
using ivec3 = glm::ivec3;
using uvec3 = glm::uvec3;
}  // namespace tinygs
