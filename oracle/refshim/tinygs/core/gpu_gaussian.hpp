// Stand-in for tinygs/include/tinygs/core/gpu_gaussian.hpp: the SoA
// container of Gaussian parameters (or gradients) in thrust device vectors,
// with the accessors the reference's optimizer uses.  Test infrastructure
// (oracle/_ref build).
#pragma once
#include <thrust/device_vector.h>

#include "tinygs/core/gaussian.hpp"
#include "tinygs/cuda/vec.hpp"

namespace tinygs {

class GPUGaussian3d {
 public:
  // n Gaussians, every array zero-filled; sh_rest holds 15 coefficients
  // each.  Every array reserves 16 spare elements: the reference's float4
  // Adam kernel (simple_adam.cu:156-213) guards its tail per 4-float group
  // and touches up to 3 floats past the end.
  explicit GPUGaussian3d(size_t n = 0) {
    m_means.reserve(n + 16);
    m_opacities.reserve(n + 16);
    m_rotations.reserve(n + 16);
    m_scales.reserve(n + 16);
    m_sh_coefficient_0.reserve(n + 16);
    m_sh_coefficients_rest.reserve(n * (kMaxSphericalHarmonicsCoefficients - 1) + 16);
    m_means.resize(n);
    m_opacities.resize(n);
    m_rotations.resize(n);
    m_scales.resize(n);
    m_sh_coefficient_0.resize(n);
    m_sh_coefficients_rest.resize(n * (kMaxSphericalHarmonicsCoefficients - 1));
  }

  size_t size() const { return m_means.size(); }

  thrust::device_vector<vec3>& means() { return m_means; }
  thrust::device_vector<float>& opacities() { return m_opacities; }
  thrust::device_vector<vec4>& rotations() { return m_rotations; }
  thrust::device_vector<vec3>& scales() { return m_scales; }
  thrust::device_vector<vec3>& sh_coefficient_0() { return m_sh_coefficient_0; }
  thrust::device_vector<vec3>& sh_coefficients_rest() { return m_sh_coefficients_rest; }
  const thrust::device_vector<vec3>& means() const { return m_means; }
  const thrust::device_vector<float>& opacities() const { return m_opacities; }
  const thrust::device_vector<vec4>& rotations() const { return m_rotations; }
  const thrust::device_vector<vec3>& scales() const { return m_scales; }
  const thrust::device_vector<vec3>& sh_coefficient_0() const { return m_sh_coefficient_0; }
  const thrust::device_vector<vec3>& sh_coefficients_rest() const { return m_sh_coefficients_rest; }

  float scene_scale() const { return m_scene_scale; }
  void set_scene_scale(float s) { m_scene_scale = s; }
  void set_sh_degree(int d) { m_sh_degree = d < kMaxSphericalHarmonicsDegree ? d : kMaxSphericalHarmonicsDegree; }
  int get_sh_degree() const { return m_sh_degree; }

 private:
  int m_sh_degree = 0;
  float m_scene_scale = 1.0f;
  thrust::device_vector<vec3> m_means;
  thrust::device_vector<float> m_opacities;
  thrust::device_vector<vec4> m_rotations;
  thrust::device_vector<vec3> m_scales;
  thrust::device_vector<vec3> m_sh_coefficient_0;
  thrust::device_vector<vec3> m_sh_coefficients_rest;
};

}  // namespace tinygs
