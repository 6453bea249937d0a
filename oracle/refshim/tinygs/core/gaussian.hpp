// Stand-in for tinygs/include/tinygs/core/gaussian.hpp (the parts the
// hot-path kernels use).  Test infrastructure (oracle/_ref build).
#pragma once
#include "tinygs/common.hpp"

namespace tinygs {

// gaussian.hpp:18-23: per-Gaussian densification statistics, 16 bytes.
struct DensificationInfo {
  float accum_counter = 0;
  float accum_grad_mean2d = 0;
  float accum_absgrad_mean2d = 0;
  float max_radii_screen = 0;
};

// gaussian.hpp:30-68: scales are stored as logs, opacities as logits.
TINYGS_HOST_DEVICE inline float activate_scale(float x) { return ::expf(x); }
TINYGS_HOST_DEVICE inline float deactivate_scale(float x) { return ::logf(x); }
TINYGS_HOST_DEVICE inline float activate_scale_deriv(float x) { return ::expf(x); }
TINYGS_HOST_DEVICE inline float activate_opacity(float x) { return logistic(x); }
TINYGS_HOST_DEVICE inline float deactivate_opacity(float x) { return logit(x); }
TINYGS_HOST_DEVICE inline float activate_opacity_deriv(float x) {
  const float s = activate_opacity(x);
  return s * (1 - s);
}

}  // namespace tinygs
