// ref_adam.cu -- the reference's SimpleAdam (tinygs/src/optim/simple_adam.cu,
// compiled unchanged) over a parameter and a gradient container, plus the
// OptimizerBase / GaussianOptimizationParams plumbing it links against,
// restated from tinygs/src/optim/optim.cu:9-80 (config fields only; the
// optimizer factory is left out).  Test infrastructure (oracle/_ref build).
#include <memory>
#include <string>

#include "ref_common.h"
#include "tinygs/optim/simple_adam.hpp"

namespace tinygs {

OptimizerBase::OptimizerBase(std::shared_ptr<GPUGaussian3d> gaussians, std::shared_ptr<GPUGaussian3d> gaussians_grad)
    : m_gaussians(gaussians), m_gaussians_grad(gaussians_grad) {}
void OptimizerBase::set_params(const json& config) { m_params.from_json(config); }
json OptimizerBase::get_params() const { return m_params.to_json(); }
void OptimizerBase::set_lr(float lr) { m_global_lr = lr; }
float OptimizerBase::get_lr() const { return m_global_lr; }
void OptimizerBase::reset() {}
void OptimizerBase::set_gaussians(std::shared_ptr<GPUGaussian3d> g, std::shared_ptr<GPUGaussian3d> gg) {
  m_gaussians = g;
  m_gaussians_grad = gg;
}

json GaussianOptimizationParams::to_json() const {
  json j;
  j["max_grad_1"] = max_grad_1;
  j["skip_zero_grad"] = skip_zero_grad;
  j["means_lr"] = means_lr;
  j["shs_lr"] = shs_lr;
  j["opacities_lr"] = opacities_lr;
  j["scales_lr"] = scales_lr;
  j["rotations_lr"] = rotations_lr;
  j["opacities_l1"] = opacities_l1;
  j["scales_l1"] = scales_l1;
  return j;
}

void GaussianOptimizationParams::from_json(const json& c) {
  auto get = [&](const char* k, auto& v) {
    if (c.contains(k)) v = c[k].get<std::remove_reference_t<decltype(v)>>();
  };
  get("max_grad_1", max_grad_1);
  get("skip_zero_grad", skip_zero_grad);
  get("means_lr", means_lr);
  get("shs_lr", shs_lr);
  get("opacities_lr", opacities_lr);
  get("scales_lr", scales_lr);
  get("rotations_lr", rotations_lr);
  get("opacities_l1", opacities_l1);
  get("scales_l1", scales_l1);
}

}  // namespace tinygs

namespace {

struct RefAdam {
  std::shared_ptr<tinygs::GPUGaussian3d> params, grads;
  std::unique_ptr<tinygs::SimpleAdam> adam;
};

void fill(tinygs::GPUGaussian3d& g, TgsRefGaussians* out) {
  out->means = reinterpret_cast<float*>(thrust::raw_pointer_cast(g.means().data()));
  out->opacities = thrust::raw_pointer_cast(g.opacities().data());
  out->rotations = reinterpret_cast<float*>(thrust::raw_pointer_cast(g.rotations().data()));
  out->scales = reinterpret_cast<float*>(thrust::raw_pointer_cast(g.scales().data()));
  out->sh0 = reinterpret_cast<float*>(thrust::raw_pointer_cast(g.sh_coefficient_0().data()));
  out->sh_rest = reinterpret_cast<float*>(thrust::raw_pointer_cast(g.sh_coefficients_rest().data()));
  out->n = static_cast<int64_t>(g.size());
  out->sh_degree = g.get_sh_degree();
}

}  // namespace

extern "C" {

int tgsref_adam_create(int64_t n, int32_t sh_degree, const char* config_json, void** handle) {
  try {
    auto* r = new RefAdam();
    r->params = std::make_shared<tinygs::GPUGaussian3d>(static_cast<size_t>(n));
    r->grads = std::make_shared<tinygs::GPUGaussian3d>(static_cast<size_t>(n));
    r->params->set_sh_degree(sh_degree);
    r->grads->set_sh_degree(sh_degree);
    r->adam = std::make_unique<tinygs::SimpleAdam>(r->params, r->grads);
    if (config_json != nullptr && config_json[0] != '\0') r->adam->set_params(tinygs::json::parse(config_json));
    *handle = r;
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : 1;
  } catch (const std::exception&) {
    cudaGetLastError();
    return -1;
  }
}

void tgsref_adam_destroy(void* handle) {
  cudaDeviceSynchronize();
  delete static_cast<RefAdam*>(handle);
}

int tgsref_adam_arrays(void* handle, TgsRefGaussians* params, TgsRefGaussians* grads) {
  auto* r = static_cast<RefAdam*>(handle);
  fill(*r->params, params);
  fill(*r->grads, grads);
  return 0;
}

int tgsref_adam_step(void* handle, float gradient_scale, void* stream) {
  try {
    static_cast<RefAdam*>(handle)->adam->step(gradient_scale, static_cast<cudaStream_t>(stream));
    return cudaGetLastError() == cudaSuccess ? 0 : 1;
  } catch (const std::exception&) {
    cudaGetLastError();
    return -1;
  }
}

}  // extern "C"
