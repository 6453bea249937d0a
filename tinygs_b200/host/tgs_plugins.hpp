// tgs_plugins.hpp -- C++20 implementations of tinygs's plugin interfaces on
// top of the C ABI (include/tgs_abi.h).
//
// The classes mirror the reference's interfaces so that the B200 kernels
// drop in behind its training loop:
//   RasterizerBase / FastGSB200Rasterizer   tinygs/include/tinygs/rasterizer/rasterizer.hpp:9-63
//   LossBase / L1Loss / FusedSSIMLoss        tinygs/include/tinygs/loss/loss.hpp:6-28
//   OptimizerBase / SimpleAdam               tinygs/include/tinygs/optim/optim.hpp:8-92,
//                                            tinygs/include/tinygs/optim/simple_adam.hpp:8-89
//   GPUGaussian3d                            tinygs/include/tinygs/core/gpu_gaussian.hpp:9-73
//   StrategyBase / DefaultStrategy           tinygs/include/tinygs/strategy/strategy.hpp:9-70,
//                                            tinygs/src/strategy/default.cu:17-69
//   train_step(), reorder_gaussians()        tinygs/src/orchestrator.cu:335-439, 1038-1060
// Camera matrices are taken in the reference's glm convention (column-major
// K and w2c, fx = K[0][0], fy = K[1][1], cx = K[2][0], cy = K[2][1]).
// Errors are reported as std::runtime_error, as the reference does; the C
// ABI underneath returns status codes.  Everything runs on the caller's
// stream; the only host synchronisation is the optional capacity check of
// the rasterizer (one per forward, cheaper than the reference's four).
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "../../include/tgs_abi.h"

namespace tgs_b200 {

inline void check(int status, const char* where) {
  if (status != TGS_OK) throw std::runtime_error(std::string(where) + ": " + tgs_status_string(status));
}

inline void check_cuda(cudaError_t e, const char* where) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(where) + ": " + cudaGetErrorString(e));
}

enum class DataType { Float32 = TGS_FLOAT32, Float16 = TGS_FLOAT16 };

// tinygs::ImageShape / tinygs::Image (tinygs/include/tinygs/core/image.hpp:35-85)
struct ImageShape {
  uint32_t width = 0, height = 0, channel = 3;
  uint32_t size() const { return width * height * channel; }
  uint32_t padded_width() const { return (width + 7u) / 8u * 8u; }
  uint32_t padded_height() const { return (height + 7u) / 8u * 8u; }
  uint32_t padded_size() const { return padded_width() * padded_height() * channel; }
};

struct Image {
  ImageShape shape;
  DataType data_type = DataType::Float32;
  void* data = nullptr;
  size_t bytes() const { return size_t(shape.padded_size()) * (data_type == DataType::Float16 ? 2u : 4u); }
};

// SoA parameter arrays in one device allocation: 59 floats per Gaussian,
// every segment padded to a multiple of four Gaussians (16-byte aligned).
// The allocation holds `capacity` Gaussians; size() of them are live, so
// densification and row operations change the count without reallocating.
class GPUGaussian3d {
 public:
  static constexpr int kWidths[6] = {3, 1, 4, 3, 3, 45};

  GPUGaussian3d(int64_t n, int sh_degree, int64_t capacity = 0) : m_n(n), m_sh_degree(sh_degree) {
    m_cap = std::max<int64_t>(capacity, n);
    m_npad = (m_cap + 3) / 4 * 4;
    m_arena = alloc_arena(m_npad);
  }
  ~GPUGaussian3d() { cudaFree(m_arena); }
  GPUGaussian3d(const GPUGaussian3d&) = delete;
  GPUGaussian3d& operator=(const GPUGaussian3d&) = delete;

  int64_t size() const { return m_n; }
  int64_t capacity() const { return m_cap; }
  int get_sh_degree() const { return m_sh_degree; }
  void set_sh_degree(int d) { m_sh_degree = d; }
  // live count within the capacity (densification moves it)
  void resize(int64_t n) {
    if (n < 0 || n > m_cap) throw std::runtime_error("GPUGaussian3d::resize: beyond the capacity");
    m_n = n;
  }
  float* segment(int k) const { return segment_of(m_arena, m_npad, k); }
  float* means() const { return segment(0); }
  float* opacities() const { return segment(1); }
  float* rotations() const { return segment(2); }
  float* scales() const { return segment(3); }
  float* sh_coefficient_0() const { return segment(4); }
  float* sh_coefficients_rest() const { return segment(5); }
  float* arena() const { return m_arena; }
  size_t arena_floats() const { return 59 * static_cast<size_t>(m_npad); }

  TgsGaussians abi() const { return abi_of(m_arena, m_npad); }

  // host data per segment in the reference layout (means [n][3], ...)
  void copy_from_host(int k, const float* src, cudaStream_t s = nullptr) {
    check_cuda(cudaMemcpyAsync(segment(k), src, sizeof(float) * kWidths[k] * static_cast<size_t>(m_n),
                               cudaMemcpyHostToDevice, s),
               "GPUGaussian3d::copy_from_host");
  }
  void copy_to_host(int k, float* dst, cudaStream_t s = nullptr) const {
    check_cuda(cudaMemcpyAsync(dst, segment(k), sizeof(float) * kWidths[k] * static_cast<size_t>(m_n),
                               cudaMemcpyDeviceToHost, s),
               "GPUGaussian3d::copy_to_host");
  }
  void memset(int value, cudaStream_t s = nullptr) {
    check_cuda(cudaMemsetAsync(m_arena, value, sizeof(float) * arena_floats(), s), "GPUGaussian3d::memset");
  }

  // GPUGaussian3d::reorder (gpu_gaussian.cu:273-311): row i <- row
  // indices[i] (device indices), through a second arena that then becomes
  // this one's.
  void reorder(const uint32_t* indices, cudaStream_t s = nullptr) {
    float* other = alloc_arena(m_npad);
    TgsGaussians src = abi(), dst = abi_of(other, m_npad);
    const int st = tgs_arena_gather(&src, &dst, indices, m_n, s);
    swap_in(other, s);
    check(st, "GPUGaussian3d::reorder");
  }

  // GPUGaussian3d::remove (gpu_gaussian.cu:117-160): keeps the rows whose
  // kept_flag (device, one byte per live row) is non-zero, in order;
  // num_kept is their number.
  void remove(const char* kept_flag, int64_t num_kept, cudaStream_t s = nullptr) {
    size_t ws_bytes = 0;
    check(tgs_arena_compact_workspace_bytes(m_n, &ws_bytes), "GPUGaussian3d::remove");
    void* ws = nullptr;
    check_cuda(cudaMalloc(&ws, ws_bytes + 256), "GPUGaussian3d::remove: workspace");
    float* other = alloc_arena(m_npad);
    TgsGaussians src = abi(), dst = abi_of(other, m_npad);
    uint32_t* count = reinterpret_cast<uint32_t*>(static_cast<char*>(ws) + ws_bytes);
    const int st = tgs_arena_compact(&src, &dst, reinterpret_cast<const uint8_t*>(kept_flag), m_n, ws, ws_bytes,
                                     count, s);
    swap_in(other, s);
    cudaFree(ws);
    check(st, "GPUGaussian3d::remove");
    m_n = num_kept;
  }

  // GPUGaussian3d::append (gpu_gaussian.cu:162-171): num_dup zero rows at the
  // end, growing the allocation if the capacity is too small.
  void append(int64_t num_dup, cudaStream_t s = nullptr) {
    if (m_n + num_dup > m_cap) {
      const int64_t cap = std::max<int64_t>(m_n + num_dup, m_cap * 3 / 2);
      const int64_t npad = (cap + 3) / 4 * 4;
      float* other = alloc_arena(npad);
      for (int k = 0; k < 6; ++k)
        check_cuda(cudaMemcpyAsync(segment_of(other, npad, k), segment(k),
                                   sizeof(float) * kWidths[k] * static_cast<size_t>(m_n), cudaMemcpyDeviceToDevice, s),
                   "GPUGaussian3d::append");
      check_cuda(cudaStreamSynchronize(s), "GPUGaussian3d::append");
      cudaFree(m_arena);
      m_arena = other;
      m_cap = cap;
      m_npad = npad;
    }
    for (int k = 0; k < 6; ++k)
      check_cuda(cudaMemsetAsync(segment(k) + kWidths[k] * m_n, 0, sizeof(float) * kWidths[k] * size_t(num_dup), s),
                 "GPUGaussian3d::append");
    m_n += num_dup;
  }

 private:
  static float* alloc_arena(int64_t npad) {
    float* a = nullptr;
    const size_t bytes = sizeof(float) * 59 * static_cast<size_t>(npad > 0 ? npad : 1);
    check_cuda(cudaMalloc(&a, bytes), "GPUGaussian3d: cudaMalloc");
    check_cuda(cudaMemset(a, 0, bytes), "GPUGaussian3d: cudaMemset");
    return a;
  }
  static float* segment_of(float* arena, int64_t npad, int k) {
    size_t off = 0;
    for (int i = 0; i < k; ++i) off += size_t(kWidths[i]) * static_cast<size_t>(npad);
    return arena + off;
  }
  TgsGaussians abi_of(float* arena, int64_t npad) const {
    TgsGaussians g{};
    g.means = segment_of(arena, npad, 0);
    g.opacities = segment_of(arena, npad, 1);
    g.rotations = segment_of(arena, npad, 2);
    g.scales = segment_of(arena, npad, 3);
    g.sh0 = segment_of(arena, npad, 4);
    g.sh_rest = segment_of(arena, npad, 5);
    g.n = m_n;
    g.sh_degree = m_sh_degree;
    return g;
  }
  void swap_in(float* other, cudaStream_t s) {
    check_cuda(cudaStreamSynchronize(s), "GPUGaussian3d: sync");
    cudaFree(m_arena);
    m_arena = other;
  }

  int64_t m_n = 0, m_cap = 0, m_npad = 0;
  int m_sh_degree = 0;
  float* m_arena = nullptr;
};

// tinygs::GPUBatchInput (tinygs/include/tinygs/dataloader/dataloader.hpp:8-14)
struct GPUBatchInput {
  uint32_t width = 0, height = 0;
  float near_plane = 0.01f, far_plane = 100.0f;
  float K[9] = {};    // glm::mat3, column-major
  float w2c[16] = {}; // glm::mat4, column-major
};

inline TgsCamera to_camera(const GPUBatchInput& in) {
  TgsCamera c{};
  c.width = static_cast<int32_t>(in.width);
  c.height = static_cast<int32_t>(in.height);
  c.fx = in.K[0];
  c.fy = in.K[4];
  c.cx = in.K[6];
  c.cy = in.K[7];
  c.near_plane = in.near_plane;
  c.far_plane = in.far_plane;
  for (int r = 0; r < 4; ++r)
    for (int col = 0; col < 4; ++col) c.w2c[4 * r + col] = in.w2c[4 * col + r];
  return c;
}

// tinygs::RasterizeContext (rasterizer.hpp:9-29)
struct RasterizeContext {
  cudaStream_t stream = nullptr;
  float grad_scaler = 1.0f;
  GPUBatchInput fwd_input;
  Image fwd_output_image;
  Image grad_output_image;
  std::shared_ptr<GPUGaussian3d> gaussians_grad;
  TgsDensificationInfo* densification_info = nullptr;  // [n], optional
};

class RasterizerBase {
 public:
  virtual ~RasterizerBase() = default;
  virtual void forward(const RasterizeContext& ctx) = 0;
  virtual void backward(RasterizeContext& ctx) = 0;
  virtual void set_gaussians(std::shared_ptr<GPUGaussian3d> g) { m_gaussians = std::move(g); }

 protected:
  std::shared_ptr<GPUGaussian3d> m_gaussians;
};

// Rasterizer backed by the sm_100a kernels.  The handle and its scratch are
// created on the first forward from the model size and image size and
// re-created (larger) only when a capacity bound is hit.
class FastGSB200Rasterizer final : public RasterizerBase {
 public:
  // check_capacity: read the device counts after each forward (one host
  // sync) and re-render with larger scratch on overflow.
  explicit FastGSB200Rasterizer(bool check_capacity = true) : m_check(check_capacity) {}
  ~FastGSB200Rasterizer() override {
    if (m_handle) tgs_raster_destroy(m_handle);
  }

  // `accumulate`: 1 = grads += (reference semantics), 0 = grads overwritten
  void set_accumulate(bool a) { m_accumulate = a; }

  void forward(const RasterizeContext& ctx) override {
    if (!m_gaussians) throw std::runtime_error("Gaussians not set");
    const TgsCamera cam = to_camera(ctx.fwd_input);
    ensure(m_gaussians->size(), cam.width, cam.height, m_inst_cap);
    for (int attempt = 0; attempt < 4; ++attempt) {
      const TgsGaussians g = m_gaussians->abi();
      check(tgs_raster_forward(m_handle, &g, &cam, static_cast<int32_t>(ctx.fwd_output_image.data_type),
                               ctx.fwd_output_image.data, nullptr, ctx.densification_info, ctx.stream),
            "FastGSB200Rasterizer::forward");
      if (!m_check) return;
      TgsRasterCounts c{};
      check(tgs_raster_counts(m_handle, &c, ctx.stream), "FastGSB200Rasterizer::forward (counts)");
      m_counts = c;
      if (c.overflow == 0) return;
      ensure(m_gaussians->size(), cam.width, cam.height, int64_t(c.n_instances) * 3 / 2 + 1024, true);
    }
    throw std::runtime_error("FastGSB200Rasterizer::forward: capacity could not be met");
  }

  void backward(RasterizeContext& ctx) override {
    if (!m_gaussians || !ctx.gaussians_grad) throw std::runtime_error("Gaussians or gradient gaussians not set");
    const TgsCamera cam = to_camera(ctx.fwd_input);
    const TgsGaussians g = m_gaussians->abi();
    TgsGaussians gg = ctx.gaussians_grad->abi();
    check(tgs_raster_backward(m_handle, &g, &cam, static_cast<int32_t>(ctx.fwd_output_image.data_type),
                              ctx.fwd_output_image.data, ctx.grad_output_image.data, &gg, m_accumulate ? 1 : 0,
                              ctx.densification_info, ctx.stream),
          "FastGSB200Rasterizer::backward");
  }

  TgsRasterCounts last_counts() const { return m_counts; }

 private:
  void ensure(int64_t n, int w, int h, int64_t inst, bool force = false) {
    if (!force && m_handle && n <= m_caps.max_gaussians && w <= m_caps.max_width && h <= m_caps.max_height) return;
    if (m_handle) tgs_raster_destroy(m_handle);
    m_handle = nullptr;
    m_caps.max_gaussians = std::max<int64_t>(n, 1);
    m_caps.max_width = w;
    m_caps.max_height = h;
    m_caps.max_instances = inst;
    m_inst_cap = inst;
    check(tgs_raster_create(&m_caps, &m_handle), "FastGSB200Rasterizer: tgs_raster_create");
  }

  TgsRaster* m_handle = nullptr;
  TgsRasterCaps m_caps{};
  TgsRasterCounts m_counts{};
  int64_t m_inst_cap = 0;
  bool m_check = true;
  bool m_accumulate = true;
};

// tinygs::LossContext / LossBase (loss.hpp:6-28)
struct LossContext {
  Image pred, target, loss, grad;
  cudaStream_t stream = nullptr;
};

class LossBase {
 public:
  virtual ~LossBase() = default;
  virtual void evaluate(LossContext ctx, float scale) = 0;
  virtual std::string name() const = 0;
};

class L1Loss final : public LossBase {
 public:
  void evaluate(LossContext ctx, float scale) override {
    check(tgs_loss_l1(static_cast<int32_t>(ctx.pred.data_type), int32_t(ctx.pred.shape.width),
                      int32_t(ctx.pred.shape.height), ctx.pred.data, ctx.target.data, ctx.loss.data, ctx.grad.data,
                      scale, ctx.stream),
          "L1Loss::evaluate");
  }
  std::string name() const override { return "l1"; }
};

class FusedSSIMLoss final : public LossBase {
 public:
  ~FusedSSIMLoss() override {
    if (m_handle) tgs_loss_destroy(m_handle);
  }
  void evaluate(LossContext ctx, float scale) override {
    ensure(int32_t(ctx.pred.shape.width), int32_t(ctx.pred.shape.height));
    check(tgs_loss_fused_ssim(m_handle, static_cast<int32_t>(ctx.pred.data_type), int32_t(ctx.pred.shape.width),
                              int32_t(ctx.pred.shape.height), ctx.pred.data, ctx.target.data, ctx.loss.data,
                              ctx.grad.data, scale, ctx.stream),
          "FusedSSIMLoss::evaluate");
  }
  std::string name() const override { return "fused_ssim"; }

 protected:
  void ensure(int32_t w, int32_t h) {
    if (m_handle && w <= m_w && h <= m_h) return;
    if (m_handle) tgs_loss_destroy(m_handle);
    m_handle = nullptr;
    check(tgs_loss_create(w, h, &m_handle), "FusedSSIMLoss: tgs_loss_create");
    m_w = w;
    m_h = h;
  }
  TgsLoss* m_handle = nullptr;
  int32_t m_w = 0, m_h = 0;
};

// GaussianOptimizationParams + SimpleAdamParameters (optim.hpp:8-37,
// simple_adam.hpp:8-27) with the reference defaults.
struct SimpleAdamParameters {
  float beta1 = 0.9f, beta2 = 0.999f, epsilon = 1e-8f;
  bool decay_reduction_mean = true;
};
struct GaussianOptimizationParams {
  float max_grad_1 = 1.0f;
  float means_lr = 1.6e-4f, shs_lr = 2.5e-3f, opacities_lr = 5.0e-2f, scales_lr = 5.0e-3f, rotations_lr = 1.0e-3f;
  float opacities_l1 = 0.0f, scales_l1 = 0.0f;
};

class OptimizerBase {
 public:
  OptimizerBase(std::shared_ptr<GPUGaussian3d> g, std::shared_ptr<GPUGaussian3d> grad)
      : m_gaussians(std::move(g)), m_gaussians_grad(std::move(grad)) {}
  virtual ~OptimizerBase() = default;
  virtual void step(float scale, cudaStream_t stream) = 0;
  // optim.hpp:61-76: row hooks the strategy and the reorder call
  virtual void remove(char* /*kept_flag*/, int /*num_kept*/) {}
  virtual void duplicate(int* /*indices*/, int* /*new_indices*/, int /*num_duplicate*/) {}
  virtual void reset(int* indices, int num_reset) = 0;
  virtual void reset_opacity() = 0;
  virtual void reorder(uint32_t* indices) = 0;
  void set_lr(float lr) { m_global_lr = lr; }
  float get_lr() const { return m_global_lr; }
  GaussianOptimizationParams& params() { return m_params; }
  std::shared_ptr<GPUGaussian3d> get_gaussians() const { return m_gaussians; }
  std::shared_ptr<GPUGaussian3d> get_gaussians_grad() const { return m_gaussians_grad; }

 protected:
  std::shared_ptr<GPUGaussian3d> m_gaussians, m_gaussians_grad;
  float m_global_lr = 1.0f;
  GaussianOptimizationParams m_params;
};

class SimpleAdam final : public OptimizerBase {
 public:
  SimpleAdam(std::shared_ptr<GPUGaussian3d> g, std::shared_ptr<GPUGaussian3d> grad)
      : OptimizerBase(g, grad),
        m_first(std::make_shared<GPUGaussian3d>(g->size(), g->get_sh_degree(), g->capacity())),
        m_second(std::make_shared<GPUGaussian3d>(g->size(), g->get_sh_degree(), g->capacity())) {}

  SimpleAdamParameters& adam_params() { return m_adam; }
  void set_scene_scale(float s) { m_scene_scale = s; }
  void set_zero_grads_after_step(bool z) { m_zero_grads = z; }
  void set_stream(cudaStream_t s) { m_stream = s; }
  GPUGaussian3d& first() { return *m_first; }
  GPUGaussian3d& second() { return *m_second; }

  void step(float scale, cudaStream_t stream) override {
    ++m_global_steps;
    const TgsAdamConfig cfg{m_adam.beta1,          m_adam.beta2,         m_adam.epsilon,   m_params.max_grad_1,
                            m_params.means_lr,     m_params.shs_lr,      m_params.opacities_lr,
                            m_params.scales_lr,    m_params.rotations_lr, m_params.opacities_l1,
                            m_params.scales_l1,    m_scene_scale,        m_global_lr,
                            m_adam.decay_reduction_mean ? 1 : 0};
    const TgsGaussians p = m_gaussians->abi(), g = m_gaussians_grad->abi(), m = m_first->abi(),
                       v = m_second->abi();
    check(tgs_adam_step(&p, &g, &m, &v, &cfg, m_global_steps, scale, m_zero_grads ? 1 : 0, stream),
          "SimpleAdam::step");
  }

  // SimpleAdam::remove (simple_adam.cu:841-903): both moments compacted to
  // the kept rows.
  void remove(char* kept_flag, int num_kept) override {
    m_first->remove(kept_flag, num_kept, m_stream);
    m_second->remove(kept_flag, num_kept, m_stream);
  }
  // SimpleAdam::duplicate (simple_adam.cu:905-924): the moments grow to the
  // new size with zero rows (the indices are not used).
  void duplicate(int*, int*, int num_duplicate) override {
    if (num_duplicate <= 0) return;
    m_first->append(num_duplicate, m_stream);
    m_second->append(num_duplicate, m_stream);
  }
  // SimpleAdam::reset (simple_adam.cu:944-982): both moments of the rows
  // zeroed (indices on the device).
  void reset(int* indices, int num_reset) override {
    if (num_reset <= 0) return;
    for (auto* m : {m_first.get(), m_second.get()}) {
      TgsGaussians a = m->abi();
      check(tgs_arena_fill_rows(&a, indices, num_reset, 0.0f, -1, m_stream), "SimpleAdam::reset");
    }
  }
  // SimpleAdam::reset_opacity (simple_adam.cu:984-987): every opacity moment
  // zeroed.
  void reset_opacity() override {
    for (auto* m : {m_first.get(), m_second.get()})
      check_cuda(cudaMemsetAsync(m->opacities(), 0, sizeof(float) * static_cast<size_t>(m->size()), m_stream),
                 "SimpleAdam::reset_opacity");
  }
  // SimpleAdam::reorder (simple_adam.cu:1036-1099): both moments gathered.
  void reorder(uint32_t* indices) override {
    m_first->reorder(indices, m_stream);
    m_second->reorder(indices, m_stream);
  }
  // live count of both moments (after an in-place densification)
  void resize(int64_t n) {
    m_first->resize(n);
    m_second->resize(n);
  }
  // Adam's step count (bias correction); restored by a resume
  uint32_t global_steps() const { return m_global_steps; }
  void set_global_steps(uint32_t s) { m_global_steps = s; }

 private:
  SimpleAdamParameters m_adam;
  std::shared_ptr<GPUGaussian3d> m_first, m_second;
  uint32_t m_global_steps = 0;
  float m_scene_scale = 1.0f;
  bool m_zero_grads = false;
  cudaStream_t m_stream = nullptr;
};

// tinygs::StrategyParams (tinygs/include/tinygs/strategy/strategy.hpp:9-29)
// with the reference defaults.
struct StrategyParams {
  float pruning_opacity_threshold = 0.005f;
  float pruning_scale_threshold = 0.1f;
  float max_screen_size = 10.0f;
  float duplicate_grad_threshold = 0.0002f;
  float duplicate_scale_threshold = 0.01f;
  bool absgrad = false;
  int refine_every = 100;
  int start_refine = 500;
  int end_refine = 15000;
  int64_t max_num_gaussians = 10000000;
  int reset_every = 3000;
  uint64_t seed = 42;
};

// tinygs::StrategyBase / DefaultStrategy (strategy.hpp:31-70,
// tinygs/src/strategy/default.cu:17-69, strategy.cpp:20-46).  The reference
// reallocates every array through on_remove / on_duplicate; here the whole
// refine (clone, split, prune, opacity reset) runs in place through
// tgs_densify_step over the parameters, gradients and both Adam moments,
// which therefore need spare capacity (GPUGaussian3d's capacity argument).
class StrategyBase {
 public:
  StrategyBase(std::shared_ptr<GPUGaussian3d> g, std::shared_ptr<GPUGaussian3d> grad, std::shared_ptr<SimpleAdam> opt)
      : m_gaussians(std::move(g)), m_gaussians_grad(std::move(grad)), m_optimizer(std::move(opt)) {}
  virtual ~StrategyBase() = default;
  // strategy.cpp:9-12: one step of the strategy after the optimizer step
  void step(RasterizeContext& ctx) {
    step_impl(ctx);
    ++m_step_count;
  }
  int64_t this_step() const { return m_step_count; }
  void set_this_step(int64_t s) { m_step_count = s; }

 protected:
  virtual void step_impl(RasterizeContext& ctx) = 0;
  std::shared_ptr<GPUGaussian3d> m_gaussians, m_gaussians_grad;
  std::shared_ptr<SimpleAdam> m_optimizer;
  int64_t m_step_count = 0;
};

class DefaultStrategyB200 final : public StrategyBase {
 public:
  DefaultStrategyB200(std::shared_ptr<GPUGaussian3d> g, std::shared_ptr<GPUGaussian3d> grad,
                      std::shared_ptr<SimpleAdam> opt, StrategyParams p = {}, float scene_scale = 1.0f)
      : StrategyBase(std::move(g), std::move(grad), std::move(opt)), m_params(p), m_scene_scale(scene_scale) {
    check(tgs_densify_create(m_gaussians->capacity(), &m_handle), "DefaultStrategyB200: tgs_densify_create");
    tgs_pcg32_seed(&m_rng, m_params.seed, 1);
    check_cuda(cudaMalloc(&m_dens, sizeof(TgsDensificationInfo) * static_cast<size_t>(m_gaussians->capacity())),
               "DefaultStrategyB200: densification records");
    check_cuda(cudaMemset(m_dens, 0, sizeof(TgsDensificationInfo) * static_cast<size_t>(m_gaussians->capacity())),
               "DefaultStrategyB200: densification records");
  }
  ~DefaultStrategyB200() override {
    if (m_handle) tgs_densify_destroy(m_handle);
    cudaFree(m_dens);
  }
  // the records the rasterizer accumulates into (RasterizeContext::densification_info)
  TgsDensificationInfo* densification_info() const { return m_dens; }
  // the random stream of the splits; saved and restored with a checkpoint
  TgsPcg32 rng() const { return m_rng; }
  void set_rng(TgsPcg32 r) { m_rng = r; }

 protected:
  void step_impl(RasterizeContext& ctx) override {
    TgsDensifyConfig c{};
    c.duplicate_grad_threshold = m_params.duplicate_grad_threshold;
    c.duplicate_scale_threshold = m_params.duplicate_scale_threshold;
    c.pruning_opacity_threshold = m_params.pruning_opacity_threshold;
    c.pruning_scale_threshold = m_params.pruning_scale_threshold;
    c.max_screen_size = m_params.max_screen_size;
    c.scene_scale = m_scene_scale;
    c.grad_scaler = ctx.grad_scaler;
    c.absgrad = m_params.absgrad ? 1 : 0;
    c.refine_every = m_params.refine_every;
    c.start_refine = m_params.start_refine;
    c.end_refine = m_params.end_refine;
    c.reset_every = m_params.reset_every;
    c.image_width = static_cast<int32_t>(ctx.fwd_input.width);
    c.image_height = static_cast<int32_t>(ctx.fwd_input.height);
    c.max_num_gaussians = m_params.max_num_gaussians;
    TgsGaussians p = m_gaussians->abi(), m = m_optimizer->first().abi(), v = m_optimizer->second().abi();
    TgsGaussians g{};
    if (m_gaussians_grad) g = m_gaussians_grad->abi();
    int64_t n = m_gaussians->size();
    check(tgs_densify_step(m_handle, &p, m_gaussians_grad ? &g : nullptr, &m, &v, m_dens, &c,
                           static_cast<int32_t>(m_step_count), &m_rng, &n, ctx.stream),
          "DefaultStrategyB200::step");
    m_gaussians->resize(n);
    if (m_gaussians_grad) m_gaussians_grad->resize(n);
    m_optimizer->resize(n);
    ctx.densification_info = m_dens;
  }

 private:
  StrategyParams m_params;
  float m_scene_scale;
  TgsDensifier* m_handle = nullptr;
  TgsPcg32 m_rng{};
  TgsDensificationInfo* m_dens = nullptr;
};

// Orchestrator::reorder_gaussians (tinygs/src/orchestrator.cu:1038-1060):
// Morton order of the means, applied to the parameters, the gradients, the
// optimizer's moments and the densification records.
inline void reorder_gaussians(GPUGaussian3d& g, GPUGaussian3d* grad, OptimizerBase* opt,
                              TgsDensificationInfo* dens, cudaStream_t s) {
  const int64_t n = g.size();
  if (n == 0) return;
  size_t ws_bytes = 0;
  check(tgs_morton_workspace_bytes(n, &ws_bytes), "reorder_gaussians");
  void* ws = nullptr;
  uint32_t* perm = nullptr;
  check_cuda(cudaMalloc(&ws, ws_bytes), "reorder_gaussians: workspace");
  check_cuda(cudaMalloc(&perm, sizeof(uint32_t) * static_cast<size_t>(n)), "reorder_gaussians: permutation");
  int st = tgs_morton_order(g.means(), n, ws, ws_bytes, perm, s);
  if (st == TGS_OK) {
    g.reorder(perm, s);
    if (grad) grad->reorder(perm, s);
    if (opt) opt->reorder(perm);
    if (dens) {
      TgsDensificationInfo* tmp = nullptr;
      check_cuda(cudaMalloc(&tmp, sizeof(TgsDensificationInfo) * static_cast<size_t>(n)), "reorder_gaussians");
      st = tgs_dens_gather(dens, tmp, perm, n, s);
      cudaMemcpyAsync(dens, tmp, sizeof(TgsDensificationInfo) * static_cast<size_t>(n), cudaMemcpyDeviceToDevice, s);
      cudaStreamSynchronize(s);
      cudaFree(tmp);
    }
  }
  cudaStreamSynchronize(s);
  cudaFree(ws);
  cudaFree(perm);
  check(st, "reorder_gaussians");
}

// One Orchestrator::train_step (orchestrator.cu:335-439) without the data
// loader, pose optimisation and strategy: zero the gradient and image
// buffers, forward, each loss with weight * grad_scaler, backward, and the
// optimizer step with gradient scale 1 / (grad_scaler * accumulate_steps).
struct WeightedLoss {
  std::unique_ptr<LossBase> loss;
  float weight;
};

class TrainStep {
 public:
  TrainStep(std::shared_ptr<GPUGaussian3d> g, std::shared_ptr<GPUGaussian3d> grad, RasterizerBase& rast,
            OptimizerBase& opt, float grad_scaler = 10.0f)
      : m_g(std::move(g)), m_grad(std::move(grad)), m_rast(rast), m_opt(opt), m_grad_scaler(grad_scaler) {}

  void add_loss(std::unique_ptr<LossBase> l, float w) { m_losses.push_back({std::move(l), w}); }
  // the densification strategy stepped after the optimizer
  void set_strategy(StrategyBase* s) { m_strategy = s; }
  // OrchestratorConfig::reorder_gaussians_interval (0: never)
  void set_reorder_interval(int k) { m_reorder_every = k; }
  int64_t current_step() const { return m_step; }
  void set_current_step(int64_t s) { m_step = s; }

  void run(RasterizeContext& ctx, const Image& target, const Image& loss_map) {
    m_grad->memset(0, ctx.stream);
    check_cuda(cudaMemsetAsync(loss_map.data, 0, loss_map.bytes(), ctx.stream), "TrainStep: loss memset");
    check_cuda(cudaMemsetAsync(ctx.grad_output_image.data, 0, ctx.grad_output_image.bytes(), ctx.stream),
               "TrainStep: grad memset");
    ctx.gaussians_grad = m_grad;
    m_rast.forward(ctx);
    LossContext lc{ctx.fwd_output_image, target, loss_map, ctx.grad_output_image, ctx.stream};
    for (auto& wl : m_losses) wl.loss->evaluate(lc, wl.weight * m_grad_scaler);
    m_rast.backward(ctx);
    m_opt.step(1.0f / m_grad_scaler, ctx.stream);
    if (m_strategy) m_strategy->step(ctx);
    if (m_step > 0 && m_reorder_every > 0 && m_step % m_reorder_every == 0)
      reorder_gaussians(*m_g, m_grad.get(), &m_opt, ctx.densification_info, ctx.stream);
    ++m_step;
  }

 private:
  std::shared_ptr<GPUGaussian3d> m_g, m_grad;
  RasterizerBase& m_rast;
  OptimizerBase& m_opt;
  float m_grad_scaler;
  std::vector<WeightedLoss> m_losses;
  StrategyBase* m_strategy = nullptr;
  int m_reorder_every = 0;
  int64_t m_step = 0;
};

// Checkpoint of a run (tgs_checkpoint_save): the parameters, the optimizer's
// moments and step count, the strategy's statistics, step count and random
// stream, and the training step.  The reference has only the callback hook
// (Orchestrator::set_checkpoint_callback, orchestrator.cu:291-293,433-435).
inline void save_checkpoint(const std::string& path, GPUGaussian3d& g, SimpleAdam* opt,
                            DefaultStrategyB200* strategy, int64_t step, cudaStream_t s) {
  TgsTrainState st{};
  st.step = static_cast<uint64_t>(step);
  const TgsGaussians p = g.abi();
  TgsGaussians m{}, v{};
  if (opt) {
    st.adam_step = opt->global_steps();
    m = opt->first().abi();
    v = opt->second().abi();
  }
  if (strategy) {
    st.strategy_step = static_cast<uint64_t>(strategy->this_step());
    st.rng = strategy->rng();
  }
  check(tgs_checkpoint_save(path.c_str(), &p, opt ? &m : nullptr, opt ? &v : nullptr,
                            strategy ? strategy->densification_info() : nullptr, &st, s),
        "save_checkpoint");
}

// Resume from a checkpoint written by save_checkpoint (or by the Python
// binding): every array moves to the saved count; returns the saved step.
inline int64_t load_checkpoint(const std::string& path, GPUGaussian3d& g, GPUGaussian3d* grad, SimpleAdam* opt,
                               DefaultStrategyB200* strategy, cudaStream_t s) {
  TgsTrainState st{};
  TgsGaussians p = g.abi(), m{}, v{};
  if (opt) {
    m = opt->first().abi();
    v = opt->second().abi();
  }
  check(tgs_checkpoint_load(path.c_str(), g.capacity(), &p, opt ? &m : nullptr, opt ? &v : nullptr,
                            strategy ? strategy->densification_info() : nullptr, &st, s),
        "load_checkpoint");
  g.resize(p.n);
  g.set_sh_degree(p.sh_degree);
  if (grad) grad->resize(p.n);
  if (opt) {
    opt->resize(p.n);
    opt->set_global_steps(static_cast<uint32_t>(st.adam_step));
  }
  if (strategy) {
    strategy->set_this_step(static_cast<int64_t>(st.strategy_step));
    strategy->set_rng(st.rng);
  }
  return static_cast<int64_t>(st.step);
}

// Factory in the shape of create_rasterizer (rasterizer.cpp:44-53).
inline std::unique_ptr<RasterizerBase> create_rasterizer(const std::string& type) {
  if (type == "fastgs_b200") return std::make_unique<FastGSB200Rasterizer>();
  throw std::runtime_error("unknown rasterizer type: " + type);
}

inline std::unique_ptr<LossBase> create_loss(const std::string& type) {
  if (type == "l1") return std::make_unique<L1Loss>();
  if (type == "fused_ssim") return std::make_unique<FusedSSIMLoss>();
  throw std::runtime_error("unknown loss type: " + type);
}

}  // namespace tgs_b200
