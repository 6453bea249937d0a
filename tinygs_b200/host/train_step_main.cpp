// train_step_main.cpp -- C++ driver of the B200 training step through the
// plugin adapters of tgs_plugins.hpp, in the shape of the reference's
// config_train loop (examples/config_train.cpp:240-288 ->
// Orchestrator::train_step, orchestrator.cu:335-439) on one resident view.
//
// Usage: tgs_train_step <scene.bin> <out_params.bin> [--save-at K ckpt]
//                       [--resume ckpt]
//   --save-at K ckpt: write a checkpoint after K steps (and carry on);
//   --resume ckpt:    start from a checkpoint and run the steps left of the
//                     scene's step count.
// scene.bin (little endian):
//   char[4] "TGSB"; int32 version (1 or 2); int64 n; int32 sh_degree;
//   int32 width, height; int32 dtype (0 fp32, 1 fp16); int32 steps;
//   float grad_scaler; float max_grad_1;
//   version 2 only: int64 capacity; int32 densify (0/1); int32 refine_every,
//     start_refine, reset_every, reorder_every; float grad_threshold
//     (DefaultStrategy run after every optimizer step, Morton reorder every
//     reorder_every steps; 0 = never);
//   float params[59 * n]  segments means, opacities, rotations, scales,
//                         sh0, sh_rest in the reference layout;
//   float K[9], w2c[16]   glm column-major; float near, far;
//   target image          3 * Wp * Hp elements of dtype, 8x8-tiled CHW.
// out_params.bin: version 1: float params[59 * n]; version 2: int64 n_final
// then float params[59 * n_final], in the same segment layout.
// Prints one line per step: "step <k> loss <sum of the loss map> n <count>".
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iostream>
#include <string>
#include <vector>

#include "tgs_plugins.hpp"

using namespace tgs_b200;

namespace {

template <typename T>
void read_pod(std::ifstream& f, T& v) {
  f.read(reinterpret_cast<char*>(&v), sizeof(T));
  if (!f) throw std::runtime_error("truncated scene file");
}

float half_to_float(uint16_t h) {
  const uint32_t sign = (h & 0x8000u) << 16, exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
  float v;
  if (exp == 0) v = std::ldexp(static_cast<float>(man), -24);
  else if (exp == 31) v = man ? NAN : INFINITY;
  else v = std::ldexp(static_cast<float>(man | 0x400u), static_cast<int>(exp) - 25);
  uint32_t bits;
  std::memcpy(&bits, &v, 4);
  bits |= sign;
  std::memcpy(&v, &bits, 4);
  return v;
}

}  // namespace

int main(int argc, char** argv) {
  int save_at = -1;
  std::string save_path, resume_path;
  for (int a = 3; a < argc; ++a) {
    const std::string arg = argv[a];
    if (arg == "--save-at" && a + 2 < argc) {
      save_at = std::atoi(argv[a + 1]);
      save_path = argv[a + 2];
      a += 2;
    } else if (arg == "--resume" && a + 1 < argc) {
      resume_path = argv[++a];
    } else {
      argc = 0;
    }
  }
  if (argc < 3) {
    std::fprintf(stderr, "usage: %s scene.bin out_params.bin [--save-at K ckpt] [--resume ckpt]\n", argv[0]);
    return 2;
  }
  try {
    std::ifstream f(argv[1], std::ios::binary);
    char magic[4];
    f.read(magic, 4);
    if (!f || std::memcmp(magic, "TGSB", 4) != 0) throw std::runtime_error("not a TGSB scene file");
    int32_t version, sh, w, h, dtype, steps;
    int64_t n;
    float grad_scaler, max_grad_1;
    read_pod(f, version);
    read_pod(f, n);
    read_pod(f, sh);
    read_pod(f, w);
    read_pod(f, h);
    read_pod(f, dtype);
    read_pod(f, steps);
    read_pod(f, grad_scaler);
    read_pod(f, max_grad_1);
    int64_t capacity = 0;
    int32_t densify = 0, refine_every = 100, start_refine = 500, reset_every = 3000, reorder_every = 0;
    float grad_threshold = 0.0002f;
    if (version == 2) {
      read_pod(f, capacity);
      read_pod(f, densify);
      read_pod(f, refine_every);
      read_pod(f, start_refine);
      read_pod(f, reset_every);
      read_pod(f, reorder_every);
      read_pod(f, grad_threshold);
    }
    if ((version != 1 && version != 2) || n <= 0 || (dtype != 0 && dtype != 1))
      throw std::runtime_error("bad scene header");
    std::vector<float> params(59 * static_cast<size_t>(n));
    f.read(reinterpret_cast<char*>(params.data()), sizeof(float) * params.size());
    GPUBatchInput in;
    in.width = static_cast<uint32_t>(w);
    in.height = static_cast<uint32_t>(h);
    f.read(reinterpret_cast<char*>(in.K), sizeof(in.K));
    f.read(reinterpret_cast<char*>(in.w2c), sizeof(in.w2c));
    read_pod(f, in.near_plane);
    read_pod(f, in.far_plane);
    Image img;
    img.shape = ImageShape{static_cast<uint32_t>(w), static_cast<uint32_t>(h), 3};
    img.data_type = dtype ? DataType::Float16 : DataType::Float32;
    std::vector<char> target_host(img.bytes());
    f.read(target_host.data(), static_cast<std::streamsize>(target_host.size()));
    if (!f) throw std::runtime_error("truncated scene file");

    cudaStream_t stream;
    check_cuda(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate");
    auto g = std::make_shared<GPUGaussian3d>(n, sh, capacity);
    auto grad = std::make_shared<GPUGaussian3d>(n, sh, capacity);
    size_t off = 0;
    for (int k = 0; k < 6; ++k) {
      g->copy_from_host(k, params.data() + off, stream);
      off += size_t(GPUGaussian3d::kWidths[k]) * static_cast<size_t>(n);
    }
    void *d_image, *d_grad, *d_target, *d_loss;
    for (void** p : {&d_image, &d_grad, &d_target, &d_loss}) check_cuda(cudaMalloc(p, img.bytes()), "cudaMalloc");
    check_cuda(cudaMemcpyAsync(d_target, target_host.data(), img.bytes(), cudaMemcpyHostToDevice, stream),
               "target upload");

    auto rast = create_rasterizer("fastgs_b200");
    rast->set_gaussians(g);
    auto adam = std::make_shared<SimpleAdam>(g, grad);
    adam->params().max_grad_1 = max_grad_1;
    adam->set_stream(stream);
    TrainStep train(g, grad, *rast, *adam, grad_scaler);
    std::unique_ptr<DefaultStrategyB200> strategy;
    if (densify) {
      StrategyParams sp;
      sp.refine_every = refine_every;
      sp.start_refine = start_refine;
      sp.reset_every = reset_every;
      sp.duplicate_grad_threshold = grad_threshold;
      sp.max_num_gaussians = capacity > 0 ? capacity : n;
      strategy = std::make_unique<DefaultStrategyB200>(g, grad, adam, sp);
      train.set_strategy(strategy.get());
    }
    train.set_reorder_interval(reorder_every);
    // the reference's default loss mix (configs/default.json:30-39)
    train.add_loss(create_loss("l1"), 0.8f);
    train.add_loss(create_loss("fused_ssim"), 0.2f);

    RasterizeContext ctx;
    ctx.stream = stream;
    ctx.grad_scaler = grad_scaler;
    ctx.fwd_input = in;
    if (strategy) ctx.densification_info = strategy->densification_info();
    Image out = img, gimg = img, target = img, loss = img;
    out.data = d_image;
    gimg.data = d_grad;
    target.data = d_target;
    loss.data = d_loss;
    ctx.fwd_output_image = out;
    ctx.grad_output_image = gimg;
    std::vector<char> loss_host(img.bytes());
    int first_step = 0;
    if (!resume_path.empty()) {
      first_step = static_cast<int>(load_checkpoint(resume_path, *g, grad.get(), adam.get(), strategy.get(), stream));
      train.set_current_step(first_step);
      rast->set_gaussians(g);
    }
    for (int s = first_step; s < steps; ++s) {
      if (s == save_at) save_checkpoint(save_path, *g, adam.get(), strategy.get(), s, stream);
      train.run(ctx, target, loss);
      check_cuda(cudaMemcpyAsync(loss_host.data(), d_loss, img.bytes(), cudaMemcpyDeviceToHost, stream), "loss");
      check_cuda(cudaStreamSynchronize(stream), "sync");
      double sum = 0.0;
      const size_t cnt = img.shape.padded_size();
      for (size_t i = 0; i < cnt; ++i)
        sum += dtype ? half_to_float(reinterpret_cast<uint16_t*>(loss_host.data())[i])
                     : reinterpret_cast<float*>(loss_host.data())[i];
      std::printf("step %d loss %.9g n %lld\n", s, sum, static_cast<long long>(g->size()));
    }
    if (save_at == steps) save_checkpoint(save_path, *g, adam.get(), strategy.get(), steps, stream);
    const int64_t n_final = g->size();
    params.assign(59 * static_cast<size_t>(n_final), 0.0f);
    off = 0;
    for (int k = 0; k < 6; ++k) {
      g->copy_to_host(k, params.data() + off, stream);
      off += size_t(GPUGaussian3d::kWidths[k]) * static_cast<size_t>(n_final);
    }
    check_cuda(cudaStreamSynchronize(stream), "sync");
    std::ofstream o(argv[2], std::ios::binary);
    if (version == 2) o.write(reinterpret_cast<const char*>(&n_final), sizeof(n_final));
    o.write(reinterpret_cast<const char*>(params.data()), sizeof(float) * params.size());
    for (void* p : {d_image, d_grad, d_target, d_loss}) cudaFree(p);
    cudaStreamDestroy(stream);
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "tgs_train_step: %s\n", e.what());
    return 1;
  }
}
