// checkpoint.cu -- training-state checkpoint and resume: the live rows of
// the parameters, both Adam moments and the densification statistics, the
// step counters and the strategy's PCG32 state, in one binary file.
//
// The reference has no such state dump: Orchestrator calls a user
// CheckpointCallback every checkpoint_interval steps (tinygs/src/
// orchestrator.cu:433-435, include/tinygs/orchestrator.hpp:33,90) that its
// example never sets, and exports only a PLY of the parameters at the end
// (core/pointcloud.cpp:111).  A resumed run here continues bit for bit where
// the saved one stopped (same parameters, moments, bias-correction step,
// refine schedule and random splits).
//
// File (little endian):
//   char magic[8] "TGSCKPT1"; uint32 version 1; uint32 flags
//   (bit 0 moments, bit 1 densification statistics); int64 n;
//   int32 sh_degree; int32 reserved 0; TgsTrainState (5 x uint64);
//   float params: the six segments in ABI order, n rows each;
//   flags bit 0: exp_avg, then exp_avg_sq, same layout;
//   flags bit 1: float dens[n][4];
//   uint64 FNV-1a hash of every byte before it.
// Saving writes `path`.tmp and renames it over `path`, so an interrupted
// save leaves the previous checkpoint intact.
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "kernels.h"
#include "tgs_abi.h"

namespace {

constexpr char kMagic[8] = {'T', 'G', 'S', 'C', 'K', 'P', 'T', '1'};
constexpr int kWidths[6] = {3, 1, 4, 3, 3, 45};
constexpr uint64_t kFnvOffset = 1469598103934665603ULL, kFnvPrime = 1099511628211ULL;

struct Header {
  char magic[8];
  uint32_t version;
  uint32_t flags;
  int64_t n;
  int32_t sh_degree;
  int32_t reserved;
  TgsTrainState state;
};
static_assert(sizeof(Header) == 72, "checkpoint header layout");

uint64_t fnv(uint64_t h, const void* p, size_t bytes) {
  const auto* b = static_cast<const unsigned char*>(p);
  for (size_t i = 0; i < bytes; ++i) h = (h ^ b[i]) * kFnvPrime;
  return h;
}

float* seg(const TgsGaussians* g, int k) {
  float* const p[6] = {g->means, g->opacities, g->rotations, g->scales, g->sh0, g->sh_rest};
  return p[k];
}

bool set_ok(const TgsGaussians* g) {
  if (g == nullptr || g->n < 0) return false;
  for (int k = 0; k < 6; ++k)
    if (g->n > 0 && seg(g, k) == nullptr) return false;
  return true;
}

// Writer that hashes what it writes.
struct Out {
  FILE* f = nullptr;
  uint64_t h = kFnvOffset;
  bool ok = true;
  void put(const void* p, size_t bytes) {
    if (!ok || bytes == 0) return;
    h = fnv(h, p, bytes);
    ok = std::fwrite(p, 1, bytes, f) == bytes;
  }
};

struct In {
  FILE* f = nullptr;
  uint64_t h = kFnvOffset;
  bool ok = true;
  void get(void* p, size_t bytes) {
    if (!ok || bytes == 0) return;
    ok = std::fread(p, 1, bytes, f) == bytes;
    if (ok) h = fnv(h, p, bytes);
  }
};

// device rows -> file, through one host buffer of the largest segment
int put_set(Out& o, const TgsGaussians* g, int64_t n, std::vector<float>& buf, cudaStream_t st) {
  for (int k = 0; k < 6; ++k) {
    const size_t cnt = static_cast<size_t>(n) * kWidths[k];
    if (cnt == 0) continue;
    buf.resize(cnt);
    if (cudaMemcpyAsync(buf.data(), seg(g, k), cnt * sizeof(float), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess) {
      cudaGetLastError();
      return TGS_ERR_CUDA;
    }
    o.put(buf.data(), cnt * sizeof(float));
  }
  return o.ok ? TGS_OK : TGS_ERR_INVALID_ARGUMENT;
}

bool header_ok(const Header& h) {
  return std::memcmp(h.magic, kMagic, 8) == 0 && h.version == 1 && h.n >= 0 && h.n <= (int64_t{1} << 31) &&
         h.sh_degree >= 0 && h.sh_degree <= 3 && (h.flags & ~3u) == 0;
}

}  // namespace

extern "C" {

int tgs_checkpoint_save(const char* path, const TgsGaussians* params, const TgsGaussians* exp_avg,
                        const TgsGaussians* exp_avg_sq, const TgsDensificationInfo* dens,
                        const TgsTrainState* state, tgs_stream_t stream) {
  if (path == nullptr || !set_ok(params) || state == nullptr || ((exp_avg == nullptr) != (exp_avg_sq == nullptr)))
    return TGS_ERR_INVALID_ARGUMENT;
  if (exp_avg != nullptr && (!set_ok(exp_avg) || !set_ok(exp_avg_sq))) return TGS_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t n = params->n;
  Header h{};
  std::memcpy(h.magic, kMagic, 8);
  h.version = 1;
  h.flags = (exp_avg != nullptr ? 1u : 0u) | (dens != nullptr ? 2u : 0u);
  h.n = n;
  h.sh_degree = params->sh_degree;
  h.state = *state;
  const std::string tmp = std::string(path) + ".tmp";
  Out o;
  o.f = std::fopen(tmp.c_str(), "wb");
  if (o.f == nullptr) return TGS_ERR_INVALID_ARGUMENT;
  std::vector<float> buf;
  o.put(&h, sizeof(h));
  int rc = put_set(o, params, n, buf, st);
  if (rc == TGS_OK && exp_avg != nullptr) rc = put_set(o, exp_avg, n, buf, st);
  if (rc == TGS_OK && exp_avg != nullptr) rc = put_set(o, exp_avg_sq, n, buf, st);
  if (rc == TGS_OK && dens != nullptr && n > 0) {
    buf.resize(4 * static_cast<size_t>(n));
    if (cudaMemcpyAsync(buf.data(), dens, buf.size() * sizeof(float), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess) {
      cudaGetLastError();
      rc = TGS_ERR_CUDA;
    } else {
      o.put(buf.data(), buf.size() * sizeof(float));
    }
  }
  if (rc == TGS_OK) {
    const uint64_t hash = o.h;
    o.put(&hash, sizeof(hash));
    if (!o.ok) rc = TGS_ERR_INVALID_ARGUMENT;
  }
  if (std::fclose(o.f) != 0 && rc == TGS_OK) rc = TGS_ERR_INVALID_ARGUMENT;
  if (rc != TGS_OK) {
    std::remove(tmp.c_str());
    return rc;
  }
  if (std::rename(tmp.c_str(), path) != 0) {
    std::remove(tmp.c_str());
    return TGS_ERR_INVALID_ARGUMENT;
  }
  return TGS_OK;
}

int tgs_checkpoint_info(const char* path, int64_t* n, int32_t* sh_degree, uint32_t* flags, TgsTrainState* state) {
  if (path == nullptr) return TGS_ERR_INVALID_ARGUMENT;
  FILE* f = std::fopen(path, "rb");
  if (f == nullptr) return TGS_ERR_INVALID_ARGUMENT;
  Header h;
  const bool ok = std::fread(&h, 1, sizeof(h), f) == sizeof(h) && header_ok(h);
  std::fclose(f);
  if (!ok) return TGS_ERR_INVALID_ARGUMENT;
  if (n != nullptr) *n = h.n;
  if (sh_degree != nullptr) *sh_degree = h.sh_degree;
  if (flags != nullptr) *flags = h.flags;
  if (state != nullptr) *state = h.state;
  return TGS_OK;
}

int tgs_checkpoint_load(const char* path, int64_t capacity, TgsGaussians* params, TgsGaussians* exp_avg,
                        TgsGaussians* exp_avg_sq, TgsDensificationInfo* dens, TgsTrainState* state,
                        tgs_stream_t stream) {
  if (path == nullptr || params == nullptr || capacity < 0) return TGS_ERR_INVALID_ARGUMENT;
  FILE* f = std::fopen(path, "rb");
  if (f == nullptr) return TGS_ERR_INVALID_ARGUMENT;
  In in;
  in.f = f;
  Header h;
  in.get(&h, sizeof(h));
  int rc = in.ok && header_ok(h) ? TGS_OK : TGS_ERR_INVALID_ARGUMENT;
  if (rc == TGS_OK && h.n > capacity) rc = TGS_ERR_CAPACITY;
  if (rc == TGS_OK && ((exp_avg != nullptr && !(h.flags & 1u)) || (dens != nullptr && !(h.flags & 2u))))
    rc = TGS_ERR_UNSUPPORTED;  // asked for state the file does not hold
  const int64_t n = h.n;
  TgsGaussians p = *params, m{}, v{};
  auto fit = [&](TgsGaussians* dst, TgsGaussians& out) {
    if (dst == nullptr) return true;
    out = *dst;
    out.n = n;
    return set_ok(&out);
  };
  if (rc == TGS_OK && (!fit(params, p) || !fit(exp_avg, m) || !fit(exp_avg_sq, v))) rc = TGS_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the whole file is read and its hash checked before any device memory is
  // written, so a damaged file leaves the caller's state untouched
  std::vector<float> staged;
  if (rc == TGS_OK) {
    const size_t rows = 59u * static_cast<size_t>(n);
    const size_t total = rows * (1u + ((h.flags & 1u) ? 2u : 0u)) + ((h.flags & 2u) ? 4u * static_cast<size_t>(n) : 0u);
    staged.resize(total);
    in.get(staged.data(), total * sizeof(float));
    uint64_t stored = 0;
    const uint64_t computed = in.h;
    if (in.ok) {
      if (std::fread(&stored, 1, sizeof(stored), f) != sizeof(stored)) in.ok = false;
    }
    char extra;
    if (!in.ok || stored != computed || std::fread(&extra, 1, 1, f) != 0) rc = TGS_ERR_INVALID_ARGUMENT;
  }
  std::fclose(f);
  if (rc != TGS_OK) return rc;
  size_t off = 0;
  auto upload = [&](TgsGaussians* dst) -> int {
    for (int k = 0; k < 6; ++k) {
      const size_t cnt = static_cast<size_t>(n) * kWidths[k];
      if (dst != nullptr && cnt > 0 &&
          cudaMemcpyAsync(seg(dst, k), staged.data() + off, cnt * sizeof(float), cudaMemcpyHostToDevice, st) !=
              cudaSuccess)
        return TGS_ERR_CUDA;
      off += cnt;
    }
    return TGS_OK;
  };
  rc = upload(&p);
  if (rc == TGS_OK && (h.flags & 1u)) rc = upload(exp_avg != nullptr ? &m : nullptr);
  if (rc == TGS_OK && (h.flags & 1u)) rc = upload(exp_avg_sq != nullptr ? &v : nullptr);
  if (rc == TGS_OK && (h.flags & 2u) && dens != nullptr && n > 0 &&
      cudaMemcpyAsync(dens, staged.data() + off, 4u * static_cast<size_t>(n) * sizeof(float), cudaMemcpyHostToDevice,
                      st) != cudaSuccess)
    rc = TGS_ERR_CUDA;
  if (rc == TGS_OK && cudaStreamSynchronize(st) != cudaSuccess) rc = TGS_ERR_CUDA;
  if (rc != TGS_OK) {
    cudaGetLastError();
    return rc;
  }
  params->n = n;
  params->sh_degree = h.sh_degree;
  if (exp_avg != nullptr) exp_avg->n = n;
  if (exp_avg_sq != nullptr) exp_avg_sq->n = n;
  if (state != nullptr) *state = h.state;
  return TGS_OK;
}

}  // extern "C"
