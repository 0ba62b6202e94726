// Host-side runtime shared by every entry point: error text, workspace arena,
// memory preflight, device properties and environment switches.
#include "fe_common.cuh"

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

namespace fe {

namespace {
thread_local std::string g_last_error;
}

void set_error(const std::string& message) { g_last_error = message; }
const char* last_error() { return g_last_error.c_str(); }
void clear_error() {
  g_last_error.clear();
  cudaGetLastError();  // drop a non-sticky error left by an earlier failed call on this thread
}

int Arena::commit(const char* what) {
  release();
  planning_ = false;
  size_ = offset_;
  offset_ = 0;
  if (size_ == 0) return 0;
  const cudaError_t code = cudaMalloc(&base_, size_);
  if (code != cudaSuccess) {
    base_ = nullptr;
    set_error(std::string("cudaMalloc(") + what + ", " + std::to_string(size_) + " bytes): " +
              cudaGetErrorString(code));
    return 1;
  }
  owned_ = true;
  return 0;
}

void Arena::release() {
  if (base_ != nullptr && owned_) cudaFree(base_);
  base_ = nullptr;
  owned_ = false;
  size_ = 0;
}

int memory_preflight(std::size_t bytes, const char* where) {
  std::size_t free_bytes = 0, total_bytes = 0;
  if (cudaMemGetInfo(&free_bytes, &total_bytes) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  const std::size_t reserve = free_bytes / 20u;
  if (bytes > free_bytes - reserve) {
    set_error(std::string(where) + ": CUDA memory request exceeds available memory; required " +
              std::to_string(bytes) + " bytes, free " + std::to_string(free_bytes) + " bytes");
    return 1;
  }
  return 0;
}

int sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cache[dev] = v;
  }
  return cache[dev];
}

int env_int(const char* name, int fallback) {
  const char* raw = std::getenv(name);
  if (raw == nullptr || raw[0] == '\0') return fallback;
  char* end = nullptr;
  const long v = std::strtol(raw, &end, 10);
  if (end == raw || v <= 0 || v > 1 << 30) return fallback;
  return static_cast<int>(v);
}

int env_int_nonneg(const char* name, int fallback) {
  const char* raw = std::getenv(name);
  if (raw == nullptr || raw[0] == '\0') return fallback;
  char* end = nullptr;
  const long v = std::strtol(raw, &end, 10);
  if (end == raw || v < 0 || v > 1 << 30) return fallback;
  return static_cast<int>(v);
}

double env_double(const char* name, double fallback) {
  const char* raw = std::getenv(name);
  if (raw == nullptr || raw[0] == '\0') return fallback;
  char* end = nullptr;
  const double v = std::strtod(raw, &end);
  if (end == raw || !(v > 0.0) || v > 1e9) return fallback;
  return v;
}

bool env_flag(const char* name, bool fallback) {
  const char* raw = std::getenv(name);
  if (raw == nullptr || raw[0] == '\0') return fallback;
  return !(std::strcmp(raw, "0") == 0 || std::strcmp(raw, "false") == 0 ||
           std::strcmp(raw, "FALSE") == 0 || std::strcmp(raw, "no") == 0 ||
           std::strcmp(raw, "NO") == 0);
}

}  // namespace fe
