// Host-side runtime shared by every entry point: error text, workspace arena,
// memory preflight, device properties and environment switches.
#include "fe_common.cuh"

#include <atomic>
#include <chrono>
#include <cstdio>
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

// ---- device memory
//
// Every device buffer of the library comes from dev_malloc / dev_free.  By
// default they draw on one stream-ordered memory pool per device that keeps up
// to FASTEMBEDR_B200_RETAIN_MB (default 32768) of freed memory mapped for the
// next call: a 1M-point t-SNE call maps and unmaps several GB, and the
// driver's unmapping of such blocks took anywhere from 4 to 600 ms per call
// on this hardware.  dev_free waits for the device first, as cudaFree does,
// so a block is never handed out again while a kernel may still use it.
// FASTEMBEDR_B200_RETAIN_MB=0 uses plain cudaMalloc / cudaFree;
// fe_b200_release_memory returns the retained memory.
namespace {
constexpr int kMaxDevices = 64;
struct DevicePool {
  cudaMemPool_t pool = nullptr;
  cudaStream_t stream = nullptr;  // orders the pool's allocations and frees
  bool tried = false;
};
std::mutex g_pool_mutex;
DevicePool g_pools[kMaxDevices];

std::size_t retain_bytes() {
  static const long long mb = env_int_nonneg("FASTEMBEDR_B200_RETAIN_MB", 32768);
  return static_cast<std::size_t>(mb) << 20;
}

// The current device's pool, created on first use; nullptr when retention is
// off or the pool could not be made (then plain cudaMalloc is used).
DevicePool* current_pool() {
  if (retain_bytes() == 0) return nullptr;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_pool_mutex);
  DevicePool& dp = g_pools[dev];
  if (!dp.tried) {
    dp.tried = true;
    cudaMemPoolProps props{};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t pool = nullptr;
    cudaStream_t stream = nullptr;
    std::uint64_t threshold = retain_bytes();
    if (cudaMemPoolCreate(&pool, &props) == cudaSuccess &&
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold) == cudaSuccess &&
        cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) == cudaSuccess) {
      dp.pool = pool;
      dp.stream = stream;
    } else {
      cudaGetLastError();
      if (pool != nullptr) cudaMemPoolDestroy(pool);
    }
  }
  return dp.pool != nullptr ? &dp : nullptr;
}
}  // namespace

namespace {
// Host time spent in dev_malloc / dev_free (read by the phase trace).
std::atomic<long long> g_alloc_ns{0}, g_free_ns{0}, g_alloc_calls{0};
const bool g_trace_allocs = std::getenv("FASTEMBEDR_B200_TRACE") != nullptr;
struct AllocClock {
  std::atomic<long long>& sink;
  std::chrono::steady_clock::time_point t0 = std::chrono::steady_clock::now();
  explicit AllocClock(std::atomic<long long>& s) : sink(s) {}
  ~AllocClock() {
    sink += std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count();
  }
};
}  // namespace

void alloc_time_totals(double* alloc_ms, double* free_ms, long long* alloc_calls) {
  *alloc_ms = static_cast<double>(g_alloc_ns.load()) * 1e-6;
  *free_ms = static_cast<double>(g_free_ns.load()) * 1e-6;
  *alloc_calls = g_alloc_calls.load();
}

cudaError_t dev_malloc_bytes(void** p, std::size_t bytes) {
  *p = nullptr;
  if (bytes == 0) return cudaSuccess;
  AllocClock clock(g_alloc_ns);
  ++g_alloc_calls;
  DevicePool* dp = current_pool();
  if (dp == nullptr) return cudaMalloc(p, bytes);
  const auto t0 = std::chrono::steady_clock::now();
  const cudaError_t code = cudaMallocFromPoolAsync(p, bytes, dp->pool, dp->stream);
  if (code != cudaSuccess) return code;
  const cudaError_t sync = cudaStreamSynchronize(dp->stream);
  if (g_trace_allocs) {
    const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    if (ms > 5.0) {
      std::uint64_t reserved = 0, used = 0;
      cudaMemPoolGetAttribute(dp->pool, cudaMemPoolAttrReservedMemCurrent, &reserved);
      cudaMemPoolGetAttribute(dp->pool, cudaMemPoolAttrUsedMemCurrent, &used);
      std::fprintf(stderr, "[fastembedr_b200 trace] slow allocation: %zu bytes in %.3f ms (pool reserved %llu MiB, used %llu MiB)\n",
                   bytes, ms, static_cast<unsigned long long>(reserved >> 20), static_cast<unsigned long long>(used >> 20));
    }
  }
  return sync;
}

cudaError_t dev_free(void* p) {
  if (p == nullptr) return cudaSuccess;
  AllocClock clock(g_free_ns);
  if (retain_bytes() == 0) return cudaFree(p);
  // The block goes back to the pool of the device that holds it, after that
  // device is idle, whichever device the caller has current (as cudaFree).
  cudaPointerAttributes attr{};
  int current = 0;
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess || cudaGetDevice(&current) != cudaSuccess) {
    cudaGetLastError();
    return cudaFree(p);
  }
  const bool switch_device = attr.type == cudaMemoryTypeDevice && attr.device != current;
  if (switch_device && cudaSetDevice(attr.device) != cudaSuccess) return cudaFree(p);
  cudaError_t code;
  DevicePool* dp = current_pool();
  if (dp == nullptr) {
    code = cudaFree(p);
  } else {
    const cudaError_t sync = cudaDeviceSynchronize();
    code = cudaFreeAsync(p, dp->stream);
    if (sync != cudaSuccess) code = sync;
  }
  if (switch_device) cudaSetDevice(current);
  return code;
}

std::size_t pool_spare_bytes() {
  DevicePool* dp = current_pool();
  if (dp == nullptr) return 0;
  std::uint64_t reserved = 0, used = 0;
  if (cudaMemPoolGetAttribute(dp->pool, cudaMemPoolAttrReservedMemCurrent, &reserved) != cudaSuccess ||
      cudaMemPoolGetAttribute(dp->pool, cudaMemPoolAttrUsedMemCurrent, &used) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return reserved > used ? static_cast<std::size_t>(reserved - used) : 0;
}

int release_retained_memory() {
  int current = 0;
  if (cudaGetDevice(&current) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  std::lock_guard<std::mutex> lock(g_pool_mutex);
  for (int dev = 0; dev < kMaxDevices; ++dev) {
    DevicePool& dp = g_pools[dev];
    if (dp.pool == nullptr) continue;
    if (cudaSetDevice(dev) != cudaSuccess || cudaStreamSynchronize(dp.stream) != cudaSuccess ||
        cudaMemPoolTrimTo(dp.pool, 0) != cudaSuccess) {
      set_error("releasing retained device memory failed");
      cudaSetDevice(current);
      return 1;
    }
  }
  cudaSetDevice(current);
  return 0;
}

int Arena::commit(const char* what) {
  release();
  planning_ = false;
  size_ = offset_;
  offset_ = 0;
  if (size_ == 0) return 0;
  const cudaError_t code = dev_malloc(&base_, size_);
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
  if (base_ != nullptr && owned_) dev_free(base_);
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
  free_bytes += pool_spare_bytes();  // freed blocks the pool keeps for reuse
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
