// Shared host/device plumbing for the B200 embedding-optimizer backend.
//
// Error convention (mirrors the reference C ABI, src/embedding_cuda_kernels.cpp:55-72):
// every entry point returns 0 on success and 1 on failure, leaving a
// thread-local message readable through fastembedr_cuda_embedding_last_error().
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>

namespace fe {

// ---------------------------------------------------------------- errors

void set_error(const std::string& message);
const char* last_error();
void clear_error();

inline int check_cuda(cudaError_t code, const char* where) {
  if (code == cudaSuccess) return 0;
  set_error(std::string(where) + ": " + cudaGetErrorString(code));
  return 1;
}

#define FE_TRY(expr)          \
  do {                        \
    if ((expr) != 0) return 1; \
  } while (0)

#define FE_CUDA(call, where) FE_TRY(::fe::check_cuda((call), (where)))
#define FE_LAUNCH(where) FE_TRY(::fe::check_cuda(cudaGetLastError(), (where)))

// ---------------------------------------------------------------- memory

constexpr std::size_t kAlign = 256;

inline std::size_t align_up(std::size_t bytes, std::size_t a = kAlign) {
  return (bytes + a - 1) & ~(a - 1);
}

// One device allocation carved into aligned sub-buffers.  Sizing is done by a
// first "plan" pass (base == nullptr) that only accumulates offsets.
class Arena {
 public:
  Arena() = default;
  ~Arena() { release(); }
  Arena(const Arena&) = delete;
  Arena& operator=(const Arena&) = delete;

  void begin_plan() {
    planning_ = true;
    offset_ = 0;
  }
  template <typename T>
  T* take(std::size_t count) {
    const std::size_t bytes = align_up(count * sizeof(T) + (count == 0 ? 1 : 0));
    T* p = planning_ ? nullptr : reinterpret_cast<T*>(static_cast<char*>(base_) + offset_);
    offset_ += bytes;
    return p;
  }
  // Allocates the planned size; returns 0 on success.
  int commit(const char* what);
  // Adopts caller-owned device memory of at least planned() bytes (no allocation).
  void adopt(void* base) {
    base_ = base;
    owned_ = false;
    planning_ = false;
    size_ = offset_;
    offset_ = 0;
  }
  void rewind() { offset_ = 0; }
  std::size_t planned() const { return offset_; }
  std::size_t size() const { return size_; }
  void release();

 private:
  void* base_ = nullptr;
  bool owned_ = false;
  bool planning_ = false;
  std::size_t offset_ = 0;
  std::size_t size_ = 0;
};

// Fails cleanly when a request exceeds 95% of free device memory
// (the reference's preflight, src/embedding_cuda_kernels.cpp:224-241).
int memory_preflight(std::size_t bytes, const char* where);

// ---------------------------------------------------------------- exact KNN (knn.cu)

// Exact Euclidean KNN of n points (n x p; column-major when col_major, else
// row-major; double or float; host or device) into caller device arrays,
// column-major n x k, indices 1-based.  Synchronises `st`.
int knn_exact(const void* data, bool data_double, bool data_on_device, bool col_major, int n, int p, int k,
              bool exclude_self, int* d_indices, float* d_distances, cudaStream_t st);

// ---------------------------------------------------------------- launch shape

// SM count of the current device (cached per device).
int sm_count();

// Device memory of the library (common.cu): cudaMalloc / cudaFree semantics
// (dev_free waits for the device), served by a per-device pool that retains
// freed blocks for the next call unless FASTEMBEDR_B200_RETAIN_MB=0.
cudaError_t dev_malloc_bytes(void** p, std::size_t bytes);
cudaError_t dev_free(void* p);
template <typename T>
inline cudaError_t dev_malloc(T** p, std::size_t bytes) {
  return dev_malloc_bytes(reinterpret_cast<void**>(p), bytes);
}
std::size_t pool_spare_bytes();   // retained and unused bytes on the current device
// Host time spent in dev_malloc / dev_free since the process started.
void alloc_time_totals(double* alloc_ms, double* free_ms, long long* alloc_calls);
int release_retained_memory();    // return every device's retained memory to the driver

// Host -> device copy of a caller's buffer (pageable or pinned) that returns
// once the data is on the device; large pageable sources are staged through
// a pinned pool by several host threads (host_copy.cu).
int h2d_copy(void* dst, const void* src, std::size_t bytes, cudaStream_t stream, const char* what);

// Environment helpers.
int env_int(const char* name, int fallback);         // positive values only
int env_int_nonneg(const char* name, int fallback);  // zero allowed
bool env_flag(const char* name, bool fallback);
double env_double(const char* name, double fallback);  // positive values only

}  // namespace fe

// ---------------------------------------------------------------- device helpers

#ifdef __CUDACC__

namespace fe {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Streaming (evict-first) 16-byte loads for data read once per pass.
__device__ __forceinline__ int4 ld_stream(const int4* p) { return __ldcs(p); }
__device__ __forceinline__ float4 ld_stream(const float4* p) { return __ldcs(p); }
__device__ __forceinline__ uint2 ld_stream(const uint2* p) { return __ldcs(p); }

// The reference's counter-based uniform in [-1, 1] for coordinate `col` of
// point `row` (deterministic_unit, src/embedding_cuda_kernels.cpp:266-274):
// a 32-bit finaliser over the seed mixed with (row + 1) and (col + 1), whose
// low 24 bits are scaled.  The constants are the reference's, so that random
// starts agree with it point for point.
__device__ __forceinline__ float hashed_unit(unsigned int seed, int row, int col) {
  unsigned int x = seed;
  x ^= (static_cast<unsigned int>(row) + 1u) * 0x9e3779b9u;
  x ^= (static_cast<unsigned int>(col) + 1u) * 0x85ebca6bu;
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return static_cast<float>(x & 0x00ffffffu) / 8388607.5f - 1.0f;
}

}  // namespace fe

#endif
