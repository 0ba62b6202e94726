// Allocation-free variant of the UMAP Jacobi (delta) epoch loop.
//
// Some callers cannot let a library allocate device memory: code running
// under a framework that owns the device heap through its own caching
// allocator or memory pool, real-time loops where cudaMalloc/cudaFree would
// synchronise the device, and embedders that budget device memory up front.
// fe_b200_umap_epochs_noalloc serves them: the caller passes every input and
// output as device memory, and the only scratch the kernels need -- one
// float2 delta per vertex -- lives in the fixed file-scope array below, which
// every GPU that loads this library holds until the process exits.
//
// Host code may not take the array's address directly (its name denotes a
// host-side shadow), so the device address is looked up with
// cudaGetSymbolAddress once per device, with that device current, on the
// first call made on it.  Every call shares the array: the delta is cleared at
// the start of each call, and calls that overlap on the GPU (different streams
// or threads at the same time) race on it.
#pragma GCC visibility push(default)
#include "fastembedr_b200.h"
#pragma GCC visibility pop
#include "umap.cuh"

#include <mutex>
#include <string>

namespace {

constexpr int kNoAllocMaxVertices = 1 << 20;  // 8 MiB of float2 per device

__device__ __align__(256) float2 g_noalloc_delta[kNoAllocMaxVertices];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
float2* g_scratch_address[kMaxDevices] = {nullptr};

// Device address of g_noalloc_delta on the current device (set-up on first use).
int scratch_address(float2** out) {
  int dev = 0;
  FE_CUDA(cudaGetDevice(&dev), "cudaGetDevice(no-alloc scratch)");
  if (dev < 0 || dev >= kMaxDevices) {
    fe::set_error("no-allocation UMAP: device ordinal out of range");
    return 1;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_address[dev] == nullptr) {
    void* p = nullptr;
    FE_CUDA(cudaGetSymbolAddress(&p, g_noalloc_delta), "cudaGetSymbolAddress(no-alloc scratch)");
    g_scratch_address[dev] = static_cast<float2*>(p);
  }
  *out = g_scratch_address[dev];
  return 0;
}

}  // namespace

extern "C" int fe_b200_umap_epochs_noalloc(const int* heads, const int* tails,
                                           const float* epochs_per_sample, long long n_edges,
                                           float* layout, int n, int epoch_begin, int epoch_end,
                                           int n_epochs, int negative_sample_rate,
                                           float learning_rate, float a, float b,
                                           float repulsion_strength, unsigned int seed,
                                           int hash_key_is_tail, void* stream) {
  fe::clear_error();
  if (heads == nullptr || tails == nullptr || epochs_per_sample == nullptr || layout == nullptr) {
    fe::set_error("null device pointer");
    return 1;
  }
  if (n < 2 || n_edges < 1 || n_epochs < 1 || negative_sample_rate < 0 || !(learning_rate > 0.0f) ||
      !(repulsion_strength > 0.0f)) {
    fe::set_error("invalid CUDA COO UMAP optimization parameters");
    return 1;
  }
  if (n > kNoAllocMaxVertices) {
    fe::set_error("no-allocation UMAP: n = " + std::to_string(n) +
                  " exceeds the fixed scratch capacity of " + std::to_string(kNoAllocMaxVertices) +
                  " vertices; use fe_b200_umap_epochs for larger graphs");
    return 1;
  }
  if (epoch_begin < 0 || epoch_end < epoch_begin || epoch_end > n_epochs) {
    fe::set_error("invalid epoch range");
    return 1;
  }
  float2* delta = nullptr;
  FE_TRY(scratch_address(&delta));
  fe::UmapRun r;
  r.params = fe::UmapParams{n, n_epochs, negative_sample_rate, hash_key_is_tail, seed, learning_rate, a, b,
                            repulsion_strength};
  r.mode = fe::kUmapDelta;
  r.heads = heads;
  r.tails = tails;
  r.periods = epochs_per_sample;
  r.n_edges = n_edges;
  r.layout = reinterpret_cast<float2*>(layout);
  r.delta = delta;  // umap_run_epochs clears it before the first epoch
  r.positive_count = nullptr;
  r.stream = static_cast<cudaStream_t>(stream);
  r.edge_blocks = fe::umap_edge_blocks(n_edges);
  r.use_graphs = false;
  FE_TRY(fe::umap_run_epochs(&r, epoch_begin, epoch_end));
  FE_CUDA(cudaStreamSynchronize(r.stream), "cudaStreamSynchronize(no-alloc UMAP)");
  return 0;
}
