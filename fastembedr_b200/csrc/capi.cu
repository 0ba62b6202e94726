// extern "C" boundary of libfastembedr_b200.so (declared in include/fastembedr_b200.h).
// The library is built with hidden visibility; only the declarations of the
// public header are exported.
#pragma GCC visibility push(default)
#include "fastembedr_b200.h"
#pragma GCC visibility pop
#include "nccl_loader.cuh"
#include "tsne.cuh"
#include "umap.cuh"

#include <cfloat>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

struct fe_b200_tsne {
  fe::TsneSession* impl = nullptr;
};

namespace {

using fe::set_error;

const char* kOutOfScope = "not provided by the B200 backend (outside the optimizer hot path)";

int out_of_scope(const char* name) {
  set_error(std::string(name) + ": " + kOutOfScope);
  return 1;
}

// Grid side: the reference CPU policy by default (the parity target);
// FASTEMBEDR_B200_GRID_POLICY=cuda selects the reference CUDA sizes
// (256 / 512 / 1024 by n, src/embedding_cuda_kernels.cpp:5496-5505).
int resolve_grid(int n, int requested) {
  if (requested > 0) {
    int g = 4;
    while (g < requested && g < 1024) g <<= 1;
    return g;
  }
  const char* policy = std::getenv("FASTEMBEDR_B200_GRID_POLICY");
  if (policy != nullptr && std::strcmp(policy, "cuda") == 0) {
    int g = 512;
    if (n < 20000) g = 256;
    if (n >= 100000) g = 1024;
    const int env = fe::env_int("FASTEMBEDR_TSNE_FFT_GRID", 0);
    if (env == 128 || env == 256 || env == 512 || env == 1024) g = env;
    return g;
  }
  return fe::default_grid_size(n);
}

struct DeviceCopy {
  void* p = nullptr;
  ~DeviceCopy() {
    if (p) fe::dev_free(p);
  }
};

int copy_to_device(const void* host, size_t bytes, DeviceCopy& dst, cudaStream_t stream, const char* what) {
  FE_CUDA(fe::dev_malloc(&dst.p, bytes ? bytes : 1), what);
  return fe::h2d_copy(dst.p, host, bytes, stream, what);
}

// FASTEMBEDR_B200_TRACE=1: wall time of each phase of a call, printed to
// stderr when the call ends (the stream is synchronised at every mark, so a
// traced call is slower; without the variable nothing is added).  The last
// line covers the teardown after the final mark, measured in the destructor.
struct PhaseTrace {
  const char* name;
  cudaStream_t stream;
  bool on;
  std::chrono::steady_clock::time_point t0, last;
  std::string lines;
  double alloc_ms = 0.0, free_ms = 0.0;
  long long alloc_calls = 0;
  PhaseTrace(const char* n, cudaStream_t s) : name(n), stream(s), on(fe::env_flag("FASTEMBEDR_B200_TRACE", false)) {
    t0 = last = std::chrono::steady_clock::now();
    if (on) fe::alloc_time_totals(&alloc_ms, &free_ms, &alloc_calls);
  }
  void mark(const char* phase) {
    if (!on) return;
    cudaStreamSynchronize(stream);
    const auto now = std::chrono::steady_clock::now();
    double a = 0.0, f = 0.0;
    long long c = 0;
    fe::alloc_time_totals(&a, &f, &c);
    char buf[160];
    std::snprintf(buf, sizeof(buf), " (allocations %lld: %.3f ms, frees %.3f ms)", c - alloc_calls, a - alloc_ms,
                  f - free_ms);
    alloc_ms = a;
    free_ms = f;
    alloc_calls = c;
    lines += std::string("[fastembedr_b200 trace] ") + name + " " + phase + ": " +
             std::to_string(std::chrono::duration<double, std::milli>(now - last).count()) + " ms" + buf + "\n";
    last = now;
  }
  ~PhaseTrace() {
    if (!on) return;
    const auto now = std::chrono::steady_clock::now();
    std::fprintf(stderr, "%s[fastembedr_b200 trace] %s total: %.3f ms\n", lines.c_str(), name,
                 std::chrono::duration<double, std::milli>(now - t0).count());
  }
};

// Shared by every openTSNE entry point (the reference's
// fastembedr_cuda_opentsne_fft_from_knn_impl, src/embedding_cuda_kernels.cpp:5453-6008).
int opentsne_impl(const int* indices, const void* distances, bool dist_double, const float* init,
                  int has_init, int n, int k, int n_components, float perplexity,
                  int early_exaggeration_iter, int n_iter, float early_exaggeration,
                  float exaggeration, float learning_rate, int learning_rate_auto,
                  float initial_momentum, float final_momentum, float min_gain,
                  float max_step_norm, unsigned int seed, int index_offset, float* out,
                  bool on_device, const void* pca_values = nullptr, bool pca_double = false, int pca_p = 0) {
  fe::clear_error();
  if (indices == nullptr || distances == nullptr || out == nullptr || (has_init && init == nullptr)) {
    set_error("null CUDA openTSNE input pointer");
    return 1;
  }
  if (n < 2 || k < 1 || k > 256 || n_components != 2 || !(perplexity > 0.0f) ||
      early_exaggeration_iter < 0 || n_iter < 0 || early_exaggeration_iter + n_iter < 1 ||
      !(early_exaggeration > 0.0f) || !(exaggeration > 0.0f) ||
      (!learning_rate_auto && !(learning_rate > 0.0f)) || initial_momentum < 0.0f ||
      final_momentum < 0.0f || !(min_gain > 0.0f)) {
    set_error("invalid CUDA openTSNE FFT-grid dimensions or parameters");
    return 1;
  }
  // Learning rate per phase: n / exaggeration when automatic (src/tsne_neighbors.cpp:1734-1737).
  const float lr_early = learning_rate_auto
      ? static_cast<float>(static_cast<double>(n) / std::max(static_cast<double>(early_exaggeration), DBL_MIN))
      : learning_rate;
  const float lr_normal = learning_rate_auto
      ? static_cast<float>(static_cast<double>(n) / std::max(static_cast<double>(exaggeration), DBL_MIN))
      : learning_rate;
  const float clip = std::isfinite(max_step_norm) ? max_step_norm : NAN;
  const bool pca = !has_init && pca_values != nullptr;
  if (pca && (pca_p < 2 || pca_p < n_components)) {
    set_error("invalid dimensions in device PCA initialization");
    return 1;
  }
  std::vector<int> devices;
  FE_TRY(fe::multi_device_list(&devices));
  std::vector<float> pca_host;
  if (devices.size() >= 2 && pca) {
    // The PCA start is made once, on the calling device, and handed to every
    // rank as a host init.
    cudaStream_t ps = nullptr;
    FE_CUDA(cudaStreamCreateWithFlags(&ps, cudaStreamNonBlocking), "cudaStreamCreate(PCA)");
    float2* d_start = nullptr;
    int rc = fe::check_cuda(fe::dev_malloc(&d_start, sizeof(float2) * static_cast<size_t>(n)), "cudaMalloc(PCA start)");
    if (rc == 0) rc = fe::pca_start_layout(pca_values, pca_double, n, pca_p, ps, d_start);
    if (rc == 0) {
      pca_host.resize(2 * static_cast<size_t>(n));
      rc = fe::check_cuda(cudaMemcpy(pca_host.data(), d_start, sizeof(float2) * static_cast<size_t>(n),
                                     cudaMemcpyDeviceToHost), "D2H PCA start");
    }
    if (d_start != nullptr) fe::dev_free(d_start);
    cudaStreamDestroy(ps);
    if (rc != 0) return 1;
    init = pca_host.data();
    has_init = 1;
  }
  if (devices.size() >= 2) {
    fe::MultiDeviceTsne job;
    job.devices = devices;
    job.indices = indices;
    job.distances = distances;
    job.dist_double = dist_double;
    job.on_device = on_device;
    job.init = has_init ? init : nullptr;
    job.seed = seed;
    job.n = n;
    job.k = k;
    job.index_offset = index_offset;
    job.perplexity = perplexity;
    job.grid = resolve_grid(n, 0);
    job.early_iter = early_exaggeration_iter;
    job.early_exaggeration = early_exaggeration;
    job.initial_momentum = initial_momentum;
    job.lr_early = lr_early;
    job.n_iter = n_iter;
    job.exaggeration = exaggeration;
    job.final_momentum = final_momentum;
    job.lr_normal = lr_normal;
    job.min_gain = min_gain;
    job.max_step_norm = clip;
    job.out = out;
    return fe::opentsne_multi_device(job);
  }
  cudaStream_t stream = nullptr;
  FE_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate(openTSNE)");
  struct StreamGuard {
    cudaStream_t s;
    ~StreamGuard() {
      cudaStreamSynchronize(s);
      cudaStreamDestroy(s);
    }
  } guard{stream};
  PhaseTrace trace("opentsne", stream);

  const size_t items = static_cast<size_t>(n) * k;
  int* row_ptr = nullptr;
  int* col = nullptr;
  float* val = nullptr;
  long long nnz = 0;
  {
    DeviceCopy d_idx, d_dist;
    const int* idx_dev = indices;
    const void* dist_dev = distances;
    if (!on_device) {
      FE_TRY(copy_to_device(indices, items * sizeof(int), d_idx, stream, "H2D openTSNE indices"));
      FE_TRY(copy_to_device(distances, items * (dist_double ? sizeof(double) : sizeof(float)), d_dist,
                            stream, "H2D openTSNE distances"));
      idx_dev = static_cast<const int*>(d_idx.p);
      dist_dev = d_dist.p;
      trace.mark("H2D KNN");
    }
    FE_TRY(fe::build_p_device(idx_dev, dist_dev, dist_double, n, k, index_offset, perplexity, stream,
                              &row_ptr, &col, &val, &nnz));
    trace.mark("P build");
  }
  trace.mark("KNN copies freed");
  fe::TsneSession* s = nullptr;
  if (fe::session_create(&s, n, resolve_grid(n, 0), row_ptr, col, val, nnz, stream)) {
    fe::dev_free(row_ptr);
    fe::dev_free(col);
    fe::dev_free(val);
    return 1;
  }
  struct SessionGuard {
    fe::TsneSession* s;
    ~SessionGuard() { fe::session_destroy(s); }
  } sguard{s};
  trace.mark("session create");
  if (has_init) {
    FE_TRY(fe::session_set_layout(s, init, true, true));
  } else if (pca) {
    // The reference's PCA start (RAFT TSVD scores, scaled to sd 1e-4), made on
    // the device into a free session buffer.
    FE_TRY(fe::pca_start_layout(pca_values, pca_double, n, pca_p, s->stream, s->grad_out));
    FE_TRY(fe::session_set_layout(s, reinterpret_cast<const float*>(s->grad_out), false, true));
  } else {
    FE_TRY(fe::session_random_layout(s, seed));
  }
  trace.mark("start layout");
  FE_TRY(fe::session_iterate(s, early_exaggeration_iter, early_exaggeration, initial_momentum, lr_early,
                             min_gain, clip));
  trace.mark("early iterations");
  FE_TRY(fe::session_iterate(s, n_iter, exaggeration, final_momentum, lr_normal, min_gain, clip));
  trace.mark("iterations");
  FE_TRY(fe::session_get_layout(s, out, true));
  trace.mark("D2H layout");
  return 0;
}

int umap_validate(const void* heads, const void* tails, const void* weights, const void* eps,
                  const void* layout, int n, long long n_edges, int n_epochs, int nsr, float lr,
                  float rep) {
  if (heads == nullptr || tails == nullptr || weights == nullptr || eps == nullptr ||
      layout == nullptr) {
    set_error("null host pointer");
    return 1;
  }
  if (n < 2 || n_edges < 1 || n_epochs < 1 || nsr < 0 || !(lr > 0.0f) || !(rep > 0.0f)) {
    set_error("invalid CUDA COO UMAP optimization parameters");
    return 1;
  }
  return 0;
}

int umap_hash_key_default() {
  const char* v = std::getenv("FASTEMBEDR_B200_UMAP_NEGATIVE_KEY");
  return (v != nullptr && std::strcmp(v, "tail") == 0) ? 1 : 0;
}

int umap_host_run(const int* heads, const int* tails, const float* eps, long long n_edges,
                  const float* init, float* out, int n, int epoch_begin, int epoch_end, int n_epochs,
                  int nsr, float lr, float a, float b, float rep, unsigned int seed, int mode,
                  int hash_key_is_tail, long long* positive_samples) {
  cudaStream_t stream = nullptr;
  FE_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate(umap)");
  struct StreamGuard {
    cudaStream_t s;
    ~StreamGuard() {
      cudaStreamSynchronize(s);
      cudaStreamDestroy(s);
    }
  } guard{stream};
  fe::Arena arena;
  int* d_heads = nullptr;
  int* d_tails = nullptr;
  float* d_eps = nullptr;
  float2* d_layout = nullptr;
  float2* d_delta = nullptr;
  long long* d_count = nullptr;
  const size_t e = static_cast<size_t>(n_edges);
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 0) arena.begin_plan();
    else arena.rewind();
    d_heads = arena.take<int>(e);
    d_tails = arena.take<int>(e);
    d_eps = arena.take<float>(e);
    d_layout = arena.take<float2>(n);
    d_delta = arena.take<float2>(mode == fe::kUmapDelta ? n : 0);
    d_count = arena.take<long long>(1);
    if (pass == 0) {
      FE_TRY(fe::memory_preflight(arena.planned(), "CUDA COO UMAP optimizer allocation preflight"));
      FE_TRY(arena.commit("COO UMAP workspace"));
    }
  }
  FE_TRY(fe::h2d_copy(d_heads, heads, e * sizeof(int), stream, "H2D heads"));
  FE_TRY(fe::h2d_copy(d_tails, tails, e * sizeof(int), stream, "H2D tails"));
  FE_TRY(fe::h2d_copy(d_eps, eps, e * sizeof(float), stream, "H2D epochs_per_sample"));
  FE_TRY(fe::h2d_copy(d_layout, init, sizeof(float2) * n, stream, "H2D init"));
  FE_CUDA(cudaMemsetAsync(d_count, 0, sizeof(long long), stream), "memset count");
  fe::UmapRun r;
  r.params = fe::UmapParams{n, n_epochs, nsr, hash_key_is_tail, seed, lr, a, b, rep};
  r.mode = mode;
  r.heads = d_heads;
  r.tails = d_tails;
  r.periods = d_eps;
  r.n_edges = n_edges;
  r.layout = d_layout;
  r.delta = mode == fe::kUmapDelta ? d_delta : nullptr;
  r.positive_count = positive_samples != nullptr ? d_count : nullptr;
  r.stream = stream;
  r.edge_blocks = fe::umap_edge_blocks(n_edges);
  r.use_graphs = fe::env_flag("FASTEMBEDR_CUDA_GRAPH_CAPTURE", true);
  struct CompactionGuard {
    fe::UmapCompaction c;
    ~CompactionGuard() { fe::umap_compaction_free(&c); }
  } compaction;
  FE_TRY(fe::umap_compaction_alloc(n_edges, &compaction.c));
  r.compact = compaction.c;
  FE_TRY(fe::umap_run_epochs(&r, epoch_begin, epoch_end));
  FE_CUDA(cudaMemcpyAsync(out, d_layout, sizeof(float2) * n, cudaMemcpyDeviceToHost, stream), "D2H layout");
  if (positive_samples != nullptr) {
    FE_CUDA(cudaMemcpyAsync(positive_samples, d_count, sizeof(long long), cudaMemcpyDeviceToHost, stream),
            "D2H count");
  }
  FE_CUDA(cudaStreamSynchronize(stream), "cudaStreamSynchronize(umap)");
  return 0;
}

// Device bytes of the graph build at its peak plus the COO list and layouts.
size_t umap_graph_bytes(int n, int k) {
  const size_t nk = static_cast<size_t>(n) * k;
  const size_t slots = static_cast<size_t>(n) * fe::umap_graph_width(k);
  return 64 * nk + 24 * slots + 32 * static_cast<size_t>(n) + (64u << 20);
}

// The device-KNN UMAP path (fastembedr_cuda_umap_from_device_knn_spectral_impl,
// src/embedding_cuda_kernels.cpp:4967-5199): graph, diffusion start, rank-major
// COO list, then the epochs.  Negatives are keyed on the tail vertex, as the
// reference's COO kernels key them (:3109-3118).  The edge order matters to the
// in-place (Hogwild) mode: rank-major order puts a vertex's edges far apart in
// time, so each sees its earlier moves, as in the reference; grouped by head
// they would all start from the same stale position.
int umap_fused_impl(const int* idx, const void* dist, bool dist_double, bool on_device, int n, int k,
                    int n_epochs, int nsr, float lr, float a, float b, float rep, int spectral_n_iter,
                    unsigned int seed, int index_offset, int optimizer_mode, bool binary, float* out) {
  if (n_epochs < 1 || nsr < 0 || lr <= 0.0f || spectral_n_iter < 1) {
    set_error("invalid fused CUDA UMAP dimensions or parameters");
    return 1;
  }
  FE_TRY(fe::memory_preflight(umap_graph_bytes(n, k) +
                                  (on_device ? 0 : static_cast<size_t>(n) * k * (dist_double ? 12 : 8)),
                              "CUDA fused UMAP allocation preflight"));
  cudaStream_t stream = nullptr;
  FE_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate(fused umap)");
  struct StreamGuard {
    cudaStream_t s;
    ~StreamGuard() {
      cudaStreamSynchronize(s);
      cudaStreamDestroy(s);
    }
  } guard{stream};
  fe::UmapDenseGraph g;
  {
    DeviceCopy d_idx, d_dist;
    const int* idx_dev = idx;
    const void* dist_dev = dist;
    if (!on_device) {
      const size_t items = static_cast<size_t>(n) * k;
      FE_TRY(copy_to_device(idx, items * sizeof(int), d_idx, stream, "H2D fused umap indices"));
      FE_TRY(copy_to_device(dist, items * (dist_double ? sizeof(double) : sizeof(float)), d_dist, stream,
                            "H2D fused umap distances"));
      idx_dev = static_cast<const int*>(d_idx.p);
      dist_dev = d_dist.p;
    }
    FE_TRY(fe::umap_graph_build(idx_dev, dist_dev, dist_double, n, k, index_offset, binary, stream, &g));
  }
  fe::Arena arena;
  const size_t slots = static_cast<size_t>(n) * g.width;
  int* heads = nullptr;
  int* tails = nullptr;
  float* periods = nullptr;
  float2* layout = nullptr;
  float2* delta = nullptr;
  const int mode = optimizer_mode == 1 ? fe::kUmapDelta : fe::kUmapInplaceSample;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 0) arena.begin_plan();
    else arena.rewind();
    heads = arena.take<int>(slots);
    tails = arena.take<int>(slots);
    periods = arena.take<float>(slots);
    layout = arena.take<float2>(n);
    delta = arena.take<float2>(mode == fe::kUmapDelta ? n : 0);
    if (pass == 0) FE_TRY(arena.commit("fused UMAP workspace"));
  }
  FE_TRY(fe::umap_diffusion_init(g, seed, spectral_n_iter, layout, stream));
  long long n_edges = 0;
  FE_TRY(fe::umap_graph_pack(g, true, heads, tails, nullptr, periods, &n_edges, stream));
  if (n_edges < 1 || n_edges > static_cast<long long>(slots)) {
    set_error("invalid fused CUDA UMAP graph edge count");
    return 1;
  }
  fe::UmapRun r;
  r.params = fe::UmapParams{n, n_epochs, nsr, 1, seed, lr, a, b, rep};
  r.mode = mode;
  r.heads = heads;
  r.tails = tails;
  r.periods = periods;
  r.n_edges = n_edges;
  r.layout = layout;
  r.delta = mode == fe::kUmapDelta ? delta : nullptr;
  r.stream = stream;
  r.edge_blocks = fe::umap_edge_blocks(n_edges);
  r.use_graphs = fe::env_flag("FASTEMBEDR_CUDA_GRAPH_CAPTURE", true);
  struct CompactionGuard {
    fe::UmapCompaction c;
    ~CompactionGuard() { fe::umap_compaction_free(&c); }
  } compaction;
  FE_TRY(fe::umap_compaction_alloc(n_edges, &compaction.c));
  r.compact = compaction.c;
  FE_TRY(fe::umap_run_epochs(&r, 0, n_epochs));
  FE_CUDA(cudaMemcpyAsync(out, layout, sizeof(float2) * n, cudaMemcpyDeviceToHost, stream), "D2H fused umap layout");
  FE_CUDA(cudaStreamSynchronize(stream), "cudaStreamSynchronize(fused umap)");
  return 0;
}

int umap_fused_host(const int* idx, const void* dist, bool dist_double, int n, int k, int n_epochs, int nsr,
                    float lr, float a, float b, float rep, int spectral_n_iter, unsigned int seed,
                    int index_offset, int optimizer_mode, float* out) {
  fe::clear_error();
  if (idx == nullptr || dist == nullptr || out == nullptr) {
    set_error("null host pointer");
    return 1;
  }
  if (n < 2 || k < 1 || k > 256) {
    set_error("invalid host CUDA UMAP dimensions");
    return 1;
  }
  return umap_fused_impl(idx, dist, dist_double, false, n, k, n_epochs, nsr, lr, a, b, rep, spectral_n_iter,
                         seed, index_offset, optimizer_mode, false, out);
}

}  // namespace

extern "C" {

const char* fe_b200_version(void) { return "fastembedr_b200 0.1.0 (sm_100a)"; }

int fe_b200_release_memory(void) {
  fe::clear_error();
  return fe::release_retained_memory();
}

bool fastembedr_cuda_available(void) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0) {
    cudaGetLastError();
    return false;
  }
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return major == 10;  // the library carries sm_100a code only
}

const char* fastembedr_cuda_embedding_last_error(void) { return fe::last_error(); }

int fastembedr_cuda_opentsne_fft_from_knn(const int* indices, const double* distances,
                                          const float* init, int has_init, int n, int k,
                                          int n_components, float perplexity,
                                          int early_exaggeration_iter, int n_iter,
                                          float early_exaggeration, float exaggeration,
                                          float learning_rate, int learning_rate_auto,
                                          float initial_momentum, float final_momentum,
                                          float min_gain, float max_step_norm, unsigned int seed,
                                          int index_offset, float* out) {
  return opentsne_impl(indices, distances, true, init, has_init, n, k, n_components, perplexity,
                       early_exaggeration_iter, n_iter, early_exaggeration, exaggeration,
                       learning_rate, learning_rate_auto, initial_momentum, final_momentum,
                       min_gain, max_step_norm, seed, index_offset, out, false);
}

int fastembedr_cuda_opentsne_fft_from_knn_float(const int* indices, const float* distances,
                                                const float* init, int has_init, int n, int k,
                                                int n_components, float perplexity,
                                                int early_exaggeration_iter, int n_iter,
                                                float early_exaggeration, float exaggeration,
                                                float learning_rate, int learning_rate_auto,
                                                float initial_momentum, float final_momentum,
                                                float min_gain, float max_step_norm,
                                                unsigned int seed, int index_offset, float* out) {
  return opentsne_impl(indices, distances, false, init, has_init, n, k, n_components, perplexity,
                       early_exaggeration_iter, n_iter, early_exaggeration, exaggeration,
                       learning_rate, learning_rate_auto, initial_momentum, final_momentum,
                       min_gain, max_step_norm, seed, index_offset, out, false);
}

int fastembedr_cuda_opentsne_fft_from_device_knn_float(
    const int* indices, const float* distances, const float* init, int has_init, int n, int k,
    int n_components, float perplexity, int early_exaggeration_iter, int n_iter,
    float early_exaggeration, float exaggeration, float learning_rate, int learning_rate_auto,
    float initial_momentum, float final_momentum, float min_gain, float max_step_norm,
    unsigned int seed, int index_offset, float* out) {
  return opentsne_impl(indices, distances, false, init, has_init, n, k, n_components, perplexity,
                       early_exaggeration_iter, n_iter, early_exaggeration, exaggeration,
                       learning_rate, learning_rate_auto, initial_momentum, final_momentum,
                       min_gain, max_step_norm, seed, index_offset, out, true);
}

int fastembedr_cuda_opentsne_fft_from_device_knn_float_pca_double(
    const int* indices, const float* distances, const double* pca_init_values, int pca_init_p, int n, int k,
    int n_components, float perplexity, int early_exaggeration_iter, int n_iter, float early_exaggeration,
    float exaggeration, float learning_rate, int learning_rate_auto, float initial_momentum, float final_momentum,
    float min_gain, float max_step_norm, unsigned int seed, int index_offset, float* out) {
  if (pca_init_values == nullptr) {
    set_error("null pointer in device PCA initialization");
    return 1;
  }
  return opentsne_impl(indices, distances, false, nullptr, 0, n, k, n_components, perplexity,
                       early_exaggeration_iter, n_iter, early_exaggeration, exaggeration, learning_rate,
                       learning_rate_auto, initial_momentum, final_momentum, min_gain, max_step_norm, seed,
                       index_offset, out, true, pca_init_values, true, pca_init_p);
}

int fastembedr_cuda_opentsne_fft_from_device_knn_float_pca_float(
    const int* indices, const float* distances, const float* pca_init_values, int pca_init_p, int n, int k,
    int n_components, float perplexity, int early_exaggeration_iter, int n_iter, float early_exaggeration,
    float exaggeration, float learning_rate, int learning_rate_auto, float initial_momentum, float final_momentum,
    float min_gain, float max_step_norm, unsigned int seed, int index_offset, float* out) {
  if (pca_init_values == nullptr) {
    set_error("null pointer in device PCA initialization");
    return 1;
  }
  return opentsne_impl(indices, distances, false, nullptr, 0, n, k, n_components, perplexity,
                       early_exaggeration_iter, n_iter, early_exaggeration, exaggeration, learning_rate,
                       learning_rate_auto, initial_momentum, final_momentum, min_gain, max_step_norm, seed,
                       index_offset, out, true, pca_init_values, false, pca_init_p);
}

int fastembedr_cuda_umap_optimize_coo(const int* heads, const int* tails, const float* weights,
                                      const float* epochs_per_sample, const float* init, int n,
                                      int n_edges_capacity, int n_epochs, int negative_sample_rate,
                                      float learning_rate, float a, float b,
                                      float repulsion_strength, unsigned int seed,
                                      int optimizer_mode, float* out) {
  fe::clear_error();
  if (out == nullptr) {
    set_error("null host pointer");
    return 1;
  }
  FE_TRY(umap_validate(heads, tails, weights, epochs_per_sample, init, n, n_edges_capacity, n_epochs,
                       negative_sample_rate, learning_rate, repulsion_strength));
  const int mode = optimizer_mode == 1 ? fe::kUmapDelta : fe::kUmapInplace;
  return umap_host_run(heads, tails, epochs_per_sample, n_edges_capacity, init, out, n, 0, n_epochs,
                       n_epochs, negative_sample_rate, learning_rate, a, b, repulsion_strength, seed,
                       mode, umap_hash_key_default(), nullptr);
}

int fe_b200_umap_epochs(const int* heads, const int* tails, const float* epochs_per_sample,
                        long long n_edges, float* layout, int n, int epoch_begin, int epoch_end,
                        int n_epochs, int negative_sample_rate, float learning_rate, float a,
                        float b, float repulsion_strength, unsigned int seed, int optimizer_mode,
                        int hash_key_is_tail, long long* positive_samples) {
  fe::clear_error();
  FE_TRY(umap_validate(heads, tails, epochs_per_sample, epochs_per_sample, layout, n, n_edges,
                       n_epochs, negative_sample_rate, learning_rate, repulsion_strength));
  if (epoch_begin < 0 || epoch_end < epoch_begin || epoch_end > n_epochs) {
    set_error("invalid epoch range");
    return 1;
  }
  const int mode = optimizer_mode == 1 ? fe::kUmapDelta : fe::kUmapInplace;
  return umap_host_run(heads, tails, epochs_per_sample, n_edges, layout, layout, n, epoch_begin,
                       epoch_end, n_epochs, negative_sample_rate, learning_rate, a, b,
                       repulsion_strength, seed, mode, hash_key_is_tail, positive_samples);
}

// ---------------------------------------------------------------- t-SNE sessions

int fe_b200_tsne_create(const int* indices, const float* distances, int n, int k, int index_offset,
                        float perplexity, const float* init, unsigned int seed, int grid_size,
                        int inputs_on_device, fe_b200_tsne** out) {
  fe::clear_error();
  if (out == nullptr || indices == nullptr || distances == nullptr) {
    set_error("null CUDA openTSNE input pointer");
    return 1;
  }
  *out = nullptr;
  if (n < 2 || k < 1 || k > 256 || !(perplexity > 0.0f)) {
    set_error("invalid CUDA openTSNE FFT-grid dimensions or parameters");
    return 1;
  }
  cudaStream_t stream = nullptr;
  FE_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate(session)");
  int* row_ptr = nullptr;
  int* col = nullptr;
  float* val = nullptr;
  long long nnz = 0;
  int rc = 0;
  {
    DeviceCopy d_idx, d_dist;
    const int* idx_dev = indices;
    const float* dist_dev = distances;
    const size_t items = static_cast<size_t>(n) * k;
    if (!inputs_on_device) {
      rc = copy_to_device(indices, items * sizeof(int), d_idx, stream, "H2D indices");
      if (rc == 0) rc = copy_to_device(distances, items * sizeof(float), d_dist, stream, "H2D distances");
      idx_dev = static_cast<const int*>(d_idx.p);
      dist_dev = static_cast<const float*>(d_dist.p);
    }
    if (rc == 0) {
      rc = fe::build_p_device(idx_dev, dist_dev, false, n, k, index_offset, perplexity, stream, &row_ptr,
                              &col, &val, &nnz);
    }
  }
  fe::TsneSession* s = nullptr;
  if (rc == 0) rc = fe::session_create(&s, n, resolve_grid(n, grid_size), row_ptr, col, val, nnz, nullptr);
  if (rc != 0) {
    if (s == nullptr) {
      if (row_ptr) fe::dev_free(row_ptr);
      if (col) fe::dev_free(col);
      if (val) fe::dev_free(val);
    }
    cudaStreamDestroy(stream);
    return 1;
  }
  cudaStreamSynchronize(stream);
  cudaStreamDestroy(stream);
  rc = init != nullptr ? fe::session_set_layout(s, init, !inputs_on_device, true)
                       : fe::session_random_layout(s, seed);
  if (rc != 0) {
    fe::session_destroy(s);
    return 1;
  }
  *out = new fe_b200_tsne{s};
  return 0;
}

int fe_b200_tsne_create_csr(const int* row_ptr, const int* col, const float* val, int n,
                            const float* init, int grid_size, fe_b200_tsne** out) {
  fe::clear_error();
  if (out == nullptr || row_ptr == nullptr || col == nullptr || val == nullptr || init == nullptr || n < 2) {
    set_error("invalid CSR session arguments");
    return 1;
  }
  *out = nullptr;
  int* d_rp = nullptr;
  int* d_col = nullptr;
  float* d_val = nullptr;
  long long nnz = 0;
  FE_TRY(fe::upload_csr(row_ptr, col, val, n, nullptr, &d_rp, &d_col, &d_val, &nnz));
  fe::TsneSession* s = nullptr;
  if (fe::session_create(&s, n, resolve_grid(n, grid_size), d_rp, d_col, d_val, nnz, nullptr)) {
    fe::dev_free(d_rp);
    fe::dev_free(d_col);
    fe::dev_free(d_val);
    return 1;
  }
  if (fe::session_set_layout(s, init, true, true)) {
    fe::session_destroy(s);
    return 1;
  }
  *out = new fe_b200_tsne{s};
  return 0;
}

int fe_b200_tsne_iterate(fe_b200_tsne* h, int n_iter, float exaggeration, float momentum,
                         float learning_rate, float min_gain, float max_step_norm) {
  fe::clear_error();
  if (h == nullptr || n_iter < 0) {
    set_error("invalid t-SNE session call");
    return 1;
  }
  return fe::session_iterate(h->impl, n_iter, exaggeration, momentum, learning_rate, min_gain, max_step_norm);
}

int fe_b200_tsne_prepare(fe_b200_tsne* h, float exaggeration, float momentum, float learning_rate,
                         float min_gain, float max_step_norm) {
  fe::clear_error();
  if (h == nullptr) {
    set_error("invalid t-SNE session call");
    return 1;
  }
  return fe::session_prepare(h->impl, exaggeration, momentum, learning_rate, min_gain, max_step_norm);
}

int fe_b200_tsne_gradient(fe_b200_tsne* h, float exaggeration, float* grad, double* z) {
  fe::clear_error();
  if (h == nullptr || grad == nullptr) {
    set_error("invalid t-SNE session call");
    return 1;
  }
  return fe::session_gradient(h->impl, exaggeration, grad, z);
}

int fe_b200_tsne_get_layout(fe_b200_tsne* h, float* out, int on_device) {
  fe::clear_error();
  if (h == nullptr || out == nullptr) {
    set_error("invalid t-SNE session call");
    return 1;
  }
  return fe::session_get_layout(h->impl, out, on_device == 0);
}

int fe_b200_tsne_set_layout(fe_b200_tsne* h, const float* y, int on_device, int reset_state) {
  fe::clear_error();
  if (h == nullptr || y == nullptr) {
    set_error("invalid t-SNE session call");
    return 1;
  }
  FE_TRY(fe::session_set_layout(h->impl, y, on_device == 0, true));
  return reset_state ? fe::session_reset_state(h->impl) : 0;
}

int fe_b200_tsne_get_state(fe_b200_tsne* h, float* update, float* gains) {
  fe::clear_error();
  if (h == nullptr || update == nullptr || gains == nullptr) {
    set_error("invalid t-SNE session call");
    return 1;
  }
  return fe::session_get_state(h->impl, update, gains, true);
}

int fe_b200_tsne_set_state(fe_b200_tsne* h, const float* update, const float* gains) {
  fe::clear_error();
  if (h == nullptr || update == nullptr || gains == nullptr) {
    set_error("invalid t-SNE session call");
    return 1;
  }
  return fe::session_set_state(h->impl, update, gains, true);
}

int fe_b200_tsne_info(fe_b200_tsne* h, int* n, int* grid, long long* nnz, long long* nnz_padded) {
  if (h == nullptr) {
    set_error("invalid t-SNE session call");
    return 1;
  }
  if (n) *n = h->impl->n;
  if (grid) *grid = h->impl->grid;
  if (nnz) *nnz = h->impl->nnz;
  if (nnz_padded) *nnz_padded = 4 * h->impl->csr4_groups;
  return 0;
}

int fe_b200_tsne_get_p(fe_b200_tsne* h, int* row_ptr, int* col, float* val) {
  fe::clear_error();
  if (h == nullptr || row_ptr == nullptr || col == nullptr || val == nullptr) {
    set_error("invalid t-SNE session call");
    return 1;
  }
  return fe::session_get_p(h->impl, row_ptr, col, val);
}

int fe_b200_tsne_staged_blocks(fe_b200_tsne* h, int* staged, int* blocks) {
  fe::clear_error();
  if (h == nullptr || staged == nullptr || blocks == nullptr) {
    set_error("invalid t-SNE session call");
    return 1;
  }
  fe::TsneSession* s = h->impl;
  const int rows = std::max(0, s->row_end - s->row_begin);
  *blocks = (rows + fe::kStageRows - 1) / fe::kStageRows;
  unsigned int count = 0;
  if (s->stage_enabled) {
    FE_CUDA(cudaMemcpyAsync(&count, &s->stats->stage_count, sizeof(count), cudaMemcpyDeviceToHost, s->stream),
            "D2H staged blocks");
    FE_CUDA(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize(staged blocks)");
  }
  *staged = static_cast<int>(count);
  return 0;
}

int fe_b200_tsne_set_interpolation(fe_b200_tsne* h, int mode) {
  fe::clear_error();
  if (h == nullptr) {
    set_error("invalid t-SNE session call");
    return 1;
  }
  return fe::session_set_interpolation(h->impl, mode);
}

int fe_b200_knn_exact(const void* data, int data_double, int data_on_device, int n, int p, int k, int exclude_self,
                      int* d_indices, float* d_distances) {
  fe::clear_error();
  cudaStream_t st = nullptr;
  FE_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "cudaStreamCreate(KNN)");
  const int rc = fe::knn_exact(data, data_double != 0, data_on_device != 0, true, n, p, k, exclude_self != 0,
                               d_indices, d_distances, st);
  cudaStreamSynchronize(st);
  cudaStreamDestroy(st);
  return rc;
}

int fe_b200_pca_start(const void* values, int values_double, int n, int p, float* out) {
  fe::clear_error();
  if (values == nullptr || out == nullptr || n < 2 || p < 2) {
    set_error("invalid dimensions in device PCA initialization");
    return 1;
  }
  cudaStream_t st = nullptr;
  FE_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "cudaStreamCreate(PCA)");
  float2* d = nullptr;
  int rc = fe::check_cuda(fe::dev_malloc(&d, sizeof(float2) * static_cast<size_t>(n)), "cudaMalloc(PCA start)");
  if (rc == 0) rc = fe::pca_start_layout(values, values_double != 0, n, p, st, d);
  if (rc == 0) {
    rc = fe::check_cuda(cudaMemcpyAsync(out, d, sizeof(float2) * static_cast<size_t>(n), cudaMemcpyDeviceToHost, st),
                        "D2H PCA start");
  }
  if (rc == 0) rc = fe::check_cuda(cudaStreamSynchronize(st), "cudaStreamSynchronize(PCA start)");
  cudaStreamSynchronize(st);
  if (d != nullptr) fe::dev_free(d);
  cudaStreamDestroy(st);
  return rc;
}

void* fe_b200_tsne_stream(fe_b200_tsne* h) { return h == nullptr ? nullptr : h->impl->stream; }

int fe_b200_tsne_profile(fe_b200_tsne* h, int enable) {
  if (h == nullptr) return 1;
  h->impl->profile = enable != 0;
  for (int k = 0; k < fe::kKindCount; ++k) {
    h->impl->kernel_ms[k] = 0.0;
    h->impl->kernel_launches[k] = 0;
  }
  return 0;
}

int fe_b200_tsne_kernel_times(fe_b200_tsne* h, double* ms, long long* launches, int kinds) {
  if (h == nullptr) return 1;
  for (int k = 0; k < kinds && k < fe::kKindCount; ++k) {
    if (ms) ms[k] = h->impl->kernel_ms[k];
    if (launches) launches[k] = h->impl->kernel_launches[k];
  }
  return 0;
}

const char* fe_b200_tsne_kernel_name(int kind) { return fe::kernel_kind_name(kind); }

void fe_b200_tsne_destroy(fe_b200_tsne* h) {
  if (h == nullptr) return;
  fe::session_destroy(h->impl);
  delete h;
}

int fe_b200_nccl_unique_id(unsigned char* id, int id_bytes) {
  fe::clear_error();
  if (id == nullptr || id_bytes < static_cast<int>(sizeof(ncclUniqueId))) {
    set_error("fe_b200_nccl_unique_id: need a buffer of at least 128 bytes");
    return 1;
  }
  const fe::NcclApi* api = fe::nccl_api();
  if (api == nullptr) return 1;
  ncclUniqueId uid;
  FE_TRY(fe::check_nccl(api->GetUniqueId(&uid), "ncclGetUniqueId"));
  std::memcpy(id, &uid, sizeof(uid));
  return 0;
}

int fe_b200_tsne_shard(fe_b200_tsne* h, const unsigned char* id, int id_bytes, int nranks, int rank) {
  fe::clear_error();
  if (h == nullptr || id == nullptr || id_bytes < static_cast<int>(sizeof(ncclUniqueId))) {
    set_error("invalid t-SNE shard call");
    return 1;
  }
  return fe::session_shard(h->impl, id, nullptr, nranks, rank);
}

int fe_b200_comm_create(const unsigned char* id, int id_bytes, int nranks, int rank, fe_b200_comm** out) {
  fe::clear_error();
  if (out == nullptr || id == nullptr || id_bytes < static_cast<int>(sizeof(ncclUniqueId))) {
    set_error("invalid communicator call");
    return 1;
  }
  *out = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks) {
    set_error("communicator: need nranks >= 1 and 0 <= rank < nranks");
    return 1;
  }
  fe_b200_comm* c = new fe_b200_comm();
  if (fe::comm_init(id, nranks, rank, &c->comm)) {
    delete c;
    return 1;
  }
  c->nranks = nranks;
  c->rank = rank;
  *out = c;
  return 0;
}

void fe_b200_comm_destroy(fe_b200_comm* c) {
  if (c == nullptr) return;
  const fe::NcclApi* api = fe::nccl_api();
  if (api != nullptr && c->comm != nullptr) api->CommDestroy(c->comm);
  delete c;
}

int fe_b200_tsne_shard_comm(fe_b200_tsne* h, fe_b200_comm* comm) {
  fe::clear_error();
  if (h == nullptr || comm == nullptr || comm->comm == nullptr) {
    set_error("invalid t-SNE shard call");
    return 1;
  }
  return fe::session_shard(h->impl, nullptr, comm->comm, comm->nranks, comm->rank);
}

// ---------------------------------------------------------------- UMAP from KNN (device graph)

int fastembedr_cuda_umap_from_knn_spectral(const int* indices, const double* distances, int n, int k,
                                           int n_epochs, int negative_sample_rate, float learning_rate,
                                           float a, float b, float repulsion_strength, int spectral_n_iter,
                                           unsigned int seed, int index_offset, int optimizer_mode,
                                           float* out) {
  return umap_fused_host(indices, distances, true, n, k, n_epochs, negative_sample_rate, learning_rate, a, b,
                         repulsion_strength, spectral_n_iter, seed, index_offset, optimizer_mode, out);
}

int fastembedr_cuda_umap_from_knn_spectral_float(const int* indices, const float* distances, int n, int k,
                                                 int n_epochs, int negative_sample_rate, float learning_rate,
                                                 float a, float b, float repulsion_strength,
                                                 int spectral_n_iter, unsigned int seed, int index_offset,
                                                 int optimizer_mode, float* out) {
  return umap_fused_host(indices, distances, false, n, k, n_epochs, negative_sample_rate, learning_rate, a, b,
                         repulsion_strength, spectral_n_iter, seed, index_offset, optimizer_mode, out);
}

int fastembedr_cuda_umap_from_device_knn_spectral_float(const int* device_indices,
                                                        const float* device_distances, int n, int k,
                                                        int n_epochs, int negative_sample_rate,
                                                        float learning_rate, float a, float b,
                                                        float repulsion_strength, int spectral_n_iter,
                                                        unsigned int seed, int index_offset,
                                                        int optimizer_mode, int binary_graph, float* out) {
  fe::clear_error();
  if (device_indices == nullptr || device_distances == nullptr || out == nullptr) {
    set_error("null device pointer");
    return 1;
  }
  if (n < 2 || k < 1 || k > 256) {
    set_error("invalid fused CUDA UMAP dimensions or parameters");
    return 1;
  }
  return umap_fused_impl(device_indices, device_distances, false, true, n, k, n_epochs, negative_sample_rate,
                         learning_rate, a, b, repulsion_strength, spectral_n_iter, seed, index_offset,
                         optimizer_mode, binary_graph != 0, out);
}

// fastembedr_cuda_umap_graph_dump_from_knn_impl (src/embedding_cuda_kernels.cpp:4804-4948):
// the device graph as a rank-major COO list; the caller's buffers hold n * width entries.
int fastembedr_cuda_umap_graph_dump_from_knn(const int* indices, const double* distances, int n, int k,
                                             int index_offset, int* out_heads, int* out_tails,
                                             float* out_weights, float* out_epochs_per_sample, int* out_width,
                                             int* out_capacity) {
  fe::clear_error();
  if (indices == nullptr || distances == nullptr || out_heads == nullptr || out_tails == nullptr ||
      out_weights == nullptr || out_epochs_per_sample == nullptr || out_width == nullptr ||
      out_capacity == nullptr) {
    set_error("null host pointer");
    return 1;
  }
  if (n < 2 || k < 1 || k > 256) {
    set_error("invalid CUDA UMAP graph dump dimensions");
    return 1;
  }
  FE_TRY(fe::memory_preflight(umap_graph_bytes(n, k) + static_cast<size_t>(n) * k * 12,
                              "CUDA UMAP graph dump allocation preflight"));
  cudaStream_t stream = nullptr;
  FE_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate(umap graph dump)");
  struct StreamGuard {
    cudaStream_t s;
    ~StreamGuard() {
      cudaStreamSynchronize(s);
      cudaStreamDestroy(s);
    }
  } guard{stream};
  fe::UmapDenseGraph g;
  {
    DeviceCopy d_idx, d_dist;
    const size_t items = static_cast<size_t>(n) * k;
    FE_TRY(copy_to_device(indices, items * sizeof(int), d_idx, stream, "H2D umap dump indices"));
    FE_TRY(copy_to_device(distances, items * sizeof(double), d_dist, stream, "H2D umap dump distances"));
    FE_TRY(fe::umap_graph_build(static_cast<const int*>(d_idx.p), d_dist.p, true, n, k, index_offset, false,
                                stream, &g));
  }
  const size_t slots = static_cast<size_t>(n) * g.width;
  fe::Arena arena;
  int* heads = nullptr;
  int* tails = nullptr;
  float* weights = nullptr;
  float* periods = nullptr;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 0) arena.begin_plan();
    else arena.rewind();
    heads = arena.take<int>(slots);
    tails = arena.take<int>(slots);
    weights = arena.take<float>(slots);
    periods = arena.take<float>(slots);
    if (pass == 0) FE_TRY(arena.commit("UMAP graph dump workspace"));
  }
  long long n_edges = 0;
  FE_TRY(fe::umap_graph_pack(g, true, heads, tails, weights, periods, &n_edges, stream));
  if (n_edges < 1 || n_edges > static_cast<long long>(slots)) {
    set_error("invalid CUDA UMAP graph edge count");
    return 1;
  }
  const size_t e = static_cast<size_t>(n_edges);
  FE_CUDA(cudaMemcpyAsync(out_heads, heads, e * sizeof(int), cudaMemcpyDeviceToHost, stream), "D2H dump heads");
  FE_CUDA(cudaMemcpyAsync(out_tails, tails, e * sizeof(int), cudaMemcpyDeviceToHost, stream), "D2H dump tails");
  FE_CUDA(cudaMemcpyAsync(out_weights, weights, e * sizeof(float), cudaMemcpyDeviceToHost, stream),
          "D2H dump weights");
  FE_CUDA(cudaMemcpyAsync(out_epochs_per_sample, periods, e * sizeof(float), cudaMemcpyDeviceToHost, stream),
          "D2H dump epochs_per_sample");
  FE_CUDA(cudaStreamSynchronize(stream), "cudaStreamSynchronize(umap graph dump)");
  *out_width = g.width;
  *out_capacity = static_cast<int>(n_edges);
  return 0;
}

// ---------------------------------------------------------------- out-of-scope symbols

int fastembedr_cuda_embed(const int*, const float*, const float*, int, int, int, int, int, float,
                          float, float, float, unsigned int, float*) {
  return out_of_scope("fastembedr_cuda_embed");
}
int fastembedr_cuda_embed_from_knn(const int*, const double*, const float*, int, int, int, int, int,
                                   float, float, float, unsigned int, int, float*) {
  return out_of_scope("fastembedr_cuda_embed_from_knn");
}
int fastembedr_cuda_spectral_init_from_knn(const int*, const double*, int, int, int, unsigned int,
                                           int, float*) {
  return out_of_scope("fastembedr_cuda_spectral_init_from_knn");
}
int fastembedr_cuda_exact_tsne_from_knn(const int*, const double*, const float*, int, int, int,
                                        float, float, int, int, float, float, float, unsigned int,
                                        int, float*) {
  return out_of_scope("fastembedr_cuda_exact_tsne_from_knn");
}
int fastembedr_cuda_landmark_tsne_from_device_knn(
    const int* device_indices, const float* device_distances, int index_offset, const float* reference_data,
    const float* query_data, const float* reference_layout, int n_reference, int n_query, int n_features, int k,
    float perplexity, int n_iter, int early_exaggeration_iter, float learning_rate, float early_exaggeration,
    float exaggeration, float initial_momentum, float final_momentum, float max_grad_norm, float max_step_norm,
    int n_negatives, int exact_repulsion_threshold, unsigned int seed, int affine_neighbors, float affine_ridge,
    float max_extrapolation, float* out) {
  return fe::landmark_tsne(device_indices, device_distances, index_offset, reference_data, query_data,
                           reference_layout, n_reference, n_query, n_features, k, perplexity, n_iter,
                           early_exaggeration_iter, learning_rate, early_exaggeration, exaggeration,
                           initial_momentum, final_momentum, max_grad_norm, max_step_norm, n_negatives,
                           exact_repulsion_threshold, seed, affine_neighbors, affine_ridge, max_extrapolation, out);
}
int fastembedr_cuda_landmark_umap_from_device_knn(const int*, const float*, int, const float*,
                                                  const float*, const float*, const int*, const int*,
                                                  int, int, int, int, int, int, int, float, float,
                                                  float, float, unsigned int, int, float, float,
                                                  float*) {
  return out_of_scope("fastembedr_cuda_landmark_umap_from_device_knn");
}
int fastembedr_cuda_standardize_matrix(const double*, int, int, double*, double*, double*) {
  return out_of_scope("fastembedr_cuda_standardize_matrix");
}
int fastembedr_cuda_project_embedding(const double*, const int*, const double*, int, int, int, int,
                                      double*) {
  return out_of_scope("fastembedr_cuda_project_embedding");
}
int fastembedr_cuda_interpolate_landmark_layout(const double*, const int*, const int*, const double*,
                                                int, int, int, int, double*) {
  return out_of_scope("fastembedr_cuda_interpolate_landmark_layout");
}
int fastembedr_cuda_landmark_project_interpolate_knn_confidence(const double*, const double*,
                                                                const double*, const int*, int, int,
                                                                int, int, int, double*, int*,
                                                                double*, double*) {
  return out_of_scope("fastembedr_cuda_landmark_project_interpolate_knn_confidence");
}
int fastembedr_cuda_knn_structure_score(const double*, const int*, const int*, const int*, int, int,
                                        int, int, int, int, int, double*) {
  return out_of_scope("fastembedr_cuda_knn_structure_score");
}
int fastembedr_cuda_silhouette_score(const double*, const int*, const int*, int, int, double*) {
  return out_of_scope("fastembedr_cuda_silhouette_score");
}
int fastembedr_cuda_matrix_multiply(const double*, const double*, int, int, int, int, double*) {
  return out_of_scope("fastembedr_cuda_matrix_multiply");
}
int fastembedr_cuda_raft_tsvd_pca_init(const double*, int, int, int, float*) {
  return out_of_scope("fastembedr_cuda_raft_tsvd_pca_init");
}

}  // extern "C"
