// Harness around the reference's own CPU openTSNE implementation.
//
// TEST INFRASTRUCTURE ONLY (checker + CPU baseline, never the product).
// This translation unit #includes the reference source file
// src/tsne_neighbors.cpp from where it lies (path passed as FE_REF_TSNE_SRC
// by oracle/Makefile), compiled against the Rcpp stand-in in
// oracle/rcpp_shim/Rcpp.h, and exports plain C entry points for ctypes.
// The wrapped functions are the reference's anonymous-namespace routines:
//   build_tsne_probabilities_float     tsne_neighbors.cpp:540-648
//   compute_gradient_fft_grid_f        tsne_neighbors.cpp:1076-1182
//   compute_gradient_pair_symmetric_f  tsne_neighbors.cpp:1014-1074
//   apply_open_tsne_update_f           tsne_neighbors.cpp:1200-1245
//   zero_mean_f                        tsne_neighbors.cpp:1196-1207
//   evaluate_kl_f                      tsne_neighbors.cpp:1247-1276
//   knn_tsne_opentsne_float_cpp        tsne_neighbors.cpp:1621-1857
#include "Rcpp.h"

#include FE_REF_TSNE_SRC

#include <chrono>
#include <cstdlib>
#include <string>

namespace {

thread_local std::string g_tsne_error;

struct PHandle {
  SparseProbabilitiesF p;
};

SparseProbabilitiesF p_from_arrays(const int* row_ptr, const int* col, const float* val, int n) {
  SparseProbabilitiesF p;
  p.row_ptr.assign(row_ptr, row_ptr + n + 1);
  const std::size_t nnz = static_cast<std::size_t>(row_ptr[n]);
  p.col.assign(col, col + nnz);
  p.val.assign(val, val + nnz);
  return p;
}

// Set FASTEMBEDR_TSNE_FFT_GRID for the duration of one call (0 = leave as is).
struct GridOverride {
  bool active = false;
  std::string saved;
  bool had = false;
  explicit GridOverride(int grid) {
    if (grid <= 0) return;
    const char* old = std::getenv("FASTEMBEDR_TSNE_FFT_GRID");
    had = old != nullptr;
    if (had) saved = old;
    setenv("FASTEMBEDR_TSNE_FFT_GRID", std::to_string(grid).c_str(), 1);
    active = true;
  }
  ~GridOverride() {
    if (!active) return;
    if (had) setenv("FASTEMBEDR_TSNE_FFT_GRID", saved.c_str(), 1);
    else unsetenv("FASTEMBEDR_TSNE_FFT_GRID");
  }
};

template <typename F>
int guarded(F&& fn) {
  try {
    fn();
    rshim::collect();
    return 0;
  } catch (const std::exception& e) {
    g_tsne_error = e.what();
    rshim::collect();
    return 1;
  }
}

}  // namespace

extern "C" {

const char* feref_tsne_last_error() { return g_tsne_error.c_str(); }

int feref_tsne_grid_size(int n, int grid_override) {
  GridOverride guard(grid_override);
  return tsne_fft_grid_size(n);
}

// Column-major KNN (R layout, idx[j*n+i]); indices 0- or 1-based (auto).
void* feref_tsne_p_build(const int* idx_cm, const float* dist_cm, int n, int k,
                         double perplexity, int threads) {
  PHandle* h = nullptr;
  const int rc = guarded([&]() {
    IntegerMatrix indices = rshim::int_matrix(idx_cm, n, k);
    std::vector<float> dist(static_cast<std::size_t>(n) * k);
    for (int i = 0; i < n; ++i) {
      for (int j = 0; j < k; ++j) {
        dist[static_cast<std::size_t>(i) * k + j] = dist_cm[static_cast<std::size_t>(j) * n + i];
      }
    }
    const int t = resolve_threads(threads, n);
    ParallelExecutor executor(t);
    ParallelExecutorScope scope(&executor);
    h = new PHandle();
    h->p = build_tsne_probabilities_float(indices, dist, perplexity, t);
  });
  if (rc != 0) {
    delete h;
    return nullptr;
  }
  return h;
}

long long feref_tsne_p_nnz(void* handle) {
  return static_cast<long long>(static_cast<PHandle*>(handle)->p.col.size());
}

void feref_tsne_p_copy(void* handle, int* row_ptr, int* col, float* val) {
  const SparseProbabilitiesF& p = static_cast<PHandle*>(handle)->p;
  std::copy(p.row_ptr.begin(), p.row_ptr.end(), row_ptr);
  std::copy(p.col.begin(), p.col.end(), col);
  std::copy(p.val.begin(), p.val.end(), val);
}

void feref_tsne_p_free(void* handle) { delete static_cast<PHandle*>(handle); }

// Full openTSNE gradient (bilinear FFT-grid repulsion + sparse attraction) at y.
int feref_tsne_gradient_fft(const int* row_ptr, const int* col, const float* val, int n,
                            const float* y, float exaggeration, int threads, int grid_override,
                            float* grad_out) {
  return guarded([&]() {
    GridOverride guard(grid_override);
    SparseProbabilitiesF p = p_from_arrays(row_ptr, col, val, n);
    std::vector<float> yy(y, y + static_cast<std::size_t>(n) * 2u);
    std::vector<float> grad(yy.size(), 0.0f);
    const int t = resolve_threads(threads, n);
    ParallelExecutor executor(t);
    ParallelExecutorScope scope(&executor);
    FftGridWorkspaceT<float> ws;
    compute_gradient_fft_grid_f(p, yy, n, 2, exaggeration, t, &ws, grad);
    std::copy(grad.begin(), grad.end(), grad_out);
  });
}

// Exact O(N^2) repulsion + sparse attraction at y.
int feref_tsne_gradient_exact(const int* row_ptr, const int* col, const float* val, int n,
                              const float* y, float exaggeration, int threads, float* grad_out) {
  return guarded([&]() {
    SparseProbabilitiesF p = p_from_arrays(row_ptr, col, val, n);
    std::vector<float> yy(y, y + static_cast<std::size_t>(n) * 2u);
    std::vector<float> grad(yy.size(), 0.0f);
    const int t = resolve_threads(threads, n);
    ParallelExecutor executor(t);
    ParallelExecutorScope scope(&executor);
    compute_gradient_pair_symmetric_f(p, yy, n, 2, exaggeration, t, grad);
    std::copy(grad.begin(), grad.end(), grad_out);
  });
}

// Attractive part only (added onto grad_inout).
int feref_tsne_attractive(const int* row_ptr, const int* col, const float* val, int n,
                          const float* y, float exaggeration, int threads, float* grad_inout) {
  return guarded([&]() {
    SparseProbabilitiesF p = p_from_arrays(row_ptr, col, val, n);
    std::vector<float> yy(y, y + static_cast<std::size_t>(n) * 2u);
    std::vector<float> grad(grad_inout, grad_inout + yy.size());
    const int t = resolve_threads(threads, n);
    ParallelExecutor executor(t);
    ParallelExecutorScope scope(&executor);
    add_sparse_attractive_gradient_f(p, yy, n, 2, exaggeration, t, grad);
    std::copy(grad.begin(), grad.end(), grad_inout);
  });
}

// One optimizer update followed by re-centering (the per-iteration tail of
// run_phase, tsne_neighbors.cpp:1765-1771).
int feref_tsne_update(float* y, float* update, float* gains, const float* grad, int n,
                      float learning_rate, float momentum, float min_gain, float max_step_norm,
                      int threads) {
  return guarded([&]() {
    const std::size_t m = static_cast<std::size_t>(n) * 2u;
    std::vector<float> yy(y, y + m), uu(update, update + m), gg(gains, gains + m), gr(grad, grad + m);
    const int t = resolve_threads(threads, n);
    ParallelExecutor executor(t);
    ParallelExecutorScope scope(&executor);
    apply_open_tsne_update_f(yy, uu, gg, gr, n, 2, learning_rate, momentum, min_gain, max_step_norm, t);
    zero_mean_f(yy, n, 2);
    std::copy(yy.begin(), yy.end(), y);
    std::copy(uu.begin(), uu.end(), update);
    std::copy(gg.begin(), gg.end(), gains);
  });
}

// The reference's per-iteration loop body (run_phase, tsne_neighbors.cpp:1753-1771:
// compute_gradient_f -> apply_open_tsne_update_f -> zero_mean_f) for `iters`
// iterations with a persistent FFT workspace; *seconds receives the loop's
// wall time only (no argument marshalling).  The CPU baseline of bench.py.
int feref_tsne_iterate(const int* row_ptr, const int* col, const float* val, int n, float* y,
                       float* update, float* gains, int iters, float exaggeration, float momentum,
                       float learning_rate, float min_gain, float max_step_norm, int threads,
                       int grid_override, double* seconds) {
  return guarded([&]() {
    GridOverride guard(grid_override);
    SparseProbabilitiesF p = p_from_arrays(row_ptr, col, val, n);
    const std::size_t m = static_cast<std::size_t>(n) * 2u;
    std::vector<float> yy(y, y + m), uu(update, update + m), gg(gains, gains + m), grad(m, 0.0f);
    const int t = resolve_threads(threads, n);
    ParallelExecutor executor(t);
    ParallelExecutorScope scope(&executor);
    FftGridWorkspaceT<float> ws;
    const auto start = std::chrono::steady_clock::now();
    for (int it = 0; it < iters; ++it) {
      compute_gradient_f(p, yy, n, 2, exaggeration, t, "fft_grid", &ws, grad);
      apply_open_tsne_update_f(yy, uu, gg, grad, n, 2, learning_rate, momentum, min_gain,
                               max_step_norm, t);
      zero_mean_f(yy, n, 2);
    }
    const auto stop = std::chrono::steady_clock::now();
    *seconds = std::chrono::duration<double>(stop - start).count();
    std::copy(yy.begin(), yy.end(), y);
    std::copy(uu.begin(), uu.end(), update);
    std::copy(gg.begin(), gg.end(), gains);
  });
}

int feref_tsne_zero_mean(float* y, int n) {
  return guarded([&]() {
    const std::size_t m = static_cast<std::size_t>(n) * 2u;
    std::vector<float> yy(y, y + m);
    zero_mean_f(yy, n, 2);
    std::copy(yy.begin(), yy.end(), y);
  });
}

int feref_tsne_kl(const int* row_ptr, const int* col, const float* val, int n, const float* y,
                  int threads, double* kl_out) {
  return guarded([&]() {
    SparseProbabilitiesF p = p_from_arrays(row_ptr, col, val, n);
    std::vector<float> yy(y, y + static_cast<std::size_t>(n) * 2u);
    const int t = resolve_threads(threads, n);
    ParallelExecutor executor(t);
    ParallelExecutorScope scope(&executor);
    *kl_out = evaluate_kl_f(p, yy, n, 2, t);
  });
}

// Full CPU run through the reference's exported entry point.
// init: row-major float[n*2] or NULL (then the reference draws N(0,1e-4)).
int feref_tsne_run(const int* idx_cm, const float* dist_cm, int n, int k, const float* init,
                   double perplexity, int early_exaggeration_iter, int n_iter,
                   double early_exaggeration, double exaggeration, double learning_rate,
                   int learning_rate_auto, double initial_momentum, double final_momentum,
                   double min_gain, double max_step_norm, int threads, int seed, int grid_override,
                   float* out_rowmajor) {
  return guarded([&]() {
    GridOverride guard(grid_override);
    IntegerMatrix indices = rshim::int_matrix(idx_cm, n, k);
    SEXP distances = rshim::float32_matrix(dist_cm, n, k);
    NumericMatrix y_init(n, 2);
    if (init != nullptr) {
      for (int i = 0; i < n; ++i) {
        y_init(i, 0) = static_cast<double>(init[2 * static_cast<std::size_t>(i)]);
        y_init(i, 1) = static_cast<double>(init[2 * static_cast<std::size_t>(i) + 1]);
      }
    }
    List res = knn_tsne_opentsne_float_cpp(
      indices, distances, y_init, init != nullptr, 2, perplexity, 0.5,
      early_exaggeration_iter, n_iter, early_exaggeration, exaggeration, learning_rate,
      learning_rate_auto != 0, initial_momentum, final_momentum, min_gain, max_step_norm,
      "fft", threads, seed, false, false, false, 5000.0);
    NumericMatrix y(res["Y"]);
    for (int i = 0; i < n; ++i) {
      out_rowmajor[2 * static_cast<std::size_t>(i)] = static_cast<float>(y(i, 0));
      out_rowmajor[2 * static_cast<std::size_t>(i) + 1] = static_cast<float>(y(i, 1));
    }
  });
}

// tsne_auto_parameters_cpp (tsne_neighbors.cpp:1573-1618): perplexity,
// n_neighbors, early_exaggeration, learning_rate, ee_iter, n_iter.
int feref_tsne_auto_parameters(int n, int k, double perplexity, int perplexity_missing,
                               double* out6) {
  return guarded([&]() {
    List res = tsne_auto_parameters_cpp(n, k, perplexity, perplexity_missing != 0, "cpu", "fft");
    out6[0] = Rcpp::as<double>(res["perplexity"]);
    out6[1] = Rcpp::as<double>(res["n_neighbors"]);
    out6[2] = Rcpp::as<double>(res["early_exaggeration"]);
    out6[3] = Rcpp::as<double>(res["learning_rate"]);
    out6[4] = Rcpp::as<double>(res["early_exaggeration_iter"]);
    out6[5] = Rcpp::as<double>(res["n_iter"]);
  });
}

}  // extern "C"
