// Harness around the reference's own CPU UMAP implementation.
//
// TEST INFRASTRUCTURE ONLY (checker + CPU baseline, never the product).
// This translation unit #includes the reference source file
// src/fast_knn_umap.cpp from where it lies (path passed as FE_REF_UMAP_SRC by
// oracle/Makefile), compiled against oracle/rcpp_shim/Rcpp.h, and exports
// plain C entry points for ctypes.  Wrapped reference routines:
//   umap_graph_csr_float_cpp             fast_knn_umap.cpp:3987-4042
//   fast_knn_umap_coo_replay_cpp         fast_knn_umap.cpp:4904-5056
//   fast_knn_umap_csr_init_cpp           fast_knn_umap.cpp:4538-4574
//   umap_powf_fast                       fast_knn_umap.cpp:179-206
//   positive/negative schedules          fast_knn_umap.cpp:595-636
//   deterministic_vertex_cuda_style      fast_knn_umap.cpp:535-547
//   find_ab_params                       fast_knn_umap.cpp:428-488
#include "Rcpp.h"

#include FE_REF_UMAP_SRC

#include <string>

namespace {

thread_local std::string g_umap_error;

struct GraphHandle {
  std::vector<int> offsets;
  std::vector<int> neighbors;
  std::vector<float> weights;
  std::vector<float> epochs_per_sample;
  float max_weight = 0.0f;
};

template <typename F>
int guarded_umap(F&& fn) {
  try {
    fn();
    rshim::collect();
    return 0;
  } catch (const std::exception& e) {
    g_umap_error = e.what();
    rshim::collect();
    return 1;
  }
}

NumericMatrix init_matrix(const float* init_rowmajor, int n) {
  NumericMatrix m(n, 2);
  for (int i = 0; i < n; ++i) {
    m(i, 0) = static_cast<double>(init_rowmajor[2 * static_cast<std::size_t>(i)]);
    m(i, 1) = static_cast<double>(init_rowmajor[2 * static_cast<std::size_t>(i) + 1]);
  }
  return m;
}

void copy_out(const NumericMatrix& y, int n, float* out_rowmajor) {
  for (int i = 0; i < n; ++i) {
    out_rowmajor[2 * static_cast<std::size_t>(i)] = static_cast<float>(y(i, 0));
    out_rowmajor[2 * static_cast<std::size_t>(i) + 1] = static_cast<float>(y(i, 1));
  }
}

std::vector<float> as_floats(SEXP x) {
  NumericVector v(x);
  return std::vector<float>(v.begin(), v.end());
}

}  // namespace

extern "C" {

const char* feref_umap_last_error() { return g_umap_error.c_str(); }

// Fuzzy-union CSR graph from column-major KNN (float32 distances).
void* feref_umap_graph(const int* idx_cm, const float* dist_cm, int n, int k, int threads) {
  GraphHandle* h = nullptr;
  const int rc = guarded_umap([&]() {
    IntegerMatrix indices = rshim::int_matrix(idx_cm, n, k);
    SEXP distances = rshim::float32_matrix(dist_cm, n, k);
    Rcpp::List g = umap_graph_csr_float_cpp(indices, distances, 0, k, k, threads);
    h = new GraphHandle();
    IntegerVector off(g["offsets"]);
    IntegerVector nb(g["neighbors"]);
    h->offsets.assign(off.begin(), off.end());
    h->neighbors.assign(nb.begin(), nb.end());
    h->weights = as_floats(g["weights"]);
    h->epochs_per_sample = as_floats(g["epochs_per_sample"]);
    h->max_weight = static_cast<float>(Rcpp::as<double>(g["max_weight"]));
  });
  if (rc != 0) {
    delete h;
    return nullptr;
  }
  return h;
}

long long feref_umap_graph_nnz(void* handle) {
  return static_cast<long long>(static_cast<GraphHandle*>(handle)->neighbors.size());
}

void feref_umap_graph_copy(void* handle, int* offsets, int* neighbors, float* weights,
                           float* epochs_per_sample, float* max_weight) {
  const GraphHandle* h = static_cast<GraphHandle*>(handle);
  std::copy(h->offsets.begin(), h->offsets.end(), offsets);
  std::copy(h->neighbors.begin(), h->neighbors.end(), neighbors);
  std::copy(h->weights.begin(), h->weights.end(), weights);
  std::copy(h->epochs_per_sample.begin(), h->epochs_per_sample.end(), epochs_per_sample);
  *max_weight = h->max_weight;
}

void feref_umap_graph_free(void* handle) { delete static_cast<GraphHandle*>(handle); }

// Replay of the CUDA COO schedule on the CPU (in-place; sequential when
// threads == 1).  min_dist selects a/b through find_ab_params(1, min_dist).
int feref_umap_coo_replay(const int* heads, const int* tails, const float* weights,
                          const float* epochs_per_sample, const float* init_rowmajor, int n,
                          int n_edges, int n_epochs, double min_dist, int negative_sample_rate,
                          double learning_rate, double repulsion_strength, int threads, int seed,
                          int sanitize_each_epoch, float* out_rowmajor) {
  return guarded_umap([&]() {
    IntegerVector h(heads, heads + n_edges);
    IntegerVector t(tails, tails + n_edges);
    SEXP w = rshim::float32_vector(weights, n_edges);
    SEXP e = rshim::float32_vector(epochs_per_sample, n_edges);
    NumericMatrix init = init_matrix(init_rowmajor, n);
    NumericMatrix y = fast_knn_umap_coo_replay_cpp(
      h, t, w, e, init, n_epochs, min_dist, negative_sample_rate, learning_rate,
      repulsion_strength, threads, seed, sanitize_each_epoch != 0, false);
    copy_out(y, n, out_rowmajor);
  });
}

// The reference CPU UMAP optimizer over a CSR graph (CPU backend of umap_knn).
int feref_umap_csr_optimize(const int* offsets, const int* neighbors, const float* weights,
                            const float* init_rowmajor, int n, int nnz, int n_epochs,
                            double min_dist, int negative_sample_rate, double learning_rate,
                            double repulsion_strength, int threads, int seed,
                            float* out_rowmajor) {
  return guarded_umap([&]() {
    IntegerVector off(offsets, offsets + n + 1);
    IntegerVector nb(neighbors, neighbors + nnz);
    SEXP w = rshim::float32_vector(weights, nnz);
    NumericMatrix init = init_matrix(init_rowmajor, n);
    NumericMatrix y = fast_knn_umap_csr_init_cpp(
      off, nb, w, init, n_epochs, min_dist, negative_sample_rate, learning_rate,
      repulsion_strength, threads, seed, false);
    copy_out(y, n, out_rowmajor);
  });
}

float feref_umap_powf(float x, float b) { return umap_powf_fast(x, b); }

int feref_umap_positive_samples(float period, int epoch) {
  return positive_samples_this_epoch_umap_schedule(period, epoch);
}

int feref_umap_negative_samples(float period, int negative_sample_rate, int epoch) {
  return negative_samples_this_epoch_umap_schedule(period, negative_sample_rate, epoch);
}

int feref_umap_negative_vertex(int n, int seed, int epoch, int head, long long edge, int sample) {
  return deterministic_vertex_cuda_style(n, seed, epoch, head, static_cast<std::size_t>(edge), sample);
}

void feref_find_ab(double spread, double min_dist, double* a, double* b) {
  const auto ab = find_ab_params(spread, min_dist);
  *a = ab.first;
  *b = ab.second;
}

}  // extern "C"
