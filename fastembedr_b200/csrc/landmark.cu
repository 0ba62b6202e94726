// openTSNE-style transform of query points against a fixed reference layout:
// the landmark t-SNE refinement behind fastembedr_cuda_landmark_tsne_from_device_knn
// (src/embedding_cuda_kernels.cpp:3496-3610; kernels :469-845).
//
// Per query point i, with its k reference neighbours (device KNN, column-major
// n_query x k, index_offset-based) and the reference layout Y fixed:
//   1. start: an affine projection of the query from its nearest m <= 12
//      reference neighbours (weighted ridge regression of the layout on the
//      data, displacement clamped to max_extrapolation times the
//      neighbourhood radius), falling back to a kernel-weighted mean
//      (landmark_affine_projection_kernel / landmark_affine_fallback, :504-725);
//   2. p_{j|i} over its k neighbours by a 200-step bisection on beta to the
//      perplexity (landmark_tsne_probabilities_kernel, :727-765);
//   3. early_exaggeration_iter + n_iter iterations of
//        grad = - sum_s q_s^2 (y_i - Y_s) / sum_s q_s + ex sum_j p_j q_j (y_i - Y_j)
//      over all reference points (exact repulsion) or n_negatives hashed
//      samples per iteration, the gradient clipped to max_grad_norm, then the
//      gains / momentum / step-clip update (landmark_tsne_epoch_kernel, :767-836).
//
// Queries never interact, so the B200 path runs every iteration of a query in
// one thread of ONE launch with its state in registers (the reference launches
// one kernel per iteration and round-trips the state through memory); with
// exact repulsion each block walks the reference layout in shared-memory
// tiles that all its threads read together.  The per-query arithmetic and its
// order follow the reference; the negative-sample hash and the reference's
// column-major inputs are kept as they are (parity of the sampled indices).
#include "tsne.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <string>

namespace fe {
namespace {

constexpr int kLandmarkMaxK = 128;     // kCudaProjectionMaxK, src/embedding_cuda_kernels.cpp:29
constexpr int kAffineMaxNeighbors = 12;
constexpr int kLandmarkThreads = 128;
constexpr int kRepulsionTile = 2048;   // reference points per shared-memory tile (16 KB)

struct LandmarkParams {
  int n_reference;
  int n_query;
  int k;
  int n_negatives;
  unsigned int seed;
  int exact;                 // repulsion over every reference point
  int early_iter;
  int total_iter;
  float learning_rate;
  float early_exaggeration;
  float exaggeration;
  float initial_momentum;
  float final_momentum;
  float max_grad_norm;
  float max_step_norm;
};

// Integer mixer and the per-(epoch, row, sample) reference draw of the
// reference (mix_uint :243-250, landmark_reference_sample :495-504): the same
// steps, so both pick the same negative samples.
__device__ __forceinline__ unsigned int mix32(unsigned int x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

__device__ __forceinline__ unsigned int reference_draw(unsigned int n, unsigned int seed, unsigned int epoch,
                                                       unsigned int row, unsigned int sample) {
  unsigned int x = seed;
  x ^= (epoch + 1u) * 0x9e3779b9u;
  x ^= (row + 1u) * 0x85ebca6bu;
  x ^= (sample + 1u) * 0xc2b2ae35u;
  return mix32(x) % n;
}

__device__ float median_in_place(float* v, int count) {
  for (int i = 1; i < count; ++i) {
    const float x = v[i];
    int j = i - 1;
    while (j >= 0 && v[j] > x) {
      v[j + 1] = v[j];
      --j;
    }
    v[j + 1] = x;
  }
  const int mid = count / 2;
  return (count & 1) ? v[mid] : 0.5f * (v[mid - 1] + v[mid]);
}

// Kernel-weighted mean of the valid neighbours' layout positions.
__device__ float2 weighted_mean_start(const float2* __restrict__ layout, const int* __restrict__ nbr,
                                      const float* __restrict__ dist, int n_reference, int n_query, int k,
                                      int index_offset, int row, float rho, float sigma) {
  constexpr float eps = 1.4901161193847656e-8f;
  float wsum = 0.0f;
  float2 v = make_float2(0.0f, 0.0f);
  for (int j = 0; j < k; ++j) {
    const size_t pos = static_cast<size_t>(j) * n_query + row;
    const int ref = nbr[pos] - index_offset;
    const float d = dist[pos];
    if (ref < 0 || ref >= n_reference || !isfinite(d) || d < 0.0f) continue;
    const float w = expf(-fmaxf(0.0f, d - rho) / fmaxf(sigma, eps));
    if (!isfinite(w) || w <= 0.0f) continue;
    wsum += w;
    const float2 y = layout[ref];
    v.x += w * y.x;
    v.y += w * y.y;
  }
  if (!isfinite(wsum) || wsum <= 0.0f) wsum = 1.0f;
  return make_float2(v.x / wsum, v.y / wsum);
}

// Step 1 (affine start), step 2 (calibration) and the optimizer state, one
// thread per query.
__global__ void __launch_bounds__(kLandmarkThreads) landmark_setup_kernel(
    const float* __restrict__ ref_data, const float* __restrict__ query_data, const float2* __restrict__ layout,
    const int* __restrict__ nbr, const float* __restrict__ dist, float* __restrict__ prob,
    float2* __restrict__ start, int n_reference, int n_query, int n_features, int k, int index_offset,
    int m_neighbors, float ridge, float max_extrapolation, float perplexity) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= n_query) return;
  constexpr float eps = 1.4901161193847656e-8f;

  // ---- calibration: beta bisection on squared distances (:727-765)
  {
    float beta = 1.0f, lo = -INFINITY, hi = INFINITY;
    float sum_p = FLT_MIN;
    const float target = logf(perplexity);
    for (int it = 0; it < 200; ++it) {
      sum_p = FLT_MIN;
      float ent = 0.0f;
      for (int j = 0; j < k; ++j) {
        const size_t pos = static_cast<size_t>(j) * n_query + row;
        const float d = dist[pos];
        const float d2 = d * d;
        const float p = expf(-beta * d2);
        prob[pos] = p;
        sum_p += p;
        ent += beta * d2 * p;
      }
      const float diff = ent / sum_p + logf(sum_p) - target;
      if (fabsf(diff) < 1.0e-5f) break;
      if (diff > 0.0f) {
        lo = beta;
        beta = isinf(hi) ? beta * 2.0f : 0.5f * (beta + hi);
      } else {
        hi = beta;
        beta = isinf(lo) ? beta * 0.5f : 0.5f * (beta + lo);
      }
    }
    const float inv = 1.0f / sum_p;
    for (int j = 0; j < k; ++j) prob[static_cast<size_t>(j) * n_query + row] *= inv;
  }

  // ---- affine start (:538-725)
  const int m = min(max(m_neighbors, 3), min(k, kAffineMaxNeighbors));
  float adjusted[kLandmarkMaxK];
  int zero_col = -1;
  float rho = INFINITY;
  for (int j = 0; j < k; ++j) {
    const size_t pos = static_cast<size_t>(j) * n_query + row;
    const int ref = nbr[pos] - index_offset;
    const float d = dist[pos];
    const bool valid = ref >= 0 && ref < n_reference && isfinite(d) && d >= 0.0f;
    adjusted[j] = valid ? d : INFINITY;
    if (valid && d <= eps && zero_col < 0) zero_col = j;
    if (valid) rho = fminf(rho, d);
  }
  if (!isfinite(rho)) rho = 0.0f;
  if (zero_col >= 0) {  // the query coincides with a reference point
    start[row] = layout[nbr[static_cast<size_t>(zero_col) * n_query + row] - index_offset];
    return;
  }
  // sigma: median of the positive rho-shifted distances
  float sigma;
  {
    float pos_d[kLandmarkMaxK];
    int count = 0;
    for (int j = 0; j < k; ++j) {
      const float a = fmaxf(0.0f, adjusted[j] - rho);
      if (isfinite(a) && a > eps) pos_d[count++] = a;
    }
    sigma = count > 0 ? median_in_place(pos_d, count) : fmaxf(rho, eps);
    if (!isfinite(sigma) || sigma < eps) sigma = eps;
  }
  int refs[kAffineMaxNeighbors];
  float w[kAffineMaxNeighbors];
  float wsum = 0.0f;
  for (int j = 0; j < m; ++j) {
    const int ref = nbr[static_cast<size_t>(j) * n_query + row] - index_offset;
    refs[j] = ref;
    const float a = fmaxf(0.0f, adjusted[j] - rho);
    const float wj = ref >= 0 && ref < n_reference && isfinite(a) ? expf(-a / sigma) : 0.0f;
    w[j] = wj;
    wsum += wj;
  }
  if (!isfinite(wsum) || wsum <= 0.0f) {
    start[row] = weighted_mean_start(layout, nbr, dist, n_reference, n_query, k, index_offset, row, rho, sigma);
    return;
  }
  for (int j = 0; j < m; ++j) w[j] /= wsum;
  float2 yc = make_float2(0.0f, 0.0f);
  for (int j = 0; j < m; ++j) {
    if (refs[j] < 0 || refs[j] >= n_reference) continue;
    const float2 y = layout[refs[j]];
    yc.x += w[j] * y.x;
    yc.y += w[j] * y.y;
  }
  float rhs[2 * kAffineMaxNeighbors];
  float norm[kAffineMaxNeighbors];
  float qv[kAffineMaxNeighbors];
  float gram[kAffineMaxNeighbors * kAffineMaxNeighbors];
  float radius_sq = 0.0f;
  for (int a = 0; a < m; ++a) {
    const bool ok = refs[a] >= 0 && refs[a] < n_reference;
    const float sw = sqrtf(fmaxf(w[a], 0.0f));
    const float2 y = ok ? layout[refs[a]] : make_float2(0.0f, 0.0f);
    const float d0 = ok ? y.x - yc.x : 0.0f;
    const float d1 = ok ? y.y - yc.y : 0.0f;
    rhs[2 * a] = sw * d0;
    rhs[2 * a + 1] = sw * d1;
    radius_sq = fmaxf(radius_sq, d0 * d0 + d1 * d1);
    norm[a] = 0.0f;
    qv[a] = 0.0f;
  }
  for (int i = 0; i < m * m; ++i) gram[i] = 0.0f;
  for (int f = 0; f < n_features; ++f) {
    const float* col = ref_data + static_cast<size_t>(f) * n_reference;
    float xc = 0.0f;
    for (int j = 0; j < m; ++j) {
      if (refs[j] >= 0 && refs[j] < n_reference) xc += w[j] * col[refs[j]];
    }
    const float qc = query_data[static_cast<size_t>(f) * n_query + row] - xc;
    float cen[kAffineMaxNeighbors];
    for (int a = 0; a < m; ++a) {
      const float v = refs[a] >= 0 && refs[a] < n_reference ? col[refs[a]] - xc : 0.0f;
      cen[a] = v;
      norm[a] += v * v;
      qv[a] += qc * v;
    }
    for (int a = 0; a < m; ++a) {
      for (int b = 0; b <= a; ++b) gram[a * m + b] += cen[a] * cen[b];
    }
  }
  float trace = 0.0f;
  for (int a = 0; a < m; ++a) {
    const float swa = sqrtf(fmaxf(w[a], 0.0f));
    trace += w[a] * norm[a];
    qv[a] *= swa;
    for (int b = 0; b <= a; ++b) {
      const float v = swa * sqrtf(fmaxf(w[b], 0.0f)) * gram[a * m + b];
      gram[a * m + b] = v;
      gram[b * m + a] = v;
    }
  }
  const float lambda = ridge * fmaxf(trace, eps) + eps;
  for (int a = 0; a < m; ++a) gram[a * m + a] += lambda;
  // Cholesky factor in the lower triangle, then two triangular solves per
  // layout coordinate.
  bool ok = true;
  for (int j = 0; j < m && ok; ++j) {
    float v = gram[j * m + j];
    for (int t = 0; t < j; ++t) v -= gram[j * m + t] * gram[j * m + t];
    if (!isfinite(v) || v <= eps) {
      ok = false;
      break;
    }
    const float diag = sqrtf(v);
    gram[j * m + j] = diag;
    for (int i = j + 1; i < m; ++i) {
      float s = gram[i * m + j];
      for (int t = 0; t < j; ++t) s -= gram[i * m + t] * gram[j * m + t];
      gram[i * m + j] = s / diag;
    }
  }
  if (!ok) {
    start[row] = weighted_mean_start(layout, nbr, dist, n_reference, n_query, k, index_offset, row, rho, sigma);
    return;
  }
  for (int c = 0; c < 2; ++c) {
    for (int i = 0; i < m; ++i) {
      float s = rhs[2 * i + c];
      for (int t = 0; t < i; ++t) s -= gram[i * m + t] * rhs[2 * t + c];
      rhs[2 * i + c] = s / gram[i * m + i];
    }
    for (int i = m - 1; i >= 0; --i) {
      float s = rhs[2 * i + c];
      for (int t = i + 1; t < m; ++t) s -= gram[t * m + i] * rhs[2 * t + c];
      rhs[2 * i + c] = s / gram[i * m + i];
    }
  }
  float2 disp = make_float2(0.0f, 0.0f);
  for (int a = 0; a < m; ++a) {
    disp.x += qv[a] * rhs[2 * a];
    disp.y += qv[a] * rhs[2 * a + 1];
  }
  const float max_disp = max_extrapolation * sqrtf(fmaxf(radius_sq, eps));
  const float disp_sq = disp.x * disp.x + disp.y * disp.y;
  if (disp_sq > max_disp * max_disp) {
    const float scale = max_disp / (sqrtf(disp_sq) + eps);
    disp.x *= scale;
    disp.y *= scale;
  }
  const float2 v = make_float2(yc.x + disp.x, yc.y + disp.y);
  start[row] = (isfinite(v.x) && isfinite(v.y))
                   ? v
                   : weighted_mean_start(layout, nbr, dist, n_reference, n_query, k, index_offset, row, rho, sigma);
}

__device__ __forceinline__ float q_of(float2 yi, float2 yr, float* dx, float* dy) {
  *dx = yi.x - yr.x;
  *dy = yi.y - yr.y;
  return 1.0f / (1.0f + *dx * *dx + *dy * *dy);
}

// Step 3: every iteration of one query in one thread.  With exact repulsion
// every thread of the block walks the whole reference layout, tile by tile,
// in shared memory (all read the same point at once: broadcast reads); the
// block's threads therefore stay in lock step across iterations, and threads
// past n_query take part without writing.
__global__ void __launch_bounds__(kLandmarkThreads) landmark_optimize_kernel(
    const float2* __restrict__ layout, const int* __restrict__ nbr, const float* __restrict__ prob,
    const float2* __restrict__ start, float2* __restrict__ out, LandmarkParams p, int index_offset) {
  __shared__ float2 tile[kRepulsionTile];
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  const bool live = row < p.n_query;
  constexpr float eps = 1.0e-12f;
  float2 yi = live ? start[row] : make_float2(0.0f, 0.0f);
  float2 gain = make_float2(1.0f, 1.0f);
  float2 upd = make_float2(0.0f, 0.0f);
  for (int it = 0; it < p.total_iter; ++it) {
    const bool early = it < p.early_iter;
    const float ex = early ? p.early_exaggeration : p.exaggeration;
    const float mom = early ? p.initial_momentum : p.final_momentum;
    float2 grad = make_float2(0.0f, 0.0f);
    float sum_q = eps;
    if (p.exact) {
      // Two passes over the layout, as the reference: the normaliser first.
      for (int pass = 0; pass < 2; ++pass) {
        for (int t0 = 0; t0 < p.n_reference; t0 += kRepulsionTile) {
          const int cnt = min(kRepulsionTile, p.n_reference - t0);
          __syncthreads();
          for (int i = threadIdx.x; i < cnt; i += blockDim.x) tile[i] = layout[t0 + i];
          __syncthreads();
          if (pass == 0) {
            for (int i = 0; i < cnt; ++i) {
              float dx, dy;
              sum_q += q_of(yi, tile[i], &dx, &dy);
            }
          } else {
            for (int i = 0; i < cnt; ++i) {
              float dx, dy;
              const float q = q_of(yi, tile[i], &dx, &dy);
              const float coeff = -(q * q) / sum_q;
              grad.x += coeff * dx;
              grad.y += coeff * dy;
            }
          }
        }
      }
    } else if (live) {
      for (int s = 0; s < p.n_negatives; ++s) {
        const unsigned int ref = reference_draw(static_cast<unsigned int>(p.n_reference), p.seed,
                                                static_cast<unsigned int>(it), static_cast<unsigned int>(row),
                                                static_cast<unsigned int>(s));
        float dx, dy;
        sum_q += q_of(yi, layout[ref], &dx, &dy);
      }
      for (int s = 0; s < p.n_negatives; ++s) {
        const unsigned int ref = reference_draw(static_cast<unsigned int>(p.n_reference), p.seed,
                                                static_cast<unsigned int>(it), static_cast<unsigned int>(row),
                                                static_cast<unsigned int>(s));
        float dx, dy;
        const float q = q_of(yi, layout[ref], &dx, &dy);
        const float coeff = -(q * q) / sum_q;
        grad.x += coeff * dx;
        grad.y += coeff * dy;
      }
    }
    if (!live) continue;
    for (int j = 0; j < p.k; ++j) {
      const size_t pos = static_cast<size_t>(j) * p.n_query + row;
      const int ref = nbr[pos] - index_offset;
      if (ref < 0 || ref >= p.n_reference) continue;
      float dx, dy;
      const float q = q_of(yi, layout[ref], &dx, &dy);
      const float coeff = ex * prob[pos] * q;
      grad.x += coeff * dx;
      grad.y += coeff * dy;
    }
    const float g2 = grad.x * grad.x + grad.y * grad.y;
    if (isfinite(p.max_grad_norm) && p.max_grad_norm > 0.0f && g2 > p.max_grad_norm * p.max_grad_norm) {
      const float scale = p.max_grad_norm / (sqrtf(g2) + eps);
      grad.x *= scale;
      grad.y *= scale;
    }
    gain.x = ((upd.x > 0.0f) != (grad.x > 0.0f)) ? gain.x + 0.2f : gain.x * 0.8f + 0.01f;
    gain.y = ((upd.y > 0.0f) != (grad.y > 0.0f)) ? gain.y + 0.2f : gain.y * 0.8f + 0.01f;
    gain.x = fmaxf(gain.x, 0.01f);
    gain.y = fmaxf(gain.y, 0.01f);
    upd.x = mom * upd.x - p.learning_rate * gain.x * grad.x;
    upd.y = mom * upd.y - p.learning_rate * gain.y * grad.y;
    const float s2 = upd.x * upd.x + upd.y * upd.y;
    if (isfinite(p.max_step_norm) && p.max_step_norm > 0.0f && s2 > p.max_step_norm * p.max_step_norm) {
      const float scale = p.max_step_norm / (sqrtf(s2) + eps);
      upd.x *= scale;
      upd.y *= scale;
    }
    yi = make_float2(yi.x + upd.x, yi.y + upd.y);
  }
  if (live) out[row] = yi;
}

// Column-major n x 2 layout -> interleaved float2 (one 8-byte gather per point).
__global__ void interleave_layout_kernel(const float* __restrict__ cm, int n, float2* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = make_float2(cm[i], cm[static_cast<size_t>(n) + i]);
}

}  // namespace

int landmark_tsne(const int* device_indices, const float* device_distances, int index_offset,
                  const float* reference_data, const float* query_data, const float* reference_layout,
                  int n_reference, int n_query, int n_features, int k, float perplexity, int n_iter,
                  int early_exaggeration_iter, float learning_rate, float early_exaggeration, float exaggeration,
                  float initial_momentum, float final_momentum, float max_grad_norm, float max_step_norm,
                  int n_negatives, int exact_repulsion_threshold, unsigned int seed, int affine_neighbors,
                  float affine_ridge, float max_extrapolation, float* out) {
  clear_error();
  if (device_indices == nullptr || device_distances == nullptr || reference_data == nullptr ||
      query_data == nullptr || reference_layout == nullptr || out == nullptr) {
    set_error("null CUDA landmark t-SNE pointer");
    return 1;
  }
  if (n_reference < 1 || n_query < 1 || n_features < 1 || k < 1 || k > kLandmarkMaxK || perplexity <= 0.0f ||
      n_iter < 0 || early_exaggeration_iter < 0 || n_iter + early_exaggeration_iter < 0) {
    set_error("invalid CUDA landmark t-SNE dimensions or parameters");
    return 1;
  }
  n_negatives = std::max(1, std::min(n_negatives, n_reference));
  affine_neighbors = std::max(3, std::min(affine_neighbors, std::min(k, kAffineMaxNeighbors)));
  const size_t ref_items = static_cast<size_t>(n_reference) * n_features;
  const size_t query_items = static_cast<size_t>(n_query) * n_features;
  const size_t graph_items = static_cast<size_t>(n_query) * k;
  Arena a;
  float* d_ref = nullptr;
  float* d_query = nullptr;
  float* d_layout_cm = nullptr;
  float2* d_layout = nullptr;
  float* d_prob = nullptr;
  float2* d_start = nullptr;
  float2* d_out = nullptr;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 0) a.begin_plan();
    else a.rewind();
    d_ref = a.take<float>(ref_items);
    d_query = a.take<float>(query_items);
    d_layout_cm = a.take<float>(2 * static_cast<size_t>(n_reference));
    d_layout = a.take<float2>(n_reference);
    d_prob = a.take<float>(graph_items);
    d_start = a.take<float2>(n_query);
    d_out = a.take<float2>(n_query);
    if (pass == 0) {
      FE_TRY(memory_preflight(a.planned(), "CUDA landmark t-SNE workspace"));
      FE_TRY(a.commit("landmark t-SNE workspace"));
    }
  }
  cudaStream_t st = nullptr;
  FE_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "cudaStreamCreate(landmark t-SNE)");
  struct StreamGuard {
    cudaStream_t s;
    ~StreamGuard() {
      cudaStreamSynchronize(s);
      cudaStreamDestroy(s);
    }
  } guard{st};
  FE_TRY(h2d_copy(d_ref, reference_data, ref_items * sizeof(float), st, "H2D landmark reference data"));
  FE_TRY(h2d_copy(d_query, query_data, query_items * sizeof(float), st, "H2D landmark query data"));
  FE_CUDA(cudaMemcpyAsync(d_layout_cm, reference_layout, 2 * static_cast<size_t>(n_reference) * sizeof(float),
                          cudaMemcpyHostToDevice, st),
          "H2D landmark reference layout");
  interleave_layout_kernel<<<(n_reference + 255) / 256, 256, 0, st>>>(d_layout_cm, n_reference, d_layout);
  FE_LAUNCH("interleave_layout_kernel");
  const int blocks = (n_query + kLandmarkThreads - 1) / kLandmarkThreads;
  landmark_setup_kernel<<<blocks, kLandmarkThreads, 0, st>>>(
      d_ref, d_query, d_layout, device_indices, device_distances, d_prob, d_start, n_reference, n_query,
      n_features, k, index_offset, affine_neighbors, affine_ridge, max_extrapolation, perplexity);
  FE_LAUNCH("landmark_setup_kernel");
  LandmarkParams p{};
  p.n_reference = n_reference;
  p.n_query = n_query;
  p.k = k;
  p.n_negatives = n_negatives;
  p.seed = seed;
  p.exact = (n_reference <= exact_repulsion_threshold || n_negatives >= n_reference) ? 1 : 0;
  p.early_iter = early_exaggeration_iter;
  p.total_iter = n_iter + early_exaggeration_iter;
  p.learning_rate = learning_rate;
  p.early_exaggeration = early_exaggeration;
  p.exaggeration = exaggeration;
  p.initial_momentum = initial_momentum;
  p.final_momentum = final_momentum;
  p.max_grad_norm = max_grad_norm;
  p.max_step_norm = max_step_norm;
  landmark_optimize_kernel<<<blocks, kLandmarkThreads, 0, st>>>(d_layout, device_indices, d_prob, d_start, d_out,
                                                                 p, index_offset);
  FE_LAUNCH("landmark_optimize_kernel");
  FE_CUDA(cudaMemcpyAsync(out, d_out, static_cast<size_t>(n_query) * sizeof(float2), cudaMemcpyDeviceToHost, st),
          "D2H landmark t-SNE layout");
  FE_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize(landmark t-SNE)");
  return 0;
}

}  // namespace fe
