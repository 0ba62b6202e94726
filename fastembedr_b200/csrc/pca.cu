// PCA start of the openTSNE device-KNN entry points with a data matrix
// (fastembedr_cuda_opentsne_fft_from_device_knn_float_pca_{double,float},
// src/embedding_cuda_impl.cpp:142-183; the reference computes it with RAFT's
// TSVD, src/embedding_cuda_kernels.cpp:3357-3495, used at :5692-5724).
//
// Steps (the reference's, with its RAFT call restated as a covariance
// eigen-decomposition, which is what its COV_EIG_DQ solver does):
//   1. column means of the n x p data (column-major, R's order) in double, and
//      the data centred in float;
//   2. the p x p covariance X^T X of the centred data, in double: a tiled
//      symmetric product (pca_cov_kernel) over row chunks, partial tiles summed
//      in a fixed order, so the result does not depend on timing;
//   3. its two leading eigenvectors on the host (cyclic Jacobi; p x p is small);
//   4. scores = X V (n x 2), each component's sign chosen so that its
//      largest-magnitude score is positive (RAFT TSVD's sign flip);
//   5. the t-SNE PCA scaling of the reference (finalize_tsne_pca_init_stats_kernel
//      / scale_tsne_pca_init_kernel, :1336-1404): centred, then scaled so the
//      larger of the two standard deviations is 1e-4.
#include "tsne.cuh"

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <string>
#include <vector>

namespace fe {
namespace {

constexpr int kPcaTile = 16;          // covariance tile side (threads per block: 16 x 16)
constexpr int kPcaChunkRows = 8192;   // rows per covariance partial

template <typename T>
__global__ void pca_mean_kernel(const T* __restrict__ x, int n, double* __restrict__ mean) {
  // one block per column; fixed reduction order
  const int j = blockIdx.x;
  const T* col = x + static_cast<size_t>(j) * n;
  double s = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += static_cast<double>(col[i]);
  __shared__ double part[32];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += part[w];
    mean[j] = t / static_cast<double>(n);
  }
}

template <typename T>
__global__ void pca_center_kernel(const T* __restrict__ x, size_t items, int n, const double* __restrict__ mean,
                                  float* __restrict__ xc) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= items) return;
  const int j = static_cast<int>(i / static_cast<size_t>(n));
  xc[i] = static_cast<float>(x[i]) - static_cast<float>(mean[j]);
}

// Partial covariance tile (ta, tb), ta <= tb, over one chunk of rows:
// part[chunk][ta*tiles+tb][a][b] = sum_rows xc[row][a] * xc[row][b] in double.
__global__ void pca_cov_kernel(const float* __restrict__ xc, int n, int p, int tiles,
                               const int2* __restrict__ tile_pairs, double* __restrict__ part) {
  __shared__ float sa[kPcaTile][kPcaTile + 1];
  __shared__ float sb[kPcaTile][kPcaTile + 1];
  const int2 tp = tile_pairs[blockIdx.x];
  const int chunk = blockIdx.y;
  const int r0 = chunk * kPcaChunkRows;
  const int r1 = min(n, r0 + kPcaChunkRows);
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int a = tp.x * kPcaTile + ty;  // row of the tile
  const int b = tp.y * kPcaTile + tx;  // column of the tile
  double acc = 0.0;
  for (int rr = r0; rr < r1; rr += kPcaTile) {
    // load rows rr..rr+15 of the two column tiles (column-major: coalesced in rows)
    const int row = rr + tx;
    const int ca = tp.x * kPcaTile + ty;
    const int cb = tp.y * kPcaTile + ty;
    sa[ty][tx] = (row < r1 && ca < p) ? xc[static_cast<size_t>(ca) * n + row] : 0.0f;
    sb[ty][tx] = (row < r1 && cb < p) ? xc[static_cast<size_t>(cb) * n + row] : 0.0f;
    __syncthreads();
#pragma unroll
    for (int t = 0; t < kPcaTile; ++t) acc += static_cast<double>(sa[ty][t]) * static_cast<double>(sb[tx][t]);
    __syncthreads();
  }
  const size_t base = (static_cast<size_t>(chunk) * tiles * tiles + static_cast<size_t>(tp.x) * tiles + tp.y) *
                      (kPcaTile * kPcaTile);
  part[base + ty * kPcaTile + tx] = (a < p && b < p) ? acc : 0.0;
}

// Sums the chunk partials in chunk order into cov (p x p, symmetric).
__global__ void pca_cov_reduce_kernel(const double* __restrict__ part, int p, int tiles, int chunks,
                                      double* __restrict__ cov) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= p * p) return;
  int a = idx / p, b = idx - (idx / p) * p;
  if (a > b) {
    const int t = a;
    a = b;
    b = t;
  }
  const int ta = a / kPcaTile, tb = b / kPcaTile;
  const size_t off = (static_cast<size_t>(ta) * tiles + tb) * (kPcaTile * kPcaTile) +
                     static_cast<size_t>(a - ta * kPcaTile) * kPcaTile + (b - tb * kPcaTile);
  double s = 0.0;
  for (int c = 0; c < chunks; ++c) s += part[static_cast<size_t>(c) * tiles * tiles * kPcaTile * kPcaTile + off];
  cov[idx] = s;
}

// Scores of the two components (double accumulation), written as float2.
__global__ void pca_scores_kernel(const float* __restrict__ xc, int n, int p, const double* __restrict__ v,
                                  float2* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  double s0 = 0.0, s1 = 0.0;
  for (int j = 0; j < p; ++j) {
    const double xv = static_cast<double>(xc[static_cast<size_t>(j) * n + i]);
    s0 += xv * v[j];
    s1 += xv * v[p + j];
  }
  const float x = static_cast<float>(s0), y = static_cast<float>(s1);
  out[i] = make_float2(isfinite(x) ? x : 0.0f, isfinite(y) ? y : 0.0f);
}

// Per block: sums {x, y, x^2, xy, y^2} and, per component, the score of
// largest magnitude (ties: lowest row) for the sign convention.
struct PcaPartial {
  double s[5];
  float best[2];
  int best_row[2];
};

__device__ __forceinline__ void better(float& v, int& r, float ov, int orow) {
  const float a = fabsf(v), b = fabsf(ov);
  if (b > a || (b == a && orow < r)) {
    v = ov;
    r = orow;
  }
}

__global__ void pca_stats_kernel(const float2* __restrict__ y, int n, PcaPartial* __restrict__ part) {
  double s[5] = {0, 0, 0, 0, 0};
  float bv[2] = {0.0f, 0.0f};
  int br[2] = {INT_MAX, INT_MAX};
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float2 p = y[i];
    const double x = p.x, z = p.y;
    s[0] += x;
    s[1] += z;
    s[2] += x * x;
    s[3] += x * z;
    s[4] += z * z;
    better(bv[0], br[0], p.x, i);
    better(bv[1], br[1], p.y, i);
  }
  __shared__ PcaPartial sh[256];
  PcaPartial me;
  for (int t = 0; t < 5; ++t) me.s[t] = s[t];
  me.best[0] = bv[0];
  me.best[1] = bv[1];
  me.best_row[0] = br[0];
  me.best_row[1] = br[1];
  sh[threadIdx.x] = me;
  __syncthreads();
  for (int stride = blockDim.x / 2; stride > 0; stride >>= 1) {
    if (static_cast<int>(threadIdx.x) < stride) {
      PcaPartial& a = sh[threadIdx.x];
      const PcaPartial& b = sh[threadIdx.x + stride];
      for (int t = 0; t < 5; ++t) a.s[t] += b.s[t];
      better(a.best[0], a.best_row[0], b.best[0], b.best_row[0]);
      better(a.best[1], a.best_row[1], b.best[1], b.best_row[1]);
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) part[blockIdx.x] = sh[0];
}

// Sign flip and the t-SNE PCA scaling, from the block partials (one thread
// folds them in block order, then every thread applies).
__global__ void pca_finish_kernel(float2* __restrict__ y, int n, const PcaPartial* __restrict__ part, int blocks) {
  __shared__ double st[5];
  if (threadIdx.x == 0) {
    PcaPartial t = part[0];
    for (int b = 1; b < blocks; ++b) {
      for (int k = 0; k < 5; ++k) t.s[k] += part[b].s[k];
      better(t.best[0], t.best_row[0], part[b].best[0], part[b].best_row[0]);
      better(t.best[1], t.best_row[1], part[b].best[1], part[b].best_row[1]);
    }
    const double sgx = t.best[0] < 0.0f ? -1.0 : 1.0;
    const double sgy = t.best[1] < 0.0f ? -1.0 : 1.0;
    // statistics of the sign-flipped scores (flipping negates the sums of x,
    // y and xy as needed; squares are unchanged)
    const double dn = static_cast<double>(max(n, 1));
    const double denom = static_cast<double>(max(n - 1, 1));
    const double sx = sgx * t.s[0], sy = sgy * t.s[1];
    const double mean_x = sx / dn, mean_y = sy / dn;
    const double ss_x = fmax(t.s[2] - sx * sx / dn, 0.0);
    const double ss_y = fmax(t.s[4] - sy * sy / dn, 0.0);
    const double sd_x = sqrt(ss_x / denom), sd_y = sqrt(ss_y / denom);
    const double max_sd = fmax(sd_x, sd_y);
    st[0] = mean_x;
    st[1] = mean_y;
    st[2] = (isfinite(max_sd) && max_sd > 0.0) ? 1.0e-4 / max_sd : 1.0;
    st[3] = sgx;
    st[4] = sgy;
  }
  __syncthreads();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float2 p = y[i];
    const float fx = static_cast<float>(st[3] * static_cast<double>(p.x));
    const float fy = static_cast<float>(st[4] * static_cast<double>(p.y));
    y[i] = make_float2(static_cast<float>((static_cast<double>(fx) - st[0]) * st[2]),
                       static_cast<float>((static_cast<double>(fy) - st[1]) * st[2]));
  }
}

// Leading two eigenvectors of a symmetric p x p matrix (cyclic Jacobi), as
// columns of v2 (p x 2, column-major), largest eigenvalue first.
void top_two_eigenvectors(std::vector<double> a, int p, std::vector<double>* v2) {
  std::vector<double> v(static_cast<size_t>(p) * p, 0.0);
  for (int i = 0; i < p; ++i) v[static_cast<size_t>(i) * p + i] = 1.0;
  auto A = [&](int i, int j) -> double& { return a[static_cast<size_t>(i) * p + j]; };
  for (int sweep = 0; sweep < 100; ++sweep) {
    double off = 0.0, diag = 0.0;
    for (int i = 0; i < p; ++i) {
      diag += A(i, i) * A(i, i);
      for (int j = i + 1; j < p; ++j) off += A(i, j) * A(i, j);
    }
    if (off <= 1e-30 * std::max(diag, 1e-300)) break;
    for (int pi = 0; pi < p; ++pi) {
      for (int q = pi + 1; q < p; ++q) {
        const double apq = A(pi, q);
        if (std::fabs(apq) < 1e-300) continue;
        const double theta = (A(q, q) - A(pi, pi)) / (2.0 * apq);
        const double t = (theta >= 0.0 ? 1.0 : -1.0) / (std::fabs(theta) + std::sqrt(theta * theta + 1.0));
        const double c = 1.0 / std::sqrt(t * t + 1.0), s = t * c;
        for (int k = 0; k < p; ++k) {  // rotate columns pi, q
          const double akp = A(k, pi), akq = A(k, q);
          A(k, pi) = c * akp - s * akq;
          A(k, q) = s * akp + c * akq;
        }
        for (int k = 0; k < p; ++k) {  // rotate rows pi, q
          const double apk = A(pi, k), aqk = A(q, k);
          A(pi, k) = c * apk - s * aqk;
          A(q, k) = s * apk + c * aqk;
        }
        for (int k = 0; k < p; ++k) {
          const double vkp = v[static_cast<size_t>(k) * p + pi], vkq = v[static_cast<size_t>(k) * p + q];
          v[static_cast<size_t>(k) * p + pi] = c * vkp - s * vkq;
          v[static_cast<size_t>(k) * p + q] = s * vkp + c * vkq;
        }
      }
    }
  }
  std::vector<int> order(p);
  for (int i = 0; i < p; ++i) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](int x, int y) { return A(x, x) > A(y, y); });
  v2->assign(2 * static_cast<size_t>(p), 0.0);
  for (int c = 0; c < 2 && c < p; ++c) {
    for (int k = 0; k < p; ++k) (*v2)[static_cast<size_t>(c) * p + k] = v[static_cast<size_t>(k) * p + order[c]];
  }
}

}  // namespace

int pca_start_layout(const void* values, bool values_double, int n, int p, cudaStream_t st, float2* d_out) {
  if (values == nullptr || d_out == nullptr) {
    set_error("null pointer in device PCA initialization");
    return 1;
  }
  if (n < 2 || p < 2) {
    set_error("invalid dimensions in device PCA initialization");
    return 1;
  }
  const size_t items = static_cast<size_t>(n) * p;
  const int tiles = (p + kPcaTile - 1) / kPcaTile;
  const int chunks = (n + kPcaChunkRows - 1) / kPcaChunkRows;
  const int pairs = tiles * (tiles + 1) / 2;
  constexpr int kStatBlocks = 296;
  Arena a;
  void* d_raw = nullptr;
  float* d_xc = nullptr;
  double* d_mean = nullptr;
  double* d_part = nullptr;
  double* d_cov = nullptr;
  double* d_v = nullptr;
  int2* d_pairs = nullptr;
  PcaPartial* d_stats = nullptr;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 0) a.begin_plan();
    else a.rewind();
    d_raw = a.take<char>(items * (values_double ? sizeof(double) : sizeof(float)));
    d_xc = a.take<float>(items);
    d_mean = a.take<double>(p);
    d_part = a.take<double>(static_cast<size_t>(chunks) * tiles * tiles * kPcaTile * kPcaTile);
    d_cov = a.take<double>(static_cast<size_t>(p) * p);
    d_v = a.take<double>(2 * static_cast<size_t>(p));
    d_pairs = a.take<int2>(pairs);
    d_stats = a.take<PcaPartial>(kStatBlocks);
    if (pass == 0) {
      FE_TRY(memory_preflight(a.planned(), "device PCA initialization"));
      FE_TRY(a.commit("device PCA initialization"));
    }
  }
  FE_TRY(h2d_copy(d_raw, values, items * (values_double ? sizeof(double) : sizeof(float)), st, "H2D PCA data"));
  FE_CUDA(cudaMemsetAsync(d_part, 0, static_cast<size_t>(chunks) * tiles * tiles * kPcaTile * kPcaTile * sizeof(double),
                          st),
          "memset PCA partials");
  std::vector<int2> tp;
  for (int ta = 0; ta < tiles; ++ta) {
    for (int tb = ta; tb < tiles; ++tb) tp.push_back(make_int2(ta, tb));
  }
  FE_CUDA(cudaMemcpyAsync(d_pairs, tp.data(), sizeof(int2) * tp.size(), cudaMemcpyHostToDevice, st), "H2D pairs");
  const unsigned center_blocks = static_cast<unsigned>((items + 255) / 256);
  if (values_double) {
    pca_mean_kernel<double><<<p, 256, 0, st>>>(static_cast<const double*>(d_raw), n, d_mean);
    pca_center_kernel<double><<<center_blocks, 256, 0, st>>>(static_cast<const double*>(d_raw), items, n, d_mean,
                                                             d_xc);
  } else {
    pca_mean_kernel<float><<<p, 256, 0, st>>>(static_cast<const float*>(d_raw), n, d_mean);
    pca_center_kernel<float><<<center_blocks, 256, 0, st>>>(static_cast<const float*>(d_raw), items, n, d_mean,
                                                            d_xc);
  }
  FE_LAUNCH("pca_center_kernel");
  pca_cov_kernel<<<dim3(pairs, chunks), dim3(kPcaTile, kPcaTile), 0, st>>>(d_xc, n, p, tiles, d_pairs, d_part);
  FE_LAUNCH("pca_cov_kernel");
  pca_cov_reduce_kernel<<<(p * p + 255) / 256, 256, 0, st>>>(d_part, p, tiles, chunks, d_cov);
  FE_LAUNCH("pca_cov_reduce_kernel");
  std::vector<double> cov(static_cast<size_t>(p) * p);
  FE_CUDA(cudaMemcpyAsync(cov.data(), d_cov, sizeof(double) * cov.size(), cudaMemcpyDeviceToHost, st), "D2H cov");
  FE_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize(PCA covariance)");
  std::vector<double> v2;
  top_two_eigenvectors(cov, p, &v2);
  FE_CUDA(cudaMemcpyAsync(d_v, v2.data(), sizeof(double) * v2.size(), cudaMemcpyHostToDevice, st), "H2D PCA axes");
  pca_scores_kernel<<<(n + 255) / 256, 256, 0, st>>>(d_xc, n, p, d_v, d_out);
  FE_LAUNCH("pca_scores_kernel");
  pca_stats_kernel<<<kStatBlocks, 256, 0, st>>>(d_out, n, d_stats);
  FE_LAUNCH("pca_stats_kernel");
  pca_finish_kernel<<<kStatBlocks, 256, 0, st>>>(d_out, n, d_stats, kStatBlocks);
  FE_LAUNCH("pca_finish_kernel");
  FE_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize(PCA start)");
  return 0;
}

}  // namespace fe
