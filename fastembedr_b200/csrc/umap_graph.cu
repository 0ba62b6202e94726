// UMAP fuzzy graph, start layout and COO edge list from a KNN on the device:
// the setup half of the device-KNN UMAP path
// (fastembedr_cuda_umap_from_device_knn_spectral_impl, src/embedding_cuda_kernels.cpp:4967-5199).
//
// Graph (prepare_device_knn_graph and its kernels, :3241-3321 and :1004-1160):
//   per row i: rho_i = smallest positive distance; sigma_i from 48 float
//   bisection steps on sum_j exp(-(d_ij - rho_i) / sigma) = log2(k);
//   w_ij = 1 if d_ij <= rho_i, else exp(-(d_ij - rho_i) / sigma_i).
//   Fuzzy union: an own entry i->j with w_ij > 0 gets w_ij + w_ji - w_ij w_ji,
//   where w_ji is the weight of the first entry of row j naming i (0 if none);
//   an entry j->i whose row i does not name j adds (j, w_ji) to row i.  Rows
//   hold min(256, 2k) slots and what does not fit is dropped.
// The reference fills the slots with atomics, so its slot order -- and, in rows
// that overflow, which incoming entries survive -- changes from run to run.
// Here the union is one stable radix sort of (row, col) records and the slot
// order is fixed: own entries in rank order, then incoming-only entries in
// ascending source order.  Rows that do not overflow hold the reference's
// entries exactly.
//
// Start layout (random_init_kernel, diffuse_init_kernel, normalize_device_init,
// :1162-1319): hashed uniform start, whitened (centred; x scaled to unit norm;
// y made orthogonal to x and scaled to unit norm), then per round every row
// takes the weighted mean of its neighbours and the result is whitened again.
// The whitening is applied while values are read, producing the same floats
// the reference materialises, so a round is one gather kernel and one
// moments reduction.
#include "umap.cuh"

#include <cub/cub.cuh>

#include <cmath>
#include <string>

namespace fe {

UmapDenseGraph::~UmapDenseGraph() {
  if (nbr) fe::dev_free(nbr);
  if (w) fe::dev_free(w);
}

namespace {

template <typename T>
struct Buf {
  T* p = nullptr;
  ~Buf() {
    if (p) fe::dev_free(p);
  }
  int alloc(size_t count, const char* what) {
    return check_cuda(fe::dev_malloc(reinterpret_cast<void**>(&p), sizeof(T) * (count ? count : 1)), what);
  }
  void free() {
    if (p) fe::dev_free(p);
    p = nullptr;
  }
  T* release() {
    T* q = p;
    p = nullptr;
    return q;
  }
};

inline unsigned grid_for(long long m, int threads) {
  return static_cast<unsigned>((m + threads - 1) / threads);
}

// ---------------------------------------------------------------- graph

// One thread per row; the KNN is column-major, so consecutive threads read
// consecutive addresses.  Writes the row's directed entries row-major:
// neighbour (-1 when invalid or self), weight, and the slot of each own entry
// that enters the union (rank among the row's entries with weight > 0).
template <typename DistT>
__global__ void calibrate_kernel(const int* __restrict__ idx, const DistT* __restrict__ dist, int n,
                                 int k, int offset, int* __restrict__ nbr_k, float* __restrict__ w_k,
                                 int* __restrict__ slot_k, int* __restrict__ out_cnt) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= n) return;
  const size_t sn = static_cast<size_t>(n);
  float rho = INFINITY;
  for (int j = 0; j < k; ++j) {
    const float d = static_cast<float>(dist[j * sn + row]);
    if (d > 0.0f && d < rho) rho = d;
  }
  if (!isfinite(rho)) rho = 0.0f;
  const float target = log2f(static_cast<float>(k < 2 ? 2 : k));
  float lo = 0.0f, hi = INFINITY, sigma = 1.0f;
  for (int step = 0; step < 48; ++step) {
    float psum = 0.0f;
    for (int j = 0; j < k; ++j) {
      const float d = static_cast<float>(dist[j * sn + row]) - rho;
      psum += d <= 0.0f ? 1.0f : expf(-d / sigma);
    }
    if (fabsf(psum - target) < 1.0e-5f) break;
    if (psum > target) {
      hi = sigma;
      sigma = 0.5f * (lo + hi);
    } else {
      lo = sigma;
      sigma = isinf(hi) ? sigma * 2.0f : 0.5f * (lo + hi);
    }
  }
  sigma = fmaxf(sigma, 1.0e-6f);
  int own = 0;
  for (int j = 0; j < k; ++j) {
    const int nb = idx[j * sn + row] - offset;
    const float d = static_cast<float>(dist[j * sn + row]);
    const bool valid = nb >= 0 && nb < n && nb != row;
    const float w = valid ? (d <= rho ? 1.0f : expf(-(d - rho) / sigma)) : 0.0f;
    const size_t e = static_cast<size_t>(row) * k + j;
    nbr_k[e] = valid ? nb : -1;
    w_k[e] = w;
    slot_k[e] = (valid && !(w <= 0.0f)) ? own++ : -1;
  }
  out_cnt[row] = own;
}

// Two records per valid entry e = (i, j): "own" (key i*n + j, value e) and
// "incoming" (key j*n + i, value nk + e).  Own records come first in the
// input, so after a stable sort a (row, col) run lists the row's own entries
// in rank order, then the entries of row col that name row, in rank order.
__global__ void records_kernel(const int* __restrict__ nbr_k, long long nk, int n, int k,
                               unsigned long long sentinel, unsigned long long* __restrict__ keys,
                               int* __restrict__ vals) {
  const long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (e >= nk) return;
  const int nb = nbr_k[e];
  const unsigned long long row = static_cast<unsigned long long>(e / k);
  if (nb < 0) {
    keys[e] = sentinel;
    keys[nk + e] = sentinel;
  } else {
    keys[e] = row * n + nb;
    keys[nk + e] = static_cast<unsigned long long>(nb) * n + row;
  }
  vals[e] = static_cast<int>(e);
  vals[nk + e] = static_cast<int>(nk + e);
}

__global__ void fill_empty_kernel(int* __restrict__ nbr, float* __restrict__ w, long long slots, int width) {
  const long long id = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (id >= slots) return;
  nbr[id] = static_cast<int>(id / width);
  w[id] = 0.0f;
}

// One thread per sorted record.  Own records with a slot write their union
// weight; incoming records of a run without own records are flagged for the
// incoming pass.
__global__ void resolve_kernel(const unsigned long long* __restrict__ keys, const int* __restrict__ vals,
                               long long m, long long nk, unsigned long long sentinel, int n, int width,
                               const float* __restrict__ w_k, const int* __restrict__ slot_k,
                               int* __restrict__ g_nbr, float* __restrict__ g_w, int* __restrict__ inc_flag) {
  const long long p = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (p >= m) return;
  const unsigned long long key = keys[p];
  if (key == sentinel) {
    inc_flag[p] = 0;
    return;
  }
  long long s = p;
  while (s > 0 && keys[s - 1] == key) --s;
  long long t = p + 1;
  while (t < m && keys[t] == key) ++t;
  bool has_own = false, have_rev = false;
  float rev = 0.0f;
  for (long long q = s; q < t; ++q) {
    const int v = vals[q];
    if (v < nk) {
      has_own = true;
    } else if (!have_rev) {
      rev = w_k[v - nk];
      have_rev = true;
    }
  }
  const int v = vals[p];
  int flag = 0;
  if (v < nk) {
    const int slot = slot_k[v];
    if (slot >= 0) {
      const int i = static_cast<int>(key / n);
      const int j = static_cast<int>(key - static_cast<unsigned long long>(i) * n);
      const float f = w_k[v];
      const size_t out = static_cast<size_t>(i) * width + slot;
      g_nbr[out] = j;
      g_w[out] = f + rev - f * rev;
    }
  } else if (!has_own && !(w_k[v - nk] <= 0.0f)) {
    flag = 1;
  }
  inc_flag[p] = flag;
}

__global__ void row_first_kernel(const unsigned long long* __restrict__ keys, long long m,
                                 unsigned long long sentinel, int n, int* __restrict__ row_first) {
  const long long p = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (p >= m) return;
  const unsigned long long key = keys[p];
  if (key == sentinel) return;
  const unsigned long long row = key / n;
  if (p == 0 || keys[p - 1] / n != row) row_first[row] = static_cast<int>(p);
}

__global__ void incoming_kernel(const unsigned long long* __restrict__ keys, const int* __restrict__ vals,
                                const int* __restrict__ inc_flag, const int* __restrict__ inc_pos,
                                long long m, long long nk, int n, int width, const float* __restrict__ w_k,
                                const int* __restrict__ out_cnt, const int* __restrict__ row_first,
                                int* __restrict__ g_nbr, float* __restrict__ g_w) {
  const long long p = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (p >= m || !inc_flag[p]) return;
  const unsigned long long key = keys[p];
  const int i = static_cast<int>(key / n);
  const int j = static_cast<int>(key - static_cast<unsigned long long>(i) * n);
  const int slot = out_cnt[i] + (inc_pos[p] - inc_pos[row_first[i]]);
  if (slot < width) {
    const size_t out = static_cast<size_t>(i) * width + slot;
    g_nbr[out] = j;
    g_w[out] = w_k[vals[p] - nk];
  }
}

// binary_graph_weights_kernel (:1099-1109): every real slot weighs 1.
__global__ void binary_kernel(const int* __restrict__ nbr, float* __restrict__ w, int n, int width) {
  const long long id = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (id >= static_cast<long long>(n) * width) return;
  const int row = static_cast<int>(id / width);
  const int nb = nbr[id];
  w[id] = (nb >= 0 && nb < n && nb != row) ? 1.0f : 0.0f;
}

// ---------------------------------------------------------------- COO

__device__ __forceinline__ void pack_coords(long long id, int n, int width, bool rank_major, int* row,
                                            int* slot) {
  if (rank_major) {
    *slot = static_cast<int>(id / n);
    *row = static_cast<int>(id - static_cast<long long>(*slot) * n);
  } else {
    *row = static_cast<int>(id / width);
    *slot = static_cast<int>(id - static_cast<long long>(*row) * width);
  }
}

__global__ void pack_flags_kernel(const int* __restrict__ nbr, const float* __restrict__ w, int n,
                                  int width, bool rank_major, int* __restrict__ flags) {
  const long long id = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (id >= static_cast<long long>(n) * width) return;
  int row, slot;
  pack_coords(id, n, width, rank_major, &row, &slot);
  const size_t dense = static_cast<size_t>(row) * width + slot;
  const int nb = nbr[dense];
  flags[id] = (nb >= 0 && nb < n && nb != row && w[dense] > 0.0f) ? 1 : 0;
}

// pack_coo_graph_from_selected_rank_major_kernel (:2997-3022): period = 1 / max(w, 1e-6).
__global__ void pack_kernel(const int* __restrict__ nbr, const float* __restrict__ w, int n, int width,
                            bool rank_major, const int* __restrict__ flags, const int* __restrict__ pos,
                            int* __restrict__ heads, int* __restrict__ tails, float* __restrict__ weights,
                            float* __restrict__ periods) {
  const long long id = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (id >= static_cast<long long>(n) * width || !flags[id]) return;
  int row, slot;
  pack_coords(id, n, width, rank_major, &row, &slot);
  const size_t dense = static_cast<size_t>(row) * width + slot;
  const float wt = w[dense];
  const int o = pos[id];
  heads[o] = row;
  tails[o] = nbr[dense];
  if (weights) weights[o] = wt;
  periods[o] = 1.0f / fmaxf(wt, 1.0e-6f);
}

// ---------------------------------------------------------------- start layout

constexpr int kMomentThreads = 256;
constexpr int kMomentBlocks = 1024;

__global__ void random_start_kernel(float2* __restrict__ y, int n, unsigned int seed) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= n) return;
  y[row] = make_float2(hashed_unit(seed, row, 0), hashed_unit(seed, row, 1));
}

// Sums {x, y, x^2, xy, y^2} in double; block partials in a fixed order.
__global__ void moments_kernel(const float2* __restrict__ y, int n, double* __restrict__ partial) {
  __shared__ double sh[5][kMomentThreads];
  double a[5] = {0.0, 0.0, 0.0, 0.0, 0.0};
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const double x = y[i].x, v = y[i].y;
    a[0] += x;
    a[1] += v;
    a[2] += x * x;
    a[3] += x * v;
    a[4] += v * v;
  }
  for (int c = 0; c < 5; ++c) sh[c][threadIdx.x] = a[c];
  __syncthreads();
  for (int stride = blockDim.x / 2; stride > 0; stride >>= 1) {
    if (threadIdx.x < stride) {
      for (int c = 0; c < 5; ++c) sh[c][threadIdx.x] += sh[c][threadIdx.x + stride];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    for (int c = 0; c < 5; ++c) partial[blockIdx.x * 5 + c] = sh[c][0];
  }
}

// Whitening coefficients (finalize_init_stats_kernel, :1250-1306):
// {mean_x, mean_y, 1 / |x_c|, <y_c, x_hat>, 1 / |y_c - <y_c, x_hat> x_hat|}.
__global__ void whiten_stats_kernel(const double* __restrict__ partial, int blocks, int n,
                                    double* __restrict__ st) {
  __shared__ double sh[5][kMomentThreads];
  double a[5] = {0.0, 0.0, 0.0, 0.0, 0.0};
  for (int b = threadIdx.x; b < blocks; b += blockDim.x) {
    for (int c = 0; c < 5; ++c) a[c] += partial[b * 5 + c];
  }
  for (int c = 0; c < 5; ++c) sh[c][threadIdx.x] = a[c];
  __syncthreads();
  for (int stride = blockDim.x / 2; stride > 0; stride >>= 1) {
    if (threadIdx.x < stride) {
      for (int c = 0; c < 5; ++c) sh[c][threadIdx.x] += sh[c][threadIdx.x + stride];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const double dn = static_cast<double>(n > 1 ? n : 1);
    const double sx = sh[0][0], sy = sh[1][0];
    const double x_ss = fmax(sh[2][0] - sx * sx / dn, 1.0e-24);
    const double y_ss = fmax(sh[4][0] - sy * sy / dn, 1.0e-24);
    const double xy = sh[3][0] - sx * sy / dn;
    const double norm_x = sqrt(x_ss);
    const double proj = xy / norm_x;
    const double resid = fmax(y_ss - proj * proj, 1.0e-24);
    st[0] = sx / dn;
    st[1] = sy / dn;
    st[2] = 1.0 / norm_x;
    st[3] = proj;
    st[4] = 1.0 / sqrt(resid);
  }
}

// normalize_init_kernel (:1308-1319) for one value.
__device__ __forceinline__ float2 whiten(float2 v, const double* __restrict__ st) {
  const double x = (static_cast<double>(v.x) - st[0]) * st[2];
  const double yc = static_cast<double>(v.y) - st[1];
  const double y = (yc - st[3] * x) * st[4];
  return make_float2(static_cast<float>(x), static_cast<float>(y));
}

// diffuse_init_kernel (:1169-1196) over whitened inputs.
__global__ void diffuse_kernel(const int* __restrict__ nbr, const float* __restrict__ w, int n, int width,
                               const float2* __restrict__ cur, const double* __restrict__ st,
                               float2* __restrict__ next) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= n) return;
  float sx = 0.0f, sy = 0.0f, sw = 0.0f;
  const size_t base = static_cast<size_t>(row) * width;
  for (int j = 0; j < width; ++j) {
    const int nb = nbr[base + j];
    const float wt = w[base + j];
    if (nb < 0 || nb >= n || nb == row || wt <= 0.0f) continue;
    const float2 c = whiten(cur[nb], st);
    sx += wt * c.x;
    sy += wt * c.y;
    sw += wt;
  }
  next[row] = sw <= 0.0f ? whiten(cur[row], st) : make_float2(sx / sw, sy / sw);
}

__global__ void whiten_kernel(float2* __restrict__ y, int n, const double* __restrict__ st) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row < n) y[row] = whiten(y[row], st);
}

int whiten_stats(const float2* y, int n, double* partial, double* st, cudaStream_t stream) {
  moments_kernel<<<kMomentBlocks, kMomentThreads, 0, stream>>>(y, n, partial);
  FE_LAUNCH("moments_kernel");
  whiten_stats_kernel<<<1, kMomentThreads, 0, stream>>>(partial, kMomentBlocks, n, st);
  FE_LAUNCH("whiten_stats_kernel");
  return 0;
}

int bit_width(unsigned long long v) {
  int b = 0;
  while (v) {
    ++b;
    v >>= 1;
  }
  return b;
}

}  // namespace

int umap_graph_build(const int* d_idx, const void* d_dist, bool dist_is_double, int n, int k,
                     int index_offset, bool binary, cudaStream_t stream, UmapDenseGraph* g) {
  const int width = umap_graph_width(k);
  const long long nk = static_cast<long long>(n) * k;
  const long long m = 2 * nk;
  const long long slots = static_cast<long long>(n) * width;
  if (m >= (1ll << 31) - 1 || slots >= (1ll << 31) - 1) {
    set_error("UMAP graph: n * k exceeds the 32-bit entry range");
    return 1;
  }
  g->n = n;
  g->k = k;
  g->width = width;
  Buf<int> nbr_k, slot_k, out_cnt;
  Buf<float> w_k;
  FE_TRY(nbr_k.alloc(nk, "cudaMalloc(UMAP directed neighbours)"));
  FE_TRY(w_k.alloc(nk, "cudaMalloc(UMAP directed weights)"));
  FE_TRY(slot_k.alloc(nk, "cudaMalloc(UMAP own slots)"));
  FE_TRY(out_cnt.alloc(n, "cudaMalloc(UMAP own counts)"));
  if (dist_is_double) {
    calibrate_kernel<double><<<grid_for(n, 128), 128, 0, stream>>>(
        d_idx, static_cast<const double*>(d_dist), n, k, index_offset, nbr_k.p, w_k.p, slot_k.p, out_cnt.p);
  } else {
    calibrate_kernel<float><<<grid_for(n, 128), 128, 0, stream>>>(
        d_idx, static_cast<const float*>(d_dist), n, k, index_offset, nbr_k.p, w_k.p, slot_k.p, out_cnt.p);
  }
  FE_LAUNCH("calibrate_kernel");

  const unsigned long long sentinel = static_cast<unsigned long long>(n) * static_cast<unsigned long long>(n);
  const int end_bit = bit_width(sentinel);
  Buf<unsigned long long> keys, keys_sorted;
  Buf<int> vals, vals_sorted;
  FE_TRY(keys.alloc(m, "cudaMalloc(UMAP union keys)"));
  FE_TRY(vals.alloc(m, "cudaMalloc(UMAP union values)"));
  records_kernel<<<grid_for(nk, 256), 256, 0, stream>>>(nbr_k.p, nk, n, k, sentinel, keys.p, vals.p);
  FE_LAUNCH("records_kernel");
  FE_TRY(keys_sorted.alloc(m, "cudaMalloc(UMAP sorted keys)"));
  FE_TRY(vals_sorted.alloc(m, "cudaMalloc(UMAP sorted values)"));
  size_t sort_bytes = 0, scan_bytes = 0;
  FE_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, keys.p, keys_sorted.p, vals.p, vals_sorted.p,
                                          static_cast<int>(m), 0, end_bit, stream),
          "cub::DeviceRadixSort(UMAP sizing)");
  Buf<int> inc_flag, inc_pos;
  FE_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, inc_flag.p, inc_pos.p, static_cast<int>(m), stream),
          "cub::DeviceScan(UMAP sizing)");
  {
    Buf<unsigned char> temp;
    FE_TRY(temp.alloc(sort_bytes, "cudaMalloc(UMAP sort temp)"));
    FE_CUDA(cub::DeviceRadixSort::SortPairs(temp.p, sort_bytes, keys.p, keys_sorted.p, vals.p, vals_sorted.p,
                                            static_cast<int>(m), 0, end_bit, stream),
            "cub::DeviceRadixSort(UMAP union records)");
    FE_CUDA(cudaStreamSynchronize(stream), "cudaStreamSynchronize(UMAP union sort)");
  }
  keys.free();
  vals.free();

  FE_CUDA(fe::dev_malloc(reinterpret_cast<void**>(&g->nbr), sizeof(int) * slots), "cudaMalloc(UMAP graph slots)");
  FE_CUDA(fe::dev_malloc(reinterpret_cast<void**>(&g->w), sizeof(float) * slots), "cudaMalloc(UMAP graph weights)");
  fill_empty_kernel<<<grid_for(slots, 256), 256, 0, stream>>>(g->nbr, g->w, slots, width);
  FE_LAUNCH("fill_empty_kernel");
  FE_TRY(inc_flag.alloc(m, "cudaMalloc(UMAP incoming flags)"));
  FE_TRY(inc_pos.alloc(m, "cudaMalloc(UMAP incoming positions)"));
  resolve_kernel<<<grid_for(m, 256), 256, 0, stream>>>(keys_sorted.p, vals_sorted.p, m, nk, sentinel, n, width,
                                                       w_k.p, slot_k.p, g->nbr, g->w, inc_flag.p);
  FE_LAUNCH("resolve_kernel");
  {
    Buf<unsigned char> temp;
    FE_TRY(temp.alloc(scan_bytes, "cudaMalloc(UMAP scan temp)"));
    FE_CUDA(cub::DeviceScan::ExclusiveSum(temp.p, scan_bytes, inc_flag.p, inc_pos.p, static_cast<int>(m), stream),
            "cub::DeviceScan(UMAP incoming)");
    Buf<int> row_first;
    FE_TRY(row_first.alloc(n, "cudaMalloc(UMAP row starts)"));
    row_first_kernel<<<grid_for(m, 256), 256, 0, stream>>>(keys_sorted.p, m, sentinel, n, row_first.p);
    FE_LAUNCH("row_first_kernel");
    incoming_kernel<<<grid_for(m, 256), 256, 0, stream>>>(keys_sorted.p, vals_sorted.p, inc_flag.p, inc_pos.p, m,
                                                          nk, n, width, w_k.p, out_cnt.p, row_first.p, g->nbr,
                                                          g->w);
    FE_LAUNCH("incoming_kernel");
    if (binary) {
      binary_kernel<<<grid_for(slots, 256), 256, 0, stream>>>(g->nbr, g->w, n, width);
      FE_LAUNCH("binary_kernel");
    }
    FE_CUDA(cudaStreamSynchronize(stream), "cudaStreamSynchronize(UMAP graph)");
  }
  return 0;
}

int umap_graph_pack(const UmapDenseGraph& g, bool rank_major, int* heads, int* tails, float* weights,
                    float* epochs_per_sample, long long* n_edges, cudaStream_t stream) {
  const long long slots = static_cast<long long>(g.n) * g.width;
  Buf<int> flags, pos;
  FE_TRY(flags.alloc(slots, "cudaMalloc(UMAP pack flags)"));
  FE_TRY(pos.alloc(slots, "cudaMalloc(UMAP pack positions)"));
  pack_flags_kernel<<<grid_for(slots, 256), 256, 0, stream>>>(g.nbr, g.w, g.n, g.width, rank_major, flags.p);
  FE_LAUNCH("pack_flags_kernel");
  size_t scan_bytes = 0;
  FE_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, flags.p, pos.p, static_cast<int>(slots), stream),
          "cub::DeviceScan(UMAP pack sizing)");
  {
    Buf<unsigned char> temp;
    FE_TRY(temp.alloc(scan_bytes, "cudaMalloc(UMAP pack scan temp)"));
    FE_CUDA(cub::DeviceScan::ExclusiveSum(temp.p, scan_bytes, flags.p, pos.p, static_cast<int>(slots), stream),
            "cub::DeviceScan(UMAP pack)");
    pack_kernel<<<grid_for(slots, 256), 256, 0, stream>>>(g.nbr, g.w, g.n, g.width, rank_major, flags.p, pos.p,
                                                          heads, tails, weights, epochs_per_sample);
    FE_LAUNCH("pack_kernel");
    int last_pos = 0, last_flag = 0;
    FE_CUDA(cudaMemcpyAsync(&last_pos, pos.p + (slots - 1), sizeof(int), cudaMemcpyDeviceToHost, stream),
            "D2H UMAP edge count");
    FE_CUDA(cudaMemcpyAsync(&last_flag, flags.p + (slots - 1), sizeof(int), cudaMemcpyDeviceToHost, stream),
            "D2H UMAP edge count");
    FE_CUDA(cudaStreamSynchronize(stream), "cudaStreamSynchronize(UMAP pack)");
    *n_edges = static_cast<long long>(last_pos) + last_flag;
  }
  return 0;
}

int umap_diffusion_init(const UmapDenseGraph& g, unsigned int seed, int iters, float2* layout,
                        cudaStream_t stream) {
  const int n = g.n;
  Buf<float2> other;
  Buf<double> partial, st;
  FE_TRY(other.alloc(n, "cudaMalloc(UMAP diffusion buffer)"));
  FE_TRY(partial.alloc(static_cast<size_t>(kMomentBlocks) * 5, "cudaMalloc(UMAP moments)"));
  FE_TRY(st.alloc(5, "cudaMalloc(UMAP whitening)"));
  float2* cur = layout;
  float2* next = other.p;
  random_start_kernel<<<grid_for(n, 256), 256, 0, stream>>>(cur, n, seed);
  FE_LAUNCH("random_start_kernel");
  FE_TRY(whiten_stats(cur, n, partial.p, st.p, stream));
  for (int it = 0; it < iters; ++it) {
    diffuse_kernel<<<grid_for(n, 128), 128, 0, stream>>>(g.nbr, g.w, n, g.width, cur, st.p, next);
    FE_LAUNCH("diffuse_kernel");
    FE_TRY(whiten_stats(next, n, partial.p, st.p, stream));
    float2* t = cur;
    cur = next;
    next = t;
  }
  whiten_kernel<<<grid_for(n, 256), 256, 0, stream>>>(cur, n, st.p);
  FE_LAUNCH("whiten_kernel");
  if (cur != layout) {
    FE_CUDA(cudaMemcpyAsync(layout, cur, sizeof(float2) * n, cudaMemcpyDeviceToDevice, stream),
            "D2D UMAP start layout");
  }
  FE_CUDA(cudaStreamSynchronize(stream), "cudaStreamSynchronize(UMAP start layout)");
  return 0;
}

}  // namespace fe
