// Sparse t-SNE affinities on the device.
//
// Follows build_tsne_probabilities_float (src/tsne_neighbors.cpp:540-648) and
// compute_row_probabilities_float (:482-532):
//   1. per row, a float32 bisection on beta (<= 200 steps, |H - ln perp| < 1e-5)
//      over the row's k distances, then p_{j|i} normalised to 1;
//   2. every non-self entry becomes the unordered pair (min, max) with value
//      p_{j|i}; equal pairs are summed (in double, as the reference does);
//   3. P_ij = sum_ij * (0.5 / total) stored in both directions, rows sorted by
//      column -- the exact row order the reference CSR has.
// The reference's global sort is replaced by device radix sorts.  Entries with
// an out-of-range index or a non-finite / negative distance are skipped (the
// reference CUDA ABI skips them too; the CPU reference rejects such input).
#include "tsne.cuh"

#include <cub/cub.cuh>

#include <cfloat>
#include <cmath>
#include <vector>

namespace fe {
namespace {

// Edge keys pack (row, col) as row << sh | col with sh = bits(n), so both
// radix sorts run over 2 sh bits (40 at n = 1M) instead of 64; the key with
// every one of those bits set marks a dropped entry and sorts last (a valid
// key is at most (n - 1) << sh | (n - 1) < 2^(2 sh) - 1).
struct KeyPack {
  int sh;
  unsigned long long none;
  unsigned long long mask;
};

inline KeyPack key_pack(int n) {
  int sh = 1;
  while (sh < 31 && (1ll << sh) <= static_cast<long long>(n)) ++sh;
  return KeyPack{sh, (1ull << (2 * sh)) - 1ull, (1ull << sh) - 1ull};
}

template <typename DistT>
__device__ __forceinline__ bool entry_valid(int nb, float d, int n) {
  return nb >= 0 && nb < n && isfinite(d) && d >= 0.0f;
}

// One thread per row; distances/indices are R column-major (entry j of row i at j*n+i),
// so consecutive threads read consecutive addresses.
template <typename DistT>
__global__ void row_affinity_kernel(const int* __restrict__ idx, const DistT* __restrict__ dist,
                                    int n, int k, int offset, float log_perp, KeyPack kp,
                                    unsigned long long* __restrict__ keys,
                                    float* __restrict__ vals) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= n) return;
  const size_t nn = static_cast<size_t>(n);

  float beta = 1.0f;
  float min_beta = -FLT_MAX;
  float max_beta = FLT_MAX;
  const float tol = 1e-5f;
  float sum_p = FLT_MIN;
  float used_beta = beta;  // beta of the last evaluated pass (the reference keeps those p_j)
  bool found = false;
  for (int iter = 0; !found && iter < 200; ++iter) {
    used_beta = beta;
    sum_p = FLT_MIN;
    float entropy = 0.0f;
    // Two passes as in the reference (the second re-reads p_j = exp(-beta d^2)).
    for (int j = 0; j < k; ++j) {
      const int nb = idx[j * nn + row] - offset;
      const float d = static_cast<float>(dist[j * nn + row]);
      if (!entry_valid<DistT>(nb, d, n)) continue;
      sum_p += expf(-beta * (d * d));
    }
    for (int j = 0; j < k; ++j) {
      const int nb = idx[j * nn + row] - offset;
      const float d = static_cast<float>(dist[j * nn + row]);
      if (!entry_valid<DistT>(nb, d, n)) continue;
      const float p = expf(-beta * (d * d));
      entropy += beta * (d * d * p);
    }
    entropy = entropy / sum_p + logf(sum_p);
    const float diff = entropy - log_perp;
    if (fabsf(diff) < tol) {
      found = true;
    } else if (diff > 0.0f) {
      min_beta = beta;
      beta = (max_beta == FLT_MAX || max_beta == -FLT_MAX) ? beta * 2.0f : (beta + max_beta) * 0.5f;
    } else {
      max_beta = beta;
      beta = (min_beta == -FLT_MAX || min_beta == FLT_MAX) ? beta * 0.5f : (beta + min_beta) * 0.5f;
    }
  }
  const float inv_sum_p = 1.0f / sum_p;
  for (int j = 0; j < k; ++j) {
    const int nb = idx[j * nn + row] - offset;
    const float d = static_cast<float>(dist[j * nn + row]);
    const size_t slot = j * nn + row;
    if (!entry_valid<DistT>(nb, d, n) || nb == row) {
      keys[slot] = kp.none;
      vals[slot] = 0.0f;
      continue;
    }
    const unsigned int a = static_cast<unsigned int>(min(row, nb));
    const unsigned int b = static_cast<unsigned int>(max(row, nb));
    keys[slot] = (static_cast<unsigned long long>(a) << kp.sh) | b;
    vals[slot] = expf(-used_beta * (d * d)) * inv_sum_p;
  }
}

__global__ void mark_heads_kernel(const unsigned long long* __restrict__ keys, long long m, KeyPack kp,
                                  int* __restrict__ flags) {
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i >= m) return;
  const unsigned long long key = keys[i];
  flags[i] = (key != kp.none && (i == 0 || keys[i - 1] != key)) ? 1 : 0;
}

// Sums each run of equal keys in double (src/tsne_neighbors.cpp:601-617).
__global__ void reduce_runs_kernel(const unsigned long long* __restrict__ keys,
                                   const float* __restrict__ vals, const int* __restrict__ flags,
                                   const int* __restrict__ pos, long long m,
                                   unsigned long long* __restrict__ ukeys,
                                   float* __restrict__ uvals, double* __restrict__ total) {
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  double local = 0.0;
  if (i < m && flags[i]) {
    const unsigned long long key = keys[i];
    double sum = 0.0;
    for (long long t = i; t < m && keys[t] == key; ++t) sum += static_cast<double>(vals[t]);
    ukeys[pos[i]] = key;
    uvals[pos[i]] = static_cast<float>(sum);
    local = sum;
  }
  local = warp_sum(local);
  __shared__ double warp_part[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) warp_part[wid] = local;
  __syncthreads();
  if (wid == 0) {
    double v = lane < (blockDim.x >> 5) ? warp_part[lane] : 0.0;
    v = warp_sum(v);
    if (lane == 0 && v != 0.0) atomicAdd(total, v);
  }
}

__global__ void expand_pairs_kernel(const unsigned long long* __restrict__ ukeys,
                                    const float* __restrict__ uvals, long long u, float norm, KeyPack kp,
                                    unsigned long long* __restrict__ keys2,
                                    float* __restrict__ vals2) {
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i >= u) return;
  const unsigned long long key = ukeys[i];
  const unsigned long long a = key >> kp.sh, b = key & kp.mask;
  const float v = uvals[i] * norm;
  keys2[2 * i] = (a << kp.sh) | b;
  keys2[2 * i + 1] = (b << kp.sh) | a;
  vals2[2 * i] = v;
  vals2[2 * i + 1] = v;
}

// row_start[r] = first entry of row r in the (row, col)-sorted list.
__global__ void row_bounds_kernel(const unsigned long long* __restrict__ keys, long long m, int n, KeyPack kp,
                                  int* __restrict__ row_start) {
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i > m) return;
  const int r = i < m ? static_cast<int>(keys[i] >> kp.sh) : n;
  const int rp = i == 0 ? -1 : static_cast<int>(keys[i - 1] >> kp.sh);
  for (int t = rp + 1; t <= r; ++t) row_start[t] = static_cast<int>(i);
}

__global__ void split_keys_kernel(const unsigned long long* __restrict__ keys, long long m, KeyPack kp,
                                  int* __restrict__ col) {
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i < m) col[i] = static_cast<int>(keys[i] & kp.mask);
}

template <typename T>
struct DevBuf {
  T* p = nullptr;
  ~DevBuf() {
    if (p) fe::dev_free(p);
  }
  int alloc(size_t count, const char* what) {
    return check_cuda(fe::dev_malloc(reinterpret_cast<void**>(&p), sizeof(T) * (count ? count : 1)), what);
  }
  T* release() {
    T* q = p;
    p = nullptr;
    return q;
  }
};

inline unsigned blocks_for(long long m, int threads) {
  return static_cast<unsigned>((m + threads - 1) / threads);
}

// Sorted (row, col) entry list -> CSR; the values array is adopted as is.
int assemble_csr(const unsigned long long* d_keys, float* d_vals, long long m, int n, KeyPack kp,
                 cudaStream_t stream, int** out_row_ptr, int** out_col) {
  DevBuf<int> row_ptr, col;
  FE_TRY(row_ptr.alloc(n + 1, "cudaMalloc(row_ptr)"));
  FE_TRY(col.alloc(m, "cudaMalloc(P col)"));
  row_bounds_kernel<<<blocks_for(m + 1, 256), 256, 0, stream>>>(d_keys, m, n, kp, row_ptr.p);
  FE_LAUNCH("row_bounds_kernel");
  split_keys_kernel<<<blocks_for(m, 256), 256, 0, stream>>>(d_keys, m, kp, col.p);
  FE_LAUNCH("split_keys_kernel");
  FE_CUDA(cudaStreamSynchronize(stream), "cudaStreamSynchronize(P assemble)");
  *out_row_ptr = row_ptr.release();
  *out_col = col.release();
  (void)d_vals;
  return 0;
}

}  // namespace

int build_p_device(const int* d_idx, const void* d_dist, bool dist_is_double, int n, int k,
                   int index_offset, float perplexity, cudaStream_t stream, int** out_row_ptr,
                   int** out_col, float** out_val, long long* out_nnz) {
  const long long m = static_cast<long long>(n) * k;
  if (m >= (1ll << 31) - 1) {
    set_error("t-SNE affinities: n*k exceeds the 32-bit entry range");
    return 1;
  }
  DevBuf<unsigned long long> keys, keys_sorted;
  DevBuf<float> vals, vals_sorted;
  FE_TRY(keys.alloc(m, "cudaMalloc(edge keys)"));
  FE_TRY(vals.alloc(m, "cudaMalloc(edge values)"));
  const float log_perp = static_cast<float>(std::log(static_cast<double>(perplexity)));
  const KeyPack kp = key_pack(n);
  if (dist_is_double) {
    row_affinity_kernel<double><<<blocks_for(n, 128), 128, 0, stream>>>(
        d_idx, static_cast<const double*>(d_dist), n, k, index_offset, log_perp, kp, keys.p, vals.p);
  } else {
    row_affinity_kernel<float><<<blocks_for(n, 128), 128, 0, stream>>>(
        d_idx, static_cast<const float*>(d_dist), n, k, index_offset, log_perp, kp, keys.p, vals.p);
  }
  FE_LAUNCH("row_affinity_kernel");

  FE_TRY(keys_sorted.alloc(m, "cudaMalloc(sorted keys)"));
  FE_TRY(vals_sorted.alloc(m, "cudaMalloc(sorted values)"));
  size_t temp_bytes = 0;
  FE_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, temp_bytes, keys.p, keys_sorted.p, vals.p,
                                          vals_sorted.p, static_cast<int>(m), 0, 2 * kp.sh, stream),
          "cub::DeviceRadixSort(sizing)");
  {
    DevBuf<unsigned char> temp;
    FE_TRY(temp.alloc(temp_bytes, "cudaMalloc(sort temp)"));
    FE_CUDA(cub::DeviceRadixSort::SortPairs(temp.p, temp_bytes, keys.p, keys_sorted.p, vals.p,
                                            vals_sorted.p, static_cast<int>(m), 0, 2 * kp.sh, stream),
            "cub::DeviceRadixSort(pair keys)");
    FE_CUDA(cudaStreamSynchronize(stream), "cudaStreamSynchronize(pair sort)");
  }
  // Merge equal pairs.
  DevBuf<int> flags, pos;
  FE_TRY(flags.alloc(m, "cudaMalloc(head flags)"));
  FE_TRY(pos.alloc(m, "cudaMalloc(head positions)"));
  mark_heads_kernel<<<blocks_for(m, 256), 256, 0, stream>>>(keys_sorted.p, m, kp, flags.p);
  FE_LAUNCH("mark_heads_kernel");
  FE_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, temp_bytes, flags.p, pos.p, static_cast<int>(m), stream),
          "cub::DeviceScan(sizing)");
  {
    DevBuf<unsigned char> temp;
    FE_TRY(temp.alloc(temp_bytes, "cudaMalloc(scan temp)"));
    FE_CUDA(cub::DeviceScan::ExclusiveSum(temp.p, temp_bytes, flags.p, pos.p, static_cast<int>(m), stream),
            "cub::DeviceScan(head positions)");
  }
  int last_pos = 0, last_flag = 0;
  FE_CUDA(cudaMemcpyAsync(&last_pos, pos.p + (m - 1), sizeof(int), cudaMemcpyDeviceToHost, stream), "D2H");
  FE_CUDA(cudaMemcpyAsync(&last_flag, flags.p + (m - 1), sizeof(int), cudaMemcpyDeviceToHost, stream), "D2H");
  FE_CUDA(cudaStreamSynchronize(stream), "cudaStreamSynchronize(head scan)");
  const long long u = static_cast<long long>(last_pos) + last_flag;
  if (u == 0) {
    set_error("KNN graph produced no non-self t-SNE edges.");
    return 1;
  }
  DevBuf<unsigned long long> ukeys;
  DevBuf<float> uvals;
  DevBuf<double> total;
  FE_TRY(ukeys.alloc(u, "cudaMalloc(unique pairs)"));
  FE_TRY(uvals.alloc(u, "cudaMalloc(unique values)"));
  FE_TRY(total.alloc(1, "cudaMalloc(total mass)"));
  FE_CUDA(cudaMemsetAsync(total.p, 0, sizeof(double), stream), "cudaMemsetAsync(total)");
  reduce_runs_kernel<<<blocks_for(m, 256), 256, 0, stream>>>(keys_sorted.p, vals_sorted.p, flags.p,
                                                            pos.p, m, ukeys.p, uvals.p, total.p);
  FE_LAUNCH("reduce_runs_kernel");
  double total_mass = 0.0;
  FE_CUDA(cudaMemcpyAsync(&total_mass, total.p, sizeof(double), cudaMemcpyDeviceToHost, stream), "D2H");
  FE_CUDA(cudaStreamSynchronize(stream), "cudaStreamSynchronize(total)");
  if (!std::isfinite(total_mass) || total_mass <= 0.0) {
    set_error("t-SNE probability normalization failed.");
    return 1;
  }
  const float norm = static_cast<float>(0.5 / total_mass);
  // Release the first-stage buffers before the second sort.
  fe::dev_free(keys.release());
  fe::dev_free(vals.release());
  fe::dev_free(flags.release());
  fe::dev_free(pos.release());

  const long long m2 = 2 * u;
  DevBuf<unsigned long long> k2, k2s;
  DevBuf<float> v2, v2s;
  FE_TRY(k2.alloc(m2, "cudaMalloc(directed keys)"));
  FE_TRY(v2.alloc(m2, "cudaMalloc(directed values)"));
  expand_pairs_kernel<<<blocks_for(u, 256), 256, 0, stream>>>(ukeys.p, uvals.p, u, norm, kp, k2.p, v2.p);
  FE_LAUNCH("expand_pairs_kernel");
  fe::dev_free(ukeys.release());
  fe::dev_free(uvals.release());
  fe::dev_free(keys_sorted.release());
  fe::dev_free(vals_sorted.release());
  FE_TRY(k2s.alloc(m2, "cudaMalloc(sorted directed keys)"));
  FE_TRY(v2s.alloc(m2, "cudaMalloc(sorted directed values)"));
  FE_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, temp_bytes, k2.p, k2s.p, v2.p, v2s.p,
                                          static_cast<int>(m2), 0, 2 * kp.sh, stream),
          "cub::DeviceRadixSort(sizing)");
  {
    DevBuf<unsigned char> temp;
    FE_TRY(temp.alloc(temp_bytes, "cudaMalloc(sort temp)"));
    FE_CUDA(cub::DeviceRadixSort::SortPairs(temp.p, temp_bytes, k2.p, k2s.p, v2.p, v2s.p,
                                            static_cast<int>(m2), 0, 2 * kp.sh, stream),
            "cub::DeviceRadixSort(directed keys)");
    FE_CUDA(cudaStreamSynchronize(stream), "cudaStreamSynchronize(directed sort)");
  }
  FE_TRY(assemble_csr(k2s.p, v2s.p, m2, n, kp, stream, out_row_ptr, out_col));
  *out_val = v2s.release();
  *out_nnz = m2;
  return 0;
}

int upload_csr(const int* row_ptr, const int* col, const float* val, int n, cudaStream_t stream,
               int** out_row_ptr, int** out_col, float** out_val, long long* out_nnz) {
  if (row_ptr[0] != 0) {
    set_error("CSR row_ptr must start at 0");
    return 1;
  }
  for (int r = 0; r < n; ++r) {
    if (row_ptr[r + 1] < row_ptr[r]) {
      set_error("CSR row_ptr is not monotone");
      return 1;
    }
  }
  const size_t nnz = static_cast<size_t>(row_ptr[n]);
  for (size_t t = 0; t < nnz; ++t) {
    if (col[t] < 0 || col[t] >= n) {
      set_error("CSR column index out of range");
      return 1;
    }
  }
  DevBuf<int> d_rp, d_c;
  DevBuf<float> d_v;
  FE_TRY(d_rp.alloc(n + 1, "cudaMalloc(row_ptr)"));
  FE_TRY(d_c.alloc(nnz, "cudaMalloc(col)"));
  FE_TRY(d_v.alloc(nnz, "cudaMalloc(val)"));
  FE_CUDA(cudaMemcpyAsync(d_rp.p, row_ptr, sizeof(int) * (n + 1), cudaMemcpyHostToDevice, stream), "H2D row_ptr");
  FE_TRY(h2d_copy(d_c.p, col, sizeof(int) * nnz, stream, "H2D col"));
  FE_TRY(h2d_copy(d_v.p, val, sizeof(float) * nnz, stream, "H2D val"));
  FE_CUDA(cudaStreamSynchronize(stream), "cudaStreamSynchronize(csr upload)");
  *out_row_ptr = d_rp.release();
  *out_col = d_c.release();
  *out_val = d_v.release();
  *out_nnz = static_cast<long long>(nnz);
  return 0;
}

}  // namespace fe
