// Exact Euclidean KNN on the device: the producer of the GPU-KNN contract the
// optimizer's device-KNN entry points consume (the reference builds it with
// FAISS / cuVS brute force, src/native_knn_cuda_impl.cpp:511-700, and its own
// finalize kernel, src/embedding_cuda_kernels.cpp:1412-1464 / 3767-3836):
// int32 indices (1-based) and float32 Euclidean distances of the k nearest
// non-self points, column-major n x k, in device memory.
//
// B200 design: every block owns kQueries query points and streams the whole
// data set through shared memory in tiles of kTile points, 64 features at a
// time (double-buffered with cp.async).  Each thread forms 2 x 8 dot products
// per tile (FP32 FMA) and ranks points by |x|^2 - 2 q.x (|q|^2
// is common to a query); a point below the query's current threshold -- the
// (k_sel)-th best so far -- is appended to the query's candidate array in
// shared memory.  When an array could overflow on the next tile, each warp
// sorts its queries' arrays (bitonic, in shared memory) and keeps the best
// k_sel, which also lowers the thresholds.  At the end the k + 1 + kMargin
// best candidates are re-ranked by the exact sum of (q - x)^2 in double, self
// is skipped (the reference's exclude_self rule: the query's own index), and
// the first k are written.  kMargin absorbs the rounding of the dot-product
// form near the k-th distance.
#include "fe_common.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <climits>
#include <string>

namespace fe {
namespace {

constexpr int kQueries = 32;    // queries per block
constexpr int kTile = 128;      // data points per tile
constexpr int kKnnThreads = 256;
constexpr int kMargin = 8;      // extra candidates re-ranked exactly
constexpr int kMaxK = 256;      // kMaxNativeCudaK, src/native_knn_cuda_impl.cpp:64

struct Cand {
  float d;
  int i;
};

// Row-major float copy of the data, features padded to a multiple of 4 with
// zeros, and the squared norms.
template <typename T>
__global__ void knn_pack_kernel(const T* __restrict__ x, int n, int p, int pp, int col_major,
                                float* __restrict__ out, float* __restrict__ norms) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  double s = 0.0;
  for (int f = 0; f < pp; ++f) {
    float v = 0.0f;
    if (f < p) v = static_cast<float>(col_major ? x[static_cast<size_t>(f) * n + i] : x[static_cast<size_t>(i) * p + f]);
    out[static_cast<size_t>(i) * pp + f] = v;
    s += static_cast<double>(v) * v;
  }
  norms[i] = static_cast<float>(s);
}

__device__ __forceinline__ bool cand_less(const Cand& a, const Cand& b) {
  return a.d < b.d || (a.d == b.d && a.i < b.i);
}

// Bitonic sort of `len` (a power of two) candidates by one warp.
__device__ void warp_bitonic_sort(Cand* a, int len) {
  const int lane = threadIdx.x & 31;
  for (int size = 2; size <= len; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int t = lane; t < (len >> 1); t += 32) {
        const int lo = 2 * stride * (t / stride) + (t % stride);
        const int hi = lo + stride;
        const bool up = ((lo & size) == 0);
        Cand x = a[lo], y = a[hi];
        if (cand_less(y, x) == up) {
          a[lo] = y;
          a[hi] = x;
        }
      }
      __syncwarp();
    }
  }
}

constexpr int kChunk = 64;  // features per step (a multiple of 4)
// Shared-memory row stride of the data tile: 16 bytes past a multiple of 128,
// so the 16 rows a warp reads with one 16-byte load fall on distinct banks
// (a 256-byte stride put all 16 on the same ones).
constexpr int kRowStride = kChunk + 4;

// Steps run over (tile, feature chunk): the data chunk [kTile][cw] and the
// query chunk [cw][kQueries] of step s + 1 are copied (cp.async) while step s
// is computed; the dot products of a tile accumulate across its chunks.
__global__ void __launch_bounds__(kKnnThreads) knn_kernel(const float* __restrict__ data, const float* __restrict__ norms,
                                                          int n, int pp, int k_sel, int cap, int k_out, int exclude_self,
                                                          int* __restrict__ out_idx, float* __restrict__ out_dist) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* xs = reinterpret_cast<float*>(smem);                        // 2 x [kTile][kRowStride]
  float* qs = xs + 2 * kTile * kRowStride;                           // 2 x [kChunk][kQueries]
  float* xn = qs + 2 * kChunk * kQueries;                            // [kTile] norms of the current tile
  Cand* cands = reinterpret_cast<Cand*>(xn + kTile);                 // [kQueries][cap]
  __shared__ int s_count[kQueries];
  __shared__ float s_tau[kQueries];
  __shared__ int s_merge;
  const int tid = threadIdx.x;
  const int lane = tid & 31, wid = tid >> 5;
  const int q0 = blockIdx.x * kQueries;
  for (int t = tid; t < kQueries * cap; t += kKnnThreads) cands[t] = Cand{FLT_MAX, INT_MAX};
  if (tid < kQueries) {
    s_count[tid] = 0;
    s_tau[tid] = FLT_MAX;
  }
  const int tiles = (n + kTile - 1) / kTile;
  const int chunks = (pp + kChunk - 1) / kChunk;
  const int steps = tiles * chunks;
  auto load_step = [&](int step, int buf) {
    const int tile = step / chunks, c = step - (step / chunks) * chunks;
    const int base = tile * kTile, f0 = c * kChunk;
    const int cw = min(kChunk, pp - f0);
    const int vec = cw / 4;
    float* xd = xs + buf * kTile * kRowStride;
    for (int t = tid; t < kTile * vec; t += kKnnThreads) {
      const int pnt = t / vec, v = t - (t / vec) * vec;
      float4* d4 = reinterpret_cast<float4*>(xd + pnt * kRowStride) + v;
      if (base + pnt < n) {
        const float4* s4 = reinterpret_cast<const float4*>(data + static_cast<size_t>(base + pnt) * pp + f0) + v;
        const unsigned int sa = static_cast<unsigned int>(__cvta_generic_to_shared(d4));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(s4) : "memory");
      } else {
        *d4 = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    float* qd = qs + buf * kChunk * kQueries;
    for (int t = tid; t < kQueries * cw; t += kKnnThreads) {
      const int q = t / cw, f = t - (t / cw) * cw;
      float* d = qd + f * kQueries + q;
      if (q0 + q < n) {
        const unsigned int sa = static_cast<unsigned int>(__cvta_generic_to_shared(d));
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(sa),
                     "l"(data + static_cast<size_t>(q0 + q) * pp + f0 + f) : "memory");
      } else {
        *d = 0.0f;
      }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };
  // thread layout: 16 query pairs x 16 point lanes; a thread owns queries
  // {2*qy, 2*qy+1} and points {px + 16*j, j < 8} of each tile
  const int qy = tid >> 4, px = tid & 15;
  float acc[2][8];
  load_step(0, 0);
  for (int step = 0; step < steps; ++step) {
    const int buf = step & 1;
    const int tile = step / chunks, c = step - (step / chunks) * chunks;
    const int base = tile * kTile;
    const int cw = min(kChunk, pp - c * kChunk);
    if (c == 0) {
#pragma unroll
      for (int a = 0; a < 2; ++a) {
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[a][j] = 0.0f;
      }
      if (tid < kTile) xn[tid] = base + tid < n ? norms[base + tid] : FLT_MAX;
    }
    if (step + 1 < steps) {
      load_step(step + 1, buf ^ 1);
      asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    }
    __syncthreads();
    const float* xt = xs + buf * kTile * kRowStride;
    const float* qt = qs + buf * kChunk * kQueries;
    for (int f = 0; f < cw; f += 4) {
      float4 xv[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) xv[j] = *reinterpret_cast<const float4*>(xt + (px + 16 * j) * kRowStride + f);
#pragma unroll
      for (int ff = 0; ff < 4; ++ff) {
        const float2 qq = *reinterpret_cast<const float2*>(qt + (f + ff) * kQueries + 2 * qy);
        const float qa = qq.x;
        const float qb = qq.y;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float xf = ff == 0 ? xv[j].x : (ff == 1 ? xv[j].y : (ff == 2 ? xv[j].z : xv[j].w));
          acc[0][j] = fmaf(qa, xf, acc[0][j]);
          acc[1][j] = fmaf(qb, xf, acc[1][j]);
        }
      }
    }
    if (c + 1 < chunks) {
      __syncthreads();  // the buffer is refilled by the step after next
      continue;
    }
#pragma unroll
    for (int a = 0; a < 2; ++a) {
      const int q = 2 * qy + a;
      const float tau = s_tau[q];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int pnt = px + 16 * j;
        const float score = xn[pnt] - 2.0f * acc[a][j];
        if (base + pnt < n && score < tau) {
          const int pos = atomicAdd(&s_count[q], 1);
          cands[q * cap + k_sel + pos] = Cand{score, base + pnt};
        }
      }
    }
    __syncthreads();
    // Merge when the next tile could overflow some array (at most kTile
    // appends per query per tile), and after the last tile.
    if (tid == 0) {
      int need = 0;
      for (int q = 0; q < kQueries; ++q) need |= (s_count[q] > cap - k_sel - 2 * kTile);
      s_merge = need || tile + 1 == tiles;
    }
    __syncthreads();
    if (s_merge) {
      for (int q = wid; q < kQueries; q += kKnnThreads / 32) {
        Cand* a = cands + q * cap;
        warp_bitonic_sort(a, cap);
        for (int t = k_sel + lane; t < cap; t += 32) a[t] = Cand{FLT_MAX, INT_MAX};
        __syncwarp();
        if (lane == 0) {
          s_count[q] = 0;
          s_tau[q] = a[k_sel - 1].d;
        }
      }
      __syncthreads();
    }
  }
  // Exact re-ranking of the k_sel best, self skipped, first k_out written.
  for (int q = wid; q < kQueries; q += kKnnThreads / 32) {
    const int qi = q0 + q;
    if (qi >= n) continue;
    Cand* a = cands + q * cap;
    const float* xq = data + static_cast<size_t>(qi) * pp;
    for (int t = lane; t < k_sel; t += 32) {
      const int j = a[t].i;
      if (j < 0 || j >= n || (exclude_self && j == qi)) {
        a[t] = Cand{FLT_MAX, INT_MAX};
        continue;
      }
      double s = 0.0;
      const float* xj = data + static_cast<size_t>(j) * pp;
      for (int f = 0; f < pp; ++f) {
        const double d = static_cast<double>(xq[f]) - static_cast<double>(xj[f]);
        s += d * d;
      }
      a[t] = Cand{static_cast<float>(sqrt(s)), j};
    }
    for (int t = k_sel + lane; t < cap; t += 32) a[t] = Cand{FLT_MAX, INT_MAX};
    __syncwarp();
    warp_bitonic_sort(a, cap);
    for (int t = lane; t < k_out; t += 32) {
      const Cand c = a[t];
      const size_t o = static_cast<size_t>(t) * n + qi;
      out_idx[o] = c.i == INT_MAX ? 0 : c.i + 1;  // 1-based; 0 marks a missing neighbour
      out_dist[o] = c.i == INT_MAX ? FLT_MAX : c.d;
    }
  }
}

}  // namespace

int knn_exact(const void* data, bool data_double, bool data_on_device, bool col_major, int n, int p, int k,
              bool exclude_self, int* d_indices, float* d_distances, cudaStream_t st) {
  if (data == nullptr || d_indices == nullptr || d_distances == nullptr) {
    set_error("null pointer in CUDA exact KNN");
    return 1;
  }
  if (n < 2 || p < 1 || k < 1 || k > kMaxK || k >= n) {
    set_error("CUDA exact KNN requires n >= 2, p >= 1 and k in [1, min(n - 1, 256)]");
    return 1;
  }
  const int pp = (p + 3) / 4 * 4;
  const int k_sel = std::min(n, k + 1 + kMargin);
  int cap = 1;
  while (cap < k_sel + 2 * kTile) cap <<= 1;
  const size_t smem = sizeof(float) * (2 * static_cast<size_t>(kTile) * kRowStride +
                                       2 * static_cast<size_t>(kChunk) * kQueries + kTile) +
                      sizeof(Cand) * static_cast<size_t>(kQueries) * cap;
  int dev = 0, max_smem = 0;
  FE_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  FE_CUDA(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev), "cudaDeviceGetAttribute");
  if (smem + 1024 > static_cast<size_t>(max_smem)) {
    set_error("CUDA exact KNN: k = " + std::to_string(k) + " exceeds the shared-memory candidate arrays");
    return 1;
  }
  const size_t elt = data_double ? sizeof(double) : sizeof(float);
  Arena a;
  void* raw = nullptr;
  float* packed = nullptr;
  float* norms = nullptr;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 0) a.begin_plan();
    else a.rewind();
    raw = data_on_device ? nullptr : a.take<char>(static_cast<size_t>(n) * p * elt);
    packed = a.take<float>(static_cast<size_t>(n) * pp);
    norms = a.take<float>(n);
    if (pass == 0) {
      FE_TRY(memory_preflight(a.planned(), "CUDA exact KNN workspace"));
      FE_TRY(a.commit("CUDA exact KNN workspace"));
    }
  }
  const void* src = data;
  if (!data_on_device) {
    FE_TRY(h2d_copy(raw, data, static_cast<size_t>(n) * p * elt, st, "H2D KNN data"));
    src = raw;
  }
  if (data_double) {
    knn_pack_kernel<double><<<(n + 255) / 256, 256, 0, st>>>(static_cast<const double*>(src), n, p, pp,
                                                             col_major ? 1 : 0, packed, norms);
  } else {
    knn_pack_kernel<float><<<(n + 255) / 256, 256, 0, st>>>(static_cast<const float*>(src), n, p, pp,
                                                            col_major ? 1 : 0, packed, norms);
  }
  FE_LAUNCH("knn_pack_kernel");
  FE_CUDA(cudaFuncSetAttribute(knn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)),
          "cudaFuncSetAttribute(knn_kernel)");
  knn_kernel<<<(n + kQueries - 1) / kQueries, kKnnThreads, smem, st>>>(packed, norms, n, pp, k_sel, cap, k,
                                                                       exclude_self ? 1 : 0, d_indices, d_distances);
  FE_LAUNCH("knn_kernel");
  FE_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize(KNN)");
  return 0;
}

}  // namespace fe
