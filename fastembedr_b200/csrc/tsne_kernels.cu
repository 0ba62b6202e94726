// Per-iteration kernels of the openTSNE FFT-grid optimizer.
//
// Algorithm (restating compute_gradient_fft_grid_f, src/tsne_neighbors.cpp:1076-1182,
// and apply_open_tsne_update_f / zero_mean_f, :1196-1245):
//   grad_i,d = -(y_i,d * phi_q2(y_i) - phi_dq2(y_i)) / Z + ex * sum_j P_ij q_ij (y_i,d - y_j,d)
// where phi_* are the bilinear charges {1, x, y} on a GxG grid convolved
// (linearly, zero-padded to 2G) with q = 1/(1+d^2) and q^2, and
// Z = sum_i interp(phi_q)(y_i) - n.  Because spread and gather use the same
// bilinear weights, Z = sum_nodes charge_1(node) * phi_q(node) - n, which the
// inverse FFT pass reduces directly.
//
// Kernels (all on the session stream):
//   splat_kernel           centres the layout in place and spreads {1,x,y};
//                          lanes sharing a cell combine first, then a block
//                          tile and 64-bit fixed-point atomics
//                          (order-independent, reproducible)
//   fft_rows_fwd_kernel    x-direction real FFTs of the charge rows and of the
//                          kernel rows (the kernels are even, so their
//                          transforms are real)
//   fft_cols_kernel        y-direction FFT, multiply by the real kernel
//                          spectra, inverse y-FFT -- one column tile per block
//   fft_rows_inv_kernel    inverse x-FFTs -> potentials, Z, and clears charges
//   grad_update_kernel     attraction (8 lanes per row, 32 for rounds with a
//                          hub row; 16-byte streaming loads, next pass
//                          prefetched; 32-row groups taken most expensive
//                          first), repulsive gather, gains / momentum / step
//                          clip, layout write
//   layout_stats_kernel    sums and bounds of the new layout in a fixed order;
//                          the last block derives the next grid geometry
#include "tsne.cuh"

#include <algorithm>
#include <cmath>
#include <cfloat>
#include <climits>

namespace fe {
namespace {

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 conjf2(float2 a) { return make_float2(a.x, -a.y); }
__device__ __forceinline__ float2 cscale(float2 a, float s) { return make_float2(a.x * s, a.y * s); }

// ---- shared-memory FFT
//
// In-place FFT of COUNT length-M sequences laid out back to back in shared
// memory, M = 2^LOG_M known at compile time (the three FFT kernels are
// instantiated for every grid side, 4 to 1024), so loop trips, shifts and
// masks are constants and every thread's loads are issued together.  Stockham
// radix 4, with a final radix-2 pass when LOG_M is odd: every pass reads each
// element once into registers, waits at one barrier, applies the twiddles
// w^q (q = 1, 2, 3; w = exp(-+2 pi i k / (4 ns))) and a 4-point DFT, and writes
// each element once to its Stockham position, so the output is in natural
// order without a bit-reversal pass.  The inverse is unnormalised.
//
// Twiddles: a table computed once per session on the host in double and
// rounded to float (fft_twiddle_table), copied into shared memory by every
// block.  Radix-4 pass p >= 1 (ns = 4^p) owns entries [4^p - 4, 4^(p+1) - 4):
// entry (q - 1) * ns + k holds w^q = exp(-2 pi i q k / (4 ns)), q = 1, 2, 3,
// so the lanes of a warp read consecutive entries and no twiddle is a product
// of rounded ones.  The radix-2 pass reads exp(-2 pi i j / M), j < M / 2,
// after them.  The inverse conjugates.
//
// Element i of the data buffer lives at sw(i): the low four index bits are
// XORed with 5 * ((i >> 4) & 3), so that the strided writes of the first two
// passes (ns = 1: stride 4; ns = 4: runs of 4 at stride 16) and the unit-
// stride reads and writes of every pass hit 16 different 8-byte bank pairs in
// each half-warp.  sw permutes each aligned run of 16 elements, and adding a
// multiple of 64 commutes with it.
constexpr int kFftBatch = 4;        // four-element groups per thread and pass: row passes
constexpr int kFftBatchCols = 2;    // column pass (twice the threads, so it needs no spills)

__device__ __forceinline__ int sw(int i) { return i ^ (((i >> 4) & 3) * 5); }

// Columns per block of the column pass: one once a transform fills a block,
// several for short ones (measured 1.9x faster than 4 per block at G = 256).
constexpr int fft_cols_per_block(int m) { return m >= 256 ? 1 : (2048 / m < 16 ? 2048 / m : 16); }

// Threads for a block holding `count` length-m sequences: enough for `batch`
// groups per thread and pass, and at least 256 (fewer only when there are
// fewer groups) so that short transforms keep eight warps.
constexpr int fft_threads_for(int count, int m, int batch) {
  const int groups = count * m / 4;
  const int need = (groups + batch - 1) / batch;
  const int floor_threads = groups < 64 ? 64 : (groups < 256 ? groups : 256);
  const int t = need > floor_threads ? need : floor_threads;
  return (t + 31) / 32 * 32;
}

constexpr int fft_tw4_entries(int log_m) { return (1 << (2 * (log_m / 2))) - 4; }
constexpr int fft_table_entries(int log_m) { return fft_tw4_entries(log_m) + ((log_m & 1) ? (1 << (log_m - 1)) : 0); }
constexpr int fft_data_entries(int count, int m) { return (count * m + 15) / 16 * 16; }

template <int LOG_M, int COUNT, int BATCH = kFftBatch>
struct FftShape {
  static constexpr int M = 1 << LOG_M;
  static constexpr int THREADS = fft_threads_for(COUNT, M, BATCH);
  static constexpr int DATA = fft_data_entries(COUNT, M);
  static constexpr int TABLE = fft_table_entries(LOG_M);
  static constexpr size_t SMEM = static_cast<size_t>(DATA + TABLE) * sizeof(float2);
  static_assert(THREADS <= 1024, "FFT block too large");
  static_assert((COUNT * M / 4 + THREADS - 1) / THREADS <= BATCH, "groups per thread");
};

template <int LOG_M, int THREADS>
__device__ __forceinline__ void fft_load_twiddles(const float2* __restrict__ table, float2* __restrict__ tw) {
#pragma unroll
  for (int i0 = 0; i0 < fft_table_entries(LOG_M); i0 += THREADS) {
    const int i = i0 + static_cast<int>(threadIdx.x);
    if (i < fft_table_entries(LOG_M)) tw[i] = __ldg(table + i);
  }
}

template <int LOG_M, int COUNT, int THREADS>
__device__ __forceinline__ void block_fft(float2* __restrict__ buf, const float2* __restrict__ tw, bool inverse) {
  constexpr int M = 1 << LOG_M;
  constexpr int QUARTER = M / 4;
  constexpr int LQ = LOG_M - 2;
  constexpr int GROUPS = COUNT * QUARTER;
  constexpr int BATCHES = (GROUPS + THREADS - 1) / THREADS;
  constexpr int PASSES = LOG_M / 2;
#pragma unroll
  for (int pass = 0; pass < PASSES; ++pass) {
    const int ns = 1 << (2 * pass);
    const int tw_off = ns - 4;
    float2 x[BATCHES][4];
#pragma unroll
    for (int b = 0; b < BATCHES; ++b) {
      const int t = static_cast<int>(threadIdx.x) + b * THREADS;
      if (GROUPS % THREADS == 0 || t < GROUPS) {
        const int src = ((t >> LQ) << LOG_M) + (t & (QUARTER - 1));
        if (QUARTER % 64 == 0) {
          const int s0 = sw(src);
#pragma unroll
          for (int q = 0; q < 4; ++q) x[b][q] = buf[s0 + q * QUARTER];
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) x[b][q] = buf[sw(src + q * QUARTER)];
        }
      }
    }
    __syncthreads();
#pragma unroll
    for (int b = 0; b < BATCHES; ++b) {
      const int t = static_cast<int>(threadIdx.x) + b * THREADS;
      if (GROUPS % THREADS == 0 || t < GROUPS) {
        const int j = t & (QUARTER - 1);
        const int k = j & (ns - 1);
        if (pass > 0) {
#pragma unroll
          for (int q = 1; q < 4; ++q) {
            float2 w = tw[tw_off + (q - 1) * ns + k];
            if (inverse) w.y = -w.y;
            x[b][q] = cmul(x[b][q], w);
          }
        }
        const float2 a0 = cadd(x[b][0], x[b][2]);
        const float2 a1 = csub(x[b][0], x[b][2]);
        const float2 a2 = cadd(x[b][1], x[b][3]);
        const float2 d = csub(x[b][1], x[b][3]);
        const float2 a3 = inverse ? make_float2(-d.y, d.x) : make_float2(d.y, -d.x);  // +-i d
        const float2 y[4] = {cadd(a0, a2), cadd(a1, a3), csub(a0, a2), csub(a1, a3)};
        const int dst = ((t >> LQ) << LOG_M) + ((j - k) << 2) + k;
        if (ns % 64 == 0) {
          const int d0 = sw(dst);
#pragma unroll
          for (int q = 0; q < 4; ++q) buf[d0 + q * ns] = y[q];
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) buf[sw(dst + q * ns)] = y[q];
        }
      }
    }
    __syncthreads();
  }
  if (LOG_M & 1) {
    // Last pass, radix 2 with span M / 2: each thread owns the pair (j, j + M/2).
    constexpr int HALF = M / 2;
    constexpr int TW4 = fft_tw4_entries(LOG_M);
#pragma unroll
    for (int t0 = 0; t0 < COUNT * HALF; t0 += THREADS) {
      const int t = t0 + static_cast<int>(threadIdx.x);
      if ((COUNT * HALF) % THREADS == 0 || t < COUNT * HALF) {
        const int j = t & (HALF - 1);
        const int base = (t >> (LOG_M - 1)) << LOG_M;
        float2 w = tw[TW4 + j];
        if (inverse) w.y = -w.y;
        const int i0 = sw(base + j);
        const int i1 = HALF % 64 == 0 ? i0 + HALF : sw(base + j + HALF);
        const float2 a = buf[i0];
        const float2 b = cmul(buf[i1], w);
        buf[i0] = cadd(a, b);
        buf[i1] = csub(a, b);
      }
    }
    __syncthreads();
  }
}

// Kernel value at integer offsets (dx, dy), formed in float exactly as
// src/tsne_neighbors.cpp:912-920 forms it.
__device__ __forceinline__ void kernel_values(int dx, int dy, float spacing, float* q, float* q2) {
  const float x_off = static_cast<float>(dx) * spacing;
  const float y_off = static_cast<float>(dy) * spacing;
  const float d2 = x_off * x_off + y_off * y_off;
  const float qq = 1.0f / (1.0f + d2);
  *q = qq;
  *q2 = qq * qq;
}

// ------------------------------------------------------------------ stats

struct StatsAcc {
  double sx, sy;
  float mnx, mxx, mny, mxy;
};

__device__ __forceinline__ void stats_init(StatsAcc& a) {
  a.sx = 0.0;
  a.sy = 0.0;
  a.mnx = FLT_MAX;
  a.mxx = -FLT_MAX;
  a.mny = FLT_MAX;
  a.mxy = -FLT_MAX;
}

__device__ __forceinline__ void stats_add(StatsAcc& a, float2 p) {
  a.sx += static_cast<double>(p.x);
  a.sy += static_cast<double>(p.y);
  a.mnx = fminf(a.mnx, p.x);
  a.mxx = fmaxf(a.mxx, p.x);
  a.mny = fminf(a.mny, p.y);
  a.mxy = fmaxf(a.mxy, p.y);
}

// Block-reduces `a`, writes the block partial, and lets the last block to
// finish fold all partials into *stats.  No block waits on another.
__device__ void stats_block_finish(StatsAcc a, double* __restrict__ partials,
                                   LayoutStats* __restrict__ stats, unsigned int* counter,
                                   int center, int n, int g) {
  __shared__ double s_d[2][32];
  __shared__ float s_f[4][32];
  __shared__ bool s_last;
  a.sx = warp_sum(a.sx);
  a.sy = warp_sum(a.sy);
  a.mnx = warp_min(a.mnx);
  a.mxx = warp_max(a.mxx);
  a.mny = warp_min(a.mny);
  a.mxy = warp_max(a.mxy);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (lane == 0) {
    s_d[0][wid] = a.sx;
    s_d[1][wid] = a.sy;
    s_f[0][wid] = a.mnx;
    s_f[1][wid] = a.mxx;
    s_f[2][wid] = a.mny;
    s_f[3][wid] = a.mxy;
  }
  __syncthreads();
  if (wid == 0) {
    double sx = lane < nw ? s_d[0][lane] : 0.0;
    double sy = lane < nw ? s_d[1][lane] : 0.0;
    float mnx = lane < nw ? s_f[0][lane] : FLT_MAX;
    float mxx = lane < nw ? s_f[1][lane] : -FLT_MAX;
    float mny = lane < nw ? s_f[2][lane] : FLT_MAX;
    float mxy = lane < nw ? s_f[3][lane] : -FLT_MAX;
    sx = warp_sum(sx);
    sy = warp_sum(sy);
    mnx = warp_min(mnx);
    mxx = warp_max(mxx);
    mny = warp_min(mny);
    mxy = warp_max(mxy);
    if (lane == 0) {
      double* p = partials + 6 * blockIdx.x;
      p[0] = sx;
      p[1] = sy;
      p[2] = mnx;
      p[3] = mxx;
      p[4] = mny;
      p[5] = mxy;
      __threadfence();
      const unsigned int ticket = atomicAdd(counter, 1u);
      s_last = ticket == gridDim.x - 1;
    }
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  StatsAcc t;
  stats_init(t);
  for (int b = threadIdx.x; b < static_cast<int>(gridDim.x); b += blockDim.x) {
    const volatile double* p = partials + 6 * b;
    t.sx += p[0];
    t.sy += p[1];
    t.mnx = fminf(t.mnx, static_cast<float>(p[2]));
    t.mxx = fmaxf(t.mxx, static_cast<float>(p[3]));
    t.mny = fminf(t.mny, static_cast<float>(p[4]));
    t.mxy = fmaxf(t.mxy, static_cast<float>(p[5]));
  }
  t.sx = warp_sum(t.sx);
  t.sy = warp_sum(t.sy);
  t.mnx = warp_min(t.mnx);
  t.mxx = warp_max(t.mxx);
  t.mny = warp_min(t.mny);
  t.mxy = warp_max(t.mxy);
  __syncthreads();
  if (lane == 0) {
    s_d[0][wid] = t.sx;
    s_d[1][wid] = t.sy;
    s_f[0][wid] = t.mnx;
    s_f[1][wid] = t.mxx;
    s_f[2][wid] = t.mny;
    s_f[3][wid] = t.mxy;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    StatsAcc r;
    stats_init(r);
    for (int w = 0; w < nw; ++w) {
      r.sx += s_d[0][w];
      r.sy += s_d[1][w];
      r.mnx = fminf(r.mnx, s_f[0][w]);
      r.mxx = fmaxf(r.mxx, s_f[1][w]);
      r.mny = fminf(r.mny, s_f[2][w]);
      r.mxy = fmaxf(r.mxy, s_f[3][w]);
    }
    stats->sum_x = r.sx;
    stats->sum_y = r.sy;
    stats->min_x = r.mnx;
    stats->max_x = r.mxx;
    stats->min_y = r.mny;
    stats->max_y = r.mxy;
    stats->center = center;
    const GridGeom q = grid_geometry(*stats, n, g);
    stats->geom = q;
    stats->scales = charge_scales(q, n, g);
    *counter = 0u;
  }
}

// Two points per 16-byte load; a fixed grid and fixed reduction order, so the
// result depends only on the layout.
__global__ void __launch_bounds__(512) layout_stats_kernel(const float2* __restrict__ y, int n, int g,
                                                           double* partials, LayoutStats* stats, int center) {
  StatsAcc a;
  stats_init(a);
  const int pairs = n >> 1;
  const float4* y2 = reinterpret_cast<const float4*>(y);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < pairs; i += gridDim.x * blockDim.x) {
    const float4 v = y2[i];
    stats_add(a, make_float2(v.x, v.y));
    stats_add(a, make_float2(v.z, v.w));
  }
  if ((n & 1) && blockIdx.x == 0 && threadIdx.x == 0) stats_add(a, y[n - 1]);
  stats_block_finish(a, partials, stats, &stats->stats_counter, center, n, g);
}

// ------------------------------------------------------------------ splat

// The scales are powers of two within float's range, so v * scale is exact in
// float as in double, and both conversions round the same value.
__device__ __forceinline__ long long to_fixed(float v, double scale) {
  return __float2ll_rn(v * static_cast<float>(scale));
}

constexpr int kSplatThreads = 256;
constexpr int kSplatTileNodes = 1024;  // 3 x 8 KB of 64-bit charges in shared memory

// One thread per point, blocks of 256 consecutive (Morton-ordered) points.
//  1. Lanes of a warp whose points share a grid cell sum their 12
//     contributions (4 corner nodes x {1, x, y}) -- a butterfly when the whole
//     warp shares the cell, else in lane order -- and the lowest such lane
//     converts the sums to 64-bit fixed point.  Sharded runs cut the points
//     at multiples of 32, so every warp sums the same lanes on any rank count.
//  2. When the block's cells fit in a tile of at most 1024 grid nodes (the
//     usual case: consecutive points are spatially close), those lanes add
//     into the tile with shared-memory atomics and the block then adds each
//     non-zero tile node to the grid once; otherwise they add to the grid
//     directly.  Integer sums are exact, so both routes give the same charges.
// Every point is centred; only points in [own_begin, own_end) are spread (a
// shard spreads its own rows, the charge grids of all shards are then summed).
__global__ void __launch_bounds__(kSplatThreads) splat_kernel(float2* __restrict__ y,
                                                              LayoutStats* __restrict__ stats, int n, int g,
                                                              ChargeCell* __restrict__ charges, int own_begin,
                                                              int own_end) {
  __shared__ unsigned long long tile[3][kSplatTileNodes];
  __shared__ int s_box[4][kSplatThreads / 32];
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const GridGeom q = stats->geom;
  const ChargeScales sc = stats->scales;
  if (i == 0) {
    // work counters of this iteration's attraction kernels
    stats->row_groups_taken = 0u;
    stats->stage_taken = 0u;
  }
  int key = -1;
  Cell c{0, 0, 0.f, 0.f};
  float v[12];
#pragma unroll
  for (int t = 0; t < 12; ++t) v[t] = 0.0f;
  if (i < n) {
    float2 p = y[i];
    if (stats->center) {
      p.x -= q.mean_x;
      p.y -= q.mean_y;
      y[i] = p;
    }
  }
  if (i >= own_begin && i < own_end) {
    const float2 p = y[i];
    c = grid_cell(p.x, p.y, q, g);
    key = c.y0 * g + c.x0;
    const float w[4] = {(1.0f - c.tx) * (1.0f - c.ty), c.tx * (1.0f - c.ty), (1.0f - c.tx) * c.ty,
                        c.tx * c.ty};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v[3 * k] = w[k];
      v[3 * k + 1] = w[k] * p.x;
      v[3 * k + 2] = w[k] * p.y;
    }
  }
  const unsigned int peers = __match_any_sync(0xffffffffu, key);
  const int leader = __ffs(peers) - 1;
  if (peers == 0xffffffffu) {
    // The whole warp shares one cell (dense regions, compact early layouts):
    // a five-step butterfly.  Non-spreading warps (key -1) skip it.
    if (key >= 0) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int t = 0; t < 12; ++t) v[t] += __shfl_xor_sync(0xffffffffu, v[t], o);
      }
    }
  } else if (key >= 0 && __popc(peers) > 1) {
    // Small groups: all groups of the warp step through their members in lock step.
    float sum[12];
#pragma unroll
    for (int t = 0; t < 12; ++t) sum[t] = 0.0f;
    for (unsigned int m = peers; m; m &= m - 1) {
      const int src = __ffs(m) - 1;
#pragma unroll
      for (int t = 0; t < 12; ++t) sum[t] += __shfl_sync(peers, v[t], src);
    }
#pragma unroll
    for (int t = 0; t < 12; ++t) v[t] = sum[t];
  }
  const bool active = key >= 0 && lane == leader;
  long long f[12];
  if (active) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      f[3 * k] = to_fixed(v[3 * k], sc.m);
      f[3 * k + 1] = to_fixed(v[3 * k + 1], sc.xy);
      f[3 * k + 2] = to_fixed(v[3 * k + 2], sc.xy);
    }
  }

  // Node box of the block's points (cells plus their +1 corners).
  const bool own = key >= 0;
  int x_lo = own ? c.x0 : INT_MAX, y_lo = own ? c.y0 : INT_MAX;
  int x_hi = own ? c.x0 + 1 : INT_MIN, y_hi = own ? c.y0 + 1 : INT_MIN;
  x_lo = __reduce_min_sync(0xffffffffu, x_lo);
  y_lo = __reduce_min_sync(0xffffffffu, y_lo);
  x_hi = __reduce_max_sync(0xffffffffu, x_hi);
  y_hi = __reduce_max_sync(0xffffffffu, y_hi);
  if (lane == 0) {
    s_box[0][wid] = x_lo;
    s_box[1][wid] = y_lo;
    s_box[2][wid] = x_hi;
    s_box[3][wid] = y_hi;
  }
  __syncthreads();
  x_lo = INT_MAX, y_lo = INT_MAX, x_hi = INT_MIN, y_hi = INT_MIN;
  for (int w = 0; w < kSplatThreads / 32; ++w) {
    x_lo = min(x_lo, s_box[0][w]);
    y_lo = min(y_lo, s_box[1][w]);
    x_hi = max(x_hi, s_box[2][w]);
    y_hi = max(y_hi, s_box[3][w]);
  }
  if (x_hi < x_lo) return;  // no point of this block is spread (block-uniform)
  const int box_w = x_hi - x_lo + 1, box_h = y_hi - y_lo + 1;
  const bool tiled = box_w * box_h <= kSplatTileNodes;  // block-uniform

  if (!tiled) {
    if (!active) return;
    const int corner[4] = {key, key + 1, key + g, key + g + 1};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      ChargeCell* cell = charges + corner[k];
      const long long a = f[3 * k], b = f[3 * k + 1], d = f[3 * k + 2];
      if (a != 0) atomicAdd(&cell->m, static_cast<unsigned long long>(a));
      if (b != 0) atomicAdd(&cell->mx, static_cast<unsigned long long>(b));
      if (d != 0) atomicAdd(&cell->my, static_cast<unsigned long long>(d));
    }
    return;
  }
  const int nodes = box_w * box_h;
  for (int t = threadIdx.x; t < nodes; t += kSplatThreads) {
    tile[0][t] = 0ull;
    tile[1][t] = 0ull;
    tile[2][t] = 0ull;
  }
  __syncthreads();
  if (active) {
    const int base = (c.y0 - y_lo) * box_w + (c.x0 - x_lo);
    const int corner[4] = {base, base + 1, base + box_w, base + box_w + 1};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const long long a = f[3 * k], b = f[3 * k + 1], d = f[3 * k + 2];
      if (a != 0) atomicAdd(&tile[0][corner[k]], static_cast<unsigned long long>(a));
      if (b != 0) atomicAdd(&tile[1][corner[k]], static_cast<unsigned long long>(b));
      if (d != 0) atomicAdd(&tile[2][corner[k]], static_cast<unsigned long long>(d));
    }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < nodes; t += kSplatThreads) {
    const int ty = t / box_w, tx = t - ty * box_w;
    ChargeCell* cell = charges + static_cast<size_t>(y_lo + ty) * g + (x_lo + tx);
    const unsigned long long a = tile[0][t], b = tile[1][t], d = tile[2][t];
    if (a != 0ull) atomicAdd(&cell->m, a);
    if (b != 0ull) atomicAdd(&cell->mx, b);
    if (d != 0ull) atomicAdd(&cell->my, d);
  }
}


// Lagrange mode (FIt-SNE boxes, three nodes per box and side): as
// splat_kernel with each point spreading {1, x, y} to the 3 x 3 nodes of its
// box with quadratic Lagrange weights (which can be negative; the fixed-point
// sums are two's complement).  Lanes sharing a box combine first; a block's
// nodes go through the shared-memory tile when they fit.
__global__ void __launch_bounds__(kSplatThreads) splat_lagrange_kernel(float2* __restrict__ y,
                                                                       LayoutStats* __restrict__ stats, int n, int g,
                                                                       ChargeCell* __restrict__ charges,
                                                                       int own_begin, int own_end) {
  __shared__ unsigned long long tile[3][kSplatTileNodes];
  __shared__ int s_box[4][kSplatThreads / 32];
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const GridGeom q = stats->geom;
  const ChargeScales sc = stats->scales;
  if (i == 0) {
    stats->row_groups_taken = 0u;
    stats->stage_taken = 0u;
  }
  int key = -1;
  LagrangeCell c;
  c.bx = 0;
  c.by = 0;
  float v[27];
#pragma unroll
  for (int t = 0; t < 27; ++t) v[t] = 0.0f;
  if (i < n) {
    float2 p = y[i];
    if (stats->center) {
      p.x -= q.mean_x;
      p.y -= q.mean_y;
      y[i] = p;
    }
  }
  if (i >= own_begin && i < own_end) {
    const float2 p = y[i];
    c = lagrange_cell(p.x, p.y, q);
    key = c.by * q.boxes + c.bx;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        const float w = c.wx[j] * c.wy[k];
        v[3 * (3 * k + j)] = w;
        v[3 * (3 * k + j) + 1] = w * p.x;
        v[3 * (3 * k + j) + 2] = w * p.y;
      }
    }
  }
  const unsigned int peers = __match_any_sync(0xffffffffu, key);
  const int leader = __ffs(peers) - 1;
  if (peers == 0xffffffffu) {
    if (key >= 0) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int t = 0; t < 27; ++t) v[t] += __shfl_xor_sync(0xffffffffu, v[t], o);
      }
    }
  } else if (key >= 0 && __popc(peers) > 1) {
    float sum[27];
#pragma unroll
    for (int t = 0; t < 27; ++t) sum[t] = 0.0f;
    for (unsigned int m = peers; m; m &= m - 1) {
      const int src = __ffs(m) - 1;
#pragma unroll
      for (int t = 0; t < 27; ++t) sum[t] += __shfl_sync(peers, v[t], src);
    }
#pragma unroll
    for (int t = 0; t < 27; ++t) v[t] = sum[t];
  }
  const bool active = key >= 0 && lane == leader;

  // Node box of the block's points (the 3 x 3 nodes of each box).
  const bool own = key >= 0;
  int x_lo = own ? 3 * c.bx : INT_MAX, y_lo = own ? 3 * c.by : INT_MAX;
  int x_hi = own ? 3 * c.bx + 2 : INT_MIN, y_hi = own ? 3 * c.by + 2 : INT_MIN;
  x_lo = __reduce_min_sync(0xffffffffu, x_lo);
  y_lo = __reduce_min_sync(0xffffffffu, y_lo);
  x_hi = __reduce_max_sync(0xffffffffu, x_hi);
  y_hi = __reduce_max_sync(0xffffffffu, y_hi);
  if (lane == 0) {
    s_box[0][wid] = x_lo;
    s_box[1][wid] = y_lo;
    s_box[2][wid] = x_hi;
    s_box[3][wid] = y_hi;
  }
  __syncthreads();
  x_lo = INT_MAX, y_lo = INT_MAX, x_hi = INT_MIN, y_hi = INT_MIN;
  for (int w = 0; w < kSplatThreads / 32; ++w) {
    x_lo = min(x_lo, s_box[0][w]);
    y_lo = min(y_lo, s_box[1][w]);
    x_hi = max(x_hi, s_box[2][w]);
    y_hi = max(y_hi, s_box[3][w]);
  }
  if (x_hi < x_lo) return;  // no point of this block is spread (block-uniform)
  const int box_w = x_hi - x_lo + 1, box_h = y_hi - y_lo + 1;
  const bool tiled = box_w * box_h <= kSplatTileNodes;  // block-uniform
  if (!tiled) {
    if (!active) return;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        ChargeCell* cell = charges + static_cast<size_t>(3 * c.by + k) * g + (3 * c.bx + j);
        const int t = 3 * (3 * k + j);
        const long long a = to_fixed(v[t], sc.m), b = to_fixed(v[t + 1], sc.xy), d = to_fixed(v[t + 2], sc.xy);
        if (a != 0) atomicAdd(&cell->m, static_cast<unsigned long long>(a));
        if (b != 0) atomicAdd(&cell->mx, static_cast<unsigned long long>(b));
        if (d != 0) atomicAdd(&cell->my, static_cast<unsigned long long>(d));
      }
    }
    return;
  }
  const int nodes = box_w * box_h;
  for (int t = threadIdx.x; t < nodes; t += kSplatThreads) {
    tile[0][t] = 0ull;
    tile[1][t] = 0ull;
    tile[2][t] = 0ull;
  }
  __syncthreads();
  if (active) {
#pragma unroll
    for (int k = 0; k < 3; ++k) {
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        const int node = (3 * c.by + k - y_lo) * box_w + (3 * c.bx + j - x_lo);
        const int t = 3 * (3 * k + j);
        const long long a = to_fixed(v[t], sc.m), b = to_fixed(v[t + 1], sc.xy), d = to_fixed(v[t + 2], sc.xy);
        if (a != 0) atomicAdd(&tile[0][node], static_cast<unsigned long long>(a));
        if (b != 0) atomicAdd(&tile[1][node], static_cast<unsigned long long>(b));
        if (d != 0) atomicAdd(&tile[2][node], static_cast<unsigned long long>(d));
      }
    }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < nodes; t += kSplatThreads) {
    const int ty = t / box_w, tx = t - ty * box_w;
    ChargeCell* cell = charges + static_cast<size_t>(y_lo + ty) * g + (x_lo + tx);
    const unsigned long long a = tile[0][t], b = tile[1][t], d = tile[2][t];
    if (a != 0ull) atomicAdd(&cell->m, a);
    if (b != 0ull) atomicAdd(&cell->mx, b);
    if (d != 0ull) atomicAdd(&cell->my, d);
  }
}

__device__ __forceinline__ float3 read_charge(const ChargeCell& c, const ChargeScales& sc) {
  return make_float3(static_cast<float>(static_cast<double>(static_cast<long long>(c.m)) / sc.m),
                     static_cast<float>(static_cast<double>(static_cast<long long>(c.mx)) / sc.xy),
                     static_cast<float>(static_cast<double>(static_cast<long long>(c.my)) / sc.xy));
}

// ------------------------------------------------------------------ FFT passes

// Row r of the three charge planes and kernel row dy = r as three complex
// length-M FFTs (buffer elements [0, M), [M, 2M), [2M, 3M), stored through
// sw; M = 2G): (mx + i my), (m), (Kq + i Kq2).  Two real rows packed into one
// complex transform share its rounding error, which scales with the larger of
// the two, so only rows of like magnitude are paired: the moments mx, my are
// the masses times coordinates of tens of units, and at a converged layout
// the repulsion is a small difference of their convolutions.
template <int LOG_M>
__global__ void __launch_bounds__(FftShape<LOG_M, 3>::THREADS, 2)
    fft_rows_fwd_kernel(const ChargeCell* __restrict__ charges, const LayoutStats* __restrict__ stats,
                        const float2* __restrict__ twiddles, float2* __restrict__ rowspec,
                        float2* __restrict__ krow) {
  using S = FftShape<LOG_M, 3>;
  constexpr int M = S::M, G = M / 2, ROW_LEN = G + 1;
  extern __shared__ float2 smem[];
  float2* tw = smem + S::DATA;
  const int r = blockIdx.x;
  const GridGeom q = stats->geom;
  const ChargeScales sc = stats->scales;
  fft_load_twiddles<LOG_M, S::THREADS>(twiddles, tw);
#pragma unroll
  for (int x0 = 0; x0 < M; x0 += S::THREADS) {
    const int x = x0 + static_cast<int>(threadIdx.x);
    if (M % S::THREADS == 0 || x < M) {
      float3 c = make_float3(0.f, 0.f, 0.f);
      if (x < G) c = read_charge(charges[static_cast<size_t>(r) * G + x], sc);
      float kq = 0.f, kq2 = 0.f;
      if (x <= G - 1) {
        kernel_values(x, r, q.spacing, &kq, &kq2);
      } else if (x >= G + 1) {
        kernel_values(x - M, r, q.spacing, &kq, &kq2);
      }
      smem[sw(x)] = make_float2(c.y, c.z);
      smem[sw(M + x)] = make_float2(c.x, 0.f);
      smem[sw(2 * M + x)] = make_float2(kq, kq2);
    }
  }
  __syncthreads();
  block_fft<LOG_M, 3, S::THREADS>(smem, tw, false);
  for (int k = threadIdx.x; k <= G; k += S::THREADS) {
    const int km = (M - k) & (M - 1);
    const float2 a = smem[sw(k)], ac = conjf2(smem[sw(km)]);
    const float2 b = smem[sw(2 * M + k)], bc = conjf2(smem[sw(2 * M + km)]);
    const float2 sum_a = cadd(a, ac), dif_a = csub(a, ac);
    // X = (Z + Z*)/2, Y = (Z - Z*)/(2i); the kernel spectra are real (even kernels)
    const float2 xmx = cscale(sum_a, 0.5f);
    const float2 xmy = make_float2(0.5f * dif_a.y, -0.5f * dif_a.x);
    const float2 xm = smem[sw(M + k)];
    const float kqx = 0.5f * (b.x + bc.x);
    const float kq2x = 0.5f * (b.y - bc.y);
    float2* out = rowspec + 3 * (static_cast<size_t>(r) * ROW_LEN + k);
    out[0] = xm;
    out[1] = xmx;
    out[2] = xmy;
    krow[static_cast<size_t>(r) * ROW_LEN + k] = make_float2(kqx, kq2x);
  }
}

// Columns [k0, k0 + TK) of the half spectrum: y-FFT of three charge planes and
// of the real, even kernel columns (Kq + i Kq2 packs two real spectra), product,
// inverse y-FFT, keep rows [0, G).  Columns past G (the last block's tail) are
// transformed as zeros and not stored.
template <int LOG_M>
__global__ void __launch_bounds__(FftShape<LOG_M, 4 * fft_cols_per_block(1 << LOG_M), kFftBatchCols>::THREADS,
                                  FftShape<LOG_M, 4 * fft_cols_per_block(1 << LOG_M), kFftBatchCols>::THREADS > 512 ? 1 : 2)
    fft_cols_kernel(const float2* __restrict__ rowspec, const float2* __restrict__ krow,
                    const float2* __restrict__ twiddles, float2* __restrict__ colspec) {
  constexpr int M = 1 << LOG_M, G = M / 2, ROW_LEN = G + 1;
  constexpr int TK = fft_cols_per_block(M);
  using S = FftShape<LOG_M, 4 * TK, kFftBatchCols>;
  extern __shared__ float2 smem[];
  float2* tw = smem + S::DATA;
  const int k0 = blockIdx.x * TK;
  fft_load_twiddles<LOG_M, S::THREADS>(twiddles, tw);
  // Sequence 4c + p: column c, plane p in {0: m, 1: mx, 2: my, 3: kernel pack}.
#pragma unroll
  for (int t0 = 0; t0 < TK * M; t0 += S::THREADS) {
    const int t = t0 + static_cast<int>(threadIdx.x);
    if ((TK * M) % S::THREADS == 0 || t < TK * M) {
      const int c = t >> LOG_M;
      const int r = t & (M - 1);
      const int k = k0 + c;
      const int b = (c * 4) << LOG_M;
      float2 v0 = make_float2(0.f, 0.f), v1 = v0, v2 = v0, kk = v0;
      if (k < ROW_LEN) {
        if (r < G) {
          const float2* src = rowspec + 3 * (static_cast<size_t>(r) * ROW_LEN + k);
          v0 = src[0];
          v1 = src[1];
          v2 = src[2];
        }
        const int dy = r <= G - 1 ? r : (r >= G + 1 ? M - r : -1);
        if (dy >= 0) kk = krow[static_cast<size_t>(dy) * ROW_LEN + k];
      }
      smem[sw(b + r)] = v0;
      smem[sw(b + M + r)] = v1;
      smem[sw(b + 2 * M + r)] = v2;
      smem[sw(b + 3 * M + r)] = kk;
    }
  }
  __syncthreads();
  block_fft<LOG_M, 4 * TK, S::THREADS>(smem, tw, false);
#pragma unroll
  for (int t0 = 0; t0 < TK * M; t0 += S::THREADS) {
    const int t = t0 + static_cast<int>(threadIdx.x);
    if ((TK * M) % S::THREADS == 0 || t < TK * M) {
      const int c = t >> LOG_M;
      const int r = t & (M - 1);
      const int b = (c * 4) << LOG_M;
      const float2 kk = smem[sw(b + 3 * M + r)];
      const float kq = kk.x, kq2 = kk.y;
      const float2 mm = smem[sw(b + r)];
      smem[sw(b + 3 * M + r)] = cscale(mm, kq);                        // phi_q
      smem[sw(b + r)] = cscale(mm, kq2);                               // phi_q2
      smem[sw(b + M + r)] = cscale(smem[sw(b + M + r)], kq2);          // phi_xq2
      smem[sw(b + 2 * M + r)] = cscale(smem[sw(b + 2 * M + r)], kq2);  // phi_yq2
    }
  }
  __syncthreads();
  block_fft<LOG_M, 4 * TK, S::THREADS>(smem, tw, true);
#pragma unroll
  for (int t0 = 0; t0 < TK * G; t0 += S::THREADS) {
    const int t = t0 + static_cast<int>(threadIdx.x);
    if ((TK * G) % S::THREADS == 0 || t < TK * G) {
      const int c = t >> (LOG_M - 1);
      const int r = t & (G - 1);
      const int k = k0 + c;
      if (k < ROW_LEN) {
        const int b = (c * 4) << LOG_M;
        float4* out = reinterpret_cast<float4*>(colspec + 4 * (static_cast<size_t>(r) * ROW_LEN + k));
        const float2 o0 = smem[sw(b + r)], o1 = smem[sw(b + M + r)];
        const float2 o2 = smem[sw(b + 2 * M + r)], o3 = smem[sw(b + 3 * M + r)];
        out[0] = make_float4(o0.x, o0.y, o1.x, o1.y);
        out[1] = make_float4(o2.x, o2.y, o3.x, o3.y);
      }
    }
  }
}

// Output row r: inverse x-FFTs of (phi_xq2 + i phi_yq2) and (phi_q2 + i phi_q)
// from their half spectra (pairs of like magnitude, as in the forward rows),
// potentials, this row's share of Z, and clearing of the charges for the next
// splat.  The row's masses are read (and its charge
// cells cleared) before the transform so that those loads are in flight
// during it.  The last block folds Z.
template <int LOG_M>
__global__ void __launch_bounds__(FftShape<LOG_M, 2>::THREADS, 4)
    fft_rows_inv_kernel(const float2* __restrict__ colspec, ChargeCell* __restrict__ charges, int n,
                        const float2* __restrict__ twiddles, float4* __restrict__ pot,
                        double* __restrict__ z_partials, LayoutStats* __restrict__ stats) {
  using S = FftShape<LOG_M, 2>;
  constexpr int M = S::M, G = M / 2, ROW_LEN = G + 1;
  constexpr int CELLS = (G + S::THREADS - 1) / S::THREADS;
  extern __shared__ float2 smem[];
  float2* tw = smem + S::DATA;
  const int r = blockIdx.x;
  unsigned long long mass_q[CELLS];
#pragma unroll
  for (int i = 0; i < CELLS; ++i) {
    const int x = static_cast<int>(threadIdx.x) + i * S::THREADS;
    mass_q[i] = 0ull;
    if (G % S::THREADS == 0 || x < G) {
      ChargeCell* cell = charges + static_cast<size_t>(r) * G + x;
      mass_q[i] = cell->m;
      *cell = ChargeCell{0ull, 0ull, 0ull, 0ull};
    }
  }
  fft_load_twiddles<LOG_M, S::THREADS>(twiddles, tw);
#pragma unroll
  for (int k0 = 0; k0 < M; k0 += S::THREADS) {
    const int k = k0 + static_cast<int>(threadIdx.x);
    if (M % S::THREADS == 0 || k < M) {
      const bool mirror = k > G;
      const int kk = mirror ? M - k : k;
      const float4* src = reinterpret_cast<const float4*>(colspec + 4 * (static_cast<size_t>(r) * ROW_LEN + kk));
      const float4 ab = src[0], cd = src[1];
      float2 a = make_float2(ab.x, ab.y), b = make_float2(ab.z, ab.w);
      float2 c = make_float2(cd.x, cd.y), d = make_float2(cd.z, cd.w);
      if (mirror) {
        a = conjf2(a);
        b = conjf2(b);
        c = conjf2(c);
        d = conjf2(d);
      }
      smem[sw(k)] = make_float2(b.x - c.y, b.y + c.x);
      smem[sw(M + k)] = make_float2(a.x - d.y, a.y + d.x);
    }
  }
  __syncthreads();
  block_fft<LOG_M, 2, S::THREADS>(smem, tw, true);
  const double inv_scale_m = 1.0 / stats->scales.m;
  const float scale = 1.0f / (static_cast<float>(M) * static_cast<float>(M));
  double zpart = 0.0;
#pragma unroll
  for (int i = 0; i < CELLS; ++i) {
    const int x = static_cast<int>(threadIdx.x) + i * S::THREADS;
    if (G % S::THREADS == 0 || x < G) {
      const float2 xy = smem[sw(x)], qq = smem[sw(M + x)];
      const float4 p = make_float4(qq.x * scale, xy.x * scale, xy.y * scale, qq.y * scale);
      pot[static_cast<size_t>(r) * G + x] = p;
      const double mass = static_cast<double>(static_cast<long long>(mass_q[i])) * inv_scale_m;
      zpart += mass * static_cast<double>(p.w);
    }
  }
  __shared__ double s_part[32];
  __shared__ bool s_last;
  zpart = warp_sum(zpart);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) s_part[wid] = zpart;
  __syncthreads();
  if (threadIdx.x == 0) {
    double v = 0.0;
    for (int w = 0; w < S::THREADS / 32; ++w) v += s_part[w];
    z_partials[r] = v;
    __threadfence();
    const unsigned int ticket = atomicAdd(&stats->fft_counter, 1u);
    s_last = ticket == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  double acc = 0.0;
  for (int b = threadIdx.x; b < static_cast<int>(gridDim.x); b += S::THREADS) {
    acc += static_cast<const volatile double*>(z_partials)[b];
  }
  acc = warp_sum(acc);
  __syncthreads();
  if (lane == 0) s_part[wid] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double z = 0.0;
    for (int w = 0; w < S::THREADS / 32; ++w) z += s_part[w];
    z -= static_cast<double>(n);
    stats->z = z;
    stats->inv_z = static_cast<float>(1.0 / fmax(z, static_cast<double>(FLT_MIN)));
    stats->fft_counter = 0u;
  }
}

}  // namespace

int fft_twiddle_entries(int log_m) { return fft_table_entries(log_m); }

void fft_twiddle_table(int log_m, float2* out) {
  const double two_pi = 6.283185307179586476925286766559;
  int e = 0;
  for (int pass = 1; pass < log_m / 2; ++pass) {  // radix-4 passes with twiddles
    const int ns = 1 << (2 * pass);
    for (int q = 1; q < 4; ++q) {
      for (int k = 0; k < ns; ++k) {
        const double ang = -two_pi * static_cast<double>(q * k) / static_cast<double>(4 * ns);
        out[e++] = make_float2(static_cast<float>(std::cos(ang)), static_cast<float>(std::sin(ang)));
      }
    }
  }
  for (int j = 0; e < fft_table_entries(log_m); ++j) {
    const double ang = -two_pi * static_cast<double>(j) / static_cast<double>(1 << log_m);
    out[e++] = make_float2(static_cast<float>(std::cos(ang)), static_cast<float>(std::sin(ang)));
  }
}

namespace {

// Launch and attribute helpers over the instantiated transform lengths.
#define FE_FFT_LOG_M_CASES(X) X(3) X(4) X(5) X(6) X(7) X(8) X(9) X(10) X(11)

template <int LOG_M>
int fft_configure() {
  constexpr int TK = fft_cols_per_block(1 << LOG_M);
  FE_CUDA(cudaFuncSetAttribute(fft_rows_fwd_kernel<LOG_M>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(FftShape<LOG_M, 3>::SMEM)),
          "cudaFuncSetAttribute(fft_rows_fwd_kernel)");
  FE_CUDA(cudaFuncSetAttribute(fft_cols_kernel<LOG_M>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(FftShape<LOG_M, 4 * TK, kFftBatchCols>::SMEM)),
          "cudaFuncSetAttribute(fft_cols_kernel)");
  FE_CUDA(cudaFuncSetAttribute(fft_rows_inv_kernel<LOG_M>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(FftShape<LOG_M, 2>::SMEM)),
          "cudaFuncSetAttribute(fft_rows_inv_kernel)");
  return 0;
}

// pass 0: rows forward, 1: columns, 2: rows inverse.
template <int LOG_M>
int fft_launch(TsneSession* s, int pass) {
  constexpr int M = 1 << LOG_M, G = M / 2;
  constexpr int TK = fft_cols_per_block(M);
  if (pass == 0) {
    using S = FftShape<LOG_M, 3>;
    fft_rows_fwd_kernel<LOG_M><<<G, S::THREADS, S::SMEM, s->stream>>>(s->charges, s->stats, s->twiddle, s->rowspec,
                                                                          s->krow);
    FE_LAUNCH("fft_rows_fwd_kernel");
  } else if (pass == 1) {
    using S = FftShape<LOG_M, 4 * TK, kFftBatchCols>;
    fft_cols_kernel<LOG_M><<<(G + 1 + TK - 1) / TK, S::THREADS, S::SMEM, s->stream>>>(s->rowspec, s->krow,
                                                                                   s->twiddle, s->colspec);
    FE_LAUNCH("fft_cols_kernel");
  } else {
    using S = FftShape<LOG_M, 2>;
    fft_rows_inv_kernel<LOG_M><<<G, S::THREADS, S::SMEM, s->stream>>>(s->colspec, s->charges, s->n, s->twiddle,
                                                                     s->pot, s->z_partials, s->stats);
    FE_LAUNCH("fft_rows_inv_kernel");
  }
  return 0;
}

int fft_launch_pass(TsneSession* s, int pass) {
  switch (s->log_fft) {
#define FE_FFT_LAUNCH_CASE(L) \
  case L:                     \
    return fft_launch<L>(s, pass);
    FE_FFT_LOG_M_CASES(FE_FFT_LAUNCH_CASE)
#undef FE_FFT_LAUNCH_CASE
    default:
      set_error("t-SNE FFT length outside the instantiated range (grid 4 to 1024)");
      return 1;
  }
}

// ------------------------------------------------------------------ gradient + update

struct UpdateParams {
  int n;
  int row_begin;   // rows [row_begin, row_end) are attracted and updated
  int row_end;
  int g;
  float exaggeration;
  float momentum;
  float learning_rate;
  float min_gain;
  float max_step_norm;
  int mode;
};

__device__ __forceinline__ float sign_f(float x) { return x == 0.0f ? 0.0f : (x < 0.0f ? -1.0f : 1.0f); }

// Lagrange mode: the 3 x 3 nodes of the point's box with its Lagrange weights.
__device__ __forceinline__ float3 gather_potentials_lagrange(const float4* __restrict__ pot, const LagrangeCell& c,
                                                             int g) {
  float3 r = make_float3(0.0f, 0.0f, 0.0f);
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const float4* rowp = pot + static_cast<size_t>(3 * c.by + k) * g + 3 * c.bx;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const float4 v = __ldg(rowp + j);
      const float w = c.wx[j] * c.wy[k];
      r.x += w * v.x;
      r.y += w * v.y;
      r.z += w * v.z;
    }
  }
  return r;
}

// bilinear_grid_value_t (src/tsne_neighbors.cpp:760-781) on three planes at once.
__device__ __forceinline__ float3 gather_potentials(const float4* __restrict__ pot, const Cell& c, int g) {
  const float4* base = pot + static_cast<size_t>(c.y0) * g + c.x0;
  const float4 v00 = __ldg(base), v10 = __ldg(base + 1), v01 = __ldg(base + g), v11 = __ldg(base + g + 1);
  const float a = (1.0f - c.tx) * (1.0f - c.ty);
  const float b = c.tx * (1.0f - c.ty);
  const float d = (1.0f - c.tx) * c.ty;
  const float e = c.tx * c.ty;
  float3 r;
  r.x = a * v00.x + b * v10.x + d * v01.x + e * v11.x;
  r.y = a * v00.y + b * v10.y + d * v01.y + e * v11.y;
  r.z = a * v00.z + b * v10.z + d * v01.z + e * v11.z;
  return r;
}

// The fused epilogue of one row: repulsive gather, gains / momentum / step
// clip (apply_open_tsne_update_f, src/tsne_neighbors.cpp:1213-1244), layout
// write; or the gradient alone (kGradOnly).  (ax, ay) is the row's attraction.
__device__ __forceinline__ void finish_row(int row, float ax, float ay, const float2* __restrict__ y,
                                           float2* __restrict__ y_next, float2* __restrict__ update,
                                           float2* __restrict__ gains, float2* __restrict__ grad_out,
                                           const float4* __restrict__ pot, const LayoutStats* __restrict__ stats,
                                           const UpdateParams& prm) {
  const float2 yi = y[row];
  const GridGeom q = stats->geom;
  float3 ph;
  if (q.boxes > 0) {
    ph = gather_potentials_lagrange(pot, lagrange_cell(yi.x, yi.y, q), prm.g);
  } else {
    ph = gather_potentials(pot, grid_cell(yi.x, yi.y, q, prm.g), prm.g);
  }
  const float inv_z = stats->inv_z;
  const float gx = -(yi.x * ph.x - ph.y) * inv_z + ax;
  const float gy = -(yi.y * ph.x - ph.z) * inv_z + ay;
  if (prm.mode == kGradOnly) {
    grad_out[row] = make_float2(gx, gy);
    return;
  }
  float2 u = update[row];
  float2 gn = gains[row];
  if (sign_f(u.x) != sign_f(gx)) gn.x += 0.2f;
  else gn.x = gn.x * 0.8f + prm.min_gain;
  if (gn.x < prm.min_gain) gn.x = prm.min_gain;
  u.x = prm.momentum * u.x - prm.learning_rate * gn.x * gx;
  if (sign_f(u.y) != sign_f(gy)) gn.y += 0.2f;
  else gn.y = gn.y * 0.8f + prm.min_gain;
  if (gn.y < prm.min_gain) gn.y = prm.min_gain;
  u.y = prm.momentum * u.y - prm.learning_rate * gn.y * gy;
  float norm_sq = 0.0f;
  norm_sq += u.x * u.x;
  norm_sq += u.y * u.y;
  if (isfinite(prm.max_step_norm) && prm.max_step_norm > 0.0f &&
      norm_sq > prm.max_step_norm * prm.max_step_norm) {
    if (isfinite(norm_sq)) {
      const float scale = prm.max_step_norm / sqrtf(fmaxf(norm_sq, FLT_MIN));
      u.x *= scale;
      u.y *= scale;
    } else {
      // An infinite step (Z collapsed to FLT_MIN): the reference's clip would
      // form inf * 0; keep the step's direction at the maximum length instead.
      const float sx = isinf(u.x) ? copysignf(1.0f, u.x) : 0.0f;
      const float sy = isinf(u.y) ? copysignf(1.0f, u.y) : 0.0f;
      const float len = sqrtf(sx * sx + sy * sy);
      u.x = len > 0.0f ? sx / len * prm.max_step_norm : 0.0f;
      u.y = len > 0.0f ? sy / len * prm.max_step_norm : 0.0f;
    }
  }
  const float2 yn = make_float2(yi.x + u.x, yi.y + u.y);
  update[row] = u;
  gains[row] = gn;
  y_next[row] = yn;
}

// Attraction over the internal-order P, eight lanes per row: a warp takes a
// block of 32 rows in 8 rounds of 4 rows.  Each pass a lane streams two
// 16-byte groups of columns and two of values (stride 8 groups within its
// row), gathers the eight y_j and accumulates; the next pass's loads are
// issued before the current pass's gathers (FE_ATTRACT_PREFETCH).  Three xor
// shuffles reduce a row's eight partial sums, and the row's sum is parked in
// one lane so that the epilogue -- repulsive gather, gains/momentum/step clip,
// layout write, statistics for the next iteration -- runs 32 rows wide.
#ifndef FE_ATTRACT_PREFETCH
#define FE_ATTRACT_PREFETCH 1
#endif

__device__ __forceinline__ void attract4(float yix, float yiy, int4 c, float4 v, float ex,
                                         const float2* __restrict__ y, float& ax, float& ay) {
  const float2 g0 = __ldg(y + c.x), g1 = __ldg(y + c.y), g2 = __ldg(y + c.z), g3 = __ldg(y + c.w);
  const float2 g[4] = {g0, g1, g2, g3};
  const float pv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float dx = yix - g[q].x;
    const float dy = yiy - g[q].y;
    float d2 = 0.0f;
    d2 += dx * dx;
    d2 += dy * dy;
    const float qq = 1.0f / (1.0f + d2);
    const float w = ex * pv[q] * qq;
    ax += w * dx;
    ay += w * dy;
  }
}

// Streams one row of the internal P (groups [beg, end) of four entries) with
// S lanes: each lane takes groups lane, lane + S in a pass and the next pass
// starts 2S groups on; the next pass's loads are issued before this pass's
// gathers (FE_ATTRACT_PREFETCH).  `passes` may exceed the row's own need
// (lanes then load nothing).
template <int S>
__device__ __forceinline__ void stream_row(int beg, int end, int l, int passes, float2 yi, float ex,
                                           const int4* __restrict__ col4, const float4* __restrict__ val4,
                                           const float2* __restrict__ y, float& ax, float& ay) {
  const int4 zero_c = make_int4(0, 0, 0, 0);
  const float4 zero_v = make_float4(0.f, 0.f, 0.f, 0.f);
  int e = beg + l;
#if FE_ATTRACT_PREFETCH
  int4 c0 = e < end ? ld_stream(col4 + e) : zero_c;
  float4 v0 = e < end ? ld_stream(val4 + e) : zero_v;
  int4 c1 = e + S < end ? ld_stream(col4 + e + S) : zero_c;
  float4 v1 = e + S < end ? ld_stream(val4 + e + S) : zero_v;
  for (int p = 0; p < passes; ++p) {
    const int en = e + 2 * S;
    const int4 nc0 = en < end ? ld_stream(col4 + en) : zero_c;
    const float4 nv0 = en < end ? ld_stream(val4 + en) : zero_v;
    const int4 nc1 = en + S < end ? ld_stream(col4 + en + S) : zero_c;
    const float4 nv1 = en + S < end ? ld_stream(val4 + en + S) : zero_v;
    attract4(yi.x, yi.y, c0, v0, ex, y, ax, ay);
    attract4(yi.x, yi.y, c1, v1, ex, y, ax, ay);
    c0 = nc0;
    v0 = nv0;
    c1 = nc1;
    v1 = nv1;
    e = en;
  }
#else
  for (int p = 0; p < passes; ++p, e += 2 * S) {
    const int4 c0 = e < end ? ld_stream(col4 + e) : zero_c;
    const float4 v0 = e < end ? ld_stream(val4 + e) : zero_v;
    const int4 c1 = e + S < end ? ld_stream(col4 + e + S) : zero_c;
    const float4 v1 = e + S < end ? ld_stream(val4 + e + S) : zero_v;
    attract4(yi.x, yi.y, c0, v0, ex, y, ax, ay);
    attract4(yi.x, yi.y, c1, v1, ex, y, ax, ay);
  }
#endif
}

// 64 registers: four blocks of 256 threads per SM, and the grid is exactly
// the resident capacity (one wave).  Warps take 32-row groups from a global
// counter (reset by the splat of the same iteration) in group_order, most
// expensive group first, so no warp idles while another still holds a long
// row and the heaviest groups do not form a tail; there is no block barrier.
__global__ void __launch_bounds__(256, 4) grad_update_kernel(
    const int* __restrict__ row_ptr4, const int4* __restrict__ col4, const float4* __restrict__ val4,
    const float2* __restrict__ y, float2* __restrict__ y_next, float2* __restrict__ update,
    float2* __restrict__ gains, float2* __restrict__ grad_out, const float4* __restrict__ pot,
    LayoutStats* __restrict__ stats, const int* __restrict__ group_order, UpdateParams prm) {
  const int lane = threadIdx.x & 31;
  const int sub = lane >> 3;  // which of the 4 rows of a round
  const int sl = lane & 7;    // lane within the row
  const float ex = prm.exaggeration;
  // 32-row groups not taken by staged_grad_kernel (set at each reorder).
  const int groups = static_cast<int>(stats->group_count);
  for (;;) {
    int ticket = 0;
    if (lane == 0) ticket = static_cast<int>(atomicAdd(&stats->row_groups_taken, 1u));
    ticket = __shfl_sync(0xffffffffu, ticket, 0);
    if (ticket >= groups) break;
    const int row0 = prm.row_begin + __ldg(group_order + ticket) * 32;
    float my_ax = 0.f, my_ay = 0.f;
#pragma unroll 1
    for (int it = 0; it < 8; ++it) {
      const int row = row0 + 4 * it + sub;
      const bool rv = row < prm.row_end;
      const int beg = rv ? __ldg(row_ptr4 + row) : 0;
      const int end = rv ? __ldg(row_ptr4 + row + 1) : 0;
      const float2 yi = rv ? y[row] : make_float2(0.f, 0.f);
      int passes = (end - beg + 15) >> 4;
      passes = max(passes, __shfl_xor_sync(0xffffffffu, passes, 8));
      passes = max(passes, __shfl_xor_sync(0xffffffffu, passes, 16));
      if (passes <= kLongRoundPasses) {
        // Four rows, eight lanes each.
        float ax = 0.f, ay = 0.f;
        stream_row<8>(beg, end, sl, passes, yi, ex, col4, val4, y, ax, ay);
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) {
          ax += __shfl_xor_sync(0xffffffffu, ax, o);
          ay += __shfl_xor_sync(0xffffffffu, ay, o);
        }
        if (sl == it) {
          my_ax = ax;
          my_ay = ay;
        }
      } else {
        // A long (hub) row in the round: its four rows one after another, 32
        // lanes each, so the round costs about a quarter of the longest row.
#pragma unroll 1
        for (int sr = 0; sr < 4; ++sr) {
          const int row_s = row0 + 4 * it + sr;
          const bool vs = row_s < prm.row_end;
          const int beg_s = vs ? __ldg(row_ptr4 + row_s) : 0;
          const int end_s = vs ? __ldg(row_ptr4 + row_s + 1) : 0;
          const float2 yis = vs ? y[row_s] : make_float2(0.f, 0.f);
          float ax = 0.f, ay = 0.f;
          stream_row<32>(beg_s, end_s, lane, (end_s - beg_s + 63) >> 6, yis, ex, col4, val4, y, ax, ay);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            ax += __shfl_xor_sync(0xffffffffu, ax, o);
            ay += __shfl_xor_sync(0xffffffffu, ay, o);
          }
          if (lane == 8 * sr + it) {
            my_ax = ax;
            my_ay = ay;
          }
        }
      }
    }
    // Epilogue: lane L finishes row row0 + 4 (L % 8) + L / 8.
    const int row = row0 + 4 * sl + sub;
    if (row >= prm.row_end) continue;
    finish_row(row, my_ax, my_ay, y, y_next, update, gains, grad_out, pot, stats, prm);
  }
}


// ---- staged row blocks ------------------------------------------------------

constexpr int kStagePerThread = kStageCap / kStageThreads;
static_assert(kStagePerThread * kStageThreads == kStageCap, "union capacity is a whole number of passes");
constexpr int kStageBatch = 8;  // union points whose indices a thread holds at once
static_assert(kStagePerThread % kStageBatch == 0, "whole batches");

// 8-byte asynchronous copy global -> shared (through L1), and the wait for all
// of this thread's outstanding copies.
__device__ __forceinline__ void cp_async8(float2* dst_smem, const float2* src) {
  const unsigned int d = static_cast<unsigned int>(__cvta_generic_to_shared(dst_smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}

// attract4 with y_j from the staged union: four 16-bit union indices.  The
// per-entry arithmetic and its order are attract4's, so a row's sum is the
// same bits whichever kernel computes it.
__device__ __forceinline__ void attract4_staged(float yix, float yiy, uint2 c, float4 v, float ex,
                                                const float2* __restrict__ ys, float& ax, float& ay) {
  // Union indices are below the block's union size by construction; the
  // clamp keeps every shared-memory read inside the staged array regardless.
  const float2 g[4] = {ys[min(c.x & 0xffffu, kStageCap - 1u)], ys[min(c.x >> 16, kStageCap - 1u)],
                       ys[min(c.y & 0xffffu, kStageCap - 1u)], ys[min(c.y >> 16, kStageCap - 1u)]};
  const float pv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float dx = yix - g[q].x;
    const float dy = yiy - g[q].y;
    float d2 = 0.0f;
    d2 += dx * dx;
    d2 += dy * dy;
    const float qq = 1.0f / (1.0f + d2);
    const float w = ex * pv[q] * qq;
    ax += w * dx;
    ay += w * dy;
  }
}

// stream_row over the union-local column indices (same lane/group assignment
// and prefetch as stream_row, hence the same summation order).
template <int S>
__device__ __forceinline__ void stream_row_staged(int beg, int end, int l, int passes, float2 yi, float ex,
                                                  const uint2* __restrict__ col16, const float4* __restrict__ val4,
                                                  const float2* __restrict__ ys, float& ax, float& ay) {
  const uint2 zero_c = make_uint2(0u, 0u);
  const float4 zero_v = make_float4(0.f, 0.f, 0.f, 0.f);
  int e = beg + l;
  uint2 c0 = e < end ? ld_stream(col16 + e) : zero_c;
  float4 v0 = e < end ? ld_stream(val4 + e) : zero_v;
  uint2 c1 = e + S < end ? ld_stream(col16 + e + S) : zero_c;
  float4 v1 = e + S < end ? ld_stream(val4 + e + S) : zero_v;
  for (int p = 0; p < passes; ++p) {
    const int en = e + 2 * S;
    const uint2 nc0 = en < end ? ld_stream(col16 + en) : zero_c;
    const float4 nv0 = en < end ? ld_stream(val4 + en) : zero_v;
    const uint2 nc1 = en + S < end ? ld_stream(col16 + en + S) : zero_c;
    const float4 nv1 = en + S < end ? ld_stream(val4 + en + S) : zero_v;
    attract4_staged(yi.x, yi.y, c0, v0, ex, ys, ax, ay);
    attract4_staged(yi.x, yi.y, c1, v1, ex, ys, ax, ay);
    c0 = nc0;
    v0 = nv0;
    c1 = nc1;
    v1 = nv1;
    e = en;
  }
}

// One block per SM, persistent.  A block takes staged row blocks (kStageRows
// rows each, most expensive first) from a global counter; per row block it
//   1. stages y of the block's column union in shared memory -- one union
//      point per thread, the union list sorted, so a warp's 32 loads touch a
//      few lines of L2 instead of 32 (the union of a 128-row block holds its
//      entries' columns at 0.2-0.27 lines per entry);
//   2. runs the block's 32 four-row rounds (eight lanes per row, a hub round
//      row by row with 32 lanes), taken by the warps from a shared counter in
//      the order stored at the reorder, gathering y_j from shared memory;
//   3. writes each row's attraction sum; staged_finish_kernel then finishes
//      the rows (repulsive gather and update) with one thread per row.
__global__ void __launch_bounds__(kStageThreads, 1) staged_grad_kernel(
    const int* __restrict__ row_ptr4, const uint2* __restrict__ col16, const float4* __restrict__ val4,
    const int* __restrict__ stage_union, const int4* __restrict__ stage_meta, const int* __restrict__ stage_order,
    const unsigned char* __restrict__ stage_rounds, const float2* __restrict__ y,
    float2* __restrict__ attraction, LayoutStats* __restrict__ stats, UpdateParams prm) {
  extern __shared__ float2 ys[];  // kStageCap points
  __shared__ float2 acc[kStageRows];
  __shared__ int s_ticket;
  __shared__ int s_round;
  const int lane = threadIdx.x & 31;
  const int sub = lane >> 3;
  const int sl = lane & 7;
  const float ex = prm.exaggeration;
  const int count = static_cast<int>(stats->stage_count);
  for (;;) {
    if (threadIdx.x == 0) {
      s_ticket = static_cast<int>(atomicAdd(&stats->stage_taken, 1u));
      s_round = 0;
    }
    __syncthreads();
    const int ticket = s_ticket;
    if (ticket >= count) break;  // block-uniform
    const int b = __ldg(stage_order + ticket);
    const int4 meta = __ldg(stage_meta + b);
    const int row0 = prm.row_begin + b * kStageRows;
    {
      // All union indices of this thread first (independent coalesced loads),
      // then the gathers as asynchronous global-to-shared copies: two memory
      // latencies per block instead of one per union point.
      const int* __restrict__ un = stage_union + meta.x;
#pragma unroll 1
      for (int j0 = 0; j0 < kStagePerThread; j0 += kStageBatch) {
        if (static_cast<int>(threadIdx.x) + j0 * kStageThreads >= meta.y) break;
        int idx[kStageBatch];
#pragma unroll
        for (int j = 0; j < kStageBatch; ++j) {
          const int u = static_cast<int>(threadIdx.x) + (j0 + j) * kStageThreads;
          idx[j] = u < meta.y ? __ldg(un + u) : 0;
        }
#pragma unroll
        for (int j = 0; j < kStageBatch; ++j) {
          const int u = static_cast<int>(threadIdx.x) + (j0 + j) * kStageThreads;
          if (u < meta.y) cp_async8(ys + u, y + idx[j]);
        }
      }
      cp_async_wait_all();
    }
    __syncthreads();
    for (;;) {
      int r = 0;
      if (lane == 0) r = atomicAdd(&s_round, 1);
      r = __shfl_sync(0xffffffffu, r, 0);
      if (r >= kStageRounds) break;
      const int round = __ldg(stage_rounds + static_cast<size_t>(b) * kStageRounds + r);
      const int row = row0 + 4 * round + sub;
      const bool rv = row < prm.row_end;
      const int beg = rv ? __ldg(row_ptr4 + row) : 0;
      const int end = rv ? __ldg(row_ptr4 + row + 1) : 0;
      const float2 yi = rv ? y[row] : make_float2(0.f, 0.f);
      int passes = (end - beg + 15) >> 4;
      passes = max(passes, __shfl_xor_sync(0xffffffffu, passes, 8));
      passes = max(passes, __shfl_xor_sync(0xffffffffu, passes, 16));
      if (passes <= kLongRoundPasses) {
        float ax = 0.f, ay = 0.f;
        stream_row_staged<8>(beg, end, sl, passes, yi, ex, col16, val4, ys, ax, ay);
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) {
          ax += __shfl_xor_sync(0xffffffffu, ax, o);
          ay += __shfl_xor_sync(0xffffffffu, ay, o);
        }
        if (sl == 0) acc[4 * round + sub] = make_float2(ax, ay);
      } else {
#pragma unroll 1
        for (int sr = 0; sr < 4; ++sr) {
          const int row_s = row0 + 4 * round + sr;
          const bool vs = row_s < prm.row_end;
          const int beg_s = vs ? __ldg(row_ptr4 + row_s) : 0;
          const int end_s = vs ? __ldg(row_ptr4 + row_s + 1) : 0;
          const float2 yis = vs ? y[row_s] : make_float2(0.f, 0.f);
          float ax = 0.f, ay = 0.f;
          stream_row_staged<32>(beg_s, end_s, lane, (end_s - beg_s + 63) >> 6, yis, ex, col16, val4, ys, ax, ay);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            ax += __shfl_xor_sync(0xffffffffu, ax, o);
            ay += __shfl_xor_sync(0xffffffffu, ay, o);
          }
          if (lane == 0) acc[4 * round + sr] = make_float2(ax, ay);
        }
      }
    }
    __syncthreads();
    if (threadIdx.x < kStageRows) {
      const int row = row0 + static_cast<int>(threadIdx.x);
      if (row < prm.row_end) attraction[row] = acc[threadIdx.x];
    }
  }
}

// The staged rows' epilogue (repulsive gather and update), one thread per row
// of each staged block: a streaming pass kept out of staged_grad_kernel, whose
// single block per SM would otherwise idle through its dependent loads.
__global__ void __launch_bounds__(kStageRows) staged_finish_kernel(
    const int* __restrict__ stage_order, const float2* __restrict__ attraction, const float2* __restrict__ y,
    float2* __restrict__ y_next, float2* __restrict__ update, float2* __restrict__ gains,
    float2* __restrict__ grad_out, const float4* __restrict__ pot, const LayoutStats* __restrict__ stats,
    UpdateParams prm) {
  if (static_cast<int>(blockIdx.x) >= static_cast<int>(stats->stage_count)) return;
  const int b = stage_order[blockIdx.x];
  const int row = prm.row_begin + b * kStageRows + static_cast<int>(threadIdx.x);
  if (row >= prm.row_end) return;
  const float2 a = attraction[row];
  finish_row(row, a.x, a.y, y, y_next, update, gains, grad_out, pot, stats, prm);
}

__global__ void center_copy_kernel(const float2* __restrict__ y, const LayoutStats* __restrict__ stats,
                                   int n, float2* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float2 p = y[i];
  if (stats->center) {
    const float mx = static_cast<float>(stats->sum_x / static_cast<double>(n));
    const float my = static_cast<float>(stats->sum_y / static_cast<double>(n));
    p.x -= mx;
    p.y -= my;
  }
  out[i] = p;
}

}  // namespace

const char* kernel_kind_name(int kind) {
  switch (kind) {
    case kKindSplat: return "splat_kernel";
    case kKindFftRows: return "fft_rows_fwd_kernel";
    case kKindFftCols: return "fft_cols_kernel";
    case kKindFftRowsInv: return "fft_rows_inv_kernel";
    case kKindGradUpdate: return "grad_update_kernel";
    case kKindChargeSum: return "charge_allreduce";
    case kKindLayoutGather: return "layout_allgather";
    case kKindLayoutStats: return "layout_stats_kernel";
    case kKindStagedGrad: return "staged_grad_kernel";
    default: return "?";
  }
}

void grad_update_launch_shape(int rows, int* blocks, int* threads) {
  *threads = 256;  // 8 warps, each taking 32-row groups
  *blocks = std::max(1, std::min(sm_count() * 4, (rows + 255) / 256));
}

int configure_kernels(TsneSession* s) {
  if (s->fft != 2 * s->grid) {
    set_error("t-SNE FFT length must be twice the grid side");
    return 1;
  }
  switch (s->log_fft) {
#define FE_FFT_CONFIGURE_CASE(L) \
  case L:                        \
    FE_TRY(fft_configure<L>());  \
    break;
    FE_FFT_LOG_M_CASES(FE_FFT_CONFIGURE_CASE)
#undef FE_FFT_CONFIGURE_CASE
    default:
      set_error("t-SNE FFT length outside the instantiated range (grid 4 to 1024)");
      return 1;
  }
  FE_CUDA(cudaFuncSetAttribute(staged_grad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(kStageCap * sizeof(float2))),
          "cudaFuncSetAttribute(staged_grad_kernel)");
  return 0;
}

int launch_stats(TsneSession* s, int center) {
  const int blocks = std::max(1, std::min(2 * sm_count(), (s->n / 2 + 511) / 512));
  layout_stats_kernel<<<blocks, 512, 0, s->stream>>>(s->y[s->cur], s->n, s->grid, s->update_partials, s->stats,
                                                     center);
  FE_LAUNCH("layout_stats_kernel");
  return 0;
}

namespace {

struct ProfileScope {
  TsneSession* s;
  int kind;
  ProfileScope(TsneSession* s_, int kind_) : s(s_), kind(kind_) {
    if (!s->profile) return;
    cudaEvent_t e;
    cudaEventCreate(&e);
    cudaEventRecord(e, s->stream);
    s->events.push_back(e);
  }
  ~ProfileScope() {
    if (!s->profile) return;
    cudaEvent_t e;
    cudaEventCreate(&e);
    cudaEventRecord(e, s->stream);
    s->events.push_back(e);
    s->event_kind.push_back(kind);
  }
};

}  // namespace

int launch_iteration(TsneSession* s, GradMode mode, float exaggeration, float momentum,
                     float learning_rate, float min_gain, float max_step_norm) {
  const int g = s->grid;
  {
    ProfileScope ps(s, kKindSplat);
    const unsigned blocks = static_cast<unsigned>((s->n + kSplatThreads - 1) / kSplatThreads);
    if (s->interp == 1) {
      splat_lagrange_kernel<<<blocks, kSplatThreads, 0, s->stream>>>(s->y[s->cur], s->stats, s->n, g, s->charges,
                                                                     s->row_begin, s->row_end);
      FE_LAUNCH("splat_lagrange_kernel");
    } else {
      splat_kernel<<<blocks, kSplatThreads, 0, s->stream>>>(s->y[s->cur], s->stats, s->n, g, s->charges,
                                                            s->row_begin, s->row_end);
      FE_LAUNCH("splat_kernel");
    }
  }
  if (s->sharded) {
    ProfileScope ps(s, kKindChargeSum);
    FE_TRY(shard_sum_charges(s));
  }
  {
    ProfileScope ps(s, kKindFftRows);
    FE_TRY(fft_launch_pass(s, 0));
  }
  {
    ProfileScope ps(s, kKindFftCols);
    FE_TRY(fft_launch_pass(s, 1));
  }
  {
    ProfileScope ps(s, kKindFftRowsInv);
    FE_TRY(fft_launch_pass(s, 2));
  }
  const UpdateParams prm{s->n, s->row_begin, s->row_end, g, exaggeration, momentum,
                         learning_rate, min_gain, max_step_norm, static_cast<int>(mode)};
  if (s->stage_enabled) {
    ProfileScope ps(s, kKindStagedGrad);
    staged_grad_kernel<<<sm_count(), kStageThreads, kStageCap * sizeof(float2), s->stream>>>(
        s->row_ptr4, s->stage_col16, s->csr4_val, s->stage_union, s->stage_meta, s->stage_order,
        s->stage_rounds, s->y[s->cur], s->attraction, s->stats, prm);
    FE_LAUNCH("staged_grad_kernel");
    const int blocks = std::max(1, (s->row_end - s->row_begin + kStageRows - 1) / kStageRows);
    staged_finish_kernel<<<blocks, kStageRows, 0, s->stream>>>(
        s->stage_order, s->attraction, s->y[s->cur], s->y[s->cur ^ 1], s->update, s->gains, s->grad_out,
        s->pot, s->stats, prm);
    FE_LAUNCH("staged_finish_kernel");
  }
  {
    ProfileScope ps(s, kKindGradUpdate);
    grad_update_kernel<<<s->update_blocks, s->update_threads, 0, s->stream>>>(
        s->row_ptr4, s->csr4_col, s->csr4_val, s->y[s->cur], s->y[s->cur ^ 1], s->update,
        s->gains, s->grad_out, s->pot, s->stats, s->group_order, prm);
    FE_LAUNCH("grad_update_kernel");
  }
  if (mode != kGradUpdate) return 0;
  s->cur ^= 1;
  if (s->sharded) {
    // Every rank now holds its own updated rows: gather the others'.
    ProfileScope ps(s, kKindLayoutGather);
    FE_TRY(shard_gather_rows(s, s->y[s->cur]));
  }
  // Statistics of the whole new layout for the next iteration's grid, in one
  // fixed reduction order (so identical on every rank of a sharded run).
  ProfileScope ps(s, kKindLayoutStats);
  FE_TRY(launch_stats(s, 1));
  return 0;
}

int launch_center_output(TsneSession* s, float2* out) {
  center_copy_kernel<<<(s->n + 255) / 256, 256, 0, s->stream>>>(s->y[s->cur], s->stats, s->n, out);
  FE_LAUNCH("center_copy_kernel");
  return 0;
}

}  // namespace fe
