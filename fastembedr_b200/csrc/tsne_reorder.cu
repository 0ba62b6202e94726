// Internal point order and the internal copy of P.
//
// The optimizer's arithmetic does not depend on the order in which points are
// stored; its memory behaviour does.  The attraction kernel gathers y_j for
// every entry of P, the splat scatters into the grid and the repulsion gathers
// potentials.  Storing points in Morton (Z-curve) order of their grid position
// makes all three local -- KNN neighbours end up close in the layout, hence
// close in memory -- so y_j gathers hit L1/L2 and lanes of a warp touch
// neighbouring grid nodes.
//
// P is kept twice: the caller-order CSR (canonical, never permuted) and an
// internal-order copy, rows padded to whole 16-byte groups, that the
// attraction kernel streams.  A reorder
//   1. sorts points by a 30-bit Morton key of the current layout (or keeps the
//      caller's order for the first build),
//   2. permutes the layout, optimizer state and permutation arrays,
//   3. rebuilds the internal copy from the caller-order CSR: internal row r is
//      caller row perm[r], with columns renamed through rank.
#include "tsne.cuh"

#include <cub/cub.cuh>

#include <algorithm>
#include <climits>

namespace fe {
namespace {

__device__ __forceinline__ unsigned int spread_bits_15(unsigned int v) {
  v &= 0x7fffu;
  v = (v | (v << 8)) & 0x00ff00ffu;
  v = (v | (v << 4)) & 0x0f0f0f0fu;
  v = (v | (v << 2)) & 0x33333333u;
  v = (v | (v << 1)) & 0x55555555u;
  return v;
}

__global__ void morton_keys_kernel(const float2* __restrict__ y, const LayoutStats* __restrict__ stats,
                                   int n, int g, int by_layout, unsigned int* __restrict__ keys,
                                   int* __restrict__ idx) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  idx[i] = i;
  if (!by_layout) {
    keys[i] = 0u;  // a stable sort keeps the current order
    return;
  }
  const GridGeom q = stats->geom;
  float2 p = y[i];
  p.x -= q.mean_x;
  p.y -= q.mean_y;
  const float extent = q.spacing * static_cast<float>(g - 1);
  const float sx = fminf(fmaxf((p.x - q.lower_x) / extent, 0.0f), 1.0f);
  const float sy = fminf(fmaxf((p.y - q.lower_y) / extent, 0.0f), 1.0f);
  const unsigned int ix = min(32767u, static_cast<unsigned int>(sx * 32767.0f));
  const unsigned int iy = min(32767u, static_cast<unsigned int>(sy * 32767.0f));
  keys[i] = spread_bits_15(ix) | (spread_bits_15(iy) << 1);
}

// order[r] = old internal index now at r.  New perm/rank, point arrays and the
// padded row lengths (in groups of four entries).
__global__ void permute_points_kernel(const int* __restrict__ order, int n, const int* __restrict__ perm_in,
                                      int* __restrict__ perm_out, int* __restrict__ rank_out,
                                      const int* __restrict__ row_ptr, int* __restrict__ groups,
                                      const float2* __restrict__ y_in, float2* __restrict__ y_out,
                                      const float2* __restrict__ u_in, float2* __restrict__ u_out,
                                      const float2* __restrict__ g_in, float2* __restrict__ g_out) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  const int o = order[r];
  const int caller = perm_in[o];
  perm_out[r] = caller;
  rank_out[caller] = r;
  groups[r] = (row_ptr[caller + 1] - row_ptr[caller] + 3) >> 2;
  y_out[r] = y_in[o];
  u_out[r] = u_in[o];
  g_out[r] = g_in[o];
}

// One warp per internal row: coalesced copy of caller row perm[r] with renamed
// columns, padded with (own row, 0) to a whole group.
__global__ void fill_rows_kernel(const int* __restrict__ perm, const int* __restrict__ rank,
                                 const int* __restrict__ row_ptr, const int* __restrict__ col,
                                 const float* __restrict__ val, int row_begin, int row_end,
                                 const int* __restrict__ row_ptr4, int* __restrict__ out_col,
                                 float* __restrict__ out_val) {
  const long long gid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int r = row_begin + static_cast<int>(gid >> 5);
  const int lane = static_cast<int>(gid & 31);
  if (r >= row_end) return;
  const int caller = perm[r];
  const int beg = row_ptr[caller];
  const int len = row_ptr[caller + 1] - beg;
  const long long dst = static_cast<long long>(row_ptr4[r]) * 4;
  const int padded = (row_ptr4[r + 1] - row_ptr4[r]) * 4;
  for (int e = lane; e < padded; e += 32) {
    if (e < len) {
      out_col[dst + e] = rank[col[beg + e]];
      out_val[dst + e] = val[beg + e];
    } else {
      out_col[dst + e] = r;
      out_val[dst + e] = 0.0f;
    }
  }
}

__global__ void unpermute_kernel(const float2* __restrict__ in, const int* __restrict__ perm, int n,
                                 float2* __restrict__ out) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < n) out[perm[r]] = in[r];
}

__global__ void permute_in_kernel(const float2* __restrict__ in, const int* __restrict__ perm, int n,
                                  float2* __restrict__ out) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < n) out[r] = in[perm[r]];
}

// Cost of a 32-row group for the attraction kernel: per round of four rows,
// the passes of the longest row (a pass of eight lanes covers 16 groups of
// four entries) plus one; a round past kLongRoundPasses runs its rows one by
// one with 32 lanes (64 groups a pass), plus one per row.
__global__ void group_cost_kernel(const int* __restrict__ row_ptr4, int row_begin, int row_end, int groups,
                                  const int4* __restrict__ stage_meta, unsigned int* __restrict__ cost,
                                  int* __restrict__ ids, unsigned int* __restrict__ group_count) {
  const int grp = blockIdx.x * blockDim.x + threadIdx.x;
  if (grp >= groups) return;
  if (stage_meta != nullptr && stage_meta[(grp * 32) / kStageRows].z) {
    // Staged row block: its rows belong to staged_grad_kernel; sorted last.
    cost[grp] = 0u;
    ids[grp] = grp;
    return;
  }
  const int row0 = row_begin + grp * 32;
  unsigned int total = 0;
  for (int round = 0; round < 8; ++round) {
    int passes = 0, wide = 0;
    for (int sub = 0; sub < 4; ++sub) {
      const int row = row0 + 4 * round + sub;
      if (row >= row_end) continue;
      const int len = row_ptr4[row + 1] - row_ptr4[row];
      passes = max(passes, (len + 15) >> 4);
      wide += ((len + 63) >> 6) + 1;
    }
    total += passes <= kLongRoundPasses ? static_cast<unsigned int>(passes) + 1u : static_cast<unsigned int>(wide);
  }
#ifndef FE_LPT_THRESHOLD
#define FE_LPT_THRESHOLD 0
#endif
  // Groups at or below the threshold keep their (Morton) order behind the
  // expensive ones (the descending sort is stable), ahead of staged groups.
  cost[grp] = total > FE_LPT_THRESHOLD ? total : 1u;
  ids[grp] = grp;
  atomicAdd(group_count, 1u);
}

// Cost estimate of one four-row round (group_cost_kernel's per-round term).
__device__ __forceinline__ unsigned int round_cost(const int* __restrict__ row_ptr4, int row0, int row_end) {
  int passes = 0, wide = 0;
  for (int sub = 0; sub < 4; ++sub) {
    const int row = row0 + sub;
    if (row >= row_end) continue;
    const int len = row_ptr4[row + 1] - row_ptr4[row];
    passes = max(passes, (len + 15) >> 4);
    wide += ((len + 63) >> 6) + 1;
  }
  return passes <= kLongRoundPasses ? static_cast<unsigned int>(passes) + 1u : static_cast<unsigned int>(wide);
}

// One block per staged row block candidate (kStageRows internal rows, whose
// entries are contiguous in the internal copy of P).
//   1. bounds [lo, hi] of the block's column indices; a span above kStageSpan
//      leaves the block to grad_update_kernel;
//   2. a bitmap of the columns present, then the union size as the sum of
//      popcounts (an exclusive scan gives each bitmap word its union prefix);
//      a union above kStageCap, or one spread over more than 0.6 lines of y
//      per entry, leaves the block to grad_update_kernel;
//   3. the union list (sorted internal indices) at the block's first entry
//      position, and each entry's union index: prefix of its word plus the
//      set bits below its own;
//   4. {union offset, union size, staged, entries}, a cost for the block order
//      and the block's rounds sorted by cost, most expensive first.
__global__ void __launch_bounds__(kStageBuildThreads, 1) stage_build_kernel(
    const int* __restrict__ row_ptr4, const int* __restrict__ csr_col, int row_begin, int row_end,
    unsigned short* __restrict__ col16, int* __restrict__ stage_union, int4* __restrict__ stage_meta,
    unsigned char* __restrict__ stage_rounds, unsigned int* __restrict__ stage_cost, int* __restrict__ stage_ids,
    unsigned int* __restrict__ stage_count) {
  extern __shared__ unsigned int bits[];  // kStageSpan / 32 words, then the per-word prefixes
  unsigned short* wpref = reinterpret_cast<unsigned short*>(bits + kStageSpan / 32);
  __shared__ int s_lo[kStageBuildThreads / 32], s_hi[kStageBuildThreads / 32];
  __shared__ int s_scan[kStageBuildThreads / 32];
  __shared__ unsigned int s_rcost[kStageRounds];
  const int b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  constexpr int nw = kStageBuildThreads / 32;
  const int r0 = row_begin + b * kStageRows;
  const int r1 = min(row_end, r0 + kStageRows);
  const long long e0 = static_cast<long long>(row_ptr4[r0]) * 4;
  const long long e1 = static_cast<long long>(row_ptr4[r1]) * 4;
  if (tid < kStageRounds) s_rcost[tid] = round_cost(row_ptr4, r0 + 4 * tid, r1);

  int lo = INT_MAX, hi = INT_MIN;
  for (long long e = e0 + tid; e < e1; e += kStageBuildThreads) {
    const int c = csr_col[e];
    lo = min(lo, c);
    hi = max(hi, c);
  }
  lo = __reduce_min_sync(0xffffffffu, lo);
  hi = __reduce_max_sync(0xffffffffu, hi);
  if (lane == 0) {
    s_lo[wid] = lo;
    s_hi[wid] = hi;
  }
  __syncthreads();
  lo = INT_MAX;
  hi = INT_MIN;
  for (int w = 0; w < nw; ++w) {
    lo = min(lo, s_lo[w]);
    hi = max(hi, s_hi[w]);
  }
  const long long span = e1 > e0 ? static_cast<long long>(hi) - lo + 1 : 0;
  bool staged = span <= kStageSpan;
  int total = 0;
  if (staged && span > 0) {  // block-uniform
    const int words = static_cast<int>((span + 31) >> 5);
    for (int w = tid; w < words; w += kStageBuildThreads) bits[w] = 0u;
    __syncthreads();
    for (long long e = e0 + tid; e < e1; e += kStageBuildThreads) {
      const int c = csr_col[e] - lo;
      atomicOr(&bits[c >> 5], 1u << (c & 31));
    }
    __syncthreads();
    const int per = (words + kStageBuildThreads - 1) / kStageBuildThreads;
    const int w0 = min(words, tid * per);
    const int w1 = min(words, w0 + per);
    int mine = 0, lines = 0;
    for (int w = w0; w < w1; ++w) {
      const unsigned int m = bits[w];
      mine += __popc(m);
      lines += ((m & 0xffffu) != 0u) + ((m >> 16) != 0u);  // 16 points of y per 128-byte line
    }
    lines = __reduce_add_sync(0xffffffffu, lines);
    if (lane == 0) s_lo[wid] = lines;  // the bounds are no longer needed
    int incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) s_scan[wid] = incl;
    __syncthreads();
    if (wid == 0) {
      int v = lane < nw ? s_scan[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      if (lane < nw) s_scan[lane] = v;
    }
    __syncthreads();
    total = s_scan[nw - 1];
    int all_lines = 0;
    for (int w = 0; w < nw; ++w) all_lines += s_lo[w];
    // Staging pays when the union's points share lines: at most 0.6 lines per
    // entry (ordered layouts: 0.12-0.27; the caller's order before the first
    // spatial reorder: about 1).
    staged = total <= kStageCap && 5LL * all_lines <= 3LL * (e1 - e0);
    if (staged) {
      int run = incl - mine + (wid > 0 ? s_scan[wid - 1] : 0);
      for (int w = w0; w < w1; ++w) {
        wpref[w] = static_cast<unsigned short>(run);
        for (unsigned int m = bits[w]; m; m &= m - 1u) {
          stage_union[e0 + run] = lo + 32 * w + (__ffs(m) - 1);
          ++run;
        }
      }
    }
    __syncthreads();
    if (staged) {
      for (long long e = e0 + tid; e < e1; e += kStageBuildThreads) {
        const int c = csr_col[e] - lo;
        const int w = c >> 5;
        const unsigned int below = bits[w] & ((1u << (c & 31)) - 1u);
        col16[e] = static_cast<unsigned short>(wpref[w] + __popc(below));
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    stage_meta[b] = make_int4(static_cast<int>(e0), total, staged ? 1 : 0, static_cast<int>(e1 - e0));
    stage_cost[b] = staged ? static_cast<unsigned int>((e1 - e0) + total / 4 + 1) : 0u;
    stage_ids[b] = b;
    if (staged) atomicAdd(stage_count, 1u);
    unsigned char order[kStageRounds];
    for (int r = 0; r < kStageRounds; ++r) {
      // insertion sort, most expensive first, ties in round order
      int j = r;
      while (j > 0 && s_rcost[order[j - 1]] < s_rcost[r]) {
        order[j] = order[j - 1];
        --j;
      }
      order[j] = static_cast<unsigned char>(r);
    }
    for (int r = 0; r < kStageRounds; ++r) stage_rounds[static_cast<size_t>(b) * kStageRounds + r] = order[r];
  }
}

}  // namespace

int build_group_order(TsneSession* s) {
  FE_CUDA(cudaMemsetAsync(&s->stats->stage_count, 0, sizeof(unsigned int), s->stream), "memset stage count");
  FE_CUDA(cudaMemsetAsync(&s->stats->group_count, 0, sizeof(unsigned int), s->stream), "memset group count");
  const int rows = s->row_end - s->row_begin;
  const int groups = (rows + 31) / 32;
  if (groups <= 0) return 0;
  const bool staged = s->stage_enabled && s->stage_col16 != nullptr;
  if (staged) {
    const int blocks = (rows + kStageRows - 1) / kStageRows;
    const int smem = kStageSpan / 32 * static_cast<int>(sizeof(unsigned int) + sizeof(unsigned short));
    FE_CUDA(cudaFuncSetAttribute(stage_build_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
            "cudaFuncSetAttribute(stage_build_kernel)");
    stage_build_kernel<<<blocks, kStageBuildThreads, smem, s->stream>>>(
        s->row_ptr4, reinterpret_cast<const int*>(s->csr4_col), s->row_begin, s->row_end,
        reinterpret_cast<unsigned short*>(s->stage_col16), s->stage_union, s->stage_meta, s->stage_rounds,
        s->stage_cost, s->stage_ids, &s->stats->stage_count);
    FE_LAUNCH("stage_build_kernel");
    size_t tb = s->ro_temp_bytes;
    FE_CUDA(cub::DeviceRadixSort::SortPairsDescending(s->ro_temp, tb, s->stage_cost, s->stage_cost_sorted,
                                                      s->stage_ids, s->stage_order, blocks, 0, 32, s->stream),
            "cub::DeviceRadixSort(stage cost)");
  }
  group_cost_kernel<<<(groups + 255) / 256, 256, 0, s->stream>>>(
      s->row_ptr4, s->row_begin, s->row_end, groups, staged ? s->stage_meta : nullptr, s->group_cost,
      s->group_ids, &s->stats->group_count);
  FE_LAUNCH("group_cost_kernel");
  size_t tb = s->ro_temp_bytes;
  FE_CUDA(cub::DeviceRadixSort::SortPairsDescending(s->ro_temp, tb, s->group_cost, s->group_cost_sorted,
                                                    s->group_ids, s->group_order, groups, 0, 32, s->stream),
          "cub::DeviceRadixSort(group cost)");
  return 0;
}

int reorder_temp_bytes(int n, size_t* bytes) {
  size_t sort_bytes = 0, scan_bytes = 0, desc_bytes = 0;
  FE_CUDA(cub::DeviceRadixSort::SortPairsDescending(nullptr, desc_bytes, static_cast<unsigned int*>(nullptr),
                                                    static_cast<unsigned int*>(nullptr), static_cast<int*>(nullptr),
                                                    static_cast<int*>(nullptr), n / 32 + 1, 0, 32),
          "cub::DeviceRadixSort(sizing)");
  FE_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, static_cast<unsigned int*>(nullptr),
                                          static_cast<unsigned int*>(nullptr), static_cast<int*>(nullptr),
                                          static_cast<int*>(nullptr), n, 0, 30),
          "cub::DeviceRadixSort(sizing)");
  FE_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, static_cast<int*>(nullptr),
                                        static_cast<int*>(nullptr), n + 1),
          "cub::DeviceScan(sizing)");
  *bytes = std::max(std::max(sort_bytes, scan_bytes), desc_bytes);
  return 0;
}

int session_reorder(TsneSession* s, bool by_layout) {
  const int n = s->n;
  const unsigned blocks = static_cast<unsigned>((n + 255) / 256);
  cudaStream_t st = s->stream;
  const int cur = s->cur;
  if (s->sharded) {
    // Each rank's optimizer state is current on its own rows only; rows
    // change owners with the new order.
    FE_TRY(shard_gather_rows(s, s->update));
    FE_TRY(shard_gather_rows(s, s->gains));
  }

  morton_keys_kernel<<<blocks, 256, 0, st>>>(s->y[cur], s->stats, n, s->grid, by_layout ? 1 : 0, s->ro_keys,
                                             s->ro_idx);
  FE_LAUNCH("morton_keys_kernel");
  size_t tb = s->ro_temp_bytes;
  FE_CUDA(cub::DeviceRadixSort::SortPairs(s->ro_temp, tb, s->ro_keys, s->ro_keys_sorted, s->ro_idx, s->ro_order,
                                          n, 0, 30, st),
          "cub::DeviceRadixSort(morton)");
  // The permuted layout lands in the free half of the double buffer and is
  // copied back, so the buffer parity (and every captured graph) is unchanged.
  float2* y_new = s->y[cur ^ 1];
  permute_points_kernel<<<blocks, 256, 0, st>>>(s->ro_order, n, s->perm, s->ro_perm, s->ro_rank, s->row_ptr,
                                                s->ro_groups, s->y[cur], y_new, s->update, s->ro_update,
                                                s->gains, s->ro_gains);
  FE_LAUNCH("permute_points_kernel");
  FE_CUDA(cudaMemcpyAsync(s->y[cur], y_new, sizeof(float2) * n, cudaMemcpyDeviceToDevice, st), "permute layout");
  FE_CUDA(cudaMemcpyAsync(s->update, s->ro_update, sizeof(float2) * n, cudaMemcpyDeviceToDevice, st),
          "permute update");
  FE_CUDA(cudaMemcpyAsync(s->gains, s->ro_gains, sizeof(float2) * n, cudaMemcpyDeviceToDevice, st),
          "permute gains");
  FE_CUDA(cudaMemcpyAsync(s->perm, s->ro_perm, sizeof(int) * n, cudaMemcpyDeviceToDevice, st), "permute perm");
  FE_CUDA(cudaMemcpyAsync(s->rank, s->ro_rank, sizeof(int) * n, cudaMemcpyDeviceToDevice, st), "permute rank");
  FE_CUDA(cudaMemsetAsync(s->ro_groups + n, 0, sizeof(int), st), "memset");
  tb = s->ro_temp_bytes;
  FE_CUDA(cub::DeviceScan::ExclusiveSum(s->ro_temp, tb, s->ro_groups, s->row_ptr4, n + 1, st),
          "cub::DeviceScan(row_ptr4)");
  if (s->csr4_capacity == 0) {
    // First build: size the padded copy.  The total of padded groups does not
    // depend on the point order, so later reorders reuse this allocation.
    int total = 0;
    FE_CUDA(cudaMemcpyAsync(&total, s->row_ptr4 + n, sizeof(int), cudaMemcpyDeviceToHost, st), "D2H");
    FE_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize(reorder)");
    if (total < 0) {
      set_error("padded P exceeds the 32-bit group range");
      return 1;
    }
    FE_TRY(memory_preflight(static_cast<size_t>(total) * 32, "padded P preflight"));
    const size_t groups = std::max<size_t>(1, static_cast<size_t>(total));
    FE_CUDA(fe::dev_malloc(&s->csr4_col, sizeof(int4) * groups), "cudaMalloc(P cols)");
    FE_CUDA(fe::dev_malloc(&s->csr4_val, sizeof(float4) * groups), "cudaMalloc(P vals)");
    // Staged row blocks address entries and union lists with 32-bit offsets.
    if (s->stage_enabled && static_cast<long long>(total) * 4 < INT_MAX &&
        memory_preflight(static_cast<size_t>(total) * 24, "staged P preflight") == 0) {
      FE_CUDA(fe::dev_malloc(&s->stage_col16, sizeof(uint2) * groups), "cudaMalloc(staged P cols)");
      FE_CUDA(fe::dev_malloc(&s->stage_union, sizeof(int4) * groups), "cudaMalloc(staged unions)");
    } else {
      clear_error();
      s->stage_enabled = false;
    }
    s->csr4_capacity = total;
    s->csr4_groups = total;
    drop_graphs(s);
  }
  // Only this rank's rows are streamed by its attraction kernel; each row
  // keeps its place in the whole-P layout of the copy.
  const int rows = s->row_end - s->row_begin;
  if (rows > 0) {
    const unsigned warp_blocks = static_cast<unsigned>((static_cast<long long>(rows) * 32 + 255) / 256);
    fill_rows_kernel<<<warp_blocks, 256, 0, st>>>(s->perm, s->rank, s->row_ptr, s->col, s->val, s->row_begin,
                                                  s->row_end, s->row_ptr4, reinterpret_cast<int*>(s->csr4_col),
                                                  reinterpret_cast<float*>(s->csr4_val));
  }
  FE_LAUNCH("fill_rows_kernel");
  s->identity_perm = false;
  return build_group_order(s);
}

int launch_unpermute(TsneSession* s, const float2* in, float2* out) {
  unpermute_kernel<<<(s->n + 255) / 256, 256, 0, s->stream>>>(in, s->perm, s->n, out);
  FE_LAUNCH("unpermute_kernel");
  return 0;
}

int launch_permute_in(TsneSession* s, const float2* in, float2* out) {
  permute_in_kernel<<<(s->n + 255) / 256, 256, 0, s->stream>>>(in, s->perm, s->n, out);
  FE_LAUNCH("permute_in_kernel");
  return 0;
}

}  // namespace fe
