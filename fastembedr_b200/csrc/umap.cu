// UMAP edge-sampled SGD over a COO graph (objective 0, the UMAP cross entropy).
//
// Per epoch e and edge (h, t) with period p = epochs_per_sample:
//   positives = floor(e/p) - floor((e-1)/p)  (0 at e = 0)
//   each positive: d2 = max(eps, |y_h - y_t|^2), c = -2ab d2^(b-1) / (1 + a d2^b),
//                  g = clip4(c (y_h - y_t)) * alpha;  y_h += g, y_t -= g
//   negatives (count from the negative schedule): vertex from a counter-based
//                  hash of (seed, epoch, head, key, sample); skip head/tail;
//                  c = 2 gamma b / ((0.001 + d2)(1 + a d2^b)); y_h += clip4(c d) * alpha
//   alpha = lr (1 - e / n_epochs); after the epoch: NaN -> 0, clamp to +-16.
// This restates fast_knn_umap_coo_replay_cpp (src/fast_knn_umap.cpp:4904-5056)
// and the reference kernels embed_epoch_coo_{atomic,delta}_kernel
// (src/embedding_cuda_kernels.cpp:3066-3222).  d^b uses the reference's own
// exponent-interpolation approximation (umap_powf_fast, src/fast_knn_umap.cpp:179-206).
//
// Modes (optimizer_mode 0 is Hogwild, 1 Jacobi, as in the reference):
//   kUmapInplace: Hogwild at edge granularity.  Each edge reads its endpoints
//     once, applies its positive and negative samples in turn to running copies
//     (the CPU replay's order within an edge), then adds its net move with one
//     8-byte vector atomic per endpoint (red.global.add.v2.f32); head moves of
//     consecutive edges sharing a head are first summed across the warp.  The
//     COO entry point uses it: its parity target is the CPU replay, and on the
//     70k configuration (CPU graph, COO grouped by head) it reaches 0.00773 kNN
//     preservation against the CPU replay's 0.00791 (sample granularity: 0.00725,
//     the reference CUDA kernel: 0.00708; means of 3 seeds).
//   kUmapInplaceSample: Hogwild at sample granularity, as
//     embed_epoch_coo_atomic_kernel: every sample reads its endpoints afresh from
//     L2 (ld.global.cg, so moves made since by this and concurrent edges are
//     seen) and applies its move at once with vector atomics.  The device-KNN
//     path uses it: its only reference is that CUDA kernel, and with its
//     rank-major edges and small diffusion start the edge-granularity form lost
//     7-11% kNN preservation against it on 50-D mixtures.
//   kUmapDelta: Jacobi.  Forces are evaluated against the layout frozen at epoch
//     start and accumulated into a delta buffer, which a second kernel applies
//     together with the sanitize step; head moves are combined as above.
#include "umap.cuh"

#include "nccl_loader.cuh"

#include <cub/cub.cuh>
#include <thrust/iterator/counting_iterator.h>

#include <cfloat>
#include <cmath>

namespace fe {
namespace {

__device__ __forceinline__ float umap_pow(float x, float b) {
  if (x <= 0.0f) return 0.0f;
  const unsigned int bits = __float_as_uint(x);
  const float bias_word = 1064866805.0f;
  const int whole = static_cast<int>(b);
  const float frac = b - static_cast<float>(whole);
  const unsigned int interp = static_cast<unsigned int>(frac * (static_cast<float>(bits) - bias_word) + bias_word);
  const float frac_pow = __uint_as_float(interp);
  float int_pow = 1.0f;
  float base = x;
  int e = whole;
  while (e > 0) {
    if (e & 1) int_pow *= base;
    base *= base;
    e >>= 1;
  }
  return int_pow * frac_pow;
}

__device__ __forceinline__ int positive_samples(float period, int epoch) {
  if (period <= 0.0f || !isfinite(period) || epoch == 0) return 0;
  const float now = static_cast<float>(epoch);
  const float prev = static_cast<float>(epoch - 1);
  const int s = static_cast<int>(floorf(now / period)) - static_cast<int>(floorf(prev / period));
  return s > 0 ? s : 0;
}

__device__ __forceinline__ int negative_samples(float period, int nsr, int epoch) {
  if (nsr <= 0 || period <= 0.0f || !isfinite(period) || epoch == 0) return 0;
  const float now = static_cast<float>(epoch);
  const float prev = static_cast<float>(epoch - 1);
  const int cur = static_cast<int>(floorf(now / period));
  const int old = static_cast<int>(floorf(prev / period));
  if (cur <= old) return 0;
  const float neg_period = period / static_cast<float>(nsr);
  if (neg_period <= 0.0f || !isfinite(neg_period)) return 0;
  const int cur_total = static_cast<int>(floorf((now - neg_period) / neg_period));
  int prev_total = 0;
  if (cur > 1) {
    const float prev_active = ceilf(static_cast<float>(cur - 1) * period);
    prev_total = static_cast<int>(floorf((prev_active - neg_period) / neg_period));
  }
  const int s = cur_total - prev_total;
  return s > 0 ? s : 0;
}

__device__ __forceinline__ unsigned int mix32(unsigned int x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

__device__ __forceinline__ int negative_vertex(unsigned int n, unsigned int seed, int epoch, int head,
                                               unsigned int key, int sample) {
  unsigned int x = seed;
  x ^= static_cast<unsigned int>(epoch) * 0x9e3779b9u;
  x ^= (static_cast<unsigned int>(head) + 1u) * 0x85ebca6bu;
  x ^= (key + 1u) * 0xc2b2ae35u;
  x ^= (static_cast<unsigned int>(sample) + 1u) * 0x27d4eb2du;
  return static_cast<int>(mix32(x) % n);
}

__device__ __forceinline__ float clip4(float v) { return v < -4.0f ? -4.0f : (v > 4.0f ? 4.0f : v); }

template <int Mode, bool Compact>
__global__ void __launch_bounds__(256) umap_epoch_kernel(const int* __restrict__ heads,
                                                         const int* __restrict__ tails,
                                                         const float* __restrict__ periods,
                                                         long long edge_begin, long long edge_end,
                                                         const int* __restrict__ active,
                                                         const int* __restrict__ active_count,
                                                         float2* layout, const float2* __restrict__ frozen,
                                                         float2* __restrict__ delta, UmapParams p,
                                                         int epoch, long long* positive_count) {
  const float eps = 1.1920928955078125e-7f;
  const float alpha = p.learning_rate * (1.0f - static_cast<float>(epoch) / fmaxf(1.0f, static_cast<float>(p.n_epochs)));
  const float2* src = Mode == kUmapDelta ? frozen : layout;
  float2* dst = Mode == kUmapDelta ? delta : layout;
  auto owned = [&](int v) { return v >= p.own_begin && v < p.own_end; };
  const int lane = threadIdx.x & 31;
  long long local_pos = 0;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  // Items: the edges [edge_begin, edge_end), or with Compact the firing edge
  // ids listed in active[0, *active_count) (in edge order).  Whole warps
  // iterate together so the head-run reduction sees full warps.
  const long long n_items = Compact ? static_cast<long long>(*active_count) : edge_end - edge_begin;
  const long long base0 = static_cast<long long>(blockIdx.x) * blockDim.x + (threadIdx.x & ~31);
  for (long long base = base0; base < n_items; base += stride) {
    const long long item = base + lane;
    const long long gid = item < n_items ? (Compact ? static_cast<long long>(__ldcs(active + item)) : edge_begin + item)
                                         : -1;
    int h = -1, t = -1;
    float gx_h = 0.f, gy_h = 0.f;
    if (gid >= 0) {
      h = __ldcs(heads + gid);
      t = __ldcs(tails + gid);
      const float per = __ldcs(periods + gid);
      const bool ok = h >= 0 && h < p.n && t >= 0 && t < p.n && h != t;
      const int pos = ok ? positive_samples(per, epoch) : 0;
      if (pos > 0) {
        local_pos += pos;
        const float2 yh0 = src[h];
        const float2 yt0 = src[t];
        const int neg = negative_samples(per, p.negative_sample_rate, epoch);
        const unsigned int key = p.hash_key_is_tail ? static_cast<unsigned int>(t) : static_cast<unsigned int>(gid);
        if (Mode == kUmapDelta) {
          // Jacobi: every force at the frozen epoch-start positions.
          float2 dh = make_float2(0.f, 0.f), dt = make_float2(0.f, 0.f);
          for (int s = 0; s < pos; ++s) {
            const float dx = yh0.x - yt0.x;
            const float dy = yh0.y - yt0.y;
            const float d2 = fmaxf(eps, dx * dx + dy * dy);
            const float d2b = umap_pow(d2, p.b);
            const float c = -2.0f * p.a * p.b * (d2b / d2) / (p.a * d2b + 1.0f);
            const float gx = clip4(c * dx) * alpha;
            const float gy = clip4(c * dy) * alpha;
            dh.x += gx;
            dh.y += gy;
            dt.x -= gx;
            dt.y -= gy;
          }
          for (int s = 0; s < (owned(h) ? neg : 0); ++s) {
            const int k = negative_vertex(static_cast<unsigned int>(p.n), p.seed, epoch, h, key, s);
            if (k == h || k == t) continue;
            const float2 yk = src[k];
            const float dx = yh0.x - yk.x;
            const float dy = yh0.y - yk.y;
            const float d2 = fmaxf(eps, dx * dx + dy * dy);
            const float d2b = umap_pow(d2, p.b);
            const float c = p.repulsion_strength * 2.0f * p.b / ((0.001f + d2) * (p.a * d2b + 1.0f));
            dh.x += clip4(c * dx) * alpha;
            dh.y += clip4(c * dy) * alpha;
          }
          gx_h = dh.x;
          gy_h = dh.y;
          if (owned(t)) atomicAdd(dst + t, dt);
        } else if (Mode == kUmapInplace) {
          // The edge's samples in the CPU replay's order on running copies.
          float2 yh = yh0, yt = yt0;
          for (int s = 0; s < pos; ++s) {
            const float dx = yh.x - yt.x;
            const float dy = yh.y - yt.y;
            const float d2 = fmaxf(eps, dx * dx + dy * dy);
            const float d2b = umap_pow(d2, p.b);
            const float c = -2.0f * p.a * p.b * (d2b / d2) / (p.a * d2b + 1.0f);
            const float gx = clip4(c * dx) * alpha;
            const float gy = clip4(c * dy) * alpha;
            yh.x += gx;
            yh.y += gy;
            yt.x += -gx;
            yt.y += -gy;
          }
          for (int s = 0; s < (owned(h) ? neg : 0); ++s) {
            const int k = negative_vertex(static_cast<unsigned int>(p.n), p.seed, epoch, h, key, s);
            if (k == h || k == t) continue;
            const float2 yk = src[k];
            const float dx = yh.x - yk.x;
            const float dy = yh.y - yk.y;
            const float d2 = fmaxf(eps, dx * dx + dy * dy);
            const float d2b = umap_pow(d2, p.b);
            const float c = p.repulsion_strength * 2.0f * p.b / ((0.001f + d2) * (p.a * d2b + 1.0f));
            yh.x += clip4(c * dx) * alpha;
            yh.y += clip4(c * dy) * alpha;
          }
          gx_h = yh.x - yh0.x;
          gy_h = yh.y - yh0.y;
          if (owned(t)) atomicAdd(dst + t, make_float2(yt.x - yt0.x, yt.y - yt0.y));
        } else {
          // Each sample reads fresh positions and applies its move at once.
          float2 yh, yt;
          for (int s = 0; s < pos; ++s) {
            yh = __ldcg(layout + h);
            yt = __ldcg(layout + t);
            const float dx = yh.x - yt.x;
            const float dy = yh.y - yt.y;
            const float d2 = fmaxf(eps, dx * dx + dy * dy);
            const float d2b = umap_pow(d2, p.b);
            const float c = -2.0f * p.a * p.b * (d2b / d2) / (p.a * d2b + 1.0f);
            const float gx = clip4(c * dx) * alpha;
            const float gy = clip4(c * dy) * alpha;
            if (owned(h)) atomicAdd(layout + h, make_float2(gx, gy));
            if (owned(t)) atomicAdd(layout + t, make_float2(-gx, -gy));
          }
          for (int s = 0; s < (owned(h) ? neg : 0); ++s) {
            const int k = negative_vertex(static_cast<unsigned int>(p.n), p.seed, epoch, h, key, s);
            if (k == h || k == t) continue;
            yh = __ldcg(layout + h);
            const float2 yk = __ldcg(layout + k);
            const float dx = yh.x - yk.x;
            const float dy = yh.y - yk.y;
            const float d2 = fmaxf(eps, dx * dx + dy * dy);
            const float d2b = umap_pow(d2, p.b);
            const float c = p.repulsion_strength * 2.0f * p.b / ((0.001f + d2) * (p.a * d2b + 1.0f));
            atomicAdd(layout + h, make_float2(clip4(c * dx) * alpha, clip4(c * dy) * alpha));
          }
          h = -1;  // moves already applied; nothing to combine across the warp
        }
      } else {
        h = -1;
      }
    }
    // Segmented sum of head displacements over lanes that share a head.
    const unsigned int peers = __match_any_sync(0xffffffffu, h);
    const int leader = __ffs(peers) - 1;
    float sx = 0.f, sy = 0.f;
    for (unsigned int m = peers; m; m &= m - 1) {
      const int l = __ffs(m) - 1;
      sx += __shfl_sync(peers, gx_h, l);
      sy += __shfl_sync(peers, gy_h, l);
    }
    if (lane == leader && h >= 0 && owned(h)) atomicAdd(dst + h, make_float2(sx, sy));
  }
  if (positive_count != nullptr) {
    local_pos = warp_sum(static_cast<double>(local_pos));
    if (lane == 0 && local_pos) atomicAdd(reinterpret_cast<unsigned long long*>(positive_count),
                                          static_cast<unsigned long long>(local_pos));
  }
}

__global__ void umap_sanitize_kernel(float2* layout, float2* delta, int n, float max_abs) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float2 v = layout[i];
  if (delta != nullptr) {
    const float2 d = delta[i];
    v.x += d.x;
    v.y += d.y;
    delta[i] = make_float2(0.f, 0.f);
  }
  if (!isfinite(v.x)) v.x = 0.0f;
  if (!isfinite(v.y)) v.y = 0.0f;
  v.x = fminf(max_abs, fmaxf(-max_abs, v.x));
  v.y = fminf(max_abs, fmaxf(-max_abs, v.y));
  layout[i] = v;
}

// Samples an edge applies over epochs [epoch_begin, epoch_end), with the
// epoch kernel's own schedules.
__global__ void count_samples_kernel(const float* __restrict__ periods, long long n_edges, int epoch_begin,
                                     int epoch_end, int nsr, long long* __restrict__ pos,
                                     long long* __restrict__ neg) {
  const long long e = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= n_edges) return;
  const float p = periods[e];
  long long sp = 0, sn = 0;
  for (int epoch = epoch_begin; epoch < epoch_end; ++epoch) {
    sp += positive_samples(p, epoch);
    sn += negative_samples(p, nsr, epoch);
  }
  pos[e] = sp;
  neg[e] = sn;
}

}  // namespace

int umap_count_samples(const float* periods, long long n_edges, int epoch_begin, int epoch_end, int nsr,
                       long long* pos, long long* neg, cudaStream_t stream) {
  const unsigned blocks = static_cast<unsigned>((n_edges + 255) / 256);
  count_samples_kernel<<<blocks, 256, 0, stream>>>(periods, n_edges, epoch_begin, epoch_end, nsr, pos, neg);
  FE_LAUNCH("count_samples_kernel");
  return 0;
}

namespace {

int gather_layout(UmapRun* r) {
  // Every rank's copy of the layout takes the owned rows of each rank,
  // gathered in place.  One rank has nothing to gather.
  if (r->comm == nullptr || r->shard_ranks <= 1) return 0;
  const NcclApi* api = nccl_api();
  if (api == nullptr) return 1;
  const size_t count = 2 * static_cast<size_t>(r->rows_per_rank);
  float* base = reinterpret_cast<float*>(r->layout);
  ncclComm_t comm = static_cast<ncclComm_t>(r->comm);
  return check_nccl_call(comm, api->AllGather(base + count * r->shard_rank, base, count, ncclFloat32, comm, r->stream),
                         "ncclAllGather(UMAP layout rows)");
}

// Edges whose schedule applies at least one positive sample in `epoch`
// (the only edges the epoch kernel does work for).
struct FiresInEpoch {
  const float* periods;
  int epoch;
  __device__ bool operator()(const int& e) const { return positive_samples(__ldg(periods + e), epoch) > 0; }
};

template <int Mode>
int launch_edges(UmapRun* r, int epoch, long long e0, long long e1) {
  // Edge-granularity Hogwild keeps the whole-list scan: packing the firing
  // edges puts about four times as many of them in flight at once, and this
  // mode, the one that follows the CPU replay's order, measurably lost kNN
  // preservation with it (0.00743 against 0.00773-0.00790 at 70k).
  const UmapCompaction& c = r->compact;
  if (c.active != nullptr && Mode != kUmapInplace && e1 > e0) {
    std::size_t bytes = c.temp_bytes;
    FE_CUDA(cub::DeviceSelect::If(c.temp, bytes, thrust::make_counting_iterator<int>(static_cast<int>(e0)), c.active,
                                  c.count, static_cast<int>(e1 - e0), FiresInEpoch{r->periods, epoch}, r->stream),
            "cub::DeviceSelect(firing edges)");
    umap_epoch_kernel<Mode, true><<<r->edge_blocks, 256, 0, r->stream>>>(
        r->heads, r->tails, r->periods, e0, e1, c.active, c.count, r->layout, r->layout,
        Mode == kUmapDelta ? r->delta : nullptr, r->params, epoch, r->positive_count);
  } else {
    umap_epoch_kernel<Mode, false><<<r->edge_blocks, 256, 0, r->stream>>>(
        r->heads, r->tails, r->periods, e0, e1, nullptr, nullptr, r->layout, r->layout,
        Mode == kUmapDelta ? r->delta : nullptr, r->params, epoch, r->positive_count);
  }
  FE_LAUNCH("umap_epoch_kernel");
  return 0;
}

}  // namespace

int umap_launch_epoch(UmapRun* r, int epoch) {
  const UmapParams& p = r->params;
  const bool sharded = r->comm != nullptr && r->shard_ranks > 1;
  if (r->mode == kUmapDelta) {
    // Jacobi: every force at the epoch-start layout, one gather per epoch.
    FE_TRY(launch_edges<kUmapDelta>(r, epoch, 0, r->n_edges));
  } else {
    // Hogwild: a shard sees the other shards' moves only through the gathers,
    // so its edges run in kShardGatherParts parts with a gather after each,
    // which keeps remote positions at most a part of an epoch old.
    const int parts = sharded ? kShardGatherParts : 1;
    for (int part = 0; part < parts; ++part) {
      const long long e0 = r->n_edges * part / parts;
      const long long e1 = r->n_edges * (part + 1) / parts;
      if (r->mode == kUmapInplaceSample) FE_TRY(launch_edges<kUmapInplaceSample>(r, epoch, e0, e1));
      else FE_TRY(launch_edges<kUmapInplace>(r, epoch, e0, e1));
      if (part + 1 < parts) FE_TRY(gather_layout(r));
    }
  }
  umap_sanitize_kernel<<<(p.n + 255) / 256, 256, 0, r->stream>>>(
      r->layout, r->mode == kUmapDelta ? r->delta : nullptr, p.n, 16.0f);
  FE_LAUNCH("umap_sanitize_kernel");
  return gather_layout(r);
}

int umap_run_epochs(UmapRun* r, int epoch_begin, int epoch_end) {
  if (r->mode == kUmapDelta && r->delta != nullptr) {
    FE_CUDA(cudaMemsetAsync(r->delta, 0, sizeof(float2) * r->params.n, r->stream), "memset delta");
  }
  const bool graphs = r->use_graphs && (epoch_end - epoch_begin) > 8 && r->positive_count == nullptr;
  if (!graphs) {
    for (int e = epoch_begin; e < epoch_end; ++e) FE_TRY(umap_launch_epoch(r, e));
    return 0;
  }
  // Capture chunks of epochs; the epoch index is a kernel argument, so each
  // chunk is its own graph (instantiated once, launched once).
  const int chunk = 50;
  for (int e0 = epoch_begin; e0 < epoch_end; e0 += chunk) {
    const int e1 = std::min(epoch_end, e0 + chunk);
    cudaGraph_t g = nullptr;
    FE_CUDA(cudaStreamBeginCapture(r->stream, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture(umap)");
    int rc = 0;
    for (int e = e0; e < e1 && rc == 0; ++e) rc = umap_launch_epoch(r, e);
    const cudaError_t end = cudaStreamEndCapture(r->stream, &g);
    if (rc != 0 || end != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      if (rc == 0) check_cuda(end, "cudaStreamEndCapture(umap)");
      return 1;
    }
    cudaGraphExec_t exec = nullptr;
    const cudaError_t inst = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    FE_CUDA(inst, "cudaGraphInstantiate(umap)");
    const cudaError_t launch = cudaGraphLaunch(exec, r->stream);
    cudaGraphExecDestroy(exec);
    FE_CUDA(launch, "cudaGraphLaunch(umap)");
  }
  return 0;
}

int umap_compaction_alloc(long long n_edges, UmapCompaction* c) {
  *c = UmapCompaction{};
  if (!env_flag("FASTEMBEDR_B200_UMAP_COMPACT", true) || n_edges < 1) return 0;
  if (n_edges >= (1ll << 31) - 1) return 0;  // 32-bit edge ids in the list; scan the whole list instead
  std::size_t bytes = 0;
  FE_CUDA(cub::DeviceSelect::If(nullptr, bytes, thrust::make_counting_iterator<int>(0), static_cast<int*>(nullptr),
                                static_cast<int*>(nullptr), static_cast<int>(n_edges), FiresInEpoch{nullptr, 0}),
          "cub::DeviceSelect(sizing)");
  UmapCompaction out;
  out.temp_bytes = bytes;
  if (dev_malloc(&out.active, sizeof(int) * static_cast<std::size_t>(n_edges)) != cudaSuccess ||
      dev_malloc(&out.count, sizeof(int)) != cudaSuccess || dev_malloc(&out.temp, bytes) != cudaSuccess) {
    cudaGetLastError();
    umap_compaction_free(&out);
    return 0;  // no room for the list: scan the whole list (same results)
  }
  *c = out;
  return 0;
}

void umap_compaction_free(UmapCompaction* c) {
  dev_free(c->active);
  dev_free(c->count);
  dev_free(c->temp);
  *c = UmapCompaction{};
}

int umap_edge_blocks(long long n_edges) {
  const long long want = (n_edges + 255) / 256;
  const long long cap = static_cast<long long>(sm_count()) * 8;
  return static_cast<int>(std::max(1ll, std::min(want, cap)));
}

}  // namespace fe
