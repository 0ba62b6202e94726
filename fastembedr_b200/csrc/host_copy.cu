// Host -> device copies of the caller's buffers.
//
// The reference's R wrapper hands the library pageable std::vector copies of
// its inputs (src/embedding_cuda_impl.cpp:776-784, 817), and a
// cudaMemcpyAsync from pageable memory is staged by the driver through one
// bounce buffer on the calling thread.  On some hosts that runs at 1-2 GB/s,
// so the 720 MB of a 1M-point KNN took longer than the whole optimisation.
//
// h2d_copy splits a large pageable source into chunks.  Worker threads (the
// caller is one of them) take chunks from a shared counter, copy each into
// one of their two pinned slots and send it with cudaMemcpyAsync on their own
// stream; a slot is refilled only after the event behind its last copy has
// completed, so each worker's memcpy of one chunk overlaps the DMA of the
// previous one.  The pinned slots form one pool per process, allocated on
// first use and kept.  Sources that are already pinned or registered, copies
// under kStagedMinBytes and FASTEMBEDR_B200_H2D_THREADS=1 take one direct
// cudaMemcpyAsync.  In every case the call returns once the data is on the
// device (the destination may be read on any stream) and the source may be
// reused.
#include "fe_common.cuh"

#include <algorithm>
#include <atomic>
#include <cstring>
#include <exception>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace fe {
namespace {

constexpr std::size_t kChunkBytes = std::size_t{4} << 20;
constexpr std::size_t kStagedMinBytes = std::size_t{16} << 20;
constexpr int kMaxWorkers = 8;

std::mutex g_pool_mutex;  // one staged copy at a time uses the pool
char* g_pool = nullptr;   // kMaxWorkers * 2 slots of kChunkBytes
bool g_pool_failed = false;

bool source_is_pinned(const void* src) {
  cudaPointerAttributes attr{};
  const cudaError_t code = cudaPointerGetAttributes(&attr, src);
  if (code != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return attr.type == cudaMemoryTypeHost;
}

struct StagedJob {
  char* dst = nullptr;
  const char* src = nullptr;
  std::size_t bytes = 0;
  int device = 0;
  std::atomic<std::size_t> next{0};
  std::atomic<bool> failed{false};
  std::mutex err_mutex;
  std::string err;

  void fail(cudaError_t code, const char* where) {
    std::lock_guard<std::mutex> lock(err_mutex);
    if (err.empty()) err = std::string(where) + ": " + cudaGetErrorString(code);
    failed.store(true);
  }
};

void staged_worker(StagedJob* job, int worker, bool set_device) {
  if (set_device) {
    const cudaError_t code = cudaSetDevice(job->device);
    if (code != cudaSuccess) return job->fail(code, "cudaSetDevice(H2D worker)");
  }
  cudaStream_t stream = nullptr;
  cudaEvent_t done[2] = {nullptr, nullptr};
  cudaError_t code = cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking);
  if (code != cudaSuccess) return job->fail(code, "cudaStreamCreate(H2D worker)");
  for (int s = 0; s < 2 && code == cudaSuccess; ++s) code = cudaEventCreateWithFlags(&done[s], cudaEventDisableTiming);
  char* slot[2] = {g_pool + (2 * worker) * kChunkBytes, g_pool + (2 * worker + 1) * kChunkBytes};
  bool in_flight[2] = {false, false};
  for (int k = 0; code == cudaSuccess && !job->failed.load(std::memory_order_relaxed); ++k) {
    const std::size_t chunk = job->next.fetch_add(1);
    const std::size_t off = chunk * kChunkBytes;
    if (off >= job->bytes) break;
    const std::size_t len = std::min(kChunkBytes, job->bytes - off);
    const int s = k & 1;
    if (in_flight[s]) {
      code = cudaEventSynchronize(done[s]);
      if (code != cudaSuccess) break;
    }
    std::memcpy(slot[s], job->src + off, len);
    code = cudaMemcpyAsync(job->dst + off, slot[s], len, cudaMemcpyHostToDevice, stream);
    if (code == cudaSuccess) code = cudaEventRecord(done[s], stream);
    in_flight[s] = true;
  }
  if (code != cudaSuccess) job->fail(code, "staged H2D copy");
  const cudaError_t sync = cudaStreamSynchronize(stream);
  if (sync != cudaSuccess) job->fail(sync, "cudaStreamSynchronize(H2D worker)");
  for (cudaEvent_t e : done) {
    if (e != nullptr) cudaEventDestroy(e);
  }
  cudaStreamDestroy(stream);
}

}  // namespace

int h2d_copy(void* dst, const void* src, std::size_t bytes, cudaStream_t stream, const char* what) {
  if (bytes == 0) return 0;
  int workers = std::min(env_int("FASTEMBEDR_B200_H2D_THREADS", kMaxWorkers), kMaxWorkers);
  workers = std::min<int>(workers, static_cast<int>(std::max(1u, std::thread::hardware_concurrency())));
  workers = std::min<int>(workers, static_cast<int>((bytes + kChunkBytes - 1) / kChunkBytes));
  if (workers < 2 || bytes < kStagedMinBytes || source_is_pinned(src)) {
    FE_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, stream), what);
    FE_CUDA(cudaStreamSynchronize(stream), what);
    return 0;
  }
  std::unique_lock<std::mutex> lock(g_pool_mutex);
  if (g_pool == nullptr && !g_pool_failed) {
    void* p = nullptr;
    if (cudaHostAlloc(&p, std::size_t{2} * kMaxWorkers * kChunkBytes, cudaHostAllocPortable) == cudaSuccess) {
      g_pool = static_cast<char*>(p);
    } else {
      cudaGetLastError();
      g_pool_failed = true;  // no pinned memory to spare: direct copies from now on
    }
  }
  if (g_pool == nullptr) {
    lock.unlock();
    FE_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, stream), what);
    FE_CUDA(cudaStreamSynchronize(stream), what);
    return 0;
  }
  // Work already queued on the caller's stream may still use the destination.
  FE_CUDA(cudaStreamSynchronize(stream), what);
  StagedJob job;
  job.dst = static_cast<char*>(dst);
  job.src = static_cast<const char*>(src);
  job.bytes = bytes;
  FE_CUDA(cudaGetDevice(&job.device), what);
  std::vector<std::thread> threads;
  threads.reserve(workers - 1);
  for (int w = 1; w < workers; ++w) {
    try {
      threads.emplace_back(staged_worker, &job, w, true);
    } catch (const std::exception&) {
      break;  // fewer workers: the chunks are shared through a counter
    }
  }
  staged_worker(&job, 0, false);
  for (std::thread& t : threads) t.join();
  if (job.failed.load()) {
    set_error(std::string(what) + ": " + job.err);
    return 1;
  }
  return 0;
}

}  // namespace fe
