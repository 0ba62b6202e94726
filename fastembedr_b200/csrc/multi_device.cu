// One process, several GPUs, behind the unchanged one-shot openTSNE entry
// points (fastembedr_cuda_opentsne_fft_from_*): the boundary's multi-GPU rule
// is that device selection comes from the environment and the ABI does not
// change, so a single-process caller (the reference's R wrapper,
// src/embedding_cuda_impl.cpp) can reach every GPU of a box.
//
// FASTEMBEDR_B200_DEVICES="0,1,..." (two or more distinct ordinals) runs the
// call as a sharded session per listed device, one host thread each, joined
// by one NCCL communicator: the same decomposition and bits as one process per
// GPU (tsne_shard.cu).  Failure handling never leaves a rank waiting on a peer:
//   * every rank builds its inputs, P and session first; a host barrier checks
//     them all before any rank joins the communicator;
//   * the join is bounded (the environment's limit, else kJoinLimitSeconds), so
//     a rank whose peer failed inside the join gives up instead of waiting;
//     a second barrier checks that every rank joined; ranks whose peers failed
//     to join abort their communicator instead of destroying it;
//   * during the run every collective goes through a RankGroup (rank_group.h):
//     the ranks agree on the host before each one, so a rank that fails on the
//     host stops its peers before they enqueue a collective it will not join;
//     each rank has at most one collective in flight, and a collective that
//     does not complete within the stall limit fails the group;
//   * only a rank whose own enqueue failed after its peers had enqueued theirs,
//     or a stalled collective, makes the calling thread abort the communicators
//     (each under its rank's lock, so no NCCL call follows an abort); that
//     ends the one collective each rank may have in flight;
//   * communicators are released only after every rank has finished.
// FASTEMBEDR_B200_INJECT_HOST_FAILURE="<rank>:<collective>" makes that rank
// fail on the host just before its collective number <collective> (counted
// from 0, warm-up included), with none of its collectives in flight: the
// failure path is exercised without faulting or stalling a GPU.
#include "nccl_loader.cuh"
#include "rank_group.h"
#include "tsne.cuh"

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace fe {
namespace {

class HostBarrier {
 public:
  explicit HostBarrier(int n) : n_(n) {}
  void wait() {
    std::unique_lock<std::mutex> lock(m_);
    const int gen = gen_;
    if (++count_ == n_) {
      count_ = 0;
      ++gen_;
      cv_.notify_all();
      return;
    }
    cv_.wait(lock, [&] { return gen_ != gen; });
  }

 private:
  std::mutex m_;
  std::condition_variable cv_;
  int n_;
  int count_ = 0;
  int gen_ = 0;
};

struct RankBuf {
  void* p = nullptr;
  ~RankBuf() {
    if (p) fe::dev_free(p);
  }
};

struct Shared {
  explicit Shared(int n) : barrier(n), group(n), ok(n, 0) {}
  HostBarrier barrier;  // set-up and tear-down points, which every rank reaches
  RankGroup group;      // collectives of the run, and the communicators
  std::vector<int> ok;
  std::mutex msg_lock;
  std::string first_msg;  // the first failure reported (its cause, not its echoes)
  std::atomic<int> finished{0};
  bool all_ok() const {
    for (int v : ok) {
      if (!v) return false;
    }
    return true;
  }
};

// Join limit of this mode when the environment sets none: a rank whose join
// fails must not leave the others inside a blocking ncclCommInitRank.
constexpr double kJoinLimitSeconds = 600.0;
// A collective of this mode that has not completed after this long is treated
// as a failed peer (FASTEMBEDR_B200_COLLECTIVE_TIMEOUT_S overrides).
constexpr double kStallLimitSeconds = 300.0;

// FASTEMBEDR_B200_INJECT_HOST_FAILURE="<rank>:<collective>" for `rank`, else -1.
long long injected_failure(int rank) {
  const char* v = std::getenv("FASTEMBEDR_B200_INJECT_HOST_FAILURE");
  if (v == nullptr || *v == '\0') return -1;
  char* end = nullptr;
  const long r = std::strtol(v, &end, 10);
  if (end == nullptr || *end != ':' || r != rank) return -1;
  const long long at = std::strtoll(end + 1, nullptr, 10);
  return at >= 0 ? at : -1;
}

void rank_main(const MultiDeviceTsne& job, int rank, Shared* sh) {
  const int nranks = static_cast<int>(job.devices.size());
  const int dev = job.devices[rank];
  const JoinLimit join_limit(kJoinLimitSeconds);
  auto fail = [&](const std::string& why) {
    sh->ok[rank] = 0;
    {
      std::lock_guard<std::mutex> l(sh->msg_lock);
      if (sh->first_msg.empty()) sh->first_msg = "device " + std::to_string(dev) + ": " + why;
    }
    sh->group.fail();
  };
  TsneSession* s = nullptr;
  cudaStream_t stream = nullptr;
  RankBuf d_idx, d_dist;
  int* row_ptr = nullptr;
  int* col = nullptr;
  float* val = nullptr;
  long long nnz = 0;
  int rc = check_cuda(cudaSetDevice(dev), "cudaSetDevice");
  if (rc == 0) rc = check_cuda(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate");
  // Inputs on this device.
  const size_t items = static_cast<size_t>(job.n) * job.k;
  const size_t dist_bytes = items * (job.dist_double ? sizeof(double) : sizeof(float));
  const int* idx_dev = job.indices;
  const void* dist_dev = job.distances;
  if (rc == 0 && (!job.on_device || dev != job.caller_device)) {
    rc = check_cuda(fe::dev_malloc(&d_idx.p, items * sizeof(int)), "cudaMalloc(indices)");
    if (rc == 0) rc = check_cuda(fe::dev_malloc(&d_dist.p, dist_bytes), "cudaMalloc(distances)");
    if (rc == 0 && job.on_device) {
      rc = check_cuda(cudaMemcpyPeerAsync(d_idx.p, dev, job.indices, job.caller_device, items * sizeof(int),
                                          stream), "peer copy indices");
      if (rc == 0) rc = check_cuda(cudaMemcpyPeerAsync(d_dist.p, dev, job.distances, job.caller_device,
                                                       dist_bytes, stream), "peer copy distances");
    } else if (rc == 0) {
      rc = h2d_copy(d_idx.p, job.indices, items * sizeof(int), stream, "H2D indices");
      if (rc == 0) rc = h2d_copy(d_dist.p, job.distances, dist_bytes, stream, "H2D distances");
    }
    idx_dev = static_cast<const int*>(d_idx.p);
    dist_dev = d_dist.p;
  }
  if (rc == 0) {
    rc = build_p_device(idx_dev, dist_dev, job.dist_double, job.n, job.k, job.index_offset, job.perplexity, stream,
                        &row_ptr, &col, &val, &nnz);
  }
  if (rc == 0) {
    rc = session_create(&s, job.n, job.grid, row_ptr, col, val, nnz, stream);
    if (rc != 0) {
      fe::dev_free(row_ptr);
      fe::dev_free(col);
      fe::dev_free(val);
    }
  }
  if (rc == 0) {
    rc = job.init != nullptr ? session_set_layout(s, job.init, true, true) : session_random_layout(s, job.seed);
  }
  if (rc == 0) {
    rc = check_cuda(cudaEventCreateWithFlags(&s->collective_done, cudaEventDisableTiming),
                    "cudaEventCreate(collective)");
  }
  if (rc == 0) rc = check_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize(set-up)");
  if (rc == 0) sh->ok[rank] = 1;
  else fail(last_error());

  // Every rank's set-up is checked before any rank joins the communicator.
  sh->barrier.wait();
  bool joined = false;
  if (sh->all_ok()) {
    rc = session_shard(s, job.unique_id, nullptr, nranks, rank);
    if (rc == 0) {
      joined = true;
      sh->group.set_comm(rank, s->comm);
    } else {
      fail(last_error());
    }
  }
  sh->barrier.wait();
  const bool run = sh->all_ok();
  if (run) {
    s->group = &sh->group;
    s->stall_limit_s = env_double("FASTEMBEDR_B200_COLLECTIVE_TIMEOUT_S", kStallLimitSeconds);
    s->inject_failure_at = injected_failure(rank);
    rc = shard_warm_up(s);
    if (rc == 0) {
      rc = session_iterate(s, job.early_iter, job.early_exaggeration, job.initial_momentum, job.lr_early,
                           job.min_gain, job.max_step_norm);
    }
    if (rc == 0) {
      rc = session_iterate(s, job.n_iter, job.exaggeration, job.final_momentum, job.lr_normal, job.min_gain,
                           job.max_step_norm);
    }
    // The newest collective completes (bounded) before any blocking wait on
    // the stream, so no rank blocks on a collective a failed peer left alone.
    if (rc == 0) rc = shard_quiesce(s);
    if (rc == 0) {
      rc = rank == 0 ? session_get_layout(s, job.out, true)
                     : check_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize(run)");
    }
    if (rc != 0) fail(last_error());
    if (shard_quiesce(s) != 0 && rc == 0) fail(last_error());
  }
  ++sh->finished;
  // No communicator is destroyed while a peer may still use it.
  sh->barrier.wait();
  if (s != nullptr && joined) {
    void* mine = sh->group.take_comm(rank);
    if (mine == nullptr || !run || sh->group.failed()) {
      // Aborted by the calling thread, or peers never ran or failed (a
      // destroy could wait on them): abort it here unless already done.
      // Nothing of this rank is in flight on it any more (quiesced above).
      const NcclApi* api = nccl_api();
      if (mine != nullptr && api != nullptr) api->CommAbort(static_cast<ncclComm_t>(mine));
      s->comm = nullptr;
      s->own_comm = false;
    }
  }
  if (s != nullptr) {
    s->group = nullptr;
    if (s->collective_done != nullptr) cudaEventDestroy(s->collective_done);
    s->collective_done = nullptr;
    session_destroy(s);
  }
  if (stream != nullptr) {
    cudaStreamSynchronize(stream);
    cudaStreamDestroy(stream);
  }
}

}  // namespace

int multi_device_list(std::vector<int>* devices) {
  devices->clear();
  const char* v = std::getenv("FASTEMBEDR_B200_DEVICES");
  if (v == nullptr || *v == '\0') return 0;
  const std::string text(v);
  size_t pos = 0;
  for (;;) {
    const size_t comma = text.find(',', pos);
    const std::string item = text.substr(pos, comma == std::string::npos ? std::string::npos : comma - pos);
    char* end = nullptr;
    const long d = std::strtol(item.c_str(), &end, 10);
    if (item.empty() || end == nullptr || *end != '\0' || d < 0 || d > 1 << 20) {
      set_error("FASTEMBEDR_B200_DEVICES: '" + item + "' is not a device ordinal");
      return 1;
    }
    for (int seen : *devices) {
      if (seen == d) {
        set_error("FASTEMBEDR_B200_DEVICES lists device " + item + " twice");
        return 1;
      }
    }
    devices->push_back(static_cast<int>(d));
    if (comma == std::string::npos) break;
    pos = comma + 1;
  }
  if (devices->size() < 2) {
    devices->clear();  // one listed device: the call runs on the current device
    return 0;
  }
  if (devices->size() > static_cast<size_t>(TsneSession::kMaxRanks)) {
    set_error("FASTEMBEDR_B200_DEVICES lists more devices than a sharded session supports");
    return 1;
  }
  int count = 0;
  FE_CUDA(cudaGetDeviceCount(&count), "cudaGetDeviceCount(FASTEMBEDR_B200_DEVICES)");
  for (int d : *devices) {
    if (d >= count) {
      set_error("FASTEMBEDR_B200_DEVICES: device " + std::to_string(d) + " does not exist (" +
                std::to_string(count) + " visible)");
      return 1;
    }
  }
  return 0;
}

int opentsne_multi_device(MultiDeviceTsne job) {
  const int nranks = static_cast<int>(job.devices.size());
  const NcclApi* api = nccl_api();
  if (api == nullptr) return 1;
  ncclUniqueId uid;
  FE_TRY(check_nccl(api->GetUniqueId(&uid), "ncclGetUniqueId"));
  job.unique_id = &uid;
  FE_CUDA(cudaGetDevice(&job.caller_device), "cudaGetDevice");
  Shared sh(nranks);
  std::vector<std::thread> threads;
  threads.reserve(nranks);
  for (int r = 0; r < nranks; ++r) threads.emplace_back(rank_main, std::cref(job), r, &sh);
  // A collective a rank enqueued without a peer (the peer's enqueue failed
  // after both arrived), or one that stalled, waits on the device for good:
  // abort every communicator then, which ends it.  Host-side failures need no
  // abort: the group stops the other ranks before their next collective.
  auto abort_comm = [&](void* c) { api->CommAbort(static_cast<ncclComm_t>(c)); };
  while (sh.finished.load() < nranks) {
    if (sh.group.abort_needed()) sh.group.abort_all(abort_comm);
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
  for (std::thread& t : threads) t.join();
  if (!sh.first_msg.empty()) {
    set_error("multi-device openTSNE: " + sh.first_msg);
    return 1;
  }
  if (!sh.all_ok()) {
    set_error("multi-device openTSNE: a rank stopped because a peer failed");
    return 1;
  }
  return 0;
}

}  // namespace fe
