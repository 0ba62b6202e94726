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
//   * during the run the calling thread watches a failure flag and aborts
//     every communicator if a rank fails, which ends the others' collectives;
//   * communicators are destroyed only after every rank has finished.
#include "nccl_loader.cuh"
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
    if (p) cudaFree(p);
  }
};

struct Shared {
  explicit Shared(int n) : barrier(n), ok(n, 0), msg(n), comm(n) {
    for (auto& c : comm) c = nullptr;
  }
  HostBarrier barrier;
  std::vector<int> ok;
  std::vector<std::string> msg;
  // A joined rank's communicator until whoever aborts or destroys it takes it
  // (exchange with nullptr), so that it is released exactly once.
  std::vector<std::atomic<void*>> comm;
  std::atomic<bool> failed{false};
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

void rank_main(const MultiDeviceTsne& job, int rank, Shared* sh) {
  const int nranks = static_cast<int>(job.devices.size());
  const int dev = job.devices[rank];
  const JoinLimit join_limit(kJoinLimitSeconds);
  auto fail = [&](const std::string& why) {
    sh->ok[rank] = 0;
    sh->msg[rank] = "device " + std::to_string(dev) + ": " + why;
    sh->failed = true;
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
    rc = check_cuda(cudaMalloc(&d_idx.p, items * sizeof(int)), "cudaMalloc(indices)");
    if (rc == 0) rc = check_cuda(cudaMalloc(&d_dist.p, dist_bytes), "cudaMalloc(distances)");
    if (rc == 0 && job.on_device) {
      rc = check_cuda(cudaMemcpyPeerAsync(d_idx.p, dev, job.indices, job.caller_device, items * sizeof(int),
                                          stream), "peer copy indices");
      if (rc == 0) rc = check_cuda(cudaMemcpyPeerAsync(d_dist.p, dev, job.distances, job.caller_device,
                                                       dist_bytes, stream), "peer copy distances");
    } else if (rc == 0) {
      rc = check_cuda(cudaMemcpyAsync(d_idx.p, job.indices, items * sizeof(int), cudaMemcpyHostToDevice, stream),
                      "H2D indices");
      if (rc == 0) rc = check_cuda(cudaMemcpyAsync(d_dist.p, job.distances, dist_bytes, cudaMemcpyHostToDevice,
                                                   stream), "H2D distances");
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
      cudaFree(row_ptr);
      cudaFree(col);
      cudaFree(val);
    }
  }
  if (rc == 0) {
    rc = job.init != nullptr ? session_set_layout(s, job.init, true, true) : session_random_layout(s, job.seed);
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
      sh->comm[rank] = s->comm;
    } else {
      fail(last_error());
    }
  }
  sh->barrier.wait();
  const bool run = sh->all_ok();
  if (run) {
    rc = shard_warm_up(s);
    if (rc == 0) {
      rc = session_iterate(s, job.early_iter, job.early_exaggeration, job.initial_momentum, job.lr_early,
                           job.min_gain, job.max_step_norm);
    }
    if (rc == 0) {
      rc = session_iterate(s, job.n_iter, job.exaggeration, job.final_momentum, job.lr_normal, job.min_gain,
                           job.max_step_norm);
    }
    if (rc == 0) {
      rc = rank == 0 ? session_get_layout(s, job.out, true)
                     : check_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize(run)");
    }
    if (rc != 0) fail(last_error());
  }
  ++sh->finished;
  // No communicator is destroyed while a peer may still use it.
  sh->barrier.wait();
  if (s != nullptr && joined) {
    void* mine = sh->comm[rank].exchange(nullptr);
    if (mine == nullptr || !run || sh->failed) {
      // Aborted by the calling thread, or peers never ran or failed (a
      // destroy could wait on them): abort it here unless already done.
      const NcclApi* api = nccl_api();
      if (mine != nullptr && api != nullptr) api->CommAbort(static_cast<ncclComm_t>(mine));
      s->comm = nullptr;
      s->own_comm = false;
    }
  }
  if (s != nullptr) session_destroy(s);
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
  // A failed rank stops issuing collectives, which would leave its peers'
  // collectives waiting on the device: abort every joined communicator then.
  while (sh.finished.load() < nranks) {
    if (sh.failed) {
      for (auto& slot : sh.comm) {
        void* c = slot.exchange(nullptr);
        if (c != nullptr) api->CommAbort(static_cast<ncclComm_t>(c));
      }
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
  for (std::thread& t : threads) t.join();
  for (int r = 0; r < nranks; ++r) {
    if (!sh.ok[r] && !sh.msg[r].empty()) {
      set_error("multi-device openTSNE: " + sh.msg[r]);
      return 1;
    }
  }
  if (!sh.all_ok()) {
    set_error("multi-device openTSNE: a rank stopped because a peer failed");
    return 1;
  }
  return 0;
}

}  // namespace fe
