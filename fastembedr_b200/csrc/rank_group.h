// Host-side coordination of the ranks that one process runs itself, one host
// thread per GPU (the single-process multi-device mode, multi_device.cu).
// Host C++ only, so a CPU test drives the same code with a stand-in NCCL.
//
// The rules it enforces:
//   * ranks agree on the host before every collective: a rank enqueues
//     collective c only after every rank has arrived at c, and a failed rank
//     never arrives; the others then return instead of enqueueing c, so a
//     host-side failure leaves no collective waiting on the device for it;
//   * a rank's NCCL calls and the abort of its communicator take the same
//     lock, and an aborted communicator's slot is cleared under it, so no
//     NCCL call reaches a communicator after its abort;
//   * a rank whose own enqueue failed after the others had arrived leaves
//     their collective without a peer: the group then asks for an abort of
//     every communicator (abort_needed), which ends those collectives.
// Together with at most one collective in flight per rank (the caller waits
// for the previous one to complete before arriving at the next), an abort can
// only ever end the newest collective: no later NCCL kernel is queued behind
// it on any rank's stream.
#pragma once

#include <atomic>
#include <condition_variable>
#include <memory>
#include <mutex>
#include <vector>

namespace fe {

class RankGroup {
 public:
  enum Status { kOk = 0, kPeerFailed = 1, kAborted = 2, kIssueFailed = 3 };

  explicit RankGroup(int nranks) : n_(nranks), locks_(new std::mutex[nranks]), slots_(nranks) {
    for (auto& s : slots_) s.store(nullptr);
  }

  int size() const { return n_; }

  // The communicator rank `rank` issues its collectives on (null: none yet, or aborted).
  void set_comm(int rank, void* comm) {
    std::lock_guard<std::mutex> l(locks_[rank]);
    slots_[rank].store(comm);
  }
  // Takes the communicator out of the slot (exactly once) for destroy or abort.
  void* take_comm(int rank) {
    std::lock_guard<std::mutex> l(locks_[rank]);
    return slots_[rank].exchange(nullptr);
  }

  // Waits until every rank has arrived at the same collective (true) or any
  // rank has failed (false).  A failed rank must not call this again.
  bool arrive() {
    std::unique_lock<std::mutex> g(m_);
    if (failed_) return false;
    const unsigned long long gen = gen_;
    if (++count_ == n_) {
      count_ = 0;
      ++gen_;
      cv_.notify_all();
      return true;
    }
    cv_.wait(g, [&] { return gen_ != gen || failed_; });
    return gen_ != gen;  // every rank arrived, even if one failed just after
  }

  // Marks the group failed and releases every rank waiting in arrive().
  // orphaned: the failing rank had already arrived at a collective that its
  // peers may have enqueued, so their communicators must be aborted.
  void fail(bool orphaned = false) {
    {
      std::lock_guard<std::mutex> g(m_);
      failed_ = true;
      if (orphaned) abort_needed_.store(true);
    }
    cv_.notify_all();
  }
  bool failed() const {
    std::lock_guard<std::mutex> g(m_);
    return failed_;
  }
  bool abort_needed() const { return abort_needed_.load(); }

  // One collective of rank `rank`: arrive, then, under the rank's lock and
  // only while its communicator is still in the slot, issue(comm) (0 = enqueued).
  template <typename Issue>
  Status collective(int rank, Issue&& issue) {
    if (!arrive()) return kPeerFailed;
    std::lock_guard<std::mutex> l(locks_[rank]);
    void* comm = slots_[rank].load();
    if (comm == nullptr) return kAborted;
    if (issue(comm) != 0) {
      fail(true);
      return kIssueFailed;
    }
    return kOk;
  }

  // Aborts every communicator still in a slot, each under its rank's lock,
  // and clears the slots; abort(comm) is called once per communicator.
  template <typename Abort>
  void abort_all(Abort&& abort) {
    for (int r = 0; r < n_; ++r) {
      std::lock_guard<std::mutex> l(locks_[r]);
      void* comm = slots_[r].exchange(nullptr);
      if (comm != nullptr) abort(comm);
    }
  }

 private:
  const int n_;
  mutable std::mutex m_;
  std::condition_variable cv_;
  int count_ = 0;
  unsigned long long gen_ = 0;
  bool failed_ = false;
  std::atomic<bool> abort_needed_{false};
  std::unique_ptr<std::mutex[]> locks_;
  std::vector<std::atomic<void*>> slots_;
};

}  // namespace fe
