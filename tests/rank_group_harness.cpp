// Drives fe::RankGroup (fastembedr_b200/csrc/rank_group.h, the coordination
// the single-process multi-device mode uses for its collectives) with host
// threads and the tracked stand-in NCCL (tests/fake_nccl.c built with
// -DFAKE_NCCL_TRACK).  No GPU is involved.  Built and run by
// tests/test_rank_group_cpu.py.
//
//   rank_group_harness <scenario> <nranks> <collectives> <fail_rank> <fail_at> <seed>
//
// scenario "host":    rank fail_rank fails on the host just before its
//                     collective fail_at (it never arrives there);
// scenario "enqueue": rank fail_rank's NCCL call number fail_at returns an
//                     error after every rank has arrived at it (its peers have
//                     enqueued theirs), which asks for an abort.
// Each rank thread issues collectives through RankGroup::collective on its
// fake communicator and sleeps a random few microseconds between them; a
// watcher thread aborts every communicator once the group asks for it, as
// opentsne_multi_device does.  Prints one line:
//   calls=<c0,c1,...> statuses=<s0,...> aborts=<a> after_abort=<v>
#include "../fastembedr_b200/csrc/rank_group.h"

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <thread>
#include <vector>

extern "C" {
typedef struct {
  char internal[128];
} fake_unique_id;
int ncclCommInitRank(void** comm, int nranks, fake_unique_id id, int rank);
int ncclAllGather(const void* s, void* r, unsigned long n, int t, void* c, void* st);
int ncclAllReduce(const void* s, void* r, unsigned long n, int t, int op, void* c, void* st);
int ncclCommAbort(void* comm);
int ncclCommDestroy(void* comm);
void fake_nccl_reset(void);
void fake_nccl_fail_call(int rank, int call);
int fake_nccl_calls(int rank);
int fake_nccl_calls_after_abort(void);
int fake_nccl_aborts(void);
}

int main(int argc, char** argv) {
  if (argc != 7) {
    std::fprintf(stderr, "usage: %s host|enqueue nranks collectives fail_rank fail_at seed\n", argv[0]);
    return 2;
  }
  const std::string scenario = argv[1];
  const int nranks = std::atoi(argv[2]);
  const int collectives = std::atoi(argv[3]);
  const int fail_rank = std::atoi(argv[4]);
  const int fail_at = std::atoi(argv[5]);
  const unsigned seed = static_cast<unsigned>(std::atoi(argv[6]));
  fake_nccl_reset();
  if (scenario == "enqueue") fake_nccl_fail_call(fail_rank, fail_at);

  fe::RankGroup group(nranks);
  std::vector<void*> comms(nranks, nullptr);
  fake_unique_id id;
  std::memset(&id, 0, sizeof(id));
  for (int r = 0; r < nranks; ++r) {
    ncclCommInitRank(&comms[r], nranks, id, r);
    group.set_comm(r, comms[r]);
  }
  std::vector<int> status(nranks, 0);
  std::atomic<int> finished{0};
  auto rank_main = [&](int r) {
    std::mt19937 rng(seed * 977u + static_cast<unsigned>(r));
    int st = fe::RankGroup::kOk;
    for (int c = 0; c < collectives && st == fe::RankGroup::kOk; ++c) {
      if (scenario == "host" && r == fail_rank && c == fail_at) {
        group.fail();
        st = -1;  // failed on the host
        break;
      }
      st = group.collective(r, [&](void* comm) {
        return (c & 1) ? ncclAllGather(nullptr, nullptr, 0, 0, comm, nullptr)
                       : ncclAllReduce(nullptr, nullptr, 0, 0, 0, comm, nullptr);
      });
      std::this_thread::sleep_for(std::chrono::microseconds(rng() % 50));
    }
    status[r] = st;
    ++finished;
  };
  std::vector<std::thread> threads;
  for (int r = 0; r < nranks; ++r) threads.emplace_back(rank_main, r);
  auto abort_comm = [](void* c) { ncclCommAbort(c); };
  while (finished.load() < nranks) {
    if (group.abort_needed()) group.abort_all(abort_comm);
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
  for (auto& t : threads) t.join();
  if (group.abort_needed()) group.abort_all(abort_comm);
  // Tear-down as the multi-device mode does it: whatever is still in a slot
  // is aborted after a failure, destroyed otherwise.
  for (int r = 0; r < nranks; ++r) {
    void* c = group.take_comm(r);
    if (c == nullptr) continue;
    if (group.failed()) ncclCommAbort(c);
    else ncclCommDestroy(c);
  }
  std::string calls, statuses;
  for (int r = 0; r < nranks; ++r) {
    calls += (r ? "," : "") + std::to_string(fake_nccl_calls(r));
    statuses += (r ? "," : "") + std::to_string(status[r]);
  }
  std::printf("calls=%s statuses=%s aborts=%d after_abort=%d\n", calls.c_str(), statuses.c_str(),
              fake_nccl_aborts(), fake_nccl_calls_after_abort());
  return 0;
}
