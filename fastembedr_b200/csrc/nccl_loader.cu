// Run-time resolution of the NCCL entry points used by sharded sessions.
#include "nccl_loader.cuh"

#include "fe_common.cuh"

#include <dlfcn.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

namespace fe {
namespace {

NcclApi g_api;
bool g_ok = false;
std::string g_load_error;
std::once_flag g_once;

template <typename F>
bool resolve(void* lib, const char* name, F* out) {
  *out = reinterpret_cast<F>(dlsym(lib, name));
  if (*out == nullptr) {
    g_load_error = std::string("NCCL symbol ") + name + " not found";
    return false;
  }
  return true;
}

void load_once() {
  const char* path = std::getenv("FASTEMBEDR_B200_NCCL_LIB");
  if (path == nullptr || *path == '\0') path = "libnccl.so.2";
  void* lib = dlopen(path, RTLD_NOW | RTLD_GLOBAL);
  if (lib == nullptr) {
    const char* why = dlerror();
    g_load_error = std::string("cannot load NCCL (") + path + "): " + (why ? why : "unknown error");
    return;
  }
  g_ok = resolve(lib, "ncclGetUniqueId", &g_api.GetUniqueId) &&
         resolve(lib, "ncclCommInitRank", &g_api.CommInitRank) &&
         resolve(lib, "ncclCommInitRankConfig", &g_api.CommInitRankConfig) &&
         resolve(lib, "ncclCommGetAsyncError", &g_api.CommGetAsyncError) &&
         resolve(lib, "ncclCommDestroy", &g_api.CommDestroy) &&
         resolve(lib, "ncclCommAbort", &g_api.CommAbort) &&
         resolve(lib, "ncclAllReduce", &g_api.AllReduce) &&
         resolve(lib, "ncclAllGather", &g_api.AllGather) &&
         resolve(lib, "ncclGetErrorString", &g_api.GetErrorString);
}

}  // namespace

const NcclApi* nccl_api() {
  std::call_once(g_once, load_once);
  if (!g_ok) {
    set_error(g_load_error);
    return nullptr;
  }
  return &g_api;
}

namespace {
thread_local double t_join_limit = 0.0;
}  // namespace

double join_timeout_seconds() {
  const char* v = std::getenv("FASTEMBEDR_B200_NCCL_INIT_TIMEOUT_S");
  if (v == nullptr || *v == '\0') return t_join_limit;
  const double s = std::strtod(v, nullptr);
  return s > 0.0 ? s : 0.0;
}

JoinLimit::JoinLimit(double seconds) : prev_(t_join_limit) { t_join_limit = seconds; }
JoinLimit::~JoinLimit() { t_join_limit = prev_; }

namespace {

// Polls the communicator's state while NCCL reports ncclInProgress, up to
// `limit_s` seconds (0: no limit).  Returns the last state; *timed_out tells
// whether the limit ended the wait.
ncclResult_t await_state(ncclComm_t comm, double limit_s, bool* timed_out) {
  using clock = std::chrono::steady_clock;
  const auto start = clock::now();
  ncclResult_t state = ncclInProgress;
  *timed_out = false;
  for (;;) {
    const ncclResult_t q = g_api.CommGetAsyncError(comm, &state);
    if (q != ncclSuccess) return q;
    if (state != ncclInProgress) return state;
    if (limit_s > 0.0 && std::chrono::duration<double>(clock::now() - start).count() >= limit_s) {
      *timed_out = true;
      return state;
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
}

std::string seconds_text(double s) {
  char buf[32];
  std::snprintf(buf, sizeof(buf), "%g", s);
  return buf;
}

}  // namespace

int check_nccl_call(ncclComm_t comm, ncclResult_t code, const char* where) {
  if (code == ncclInProgress && g_ok && comm != nullptr) {
    bool timed_out = false;
    const double limit = join_timeout_seconds();
    code = await_state(comm, limit, &timed_out);
    if (timed_out) {
      set_error(std::string(where) + ": still in progress after " + seconds_text(limit) + " s");
      return 1;
    }
  }
  return check_nccl(code, where);
}

int comm_init(const void* unique_id, int nranks, int rank, ncclComm_t* out) {
  const NcclApi* api = nccl_api();
  if (api == nullptr) return 1;
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  const double limit = join_timeout_seconds();
  if (limit <= 0.0) return check_nccl(api->CommInitRank(out, nranks, id, rank), "ncclCommInitRank");

  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;
  *out = nullptr;
  ncclResult_t code = api->CommInitRankConfig(out, nranks, id, rank, &config);
  bool timed_out = false;
  if (code == ncclInProgress && *out != nullptr) code = await_state(*out, limit, &timed_out);
  if (code == ncclSuccess && !timed_out) return 0;
  if (*out != nullptr) api->CommAbort(*out);  // ends NCCL's join threads; the communicator is gone
  *out = nullptr;
  if (timed_out) {
    set_error("ncclCommInitRankConfig: timed out after " + seconds_text(limit) + " s waiting for the other " +
              std::to_string(nranks - 1) + " rank(s) to join (rank " + std::to_string(rank) +
              "); communicator aborted");
    return 1;
  }
  return check_nccl(code, "ncclCommInitRankConfig");
}

int check_nccl(ncclResult_t code, const char* where) {
  if (code == ncclSuccess) return 0;
  const char* text = g_ok ? g_api.GetErrorString(code) : "NCCL unavailable";
  set_error(std::string(where) + ": " + (text ? text : "NCCL error") + " (code " + std::to_string(code) + ")");
  return 1;
}

}  // namespace fe
