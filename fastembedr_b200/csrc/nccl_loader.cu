// Run-time resolution of the NCCL entry points used by sharded sessions.
#include "nccl_loader.cuh"

#include "fe_common.cuh"

#include <dlfcn.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

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

int comm_init(const void* unique_id, int nranks, int rank, ncclComm_t* out) {
  const NcclApi* api = nccl_api();
  if (api == nullptr) return 1;
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  return check_nccl(api->CommInitRank(out, nranks, id, rank), "ncclCommInitRank");
}

int check_nccl(ncclResult_t code, const char* where) {
  if (code == ncclSuccess) return 0;
  const char* text = g_ok ? g_api.GetErrorString(code) : "NCCL unavailable";
  set_error(std::string(where) + ": " + (text ? text : "NCCL error") + " (code " + std::to_string(code) + ")");
  return 1;
}

}  // namespace fe
