#include "nccl_rt.h"

#include <dlfcn.h>

#include <cstdlib>
#include <mutex>

#include "gguf.h"

namespace wcb {

namespace {

void* sym(void* h, const char* name) {
  void* p = dlsym(h, name);
  if (!p) throw WcbError(E_BACKEND, std::string("Backend error: NCCL symbol ") + name + " not found");
  return p;
}

}  // namespace

const NcclApi& nccl() {
  static std::mutex mu;
  static NcclApi api{};
  static bool ready = false;
  std::lock_guard<std::mutex> lk(mu);
  if (ready) return api;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // one already in the process
  if (!h) {
    const char* path = std::getenv("WCB_NCCL_LIB");
    if (path && *path) h = dlopen(path, RTLD_NOW | RTLD_GLOBAL);
  }
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) throw WcbError(E_BACKEND, std::string("Backend error: cannot load NCCL: ") + dlerror());
  api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(sym(h, "ncclGetUniqueId"));
  api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(sym(h, "ncclCommInitRank"));
  api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(sym(h, "ncclCommDestroy"));
  api.CommAbort = reinterpret_cast<decltype(api.CommAbort)>(sym(h, "ncclCommAbort"));
  api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(sym(h, "ncclAllReduce"));
  api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(sym(h, "ncclGetErrorString"));
  ready = true;
  return api;
}

}  // namespace wcb
