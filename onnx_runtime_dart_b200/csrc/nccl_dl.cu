#include <dlfcn.h>

#include <cstdlib>
#include <mutex>
#include <string>

#include "common.cuh"
#include "nccl_dl.cuh"

namespace ortc {

const NcclApi* nccl() {
  static std::once_flag once;
  static NcclApi api;
  static bool ok = false;
  static std::string err;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) {
      const char* path = std::getenv("ORT_CUDA_NCCL_LIB");
      h = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    }
    if (!h) {
      err = std::string("cannot load NCCL: ") + dlerror();
      return;
    }
#define ORTC_SYM(field, name)                                             \
  api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name));      \
  if (!api.field) {                                                       \
    err = std::string("NCCL symbol missing: ") + name;                    \
    return;                                                               \
  }
    ORTC_SYM(GetUniqueId, "ncclGetUniqueId");
    ORTC_SYM(CommInitRankConfig, "ncclCommInitRankConfig");
    ORTC_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
    ORTC_SYM(CommAbort, "ncclCommAbort");
    ORTC_SYM(CommFinalize, "ncclCommFinalize");
    ORTC_SYM(CommDestroy, "ncclCommDestroy");
    ORTC_SYM(AllGather, "ncclAllGather");
    ORTC_SYM(GetErrorString, "ncclGetErrorString");
#undef ORTC_SYM
    ok = true;
  });
  if (!ok) {
    set_error(err);
    return nullptr;
  }
  return &api;
}

}  // namespace ortc
