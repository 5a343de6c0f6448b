// nls_nccl.cu -- NCCL for the vocab-sharded entry point, resolved at run time.
//
// The library does not link NCCL: a process that already holds one (a
// PyTorch process loads its own) must not get a second copy with another
// version, so the functions are looked up in the libnccl.so.2 already loaded,
// else in the one the dynamic loader finds. Only nccl.h's types are used at
// build time.
#include <dlfcn.h>

#include <mutex>

#include "nls_nccl.h"

namespace nls {

namespace {

template <class F>
bool sym(void* lib, const char* name, F* out) {
  *out = reinterpret_cast<F>(dlsym(lib, name));
  return *out != nullptr;
}

}  // namespace

const NcclApi& nccl_api() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!lib) return;
    api.ok = sym(lib, "ncclGetUniqueId", &api.GetUniqueId) &&
             sym(lib, "ncclCommInitRank", &api.CommInitRank) &&
             sym(lib, "ncclCommInitRankConfig", &api.CommInitRankConfig) &&
             sym(lib, "ncclCommGetAsyncError", &api.CommGetAsyncError) &&
             sym(lib, "ncclCommAbort", &api.CommAbort) &&
             sym(lib, "ncclCommDestroy", &api.CommDestroy) &&
             sym(lib, "ncclGroupStart", &api.GroupStart) && sym(lib, "ncclGroupEnd", &api.GroupEnd) &&
             sym(lib, "ncclSend", &api.Send) && sym(lib, "ncclRecv", &api.Recv) &&
             sym(lib, "ncclAllGather", &api.AllGather) &&
             sym(lib, "ncclGetErrorString", &api.GetErrorString);
  });
  return api;
}

}  // namespace nls
