// nccl_dyn.cpp — run-time binding of the NCCL calls used by the expert-parallel path.
#include "nccl_dyn.h"

#include <dlfcn.h>

#include <mutex>

namespace dmoe {

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      api.why = "libnccl.so.2 not found";
      return;
    }
    bool all = true;
    auto sym = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      all = all && fn != nullptr;
    };
    sym(api.GetUniqueId, "ncclGetUniqueId");
    sym(api.CommInitRankConfig, "ncclCommInitRankConfig");
    sym(api.CommSplit, "ncclCommSplit");
    sym(api.CommDestroy, "ncclCommDestroy");
    sym(api.CommAbort, "ncclCommAbort");
    sym(api.CommGetAsyncError, "ncclCommGetAsyncError");
    sym(api.Send, "ncclSend");
    sym(api.Recv, "ncclRecv");
    sym(api.Broadcast, "ncclBroadcast");
    sym(api.AllReduce, "ncclAllReduce");
    sym(api.GroupStart, "ncclGroupStart");
    sym(api.GroupEnd, "ncclGroupEnd");
    sym(api.GetErrorString, "ncclGetErrorString");
    api.ok = all;
    api.why = all ? "ok" : "libnccl.so.2 lacks a required symbol";
  });
  return api;
}

}  // namespace dmoe
