// nccl_dyn.h — NCCL entry points resolved at run time.
//
// libdiffuse_moe does not link NCCL: a single-GPU layer needs none, and a process that already
// loaded NCCL (PyTorch bundles its own libnccl.so.2) must keep using that copy. The library
// dlopen()s "libnccl.so.2" the first time an expert-parallel layer is created; glibc returns the
// already-loaded object when one with that soname exists. The types come from the system
// nccl.h (the NCCL ABI is stable across 2.x minor versions).
#pragma once
#include <nccl.h>

#include <type_traits>

namespace dmoe {

struct NcclApi {
  bool ok = false;
  const char* why = "not loaded";
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommSplit)(ncclComm_t, int, int, ncclComm_t*, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

// Loads NCCL once per process; check .ok / .why.
const NcclApi& nccl();

}  // namespace dmoe
