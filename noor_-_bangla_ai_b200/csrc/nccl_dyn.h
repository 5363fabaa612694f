// nccl_dyn.h -- NCCL entry points resolved at run time with dlopen.
//
// The library does not link libnccl: a process may already hold an NCCL
// (e.g. the one PyTorch ships), and two different libnccl.so.2 builds cannot
// share one process.  The first expert-parallel call resolves the entry points
// from whichever libnccl.so.2 the process has loaded, or loads one.
#pragma once

#include <dlfcn.h>
#include <nccl.h>

#include <mutex>

namespace noor {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  bool ok = false;
};

inline const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
#define NOOR_NCCL_SYM(field, name) api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name))
    NOOR_NCCL_SYM(GetUniqueId, "ncclGetUniqueId");
    NOOR_NCCL_SYM(CommInitRank, "ncclCommInitRank");
    NOOR_NCCL_SYM(CommDestroy, "ncclCommDestroy");
    NOOR_NCCL_SYM(CommAbort, "ncclCommAbort");
    NOOR_NCCL_SYM(GroupStart, "ncclGroupStart");
    NOOR_NCCL_SYM(GroupEnd, "ncclGroupEnd");
    NOOR_NCCL_SYM(Send, "ncclSend");
    NOOR_NCCL_SYM(Recv, "ncclRecv");
    NOOR_NCCL_SYM(AllReduce, "ncclAllReduce");
    NOOR_NCCL_SYM(AllGather, "ncclAllGather");
    NOOR_NCCL_SYM(GetErrorString, "ncclGetErrorString");
#undef NOOR_NCCL_SYM
    api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.CommAbort && api.GroupStart &&
             api.GroupEnd && api.Send && api.Recv && api.AllReduce && api.AllGather && api.GetErrorString;
  });
  return api;
}

}  // namespace noor
