// NCCL entry points the multi-GPU build uses, resolved at run time.
//
// libungx.so does not link NCCL: single-GPU callers never need it, and a process that
// already loaded an NCCL (a framework's copy, say) must not get a second one.  The
// first multi-GPU call dlopen()s $UNGX_NCCL_LIBRARY when set, else the "libnccl.so.2"
// already in the process, else "libnccl.so.2" from the loader's search path, and
// resolves the functions below.  Only one libnccl.so.2 can live in a process: a
// framework that brings its own (and needs its newer symbols) is loaded before the
// first multi-GPU call.  Types and constants come from nccl.h; the library's own ABI
// never exposes them.
#pragma once

#include <nccl.h>

#include <string>
#include <type_traits>

namespace ungx
{

struct NcclApi
{
   ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
   ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
   ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
   ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
   ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
   ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
   ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
   ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
   ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
   ncclResult_t (*GroupStart)() = nullptr;
   ncclResult_t (*GroupEnd)() = nullptr;
   const char *(*GetErrorString)(ncclResult_t) = nullptr;
   ncclResult_t (*GetVersion)(int *) = nullptr;
};

// The process-wide table; nullptr with `err` set when NCCL cannot be loaded.
const NcclApi *nccl_api(std::string &err);

} // namespace ungx
