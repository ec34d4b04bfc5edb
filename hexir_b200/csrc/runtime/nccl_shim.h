// nccl_shim.h -- NCCL resolved at run time from libnccl.so.2.
//
// Only row-sharded dispatches need it (the weight broadcast, the root's
// output descriptor and the one-word completion all-reduce, and the row
// gather where peer stores are unavailable), so it is loaded on first use
// and a single-GPU or CPU program never touches it.  Types come from nccl.h
// at build time.
#pragma once

#include <nccl.h>

#include <string>

namespace hexir {

struct Nccl {
  bool ok = false;
  std::string error;
  ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommInitAll)(ncclComm_t *, int, const int *) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*Broadcast)(const void *, void *, size_t, ncclDataType_t, int,
                            ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t,
                       cudaStream_t) = nullptr;
  ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t,
                            ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t,
                       cudaStream_t) = nullptr;
  const char *(*GetErrorString)(ncclResult_t) = nullptr;
};

const Nccl &nccl();

std::string nccl_message(const char *call, ncclResult_t result);

}  // namespace hexir
