// NCCL, loaded at run time (dlopen of libnccl.so.2) so that the library
// neither needs NCCL for single-GPU use nor brings a second copy into a
// process that already loaded one (PyTorch ships its own libnccl.so.2; dlopen
// by soname returns the copy already loaded).
#pragma once

#include <nccl.h>

namespace fz {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  // non-blocking communicators (null when the loaded NCCL lacks them)
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
};

// The loaded API; fails (FZ_ECUDA) when libnccl.so.2 or a symbol is missing.
const NcclApi& nccl();

}  // namespace fz
