// NCCL entry points resolved with dlopen on first multi-GPU use.
//
// A single-GPU session never loads NCCL.  When a process already holds an
// NCCL (e.g. one loaded by the host framework) that copy is reused
// (RTLD_NOLOAD), so two different libnccl.so.2 builds never meet in one
// process; otherwise ORT_CUDA_NCCL_LIB (if set) or "libnccl.so.2" is loaded.
#pragma once

#include <nccl.h>

namespace ortc {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*CommAbort)(ncclComm_t);
  ncclResult_t (*CommFinalize)(ncclComm_t);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t);
  const char* (*GetErrorString)(ncclResult_t);
};

// Returns the resolved table, or nullptr (with the error text set).
const NcclApi* nccl();

// Polls a non-blocking communicator until its last call has completed,
// bounded by timeout_ms (session.cu).
int nccl_wait_ready(ncclComm_t comm, int timeout_ms);

}  // namespace ortc
