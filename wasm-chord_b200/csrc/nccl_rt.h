// NCCL entry points resolved at run time. The library does not link NCCL: a
// process that also uses PyTorch must share one NCCL with it, so the first use
// takes the NCCL already loaded in the process if there is one, else the file
// named by WCB_NCCL_LIB (the Python package points it at the NCCL that
// PyTorch ships), else libnccl.so.2 from the loader's search path.
#pragma once
#include <nccl.h>

#include <string>

namespace wcb {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*CommAbort)(ncclComm_t);
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
  const char* (*GetErrorString)(ncclResult_t);
};

// The resolved table; throws WcbError (backend unsupported) when NCCL cannot be loaded.
const NcclApi& nccl();

}  // namespace wcb
