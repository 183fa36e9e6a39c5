// Minimal NCCL binding resolved at run time (dlopen). The tensor-parallel engine
// uses only AllReduce/AllGather on a communicator built from a unique id; loading
// lazily keeps single-GPU use free of any NCCL dependency and, inside a PyTorch
// process, binds the same libnccl.so.2 instance torch already loaded.
#pragma once
#include <cuda_runtime.h>

#include <string>

namespace fb {

using NcclComm = void*;
constexpr int kNcclIdBytes = 128;
enum NcclType : int { kNcclUint8 = 1, kNcclInt32 = 2, kNcclFloat32 = 7 };
constexpr int kNcclInProgress = 7;  // ncclResult_t ncclInProgress (non-blocking operation still running)

struct Nccl {
    int (*GetUniqueId)(void* id) = nullptr;
    int (*AllReduce)(const void*, void*, size_t, int, int, NcclComm, cudaStream_t) = nullptr;
    int (*AllGather)(const void*, void*, size_t, int, NcclComm, cudaStream_t) = nullptr;
    int (*CommDestroy)(NcclComm) = nullptr;
    int (*CommAbort)(NcclComm) = nullptr;
    int (*CommGetAsyncError)(NcclComm, int*) = nullptr;
    const char* (*GetErrorString)(int) = nullptr;
    bool ok = false;
    std::string error;
};

// The process-wide binding (loaded on first use). `ok` is false when libnccl.so.2
// cannot be found; `error` says why.
Nccl& nccl();

// ncclCommInitRank with the 128-byte id passed by value, as the C API expects.
int nccl_comm_init_rank(NcclComm* comm, int nranks, const void* id, int rank);

}  // namespace fb
